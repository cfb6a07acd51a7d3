"""Benchmark of the tiered paged-decode hot path (headline metric: paged-decode tok/s and
local+peer GB/s as % of roofline).

Default workload (headline config 2: one B200, all-local): a full 36-layer
Qwen3-8B-shaped KV pool of 1,048,576 token slots per plane (72 planes x 2 KiB
x (C+1) slots = 154.6 GB in HBM), batch 64, KV lengths uniform in [2048, 32768]
(seeded; redrawn with the next seed while the sum exceeds the pool), slots a
seeded random permutation of the pool, Q/K/V ~ N(0, 1) bf16.  One step = the
packer (unified read order for the batch) + 36 layers of tiered decode
(one kernel per layer; split requests are merged inside it).  Per-layer KV (4.5 GB) is far larger than L2, so no
flush is needed between iterations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl dual|reference] [--workload W]

Workloads: config2 (default), small; config3, config5, tiered-small, and config3-local / config3-r12
(config 3's batch with no remote rows / twice its remote share) (a compute GPU + a supplier GPU;
under torchrun N/2 such pairs); config4, append-small, append-mid (causal append; --stage range|rows
stages the supplier rows per layer); migration; fi-<workload> times native FlashInfer FA2 on the
same inputs (the number to beat).

Under torchrun (N > 1) the default is config 5's layout: N/2 (compute GPU r, supplier GPU r + N/2)
pairs, each compute GPU decoding its own batch with its supplier's rows read over NVLink and a
concurrent migration; `--workload config2` runs N independent all-local replicas instead.  Decode
shards by request, with no collective on the data path: scaling "weak".
``--impl reference`` times the reference's CPU attention math (the fp32 oracle
restatement of check_attention_output) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
import types
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
METRIC = "paged-decode tok/s and local+peer GB/s as % roofline at 1/2/4/8 B200"
UNIT = "tok/s"
FALLBACK_HBM_GBS = 6650.0

WORKLOADS = {
    # name: (batch, Lmin, Lmax, pool slots C, layers resident)
    "config2": (64, 2048, 32768, 1 << 20, 36),
    "small": (16, 2048, 32768, 1 << 18, 4),
}
# Tiered multi-GPU workloads (one process, compute GPU 0 + supplier GPU 1 reached by peer access):
# name: (batch, Lmin, Lmax, remote/local ratio, remote placement, RN, TN, layers resident, migrate)
TIERED = {
    "config3": (128, 2048, 32768, 0.0599, "tail", 8, 128, 6, False),
    # config 3 at equal batch with no remote rows and with twice its remote share (all-local comparison)
    "config3-local": (128, 2048, 32768, 0.0, "tail", 8, 128, 6, False),
    "config3-r12": (128, 2048, 32768, 0.12, "tail", 8, 128, 6, False),
    "config5": (128, 4096, 32768, 0.1797, "prefix", 5, 32, 6, True),
    # profiling case: config-5 ratios and read order, 16 requests, 2 resident layers (~3 GB on the device)
    "tiered-small": (16, 4096, 32768, 0.1797, "prefix", 5, 32, 2, False),
}
PEER_GBS = 770.0  # measured peer copy per direction on this pool (NVLink 5, NVSwitch)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["dual", "reference"], default="dual")
    ap.add_argument("--workload", choices=list(WORKLOADS) + list(TIERED) + ["migration"] + list(APPEND)
                    + ["fi-" + w for w in list(WORKLOADS) + list(APPEND)],
                    default=None,
                    help="default: config2 on one GPU; config5 (N/2 compute + supplier pairs) under torchrun")
    ap.add_argument("--seed", type=int, default=20261101)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-flashinfer", action="store_true",
                    help="config2: skip timing native FlashInfer FA2 on the same inputs after the dual_b200 arm")
    ap.add_argument("--mig-ctas", type=int, default=64,
                    help="tiered workloads with migration: CTAs of the side-stream copy")
    ap.add_argument("--stage", choices=["range", "rows"], default=None,
                    help="append workloads: stage each layer's supplier rows into local memory first "
                         "(LayerStager: 'range' = copy engines, one stream per bank, overlapped with the "
                         "previous layer's append; 'rows' = the row kernel before each append)")
    return ap.parse_args()


def draw_lengths(batch, lmin, lmax, capacity, seed):
    """Seeded U[lmin, lmax] lengths; redraw with seed+1, ... while the sum exceeds the pool."""
    for k in range(1000):
        rng = np.random.default_rng(seed + k)
        L = rng.integers(lmin, lmax + 1, batch)
        if L.sum() <= capacity:
            return L.astype(np.int64), seed + k
    raise RuntimeError("could not draw lengths that fit the pool")


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi SM clock / throttle sampling during the timed region (exact PID, no patterns)."""

    def __init__(self, gpu_index: int):
        self.proc = None
        self.gpu = gpu_index

    def start(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons, watts = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            try:
                watts.append(float(f[2]))
            except ValueError:
                pass
            for name, val in zip(names, f[3:7]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "power_w": statistics.median(watts) if watts else None}


# ------------------------------------------------------------ sampled parity against the oracle
# The north star's bar: bf16 attention outputs and base-2 LSEs within 2e-3 abs / 1e-2 rel of the fp32
# reference math.  After the timed region, a few requests of the last timed layer are recomputed on
# the CPU by the oracle (oracle.attention, the restatement of the reference's explicit-math check);
# the oracle is only the checker here, never part of what is timed.
ATOL, RTOL = 2e-3, 1e-2


def gather_rows(pages, C, local, banks):
    """Rows named by unified page ids (local slot p <= C, else global remote id g = p - C - 1 in
    bank g % n at row g // n), gathered on the pools' devices and returned on the CPU."""
    dev = local.device
    pages = pages.to(dev).long()
    far = pages > C
    out = torch.empty((pages.numel(), 8, 128), dtype=local.dtype, device=dev)
    near = torch.nonzero(~far).squeeze(1)
    out[near] = local.index_select(0, pages[near])
    fidx = torch.nonzero(far).squeeze(1)
    if fidx.numel():
        g = pages[fidx] - C - 1
        n = len(banks)
        for d in range(n):
            sel = torch.nonzero(g % n == d).squeeze(1)
            if sel.numel():
                out[fidx[sel]] = banks[d].index_select(0, (g[sel] // n).to(banks[d].device)).to(dev)
    return out.cpu()


class ParityTally:
    """max |err| and max |err| / |ref| over the sampled outputs, max |err| of the LSEs, and whether every
    element meets |got - ref| <= ATOL + RTOL |ref| (torch.allclose)."""

    def __init__(self):
        self.max_abs = self.max_rel = self.lse_max_abs = self.worst = 0.0
        self.ok = True
        self.samples = []

    def add(self, got, ref, got_lse, ref_lse, label):
        got, ref = got.float().cpu(), ref.float().cpu()
        got_lse, ref_lse = got_lse.float().cpu(), ref_lse.float().cpu()
        err = (got - ref).abs()
        lerr = (got_lse - ref_lse).abs()
        self.max_abs = max(self.max_abs, float(err.max()))
        big = ref.abs() > ATOL
        if big.any():
            self.max_rel = max(self.max_rel, float((err[big] / ref.abs()[big]).max()))
        self.lse_max_abs = max(self.lse_max_abs, float(lerr.max()))
        self.worst = max(self.worst, float((err / (ATOL + RTOL * ref.abs())).max()),
                         float((lerr / (ATOL + RTOL * ref_lse.abs())).max()))
        self.ok &= bool(torch.allclose(got, ref, atol=ATOL, rtol=RTOL) and
                        torch.allclose(got_lse, ref_lse, atol=ATOL, rtol=RTOL))
        self.samples.append(label)

    def result(self):
        return {"max_abs": round(self.max_abs, 6), "max_rel": round(self.max_rel, 6),
                "lse_max_abs": round(self.lse_max_abs, 6), "worst_over_tolerance": round(self.worst, 4),
                "tolerance": {"atol": ATOL, "rtol": RTOL}, "samples": self.samples,
                "checker": "oracle.attention (fp32 reference math, CPU)", "pass": self.ok}


def decode_picks(lengths, num_ctas, extra=(), limit=8):
    """Requests to check: the longest, the shortest, the median, and the requests holding the token
    where CTAs 1, G/2 and G-1 begin (their lists are split across CTAs and merged), plus `extra`."""
    lengths = np.asarray(lengths)
    order = np.argsort(lengths, kind="stable")
    ends = np.cumsum(lengths)
    T = int(ends[-1])
    picks = [int(order[-1]), int(order[0]), int(order[len(order) // 2])]
    for g in (1, num_ctas // 2, num_ctas - 1):
        tok = g * T // num_ctas
        picks.append(int(np.searchsorted(ends, tok, side="right")))
    picks += [int(x) for x in extra]
    out = []
    for b in picks:
        if 0 <= b < len(lengths) and b not in out and lengths[b] > 0:
            out.append(b)
    return out[:limit]


def decode_parity(q, out, lse, k, v, C, peer_k, peer_v, indptr_h, indices, picks, scale):
    """Sampled requests of one decode layer against the oracle."""
    from oracle.attention import attend
    tally = ParityTally()
    for b in picks:
        s, e = int(indptr_h[b]), int(indptr_h[b + 1])
        pages = indices[s:e]
        kr, vr = gather_rows(pages, C, k, peer_k), gather_rows(pages, C, v, peer_v)
        far = int((pages.long() > C).sum())
        ro, rl = attend(q[b:b + 1].cpu(), kr, vr, e - s - 1, scale)
        tally.add(out[b:b + 1], ro, lse[b:b + 1], rl, f"request {b}: L={e - s}, remote={far}")
    return tally.result()


# ------------------------------------------------------------------- dual arm
class DecodeWorkload:
    def __init__(self, args, device):
        from dual_b200 import ops
        self.ops = ops
        B, lmin, lmax, C, layers = WORKLOADS[args.workload]
        self.B, self.C, self.layers, self.device = B, C, layers, device
        self.lengths, self.seed_used = draw_lengths(B, lmin, lmax, C, args.seed)
        self.T = int(self.lengths.sum())
        g = torch.Generator(device=device).manual_seed(args.seed)
        # 36 layers x (K, V) planes, page 0 is SGLang's dummy slot
        self.k = [torch.empty((C + 1, 8, 128), dtype=torch.bfloat16, device=device) for _ in range(layers)]
        self.v = [torch.empty((C + 1, 8, 128), dtype=torch.bfloat16, device=device) for _ in range(layers)]
        for t in self.k + self.v:
            t.normal_(generator=g)
        perm = (torch.randperm(C, generator=g, device=device) + 1).to(torch.int32)
        maxL = int(self.lengths.max())
        self.tier = torch.full((B, maxL), -1, dtype=torch.int32, device=device)
        self.slot = torch.zeros((B, maxL), dtype=torch.int32, device=device)
        off = 0
        for b, L in enumerate(self.lengths.tolist()):
            self.tier[b, :L] = 0
            self.slot[b, :L] = perm[off:off + L]
            off += L
        self.req = torch.arange(B, dtype=torch.int32, device=device)
        self.seq = torch.tensor(self.lengths, dtype=torch.int32, device=device)
        self.indptr = torch.tensor(np.concatenate([[0], np.cumsum(self.lengths)]), dtype=torch.int32, device=device)
        self.indices = torch.empty(self.T, dtype=torch.int32, device=device)
        self.q = torch.randn((layers, B, 32, 128), generator=g, device=device).to(torch.bfloat16)
        self.out = torch.empty((layers, B, 32, 128), dtype=torch.bfloat16, device=device)
        self.lse = torch.empty((layers, B, 32), dtype=torch.float32, device=device)
        self.num_ctas = ops.default_ctas(device.index)
        self.ws = torch.zeros(ops.decode_workspace_size(B, self.num_ctas), dtype=torch.uint8, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.scale = 128 ** -0.5

    def step(self, events=None):
        ops = self.ops
        ops.pack_read_order(self.tier, self.slot, self.req, self.seq, self.C, 5, 32, self.indices, status=self.status)
        torch.cuda.nvtx.range_push("decode_layers")
        for i in range(self.layers):
            if events is not None:
                events[i][0].record()
            ops.tiered_decode(self.q[i], self.k[i], self.v[i], self.C, [], [], self.indptr, self.indices, self.scale,
                              self.out[i], self.lse[i], self.ws, self.num_ctas)
            if events is not None:
                events[i][1].record()
        torch.cuda.nvtx.range_pop()

    def bytes_per_layer(self):
        return 4096 * self.T + 8192 * self.B * 2 + 128 * self.B

    def launches_per_step(self):
        return 1 + self.layers

    def parity(self):
        """Sampled requests of the last layer of the last timed step against the oracle."""
        lyr = self.layers - 1
        picks = decode_picks(self.lengths, self.num_ctas)
        indptr_h = np.concatenate([[0], np.cumsum(self.lengths)])
        return decode_parity(self.q[lyr], self.out[lyr], self.lse[lyr], self.k[lyr], self.v[lyr], self.C, [], [],
                             indptr_h, self.indices, picks, self.scale)


class E2E:
    """Same metric through the public wrapper API with host buffers: per step H2D of the step's
    queries (pinned), plan(), the packer, 36 x wrapper.run, D2H of the outputs (pinned).  The copies
    are pipelined by layer inside the step, as a serving process would issue them: layer l's queries
    go up on an H2D stream and its output comes back on a D2H stream as soon as layer l is done, so
    only layer 0's upload and layer 35's download are exposed; the step ends when every output of
    the step is in host memory."""

    def __init__(self, w: DecodeWorkload):
        from dual_b200.wrapper import BatchDecodeWithPagedKVCacheWrapper
        self.w = w
        self.q_host = torch.randn(w.q.shape, dtype=torch.float32).to(torch.bfloat16).pin_memory()
        self.out_host = torch.empty(w.out.shape, dtype=torch.bfloat16).pin_memory()
        self.indptr_host = w.indptr.cpu().pin_memory()
        self.q_dev = torch.empty_like(w.q)
        self.wrapper = BatchDecodeWithPagedKVCacheWrapper(torch.empty(64 << 20, dtype=torch.uint8, device=w.device),
                                                          "NHD", use_tensor_cores=True)
        self.last = torch.ones(w.B, dtype=torch.int32)
        self.h2d = torch.cuda.Stream(w.device)
        self.d2h = torch.cuda.Stream(w.device)
        self.q_ready = [torch.cuda.Event() for _ in range(w.layers)]
        self.out_ready = [torch.cuda.Event() for _ in range(w.layers)]

    def step(self):
        w = self.w
        cur = torch.cuda.current_stream(w.device)
        self.h2d.wait_stream(cur)  # the previous step's layers are done with q_dev
        with torch.cuda.stream(self.h2d):
            for i in range(w.layers):
                self.q_dev[i].copy_(self.q_host[i], non_blocking=True)
                self.q_ready[i].record(self.h2d)
        w.ops.pack_read_order(w.tier, w.slot, w.req, w.seq, w.C, 5, 32, w.indices, status=w.status)
        self.wrapper.plan(self.indptr_host, w.indices, self.last, 32, 8, 128, 1, q_data_type=torch.bfloat16,
                          sm_scale=w.scale)
        for i in range(w.layers):
            cur.wait_event(self.q_ready[i])
            self.wrapper.run(self.q_dev[i], (w.k[i], w.v[i]), out=w.out[i])
            self.out_ready[i].record(cur)
            self.d2h.wait_event(self.out_ready[i])
            with torch.cuda.stream(self.d2h):
                self.out_host[i].copy_(w.out[i], non_blocking=True)
        cur.wait_stream(self.d2h)  # the step ends when its outputs are in host memory

    def h2d_bytes(self):
        return self.q_host.numel() * 2 + self.indptr_host.numel() * 4

    def d2h_bytes(self):
        return self.out_host.numel() * 2


def cpu_baseline(w: DecodeWorkload, budget_s=12.0):
    """Reference fp32 attention math (oracle restatement) on the host cores, bounded sample:
    a few of this batch's requests for one layer, repeated until ~budget_s; scaled to tok/s."""
    from oracle.attention import attend
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    order = np.argsort(w.lengths)
    picks = [int(order[len(order) // 2]), int(order[len(order) // 4]), int(order[3 * len(order) // 4])]
    data = []
    for b in picks:
        L = int(w.lengths[b])
        s = w.slot[b, :L].long()
        data.append((w.q[0, b:b + 1].cpu(), w.k[0].index_select(0, s).cpu(), w.v[0].index_select(0, s).cpu(), L))
    tokens, t0 = 0, time.perf_counter()
    reps = 0
    while True:
        for q, k, v, L in data:
            attend(q, k, v, L - 1, w.scale)
            tokens += L
        reps += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    per_token_layer = dt / tokens                       # seconds per KV token per layer
    step_s = per_token_layer * w.T * w.layers           # whole batch, all layers
    return {"value": w.B / step_s, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{len(picks)} of {w.B} requests (L={[d[3] for d in data]}), layer 0, x{reps} reps; "
                      f"scaled by sum(L)={w.T} and {w.layers} layers"}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device(f"cuda:{local}"))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world, device):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_dual(args):
    world, rank, local = dist_setup(args)
    device = torch.device(f"cuda:{local}")
    torch.cuda.set_device(device)
    w = DecodeWorkload(args, device)
    stream = torch.cuda.current_stream(device)
    for _ in range(max(args.warmup, 3)):
        w.step()
    torch.cuda.synchronize()
    status = int(w.status.item()) | int(w.ws[:4].view(torch.int32).item())
    # timed region
    events = [[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(w.layers)]
    layer_ms = []
    clocks = ClockSampler(device.index if "CUDA_VISIBLE_DEVICES" not in os.environ else
                          int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local]))
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    all_events = []
    for _ in range(args.steps):
        ev = [[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(w.layers)]
        w.step(ev)
        all_events.append(ev)
    t1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    ms = t0.elapsed_time(t1)
    for ev in all_events:
        layer_ms += [a.elapsed_time(b) for a, b in ev]
    ms_max = max_over_ranks(ms, world, device)
    tok = w.B * args.steps * world
    value = tok / (ms_max / 1e3)
    layer_avg = sum(layer_ms) / len(layer_ms)
    peak, peak_kind = measured_peaks()
    achieved = w.bytes_per_layer() / (layer_avg / 1e3) / 1e9
    result = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{args.workload}: 1xB200 all-local tiered paged decode, {w.layers} layers",
                   "batch_per_gpu": w.B, "kv_len": f"U[{WORKLOADS[args.workload][1]},{WORKLOADS[args.workload][2]}]",
                   "sum_kv_tokens": w.T, "length_seed": w.seed_used, "pool_slots": w.C, "layers": w.layers,
                   "heads": "32q/8kv x 128", "page_size": 1, "parallelism": f"replicas x{world} (request-sharded)",
                   "l2": f"inputs larger than L2 ({w.bytes_per_layer() / 1e9:.2f} GB per layer)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic_per_launch(w),
                     "peak_source": f"{peak_kind} hbm_gbs", "kernel": "tiered_decode_kernel",
                     "layer_ms": round(layer_avg, 4), "algorithmic_bytes_per_launch": w.bytes_per_layer()},
        "gpu_launches": w.launches_per_step() * args.steps,
        "device_status": status,
    }
    if clk:
        result["clocks"] = clk
    result["parity"] = w.parity()  # outside the timed region: the last timed step's outputs
    if not args.no_e2e:
        result["e2e"] = run_e2e(w, args, world, device)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(w)
    if world == 1 and not args.no_flashinfer:
        fi = flashinfer_decode(w, args)
        if "value" in fi:
            fi["dual_over_flashinfer"] = round(result["value"] / fi["value"], 4)
        result["flashinfer_native"] = fi
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def traffic_per_launch(w):
    """DRAM bytes per decode launch from the committed ncu summary (bytes per KV token, scaled)."""
    p = ROOT / "profiles" / "decode_traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    return int(d["dram_bytes_per_kv_token"] * w.T + d.get("dram_bytes_per_request", 0) * w.B)


def run_e2e(w, args, world, device):
    e = E2E(w)
    for _ in range(3):
        e.step()
    torch.cuda.synchronize()
    barrier(world)
    stream = torch.cuda.current_stream(device)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        e.step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(a.elapsed_time(b), world, device)
    return {"value": round(w.B * args.steps * world / (ms / 1e3), 2), "unit": UNIT,
            "h2d_bytes_per_step": e.h2d_bytes(), "d2h_bytes_per_step": e.d2h_bytes(),
            "api": "dual_b200.wrapper.BatchDecodeWithPagedKVCacheWrapper.plan/run (C ABI) + packer"}



# ------------------------------------------------------------ tiered (compute GPU + supplier GPU)
MIG_TOKENS = 2048   # token slots per migration batch (peer/policy.py:70): x 147,456 B = 302 MB
MODEL_LAYERS = 36


class TieredWorkload:
    """Compute GPU `compute` reads its local pool from HBM and its remote rows from a supplier bank in
    GPU `supplier`'s HBM (peer access).  A 36-layer pool of this batch does not fit one GPU, so
    `layers` pools are resident and the 36 layers of a step cycle through them (one layer's KV is
    several GB, far beyond L2, so a pool visited again is read from HBM again).  With `migrate`, every
    step also moves one batch of 2048 background token slots x 72 planes (36 layers x K, V = 302 MB)
    into the supplier bank on a side stream, launched after the step's packer and switched in the
    page tables at the next step boundary (the reference's launch/commit order)."""

    def __init__(self, args, compute=0, supplier=1, seed=None):
        from dual_b200 import ops, topology
        self.ops = ops
        B, lmin, lmax, rl, placement, RN, TN, layers, migrate = TIERED[args.workload]
        self.B, self.layers, self.RN, self.TN, self.migrate = B, layers, RN, TN, migrate
        self.d0, self.d1 = torch.device(f"cuda:{compute}"), torch.device(f"cuda:{supplier}")
        if supplier != compute:  # (the same GPU for both: the small one-GPU check in the tests)
            topology.enable_peer(compute, supplier)
        seed = args.seed if seed is None else seed
        rng = np.random.default_rng(seed)
        self.lengths = rng.integers(lmin, lmax + 1, B).astype(np.int64)
        self.remote = np.rint(self.lengths * rl / (1.0 + rl)).astype(np.int64)
        self.T, self.R = int(self.lengths.sum()), int(self.remote.sum())
        self.mig_tokens = MIG_TOKENS if migrate else 0
        n_bg = 4 * self.mig_tokens  # background (not decoded) slots: four batches that migrate in turn
        n_local = self.T - self.R
        C = n_local + n_bg
        R_cap = max(1, self.R + n_bg)  # a one-row bank when nothing is remote
        self.C, self.R_cap, self.n_bg, self.n_local = C, R_cap, n_bg, n_local
        g = torch.Generator(device=self.d0).manual_seed(seed)
        self.k = [torch.empty((C + 1, 8, 128), dtype=torch.bfloat16, device=self.d0) for _ in range(layers)]
        self.v = [torch.empty((C + 1, 8, 128), dtype=torch.bfloat16, device=self.d0) for _ in range(layers)]
        for t in self.k + self.v:
            t.normal_(generator=g)
        self.bank = torch.empty((layers, 2, R_cap, 8, 128), dtype=torch.bfloat16, device=self.d1)
        self.bank.normal_(generator=torch.Generator(device=self.d1).manual_seed(seed + 1))
        self.peer_k = [[self.bank[i, 0]] for i in range(layers)]
        self.peer_v = [[self.bank[i, 1]] for i in range(layers)]
        # decoded positions take a seeded permutation of local slots 1..n_local; the background slots are
        # n_local+1..C, so the migration's other 36 - layers layers live in buffers covering only them
        perm = (torch.randperm(n_local, generator=g, device=self.d0) + 1).to(torch.int32)
        maxL = int(self.lengths.max())
        self.tier = torch.full((B + 1, max(maxL, n_bg, 1)), -1, dtype=torch.int32, device=self.d0)
        self.slot = torch.zeros_like(self.tier)
        off, roff = 0, 0
        for b in range(B):
            L, r = int(self.lengths[b]), int(self.remote[b])
            far = np.zeros(L, bool)
            if placement == "tail":
                far[L - r:] = True
            else:
                far[:r] = True
            fidx = torch.from_numpy(np.nonzero(far)[0]).to(self.d0)
            nidx = torch.from_numpy(np.nonzero(~far)[0]).to(self.d0)
            s_ = torch.empty(L, dtype=torch.int32, device=self.d0)
            s_[fidx] = torch.arange(roff, roff + r, dtype=torch.int32, device=self.d0)
            s_[nidx] = perm[off:off + L - r]
            off += L - r
            roff += r
            self.tier[b, :L] = torch.from_numpy(far.astype(np.int32)).to(self.d0)
            self.slot[b, :L] = s_
        self.req = torch.arange(B, dtype=torch.int32, device=self.d0)
        self.seq = torch.tensor(self.lengths, dtype=torch.int32, device=self.d0)
        self.indptr = torch.tensor(np.concatenate([[0], np.cumsum(self.lengths)]), dtype=torch.int32, device=self.d0)
        self.indptr_h = np.concatenate([[0], np.cumsum(self.lengths)])
        self.indices = torch.empty(self.T, dtype=torch.int32, device=self.d0)
        self.q = torch.randn((layers, B, 32, 128), generator=g, device=self.d0).to(torch.bfloat16)
        self.out = torch.empty_like(self.q)
        self.lse = torch.empty((layers, B, 32), dtype=torch.float32, device=self.d0)
        self.num_ctas = ops.default_ctas(compute)
        self.ws = torch.zeros(ops.decode_workspace_size(B, self.num_ctas), dtype=torch.uint8, device=self.d0)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.d0)
        self.scale = 128 ** -0.5
        self.mig_ctas = getattr(args, "mig_ctas", 64)
        self.migrating = migrate
        if migrate:
            # background rows: table row B (never decoded); local slots n_local+1..C in a seeded order,
            # migrating into remote ids R..R_cap-1
            self.bg_local = (torch.randperm(n_bg, generator=g, device=self.d0) + n_local + 1).long()
            self.bg_remote = torch.arange(self.R, R_cap, dtype=torch.int64, device=self.d0)
            self.tier[B, :n_bg] = 0
            self.slot[B, :n_bg] = self.bg_local.to(torch.int32)
            extra = MODEL_LAYERS - layers
            self.mig_local = torch.empty((extra, 2, n_bg, 8, 128), dtype=torch.bfloat16, device=self.d0)
            self.mig_local.normal_(generator=g)
            self.mig_remote = torch.zeros((extra, 2, n_bg, 8, 128), dtype=torch.bfloat16, device=self.d1)
            # plane base pointers, layer-major (K, V): resident layers use the decode pools and the bank;
            # the others use the small buffers, based so that slot n_local+1 / remote id R is their row 0
            # (only background slots and ids, which lie in those ranges, are ever copied)
            lp, rp = [], []
            for layer in range(MODEL_LAYERS):
                for plane in range(2):
                    if layer < layers:
                        lp.append((self.k, self.v)[plane][layer].data_ptr())
                        rp.append(self.bank[layer, plane].data_ptr())
                    else:
                        lp.append(self.mig_local[layer - layers, plane].data_ptr() - (n_local + 1) * 2048)
                        rp.append(self.mig_remote[layer - layers, plane].data_ptr() - self.R * 2048)
            self.lp = torch.tensor(lp, dtype=torch.int64, device=self.d0)
            self.rp = torch.tensor(rp, dtype=torch.int64, device=self.d0)
            self.copy_stream = torch.cuda.Stream(self.d0)
            self.mig_status = torch.zeros(1, dtype=torch.int32, device=self.d0)
            self.mig_events = []
            self.batch_no = 0
            self.pending = None

    def _launch_migration(self):
        """Async copy of the next 2048 background slots x 72 planes on the side stream, ordered after
        the work issued so far on the main stream (this step's packer), as TierManager.submit does."""
        n = self.mig_tokens
        k = self.batch_no % 4
        src, dst = self.bg_local[k * n:(k + 1) * n], self.bg_remote[k * n:(k + 1) * n]
        start = torch.cuda.Event(enable_timing=True)
        done = torch.cuda.Event(enable_timing=True)
        self.copy_stream.wait_stream(torch.cuda.current_stream(self.d0))
        with torch.cuda.stream(self.copy_stream):
            start.record(self.copy_stream)
            self.ops.migrate_copy(self.lp, self.rp, 2 * MODEL_LAYERS, 1, src, dst, False, self.C + 1, self.R_cap,
                                  self.mig_status, max_ctas=self.mig_ctas)
            done.record(self.copy_stream)
        self.mig_events.append((start, done))
        self.pending = (k, done)
        self.batch_no += 1

    def _commit_migration(self):
        """Step boundary: the main stream waits for the copy, then switches the batch's page-table rows."""
        if self.pending is None:
            return
        k, done = self.pending
        torch.cuda.current_stream(self.d0).wait_event(done)
        n = self.mig_tokens
        self.tier[self.B, k * n:(k + 1) * n] = 1
        self.slot[self.B, k * n:(k + 1) * n] = self.bg_remote[k * n:(k + 1) * n].to(torch.int32)
        self.pending = None

    def step(self, events=None):
        ops = self.ops
        if self.migrating:
            self._commit_migration()
        ops.pack_read_order(self.tier, self.slot, self.req, self.seq, self.C, self.RN, self.TN, self.indices,
                            status=self.status)
        if self.migrating:
            self._launch_migration()
        for i in range(MODEL_LAYERS):
            lyr = i % self.layers
            if events is not None:
                events[i][0].record()
            ops.tiered_decode(self.q[lyr], self.k[lyr], self.v[lyr], self.C, self.peer_k[lyr], self.peer_v[lyr],
                              self.indptr, self.indices, self.scale, self.out[lyr], self.lse[lyr], self.ws,
                              self.num_ctas)
            if events is not None:
                events[i][1].record()

    def local_bytes(self):
        return 4096 * (self.T - self.R) + 8192 * self.B * 2 + 128 * self.B

    def remote_bytes(self):
        return 4096 * self.R

    def launches_per_step(self):
        return 1 + MODEL_LAYERS + (1 if self.migrating else 0)

    def parity(self):
        """Sampled requests of the last resident layer against the oracle: the CTA-boundary and length
        extremes plus the requests with the most and the fewest remote rows."""
        lyr = self.layers - 1
        picks = decode_picks(self.lengths, self.num_ctas,
                             extra=(int(np.argmax(self.remote)), int(np.argmin(self.remote))))
        return decode_parity(self.q[lyr], self.out[lyr], self.lse[lyr], self.k[lyr], self.v[lyr], self.C,
                             self.peer_k[lyr], self.peer_v[lyr], self.indptr_h, self.indices, picks, self.scale)

    def migrated_bit_exact(self):
        """Every migrated row of every one of the 72 planes equals its source, sampled every 97th slot."""
        torch.cuda.synchronize(self.d0)
        k = min(self.batch_no, 4) * self.mig_tokens
        src, dst = self.bg_local[:k:97], self.bg_remote[:k:97]
        ok = True
        for layer in range(MODEL_LAYERS):
            for plane in range(2):
                if layer < self.layers:
                    s_rows = (self.k, self.v)[plane][layer].index_select(0, src)
                    d_rows = self.bank[layer, plane].index_select(0, dst.to(self.d1)).to(self.d0)
                else:
                    s_rows = self.mig_local[layer - self.layers, plane].index_select(0, src - self.n_local - 1)
                    d_rows = self.mig_remote[layer - self.layers, plane].index_select(
                        0, (dst - self.R).to(self.d1)).to(self.d0)
                ok &= bool(torch.equal(s_rows.view(torch.int16), d_rows.view(torch.int16)))
        return ok


class TieredE2E:
    """The tiered step through the public wrapper API with host buffers: per step the commit of the
    previous migration, H2D of the step's 36 layers of queries (pinned), the packer, plan(), the next
    migration, 36 x run(q, paged_kv, peer_k0, peer_v0, unified_indices, local_capacity, sm_scale) and
    D2H of every layer's output (pinned), pipelined by layer on two side streams."""

    def __init__(self, w: TieredWorkload):
        from dual_b200.wrapper import BatchDecodeWithPagedKVCacheWrapper
        self.w = w
        shape = (MODEL_LAYERS, w.B, 32, 128)
        self.q_host = torch.randn(shape, dtype=torch.float32).to(torch.bfloat16).pin_memory()
        self.out_host = torch.empty(shape, dtype=torch.bfloat16).pin_memory()
        self.indptr_host = torch.from_numpy(w.indptr_h.astype(np.int32)).pin_memory()
        self.q_dev = torch.empty(shape, dtype=torch.bfloat16, device=w.d0)
        self.out_dev = torch.empty(shape, dtype=torch.bfloat16, device=w.d0)
        self.wrapper = BatchDecodeWithPagedKVCacheWrapper(torch.empty(64 << 20, dtype=torch.uint8, device=w.d0),
                                                          "NHD", use_tensor_cores=True)
        self.last = torch.ones(w.B, dtype=torch.int32)
        self.h2d = torch.cuda.Stream(w.d0)
        self.d2h = torch.cuda.Stream(w.d0)
        self.q_ready = [torch.cuda.Event() for _ in range(MODEL_LAYERS)]
        self.out_ready = [torch.cuda.Event() for _ in range(MODEL_LAYERS)]

    def step(self):
        w = self.w
        cur = torch.cuda.current_stream(w.d0)
        if w.migrating:
            w._commit_migration()
        self.h2d.wait_stream(cur)
        with torch.cuda.stream(self.h2d):
            for i in range(MODEL_LAYERS):
                self.q_dev[i].copy_(self.q_host[i], non_blocking=True)
                self.q_ready[i].record(self.h2d)
        w.ops.pack_read_order(w.tier, w.slot, w.req, w.seq, w.C, w.RN, w.TN, w.indices, status=w.status)
        self.wrapper.plan(self.indptr_host, w.indices, self.last, 32, 8, 128, 1, q_data_type=torch.bfloat16,
                          sm_scale=w.scale)
        if w.migrating:
            w._launch_migration()
        for i in range(MODEL_LAYERS):
            lyr = i % w.layers
            cur.wait_event(self.q_ready[i])
            self.wrapper.run(self.q_dev[i], (w.k[lyr], w.v[lyr]), w.peer_k[lyr][0], w.peer_v[lyr][0], w.indices,
                             w.C, w.scale, out=self.out_dev[i])
            self.out_ready[i].record(cur)
            self.d2h.wait_event(self.out_ready[i])
            with torch.cuda.stream(self.d2h):
                self.out_host[i].copy_(self.out_dev[i], non_blocking=True)
        cur.wait_stream(self.d2h)

    def h2d_bytes(self):
        return self.q_host.numel() * 2 + self.indptr_host.numel() * 4

    def d2h_bytes(self):
        return self.out_host.numel() * 2


def reduce_over_ranks(x, world, device, op="max"):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.MIN)
    return float(t.item())


def run_tiered(args):
    """N/2 (compute, supplier) pairs.  Under torchrun with W ranks, rank r < W/2 decodes on GPU r with
    its supplier bank on GPU r + W/2 (BASELINE config 5 = 4 pairs on 8 GPUs); the other ranks hold
    their GPUs for the supplier role and take the same collective steps.  Without torchrun: GPU 0
    computes, GPU 1 supplies.  Every rank issues the same collectives in the same order."""
    world, rank, local = dist_setup(args)
    pairs = max(1, world // 2)
    if world == 1 and torch.cuda.device_count() < 2:
        print(json.dumps({"metric": METRIC, "unavailable": f"{args.workload} needs 2 GPUs"}))
        return
    is_compute = world == 1 or local < pairs
    compute, supplier = (0, 1) if world == 1 else (local, local + pairs)
    dev = torch.device(f"cuda:{compute if is_compute else local}")
    torch.cuda.set_device(dev)
    w = TieredWorkload(args, compute, supplier, seed=args.seed + 1000 * local) if is_compute else None
    steps = args.steps
    if w is not None:
        for _ in range(max(args.warmup, 3)):
            w.step()
        torch.cuda.synchronize(w.d0)
    clocks = ClockSampler(compute) if w is not None else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    # ---- timed region: `steps` full 36-layer steps (with the step's migration when configured)
    barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    all_events = []
    if w is not None:
        if w.migrate:
            w.mig_events = []
        stream = torch.cuda.current_stream(w.d0)
        torch.cuda.synchronize(w.d0)
        t0.record(stream)
        for _ in range(steps):
            ev = [[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
                  for _ in range(MODEL_LAYERS)]
            w.step(ev)
            all_events.append(ev)
        t1.record(stream)
        torch.cuda.synchronize(w.d0)
        torch.cuda.synchronize(w.d1)
    barrier(world)
    clk = clocks.stop() if clocks else None
    ms = t0.elapsed_time(t1) if w is not None else 0.0
    mig_ms = [a.elapsed_time(b) for a, b in w.mig_events] if (w is not None and w.migrate) else []
    layer_ms = [a.elapsed_time(b) for ev in all_events for a, b in ev]
    layer_avg = sum(layer_ms) / len(layer_ms) if layer_ms else 0.0
    ms_max = reduce_over_ranks(ms, world, dev)
    layer_max = reduce_over_ranks(layer_avg, world, dev)
    step_min = reduce_over_ranks(ms / steps if w is not None else float("inf"), world, dev, "min")
    # ---- the same steps with the migration switched off (decode layer time without a copy beside it)
    nomig_layer = None
    if w is not None and w.migrate:
        w.migrating = False
        ev = [[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
              for _ in range(MODEL_LAYERS)]
        for _ in range(2):
            w.step(ev)
        torch.cuda.synchronize(w.d0)
        nomig = [a.elapsed_time(b) for a, b in ev]
        nomig_layer = sum(nomig) / len(nomig)
        w.migrating = True
    nomig_layer = reduce_over_ranks(nomig_layer or 0.0, world, dev)
    # ---- end to end through the wrapper API with host buffers
    e2e_ms = 0.0
    e = None
    if not args.no_e2e and w is not None:
        e = TieredE2E(w)
        for _ in range(2):
            e.step()
        torch.cuda.synchronize(w.d0)
    if not args.no_e2e:
        barrier(world)
        if e is not None:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(torch.cuda.current_stream(w.d0))
            for _ in range(steps):
                e.step()
            b.record(torch.cuda.current_stream(w.d0))
            torch.cuda.synchronize(w.d0)
            e2e_ms = a.elapsed_time(b)
        e2e_ms = reduce_over_ranks(e2e_ms, world, dev)
    # ---- sampled parity and migrated bytes (outside every timed region)
    parity = w.parity() if w is not None else None
    all_pass = reduce_over_ranks(1.0 if (parity is None or parity["pass"]) else 0.0, world, dev, "min")
    bit_exact = w.migrated_bit_exact() if (w is not None and w.migrate) else None
    if w is None:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    t_layer = layer_max / 1e3
    peak_hbm, peak_kind = measured_peaks()
    t_local = w.local_bytes() / (peak_hbm * 1e9)
    t_remote = w.remote_bytes() / (PEER_GBS * 1e9)
    t_star = max(t_local, t_remote)
    value = pairs * w.B * steps / (ms_max / 1e3)
    status = int(w.status.item()) | int(w.ws[:4].view(torch.int32).item())
    result = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world if world > 1 else 2,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms_max / steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{args.workload}: {pairs} x (1 compute GPU + 1 KV supplier GPU, peer access), "
                               f"tiered paged decode, 36-layer steps",
                   "pairs": pairs, "batch_per_compute_gpu": w.B, "kv_len": f"U[{TIERED[args.workload][1]},"
                                                                      f"{TIERED[args.workload][2]}]",
                   "sum_kv_tokens": w.T, "remote_tokens": w.R, "remote_over_local": round(w.R / (w.T - w.R), 4),
                   "remote_placement": TIERED[args.workload][4], "read_order_rn_tn": [w.RN, w.TN],
                   "layers_resident": w.layers, "layers_per_step": MODEL_LAYERS,
                   "concurrent_migration": bool(w.migrate),
                   "parallelism": f"{pairs} request-sharded (compute, supplier) pairs, no collective on the data path",
                   "l2": f"inputs larger than L2 ({(w.local_bytes() + w.remote_bytes()) / 1e9:.2f} GB per layer)"},
        "per_compute_gpu": {"tok_s_slowest": round(w.B / (ms_max / steps / 1e3), 2),
                            "tok_s_fastest": round(w.B / (step_min / 1e3), 2)},
        "roofline": {"bound": "nvlink" if t_remote > t_local else "hbm",
                     "achieved": round((w.local_bytes() + w.remote_bytes()) / t_layer / 1e9, 1),
                     "peak": round((w.local_bytes() + w.remote_bytes()) / t_star / 1e9, 1), "unit": "GB/s",
                     "frac": round(t_star / t_layer, 4), "traffic": None,
                     "local_gbs": round(w.local_bytes() / t_layer / 1e9, 1),
                     "peer_gbs": round(w.remote_bytes() / t_layer / 1e9, 1),
                     "t_star_ms": round(t_star * 1e3, 4), "layer_ms": round(t_layer * 1e3, 4),
                     "kernel": "tiered_decode_kernel",
                     "peak_source": f"{peak_kind} hbm_gbs {peak_hbm} + measured peer copy {PEER_GBS} GB/s per "
                                    f"direction; frac = max(local/HBM, remote/NVLink) time / layer time"},
        "gpu_launches": w.launches_per_step() * steps,
        "device_status": status,
        "parity": dict(parity, all_ranks_pass=bool(all_pass >= 1.0)),
    }
    if w.migrate and mig_ms:
        nbytes = w.mig_tokens * MODEL_LAYERS * 4096
        result["migration"] = {"tokens_per_batch": w.mig_tokens, "planes": 2 * MODEL_LAYERS,
                               "bytes_per_batch": nbytes, "copy_ctas": w.mig_ctas,
                               "avg_ms": round(sum(mig_ms) / len(mig_ms), 4),
                               "gbs": round(nbytes / (sum(mig_ms) / len(mig_ms) / 1e3) / 1e9, 1),
                               "decode_layer_ms_with_copy": round(layer_max, 4),
                               "decode_layer_ms_without_copy": round(nomig_layer, 4),
                               "status": int(w.mig_status.item()), "bit_exact_sampled": bit_exact}
    if not args.no_e2e:
        result["e2e"] = {"value": round(pairs * w.B * steps / (e2e_ms / 1e3), 2), "unit": UNIT,
                         "h2d_bytes_per_step": e.h2d_bytes(), "d2h_bytes_per_step": e.d2h_bytes(),
                         "api": "dual_b200.wrapper.BatchDecodeWithPagedKVCacheWrapper.plan/run with the peer tail "
                                "(C ABI) + packer + migration"}
    if clk:
        result["clocks"] = clk
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# ------------------------------------------------------------ migration copy (1 GPU)
def run_migration(args):
    """One 2048-slot migration batch over all 72 planes (36 layers x K, V = 302 MB) from the local
    pool into a supplier-bank layout on the same GPU, repeated; bytes moved / CUDA-event time."""
    from dual_b200 import ops
    from dual_b200.remote_bank import RemoteBank, local_plane_pointers
    dev = torch.device("cuda:0")
    layers, lslots, bslots, n = 36, 1 << 16, 1 << 13, 2048
    g = torch.Generator(device=dev).manual_seed(args.seed)
    local = [(torch.randn((lslots + 1, 8, 128), generator=g, device=dev).to(torch.bfloat16),
              torch.randn((lslots + 1, 8, 128), generator=g, device=dev).to(torch.bfloat16)) for _ in range(layers)]
    bank = RemoteBank([torch.zeros((layers, 2, bslots, 8, 128), dtype=torch.bfloat16, device=dev)])
    lp = local_plane_pointers(local, dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    src = (torch.randperm(lslots, generator=g, device=dev)[:n] + 1).long()
    dst = torch.randperm(bslots, generator=g, device=dev)[:n].long()
    for _ in range(max(args.warmup, 3)):
        ops.migrate_copy(lp, bank.pointers, 72, 1, src, dst, False, lslots + 1, bslots, status)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        ops.migrate_copy(lp, bank.pointers, 72, 1, src, dst, False, lslots + 1, bslots, status)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    nbytes = n * 147456
    ok = all(torch.equal(bank.gather(i, p, dst).view(torch.int16), local[i][p].index_select(0, src).view(torch.int16))
             for i in range(0, layers, 7) for p in range(2))
    peak, kind = measured_peaks()
    print(json.dumps({"metric": "migration copy GB/s (2048 slots x 72 planes)", "value": round(nbytes / ms / 1e6, 1),
                      "unit": "GB/s moved", "ms_per_batch": round(ms, 4), "bytes_per_batch": nbytes,
                      "roofline": {"bound": "hbm", "achieved": round(2 * nbytes / ms / 1e6, 1), "peak": peak,
                                   "unit": "GB/s (read+write)", "frac": round(2 * nbytes / ms / 1e6 / peak, 4)},
                      "bit_exact_sampled": ok, "status": int(status.item()), "gpu_launches": args.steps}), flush=True)


# ------------------------------------------------------------ causal append (config 4 shapes)
APPEND = {
    # name: (requests, qmin, qmax (log-uniform), Pmin, Pmax (uniform), remote/local, suppliers)
    "config4": (32, 128, 2048, 4096, 32768, 0.1797, 3),
    "append-small": (4, 128, 512, 1024, 4096, 0.1797, 3),
    "append-mid": (8, 128, 2048, 4096, 32768, 0.1797, 3),  # the profiling case: ~0.7 GB on the device
}


def append_setup(args, workload):
    """Inputs of one causal append layer for the 4-GPU configuration's shapes: per request a
    history prefix of P tokens (remote share R/L = 17.97 %, one request in eight ~95 % remote, remote
    only in the history) and q new tokens.  Supplier banks live on GPUs 1..3 when present (peer
    access), else in this GPU's memory.  FLOPs per request = 16384 (q P + q (q + 1) / 2)."""
    from dual_b200 import ops, topology
    B, qmin, qmax, pmin, pmax, rl, nsup = APPEND[workload]
    dev = torch.device("cuda:0")
    ngpu = torch.cuda.device_count()
    owners = [torch.device(f"cuda:{1 + i % (ngpu - 1)}") if ngpu > 1 else dev for i in range(nsup)]
    for o in set(owners):
        if o != dev:
            topology.enable_peer(0, o.index)
    rng = np.random.default_rng(args.seed)
    qlens = np.exp(rng.uniform(np.log(qmin), np.log(qmax), B)).astype(np.int64)
    pref = rng.integers(pmin, pmax + 1, B).astype(np.int64)
    lengths = pref + qlens
    frac = np.full(B, rl / (1 + rl))
    heavy = np.arange(B) % 8 == 0
    frac[heavy] = 0.95
    frac[~heavy] = max(0.0, (rl / (1 + rl) * lengths.sum() - 0.95 * lengths[heavy].sum()) / lengths[~heavy].sum())
    remote = np.minimum((frac * lengths).astype(np.int64), pref)
    T, R = int(lengths.sum()), int(remote.sum())
    C = T - R + 1
    g = torch.Generator(device=dev).manual_seed(args.seed)
    k = torch.empty((C + 1, 8, 128), dtype=torch.bfloat16, device=dev).normal_(generator=g)
    v = torch.empty((C + 1, 8, 128), dtype=torch.bfloat16, device=dev).normal_(generator=g)
    per_bank = R // nsup + 1
    pk = [torch.randn((per_bank, 8, 128), device=o).to(torch.bfloat16) for o in owners]
    pv = [torch.randn((per_bank, 8, 128), device=o).to(torch.bfloat16) for o in owners]
    tier = torch.zeros((B, int(lengths.max())), dtype=torch.int32, device=dev)
    slot = torch.zeros_like(tier)
    perm = (torch.randperm(C, generator=g, device=dev) + 1).to(torch.int32)
    off, roff = 0, 0
    for b in range(B):
        L, r = int(lengths[b]), int(remote[b])
        far = torch.zeros(L, dtype=torch.bool)
        far[torch.from_numpy(np.sort(rng.choice(int(pref[b]), r, replace=False)))] = True
        s_ = torch.empty(L, dtype=torch.int32)
        s_[far] = torch.arange(roff, roff + r, dtype=torch.int32)
        s_[~far] = perm[off:off + L - r].cpu()
        off += L - r
        roff += r
        tier[b, :L] = far.to(torch.int32).to(dev)
        slot[b, :L] = s_.to(dev)
    req = torch.arange(B, dtype=torch.int32, device=dev)
    seq = torch.tensor(lengths, dtype=torch.int32, device=dev)
    pre = torch.tensor(pref, dtype=torch.int32, device=dev)
    full = torch.empty(T, dtype=torch.int32, device=dev)
    ops.pack_read_order(tier, slot, req, seq, C, 5, 32, full, prefix_lens=pre)
    qo = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    kv = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    # per-request remote counts (the tier manager's host mirror in a server) let the plan spread the
    # mostly-remote requests' items over the launch
    work = ops.append_plan(qo, kv, True, remote.astype(np.int32)).to(dev)
    Q = int(qlens.sum())
    q = torch.empty((Q, 32, 128), dtype=torch.bfloat16, device=dev).normal_(generator=g)
    out = torch.empty_like(q)
    lse = torch.empty((Q, 32), dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    qo_d, kv_d = torch.from_numpy(qo).to(dev), torch.from_numpy(kv).to(dev)
    flops = float(sum(16384 * (int(x) * int(p_) + int(x) * (int(x) + 1) / 2) for x, p_ in zip(qlens, pref)))
    return types.SimpleNamespace(B=B, dev=dev, owners=owners, qlens=qlens, pref=pref, lengths=lengths, T=T, R=R, C=C,
                                 remote=remote,
                                 k=k, v=v, pk=pk, pv=pv, full=full, qo=qo, kv=kv, work=work, Q=Q, q=q, out=out, lse=lse,
                                 status=status, qo_d=qo_d, kv_d=kv_d, flops=flops)


def append_parity(S, scale=128 ** -0.5):
    """Sampled query rows of one append layer against the oracle: the request with the longest query,
    one whose query length is not a multiple of 64, the one with the longest prefix and a ~95 %-remote
    one; in each, three runs of up to 4 consecutive query tokens (its first, those around token 64
    where a work item's 64-token pair ends, its last)."""
    from oracle.attention import attend
    qlens, pref = np.asarray(S.qlens), np.asarray(S.pref)
    cand = [int(np.argmax(qlens)), next((b for b in range(S.B) if qlens[b] % 64), 0), int(np.argmax(pref)),
            int(np.argmax(np.asarray(S.remote) / np.asarray(S.lengths)))]
    picks = []
    for b in cand:
        if b not in picks:
            picks.append(b)
    qo, kv = np.asarray(S.qo), np.asarray(S.kv)
    tally = ParityTally()
    for b in picks:
        L, P, ql = int(S.lengths[b]), int(pref[b]), int(qlens[b])
        pages = S.full[int(kv[b]):int(kv[b]) + L]
        kr, vr = gather_rows(pages, S.C, S.k, S.pk), gather_rows(pages, S.C, S.v, S.pv)
        q0 = int(qo[b])
        for t0 in sorted({0, max(0, min(62, ql - 4)), max(0, ql - 4)}):
            n = min(4, ql - t0)
            vis = P + t0 + n
            ro, rl = attend(S.q[q0 + t0:q0 + t0 + n].cpu(), kr[:vis], vr[:vis], P + t0, scale)
            tally.add(S.out[q0 + t0:q0 + t0 + n], ro, S.lse[q0 + t0:q0 + t0 + n], rl,
                      f"request {b}: q={ql}, prefix={P}, remote={int(S.remote[b])}, tokens {t0}..{t0 + n - 1}")
    return tally.result()


def append_cpu_baseline(lengths, qlens, flops):
    """fp32 oracle (the reference's attention math) on a bounded sample: the last query tokens of the
    median request against its whole visible context, ~10 s, scaled by FLOPs to one layer."""
    from oracle.attention import attend

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    bm = int(np.argsort(lengths)[len(lengths) // 2])
    qs = min(int(qlens[bm]), 16)
    Lb = int(lengths[bm])
    kb_ = torch.randn((Lb, 8, 128)).to(torch.bfloat16)
    vb_ = torch.randn((Lb, 8, 128)).to(torch.bfloat16)
    qb_ = torch.randn((qs, 32, 128)).to(torch.bfloat16)
    pre_s = Lb - qs
    attend(qb_, kb_, vb_, pre_s, 128 ** -0.5)
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < 10.0 and reps < 50:
        attend(qb_, kb_, vb_, pre_s, 128 ** -0.5)
        reps += 1
    t_sample = (time.perf_counter() - t0) / reps
    flops_sample = 16384 * (qs * pre_s + qs * (qs + 1) / 2)
    cpu_ms = t_sample * flops / flops_sample * 1e3

    return {"value": round(cpu_ms, 1), "unit": "ms", "cores": threads, "kind": "port",
            "sample": f"fp32 oracle: last {qs} query tokens of request {bm} (L={Lb}) against its visible context, "
                      f"scaled by FLOPs"}


def run_append(args):
    """dual_b200's tiered append kernel on append_setup's inputs (one layer per step)."""
    from dual_b200 import ops
    S = append_setup(args, args.workload)
    B, dev, owners, qlens, pref, lengths, T, R, C = S.B, S.dev, S.owners, S.qlens, S.pref, S.lengths, S.T, S.R, S.C
    k, v, pk, pv, full, qo, kv, work, Q, q, out, lse, status = (S.k, S.v, S.pk, S.pv, S.full, S.qo, S.kv, S.work, S.Q,
                                                                 S.q, S.out, S.lse, S.status)
    qo_d, kv_d = S.qo_d, S.kv_d
    warm = max(args.warmup, 3)

    # Supplier rows either read in place (peer loads from the banks) or, with --stage, copied once per
    # layer into local buffers by the LayerStager on a side stream while the previous layer's append
    # runs.  Every step is one layer of a forward; the stager's start() (layer 0's copy, not overlapped)
    # is inside the timed region.
    stager = None
    if args.stage:
        from dual_b200.staging import LayerStager
        stager = LayerStager(lambda i: (pk, pv), max(warm, args.steps), dev, depth=2, mode=args.stage)

    def begin():
        if stager is not None:
            stager.start(full, C)

    def banks(i):
        if stager is None:
            return pk, pv
        t = stager.tail(i)
        return t[0::2], t[1::2]

    def done(i):
        if stager is not None:
            stager.next(i)

    def step(i):
        bk, bv = banks(i)
        ops.tiered_append(q, k, v, C, bk, bv, qo_d, kv_d, full, True, 128 ** -0.5, work, out, lse, status)
        done(i)

    begin()
    for i in range(warm):
        step(i)
    torch.cuda.synchronize()
    clocks = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0]))
    clocks.start()
    time.sleep(0.3)
    a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    begin()
    for i in range(args.steps):
        step(i)
    b_.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = a.elapsed_time(b_) / args.steps
    flops = S.flops
    tf = flops / (ms / 1e3) / 1e12
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(peaks.get("bf16_tflops", 1590.0))

    # end to end through the reference-facing wrapper, as a forward of `steps` layers: plan once (per
    # forward, as SGLang calls it), then per layer the layer's q from pinned host memory on a copy
    # stream, run_return_lse, and the layer's output and LSE back to pinned host memory on another;
    # device q / out / lse are double-buffered so layer i+1's upload and layer i-1's read-back overlap
    # layer i's attention.  The timed region ends when the last layer's outputs are in host memory.
    e2e = None
    from dual_b200.wrapper import BatchPrefillWithPagedKVCacheWrapper
    wrapper = BatchPrefillWithPagedKVCacheWrapper(torch.empty(1 << 20, dtype=torch.uint8, device=dev), "NHD")
    q_host = q.cpu().pin_memory()
    out_host = [torch.empty(out.shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    lse_host = [torch.empty(lse.shape, dtype=torch.float32).pin_memory() for _ in range(2)]
    qo_t, kv_t = torch.from_numpy(qo), torch.from_numpy(kv)
    peers = [t for pair in zip(pk, pv) for t in pair]
    q_dev = [torch.empty_like(q) for _ in range(2)]
    o_dev = [torch.empty_like(out) for _ in range(2)]
    l_dev = [torch.empty_like(lse) for _ in range(2)]
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    q_ready = [torch.cuda.Event() for _ in range(2)]
    q_free = [torch.cuda.Event() for _ in range(2)]
    o_ready = [torch.cuda.Event() for _ in range(2)]
    o_free = [torch.cuda.Event() for _ in range(2)]

    def e2e_forward(layers):
        cur = torch.cuda.current_stream(dev)
        h2d.wait_stream(cur)
        d2h.wait_stream(cur)

        def upload(i):
            s_ = i % 2
            with torch.cuda.stream(h2d):
                if i >= 2:
                    h2d.wait_event(q_free[s_])  # layer i-2's attention has read this buffer
                q_dev[s_].copy_(q_host, non_blocking=True)
                q_ready[s_].record(h2d)

        wrapper.plan(qo_t, kv_t, full, torch.ones(B, dtype=torch.int32), 32, 8, 128, 1, causal=True,
                     q_data_type=torch.bfloat16, remote_counts=S.remote)
        begin()
        upload(0)
        for i in range(layers):
            s_ = i % 2
            if i + 1 < layers:
                upload(i + 1)
            cur.wait_event(q_ready[s_])
            if i >= 2:
                cur.wait_event(o_free[s_])  # layer i-2's outputs have been read back
            tail = peers if stager is None else stager.tail(i)
            wrapper.run_return_lse(q_dev[s_], (k.unsqueeze(1), v.unsqueeze(1)), *tail, full, C, 128 ** -0.5,
                                   out=o_dev[s_], lse=l_dev[s_])
            done(i)
            q_free[s_].record(cur)
            o_ready[s_].record(cur)
            with torch.cuda.stream(d2h):
                d2h.wait_event(o_ready[s_])
                out_host[s_].copy_(o_dev[s_], non_blocking=True)
                lse_host[s_].copy_(l_dev[s_], non_blocking=True)
                o_free[s_].record(d2h)
        cur.wait_stream(d2h)  # the forward ends when its outputs are in host memory

    if not args.no_e2e:
        e2e_forward(3)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        e2e_forward(args.steps)
        e1.record()
        torch.cuda.synchronize()
        e2e = {"value": round(e0.elapsed_time(e1) / args.steps, 4), "unit": "ms",
               "h2d_bytes_per_step": q_host.numel() * 2,
               "d2h_bytes_per_step": out_host[0].numel() * 2 + lse_host[0].numel() * 4,
               "api": "dual_b200.wrapper.BatchPrefillWithPagedKVCacheWrapper.plan (once per forward) / "
                      "run_return_lse per layer, host copies pipelined by layer on two side streams"}

    # traffic: DRAM bytes of one launch from the committed ncu summary of this workload, if any
    traffic = None
    tfile = ROOT / "profiles" / "append_traffic.json"
    if tfile.exists():
        tj = json.loads(tfile.read_text())
        if tj.get("workload") == args.workload:
            traffic = tj.get("dram_bytes_per_launch")

    # CPU baseline: the fp32 oracle on a bounded sample (the last query tokens of the median request
    # against its whole visible context), scaled by FLOPs
    parity = append_parity(S)  # outside the timed regions: the last timed step's outputs
    cpu = None
    if not args.no_cpu_baseline:
        cpu = append_cpu_baseline(lengths, qlens, flops)
    print(json.dumps({"metric": "causal append attention time per layer", "value": round(ms, 4), "unit": "ms",
                      "n_gpus": len({str(dev)} | {str(o) for o in owners}), "steps": args.steps,
                      "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 4),
                      "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                      "data": "synthetic", "tflops": round(tf, 1),
                      "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak, "unit": "TFLOP/s",
                                   "frac": round(tf / peak, 4), "traffic": traffic,
                                   "kernel": "tiered_append_kernel",
                                   "peak_source": "measured bf16_tflops" if peaks else "fallback"},
                      "config": {"workload": args.workload, "requests": B, "sum_q": Q, "sum_kv": T,
                                 "remote_tokens": R, "remote_over_local": round(R / (T - R), 4),
                                 "suppliers": [str(o) for o in owners], "work_items": int(work.shape[0]),
                                 "flops_per_layer": flops,
                                 "supplier_rows": ({"range": "staged: LayerStager 'range', whole banks copied by "
                                                             "the copy engines per layer, one stream per bank, "
                                                             "overlapped with the previous layer's append",
                                                    "rows": "staged: LayerStager 'rows', the rows the index list "
                                                            "names copied by the row kernel before each append"}
                                                   [args.stage] if stager is not None else "read in place"),
                                 "l2": "K/V rows gathered from a pool larger than L2; no flush"},
                      "clocks": clk, "e2e": e2e, "cpu_baseline": cpu, "parity": parity,
                      "status": int(status.item()) | wrapper.status() | (stager.status() if stager else 0),
                      "gpu_launches": args.steps * (2 if args.stage == "rows" else 1)}), flush=True)

# ------------------------------------------------------- native FlashInfer (the number to beat)
def flashinfer_decode(w, args):
    """Native, unpatched FlashInfer FA2 decode -- the kernel the reference runs (BatchDecode with
    use_tensor_cores=True, peer/backend.py:130) -- timed on a DecodeWorkload's own pools, index list
    and queries (all local), `args.steps` steps of its layers after the warm-up, with its own clock
    record; also the largest difference from dual_b200's output of the last layer.  Prebuilt by
    baseline/build_flashinfer.py; reported as unavailable when that build is missing."""
    cache = ROOT / "baseline" / "flashinfer_jit"
    if not cache.exists() or not any(cache.rglob("*.so")):
        return {"unavailable": "native FlashInfer FA2 not prebuilt (run baseline/build_flashinfer.py)"}
    try:
        sys.path.insert(0, str(ROOT / "baseline"))
        import build_flashinfer
        build_flashinfer.configure()
        import flashinfer
    except Exception as exc:  # pragma: no cover - depends on the installed FlashInfer
        return {"unavailable": f"FlashInfer import failed: {exc}"}
    dev = w.device
    wrapper = flashinfer.BatchDecodeWithPagedKVCacheWrapper(torch.empty(256 << 20, dtype=torch.uint8, device=dev),
                                                            "NHD", use_tensor_cores=True, backend="fa2")
    wrapper.plan(w.indptr, w.indices, torch.ones(w.B, dtype=torch.int32, device=dev), 32, 8, 128, 1,
                 q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16, sm_scale=w.scale)
    fi_out = torch.empty_like(w.out[0])

    def step():
        for i in range(w.layers):
            wrapper.run(w.q[i], (w.k[i].unsqueeze(1), w.v[i].unsqueeze(1)), out=fi_out)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(dev.index)
    clocks.start()
    time.sleep(0.3)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    layer_ms = ms / w.layers
    peak, peak_kind = measured_peaks()
    gbs = w.bytes_per_layer() / (layer_ms / 1e3) / 1e9
    # dual_b200's output of the same layer again (w.out may hold other queries' outputs by now)
    dual_out = torch.empty_like(fi_out)
    lyr = w.layers - 1
    w.ops.tiered_decode(w.q[lyr], w.k[lyr], w.v[lyr], w.C, [], [], w.indptr, w.indices, w.scale, dual_out, None,
                        w.ws, w.num_ctas)
    torch.cuda.synchronize()
    diff = float((fi_out.float() - dual_out.float()).abs().max())
    return {"impl": "flashinfer-fa2-native", "value": round(w.B / (ms / 1e3), 2), "unit": UNIT,
            "ms_per_step": round(ms, 4),
            "config": {"workload": f"{args.workload} inputs, native FlashInfer {flashinfer.__version__} FA2 "
                                   f"BatchDecode(use_tensor_cores=True), all-local, same pools and index list",
                       "batch": w.B, "sum_kv_tokens": w.T, "layers": w.layers},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "layer_ms": round(layer_ms, 4),
                         "peak_source": f"{peak_kind} hbm_gbs"},
            "max_abs_vs_dual_b200_last_layer": round(diff, 6), "clocks": clk}


def run_flashinfer(args):
    """Native, unpatched FlashInfer FA2 — the kernel the reference runs (BatchDecode with
    use_tensor_cores=True, peer/backend.py:130; BatchPrefill for append) — on the same inputs as the
    dual_b200 workload named after the "fi-" prefix, all-local: remote rows are gathered into one
    local pool first (outside the timed region), as the reference's own oracle does.  Prebuilt by
    baseline/build_flashinfer.py."""
    sys.path.insert(0, str(ROOT / "baseline"))
    import build_flashinfer
    build_flashinfer.configure()
    import flashinfer
    base = args.workload[3:]
    scale = 128 ** -0.5
    if base in WORKLOADS:
        args.workload = base
        w = DecodeWorkload(args, torch.device("cuda:0"))
        w.ops.pack_read_order(w.tier, w.slot, w.req, w.seq, w.C, 5, 32, w.indices, status=w.status)
        fi = flashinfer_decode(w, args)
        fi.update({"metric": METRIC, "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
                   "higher_is_better": True, "dtype": "bf16", "data": "synthetic"})
        print(json.dumps(fi), flush=True)
        return
    S = append_setup(args, base)
    dev = S.dev
    # gather every row of the unified list into one local pool (page 0 unused), outside the timed region
    full = S.full.long()
    far = full > S.C
    n = len(S.pk)

    def gather(local, banks):
        pool = torch.empty((full.numel() + 1, 8, 128), dtype=torch.bfloat16, device=dev)
        rows = torch.empty((full.numel(), 8, 128), dtype=torch.bfloat16, device=dev)
        rows[~far] = local.index_select(0, full[~far])
        g = full[far] - S.C - 1
        for d in range(n):
            m = g % n == d
            src = banks[d].to(dev).index_select(0, (g[m] // n))
            idx = torch.nonzero(far).squeeze(1)[m]
            rows[idx] = src
        pool[1:] = rows
        return pool.unsqueeze(1)
    kp, vp = gather(S.k, S.pk), gather(S.v, S.pv)
    wrapper = flashinfer.BatchPrefillWithPagedKVCacheWrapper(torch.empty(256 << 20, dtype=torch.uint8, device=dev),
                                                             "NHD", backend="fa2")
    wrapper.plan(S.qo_d, S.kv_d, torch.arange(1, full.numel() + 1, dtype=torch.int32, device=dev),
                 torch.ones(S.B, dtype=torch.int32, device=dev), 32, 8, 128, 1, causal=True, sm_scale=scale,
                 q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16)

    def step():
        wrapper.run(S.q, (kp, vp), out=S.out)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(0)
    clocks.start()
    time.sleep(0.3)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(peaks.get("bf16_tflops", 1590.0))
    tf = S.flops / (ms / 1e3) / 1e12
    print(json.dumps({"impl": "flashinfer-fa2-native", "metric": "causal append attention time per layer",
                      "value": round(ms, 4), "unit": "ms", "n_gpus": 1, "steps": args.steps,
                      "warmup": max(args.warmup, 3), "higher_is_better": False, "dtype": "bf16", "data": "synthetic",
                      "tflops": round(tf, 1),
                      "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak, "unit": "TFLOP/s",
                                   "frac": round(tf / peak, 4)},
                      "config": {"workload": f"{base} inputs, native FlashInfer {flashinfer.__version__} FA2 "
                                             f"BatchPrefill(causal), KV gathered all-local",
                                 "requests": S.B, "sum_q": S.Q, "sum_kv": S.T, "flops_per_layer": S.flops},
                      "clocks": clk}), flush=True)


# -------------------------------------------------------------- reference arm
def run_reference(args):
    """The reference's CPU attention math (fp32 torch restatement of check_attention_output, oracle
    port) on this host's cores, on the dual arm's workload definition (config 2 at N = 1; the config-5
    pairs under torchrun, where rank 0 alone runs).  Each step is a bounded sample: one request of the
    batch (the median length) for one layer, its K/V rows gathered from scattered pools -- local rows
    and, for the tiered workloads, its remote share from a second pool.  `ms_per_step` is that measured
    sample; `value` scales it by the whole job's token-layers (sum(L) x 36 per compute GPU's batch)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle.attention import attend
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.workload in TIERED:
        B, lmin, lmax, rl, placement = TIERED[args.workload][:5]
        rng = np.random.default_rng(args.seed)  # rank 0's batch of the dual arm
        lengths = rng.integers(lmin, lmax + 1, B).astype(np.int64)
        remote = np.rint(lengths * rl / (1.0 + rl)).astype(np.int64)
        seed_used, pairs, layers = args.seed, max(1, world // 2), MODEL_LAYERS
        desc = f"{args.workload}: {pairs} (compute, supplier) pairs' decode, CPU fp32 reference attention math"
    else:
        B, lmin, lmax, C, layers = WORKLOADS[args.workload]
        lengths, seed_used = draw_lengths(B, lmin, lmax, C, args.seed)
        remote, pairs = np.zeros_like(lengths), 1
        desc = f"{args.workload}: CPU fp32 reference attention math"
    T = int(lengths.sum())
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(args.seed)
    b = int(np.argsort(lengths, kind="stable")[len(lengths) // 2])
    L, r = int(lengths[b]), int(remote[b])
    # scattered pools of 4x the rows the request reads: local rows, and its remote rows in a second pool
    pool_k = torch.randn((4 * L, 8, 128), generator=g).to(torch.bfloat16)
    pool_v = torch.randn((4 * L, 8, 128), generator=g).to(torch.bfloat16)
    bank_k = torch.randn((4 * max(r, 1), 8, 128), generator=g).to(torch.bfloat16)
    bank_v = torch.randn((4 * max(r, 1), 8, 128), generator=g).to(torch.bfloat16)
    near = torch.randperm(4 * L, generator=g)[:L - r]
    far = torch.randperm(4 * max(r, 1), generator=g)[:r]
    q = torch.randn((1, 32, 128), generator=g).to(torch.bfloat16)

    def one():
        k = torch.cat([bank_k.index_select(0, far), pool_k.index_select(0, near)])
        v = torch.cat([bank_v.index_select(0, far), pool_v.index_select(0, near)])
        attend(q, k, v, L - 1, 128 ** -0.5)

    for _ in range(max(args.warmup, 1)):
        one()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    dt = (time.perf_counter() - t0) / args.steps
    scaled_step_s = dt / L * T * pairs * layers  # every compute GPU's batch, all layers, on these cores
    value = pairs * B / scaled_step_s
    sample = (f"1 of {B} requests (L={L}, {r} remote), 1 layer per step; scaled by sum(L)={T} x {pairs} "
              f"batch(es) x {layers} layers")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": 0,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
        "ms_per_step_is": "the measured sample step (one request, one layer)",
        "scaled_ms_per_step": round(scaled_step_s * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": desc, "batch": B, "sum_kv_tokens": T, "length_seed": seed_used, "layers": layers,
                   "pairs": pairs},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    args = parse()
    if args.workload is None:
        args.workload = "config5" if int(os.environ.get("WORLD_SIZE", "1")) > 1 else "config2"
    if args.impl == "reference":
        run_reference(args)
    elif args.workload in TIERED:
        run_tiered(args)
    elif args.workload == "migration":
        run_migration(args)
    elif args.workload in APPEND:
        run_append(args)
    elif args.workload.startswith("fi-"):
        run_flashinfer(args)
    else:
        run_dual(args)


if __name__ == "__main__":
    main()
