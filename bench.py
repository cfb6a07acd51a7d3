"""Benchmark of the tiered paged-decode hot path (headline metric: paged-decode tok/s and
local+peer GB/s as % of roofline).

Default workload (headline config 2: one B200, all-local): a full 36-layer
Qwen3-8B-shaped KV pool of 1,048,576 token slots per plane (72 planes x 2 KiB
x (C+1) slots = 154.6 GB in HBM), batch 64, KV lengths uniform in [2048, 32768]
(seeded; redrawn with the next seed while the sum exceeds the pool), slots a
seeded random permutation of the pool, Q/K/V ~ N(0, 1) bf16.  One step = the
packer (unified read order for the batch) + 36 layers of tiered decode
(decode kernel + merge).  Per-layer KV (4.5 GB) is far larger than L2, so no
flush is needed between iterations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl dual|reference] [--workload W]

Workloads: config2 (default), small; config3, config5, tiered-small, and config3-local / config3-r12
(config 3's batch with no remote rows / twice its remote share) (a compute GPU + a supplier GPU;
under torchrun N/2 such pairs); config4, append-small, append-mid (causal append; --stage range|rows
stages the supplier rows per layer); migration; fi-<workload> times native FlashInfer FA2 on the
same inputs (the number to beat).

Under torchrun (N > 1) every rank serves its own independent batch (decode
shards by request; no collective on the data path): scaling "weak".
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
                    default="config2")
    ap.add_argument("--seed", type=int, default=20261101)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
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
        return 1 + 2 * self.layers


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
                     "peak_source": f"{peak_kind} hbm_gbs", "kernel": "tiered_decode_kernel + decode_merge_kernel",
                     "layer_ms": round(layer_avg, 4), "algorithmic_bytes_per_launch": w.bytes_per_layer()},
        "gpu_launches": w.launches_per_step() * args.steps,
        "device_status": status,
    }
    if clk:
        result["clocks"] = clk
    if not args.no_e2e:
        result["e2e"] = run_e2e(w, args, world, device)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(w)
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



# ------------------------------------------------------------ tiered (2 GPUs)
class TieredWorkload:
    """Compute GPU 0 reads its local pool from HBM and its remote rows from a supplier bank in
    GPU 1's HBM (peer access); per-layer pools of `layers` resident layers (a 36-layer pool of this
    batch does not fit one GPU), the per-step figure is 36 x the per-layer time."""

    def __init__(self, args, compute=0, supplier=1, seed=None):
        from dual_b200 import ops, topology
        from dual_b200.remote_bank import RemoteBank, local_plane_pointers
        self.ops = ops
        B, lmin, lmax, rl, placement, RN, TN, layers, migrate = TIERED[args.workload]
        self.B, self.layers, self.RN, self.TN, self.migrate = B, layers, RN, TN, migrate
        self.d0, self.d1 = torch.device(f"cuda:{compute}"), torch.device(f"cuda:{supplier}")
        topology.enable_peer(compute, supplier)
        seed = args.seed if seed is None else seed
        rng = np.random.default_rng(seed)
        self.lengths = rng.integers(lmin, lmax + 1, B).astype(np.int64)
        self.remote = np.rint(self.lengths * rl / (1.0 + rl)).astype(np.int64)
        self.local = self.lengths - self.remote
        self.T, self.R = int(self.lengths.sum()), int(self.remote.sum())
        self.mig_tokens = 2048 if migrate else 0
        n_bg = 4 * self.mig_tokens  # background (not decoded) positions that migrate each step
        C = int(self.local.sum()) + n_bg
        R_cap = max(1, self.R + n_bg)  # a one-row bank when nothing is remote
        self.C, self.R_cap = C, R_cap
        g = torch.Generator(device=self.d0).manual_seed(seed)
        self.k = [torch.empty((C + 1, 8, 128), dtype=torch.bfloat16, device=self.d0) for _ in range(layers)]
        self.v = [torch.empty((C + 1, 8, 128), dtype=torch.bfloat16, device=self.d0) for _ in range(layers)]
        for t in self.k + self.v:
            t.normal_(generator=g)
        bank_t = torch.empty((layers, 2, R_cap, 8, 128), dtype=torch.bfloat16, device=self.d1)
        bank_t.normal_(generator=torch.Generator(device=self.d1).manual_seed(seed + 1))
        self.bank = RemoteBank([bank_t], layers=layers)
        perm = (torch.randperm(C, generator=g, device=self.d0) + 1).to(torch.int32)
        maxL = max(int(self.lengths.max()), n_bg)
        self.tier = torch.full((B + 1, maxL), -1, dtype=torch.int32, device=self.d0)
        self.slot = torch.zeros_like(self.tier)
        off, roff = 0, 0
        for b in range(B):
            L, r = int(self.lengths[b]), int(self.remote[b])
            far = np.zeros(L, bool)
            if placement == "tail":
                far[L - r:] = True
            else:
                far[:r] = True
            t = torch.from_numpy(far.astype(np.int32)).to(self.d0)
            s_ = torch.empty(L, dtype=torch.int32, device=self.d0)
            fidx = torch.from_numpy(np.nonzero(far)[0]).to(self.d0)
            nidx = torch.from_numpy(np.nonzero(~far)[0]).to(self.d0)
            s_[fidx] = torch.arange(roff, roff + r, dtype=torch.int32, device=self.d0)
            s_[nidx] = perm[off:off + L - r]
            off += L - r
            roff += r
            self.tier[b, :L] = t
            self.slot[b, :L] = s_
        # background positions (row B): local slots perm[off:off+n_bg], migrating into ids R .. R_cap-1
        self.bg_local = perm[off:off + n_bg].long()
        self.bg_remote = torch.arange(self.R, R_cap, dtype=torch.int64, device=self.d0)
        self.req = torch.arange(B, dtype=torch.int32, device=self.d0)
        self.seq = torch.tensor(self.lengths, dtype=torch.int32, device=self.d0)
        self.indptr = torch.tensor(np.concatenate([[0], np.cumsum(self.lengths)]), dtype=torch.int32, device=self.d0)
        self.indices = torch.empty(self.T, dtype=torch.int32, device=self.d0)
        self.q = torch.randn((layers, B, 32, 128), generator=g, device=self.d0).to(torch.bfloat16)
        self.out = torch.empty_like(self.q)
        self.lse = torch.empty((layers, B, 32), dtype=torch.float32, device=self.d0)
        self.num_ctas = ops.default_ctas(compute)
        self.ws = torch.zeros(ops.decode_workspace_size(B, self.num_ctas), dtype=torch.uint8, device=self.d0)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.d0)
        self.scale = 128 ** -0.5
        self.peer_k = [[self.bank.banks[0][i, 0]] for i in range(layers)]
        self.peer_v = [[self.bank.banks[0][i, 1]] for i in range(layers)]
        if migrate:
            self.lp = local_plane_pointers(list(zip(self.k, self.v)), self.d0)
            self.rp = self.bank.pointers.to(self.d0)
            self.copy_stream = torch.cuda.Stream(self.d0)
            self.mig_status = torch.zeros(1, dtype=torch.int32, device=self.d0)
            self.mig_events = []
            self.batch_no = 0
            self.pending = None

    def _launch_migration(self):
        """Async copy of the next 2048 background slots (all resident planes) on the side stream."""
        k = self.batch_no % 4
        src = self.bg_local[k * self.mig_tokens:(k + 1) * self.mig_tokens]
        dst = self.bg_remote[k * self.mig_tokens:(k + 1) * self.mig_tokens]
        start = torch.cuda.Event(enable_timing=True)
        done = torch.cuda.Event(enable_timing=True)
        self.copy_stream.wait_stream(torch.cuda.current_stream(self.d0))
        with torch.cuda.stream(self.copy_stream):
            start.record(self.copy_stream)
            self.ops.migrate_copy(self.lp, self.rp, 2 * self.layers, 1, src, dst, False, self.C + 1, self.R_cap,
                                  self.mig_status, max_ctas=32)
            done.record(self.copy_stream)
        self.mig_events.append((start, done))
        self.pending = (k, done)
        self.batch_no += 1

    def _commit_migration(self):
        """Step boundary: the main stream waits for the copy, then switches the background rows' tables."""
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
        if self.migrate:
            self._commit_migration()
        ops.pack_read_order(self.tier, self.slot, self.req, self.seq, self.C, self.RN, self.TN, self.indices,
                            status=self.status)
        if self.migrate:
            self._launch_migration()
        for i in range(self.layers):
            if events is not None:
                events[i][0].record()
            ops.tiered_decode(self.q[i], self.k[i], self.v[i], self.C, self.peer_k[i], self.peer_v[i], self.indptr,
                              self.indices, self.scale, self.out[i], self.lse[i], self.ws, self.num_ctas)
            if events is not None:
                events[i][1].record()

    def local_bytes(self):
        return 4096 * (self.T - self.R) + 8192 * self.B * 2 + 128 * self.B

    def remote_bytes(self):
        return 4096 * self.R


def run_tiered(args):
    """One (compute, supplier) pair per process.  Under torchrun with W ranks, ranks r < W/2 each
    decode on GPU r with their supplier bank on GPU r + W/2 (BASELINE config 5 = 4 pairs on 8 GPUs);
    the other ranks only hold their GPU for the supplier role and join the barriers.  Without
    torchrun: GPU 0 computes, GPU 1 supplies."""
    world, rank, local = dist_setup(args)
    pairs = max(1, world // 2)
    if world == 1 and torch.cuda.device_count() < 2:
        print(json.dumps({"metric": METRIC, "unavailable": f"{args.workload} needs 2 GPUs"}))
        return
    is_compute = world == 1 or local < pairs
    compute, supplier = (0, 1) if world == 1 else (local, local + pairs)
    if not is_compute:  # supplier rank: its GPU holds a compute rank's bank; take part in the timing collectives
        dev = torch.device(f"cuda:{local}")
        torch.cuda.set_device(dev)
        barrier(world)
        barrier(world)
        max_over_ranks(0.0, world, dev)
        max_over_ranks(0.0, world, dev)
        import torch.distributed as dist
        dist.destroy_process_group()
        return
    torch.cuda.set_device(compute)
    w = TieredWorkload(args, compute, supplier, seed=args.seed + 1000 * local)
    stream = torch.cuda.current_stream(w.d0)
    for _ in range(max(args.warmup, 3)):
        w.step()
    torch.cuda.synchronize(w.d0)
    clocks = ClockSampler(compute)
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    if w.migrate:
        w.mig_events = []
    all_events = []
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        ev = [[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(w.layers)]
        w.step(ev)
        all_events.append(ev)
    t1.record(stream)
    torch.cuda.synchronize(w.d0)
    torch.cuda.synchronize(w.d1)
    barrier(world)
    clk = clocks.stop()
    layer_ms = [a.elapsed_time(b) for ev in all_events for a, b in ev]
    t_layer = max_over_ranks(sum(layer_ms) / len(layer_ms), world, w.d0) / 1e3
    step_ms = max_over_ranks(t0.elapsed_time(t1) / args.steps, world, w.d0)
    peak_hbm, peak_kind = measured_peaks()
    t_local = w.local_bytes() / (peak_hbm * 1e9)
    t_remote = w.remote_bytes() / (PEER_GBS * 1e9)
    t_star = max(t_local, t_remote)
    tok_s = pairs * w.B / (36 * t_layer)
    status = int(w.status.item()) | int(w.ws[:4].view(torch.int32).item())
    result = {
        "metric": METRIC, "value": round(tok_s, 2), "unit": UNIT, "n_gpus": 2 * pairs, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(36 * t_layer * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{args.workload}: {pairs} x (1 compute GPU + 1 KV supplier GPU, peer access), "
                               f"tiered decode",
                   "pairs": pairs, "timed_36_layer_equivalent_step_ms": round(36 * step_ms / w.layers, 4),
                   "batch": w.B, "sum_kv_tokens": w.T, "remote_tokens": w.R,
                   "remote_over_local": round(w.R / (w.T - w.R), 4), "read_order_rn_tn": [w.RN, w.TN],
                   "layers_resident": w.layers, "per_step": "36 x per-layer time",
                   "concurrent_migration": bool(w.migrate)},
        "roofline": {"bound": "nvlink" if t_remote > t_local else "hbm",
                     "achieved": round((w.local_bytes() + w.remote_bytes()) / t_layer / 1e9, 1),
                     "peak": round((w.local_bytes() + w.remote_bytes()) / t_star / 1e9, 1), "unit": "GB/s",
                     "frac": round(t_star / t_layer, 4), "traffic": None,
                     "local_gbs": round(w.local_bytes() / t_layer / 1e9, 1),
                     "peer_gbs": round(w.remote_bytes() / t_layer / 1e9, 1),
                     "t_star_ms": round(t_star * 1e3, 4), "layer_ms": round(t_layer * 1e3, 4),
                     "peak_source": f"{peak_kind} hbm_gbs {peak_hbm} + peer copy {PEER_GBS} GB/s per direction"},
        "gpu_launches": (1 + 2 * w.layers + (1 if w.migrate else 0)) * args.steps,
        "device_status": status,
    }
    if w.migrate and w.mig_events:
        mig_ms = [a.elapsed_time(b) for a, b in w.mig_events]
        nbytes = w.mig_tokens * w.layers * 4096
        result["migration"] = {"tokens_per_batch": w.mig_tokens, "planes": 2 * w.layers,
                               "bytes_per_batch": nbytes, "bytes_per_batch_36_layers": w.mig_tokens * 147456,
                               "avg_ms": round(sum(mig_ms) / len(mig_ms), 4),
                               "gbs": round(nbytes / (sum(mig_ms) / len(mig_ms) / 1e3) / 1e9, 1),
                               "status": int(w.mig_status.item())}
        # bit-exactness of everything migrated so far (sampled rows of every plane)
        torch.cuda.synchronize(w.d0)
        k = min(w.batch_no, 4) * w.mig_tokens
        ok = True
        for i in range(w.layers):
            for plane, t in enumerate((w.k[i], w.v[i])):
                src = w.bg_local[:k:97]
                dst = w.bg_remote[:k:97]
                got = w.bank.banks[0][i, plane].index_select(0, dst.to(w.d1)).to(w.d0)
                ok &= bool(torch.equal(got.view(torch.int16), t.index_select(0, src).view(torch.int16)))
        result["migration"]["bit_exact_sampled"] = ok
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
    work = ops.append_plan(qo, kv, True).to(dev)
    Q = int(qlens.sum())
    q = torch.empty((Q, 32, 128), dtype=torch.bfloat16, device=dev).normal_(generator=g)
    out = torch.empty_like(q)
    lse = torch.empty((Q, 32), dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    qo_d, kv_d = torch.from_numpy(qo).to(dev), torch.from_numpy(kv).to(dev)
    flops = float(sum(16384 * (int(x) * int(p_) + int(x) * (int(x) + 1) / 2) for x, p_ in zip(qlens, pref)))
    return types.SimpleNamespace(B=B, dev=dev, owners=owners, qlens=qlens, pref=pref, lengths=lengths, T=T, R=R, C=C,
                                 k=k, v=v, pk=pk, pv=pv, full=full, qo=qo, kv=kv, work=work, Q=Q, q=q, out=out, lse=lse,
                                 status=status, qo_d=qo_d, kv_d=kv_d, flops=flops)


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

    # end to end through the reference-facing wrapper: q from pinned host memory, plan + run_return_lse,
    # outputs and LSE back to pinned host memory, every step
    e2e = None
    from dual_b200.wrapper import BatchPrefillWithPagedKVCacheWrapper
    wrapper = BatchPrefillWithPagedKVCacheWrapper(torch.empty(1 << 20, dtype=torch.uint8, device=dev), "NHD")
    q_host = q.cpu().pin_memory()
    out_host = torch.empty(out.shape, dtype=torch.bfloat16).pin_memory()
    lse_host = torch.empty(lse.shape, dtype=torch.float32).pin_memory()
    qo_t, kv_t = torch.from_numpy(qo), torch.from_numpy(kv)
    peers = [t for pair in zip(pk, pv) for t in pair]
    q_dev = torch.empty_like(q)

    def e2e_step(i):
        q_dev.copy_(q_host, non_blocking=True)
        wrapper.plan(qo_t, kv_t, full, torch.ones(B, dtype=torch.int32), 32, 8, 128, 1, causal=True,
                     q_data_type=torch.bfloat16)
        tail = peers if stager is None else stager.tail(i)
        o_, l_ = wrapper.run_return_lse(q_dev, (k.unsqueeze(1), v.unsqueeze(1)), *tail, full, C, 128 ** -0.5)
        done(i)
        out_host.copy_(o_, non_blocking=True)
        lse_host.copy_(l_, non_blocking=True)

    if not args.no_e2e:
        begin()
        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        begin()
        for i in range(args.steps):
            e2e_step(i)
        e1.record()
        torch.cuda.synchronize()
        e2e = {"value": round(e0.elapsed_time(e1) / args.steps, 4), "unit": "ms",
               "h2d_bytes_per_step": q_host.numel() * 2,
               "d2h_bytes_per_step": out_host.numel() * 2 + lse_host.numel() * 4,
               "api": "dual_b200.wrapper.BatchPrefillWithPagedKVCacheWrapper.plan/run_return_lse"}

    # traffic: DRAM bytes of one launch from the committed ncu summary of this workload, if any
    traffic = None
    tfile = ROOT / "profiles" / "append_traffic.json"
    if tfile.exists():
        tj = json.loads(tfile.read_text())
        if tj.get("workload") == args.workload:
            traffic = tj.get("dram_bytes_per_launch")

    # CPU baseline: the fp32 oracle on a bounded sample (the last query tokens of the median request
    # against its whole visible context), scaled by FLOPs
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
                      "clocks": clk, "e2e": e2e, "cpu_baseline": cpu,
                      "status": int(status.item()) | wrapper.status() | (stager.status() if stager else 0),
                      "gpu_launches": args.steps * (2 if args.stage == "rows" else 1)}), flush=True)

# ------------------------------------------------------- native FlashInfer (the number to beat)
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
        dev = torch.device("cuda:0")
        args.workload = base
        w = DecodeWorkload(args, dev)
        w.ops.pack_read_order(w.tier, w.slot, w.req, w.seq, w.C, 5, 32, w.indices, status=w.status)
        wrapper = flashinfer.BatchDecodeWithPagedKVCacheWrapper(torch.empty(256 << 20, dtype=torch.uint8, device=dev),
                                                                "NHD", use_tensor_cores=True, backend="fa2")
        wrapper.plan(w.indptr, w.indices, torch.ones(w.B, dtype=torch.int32, device=dev), 32, 8, 128, 1,
                     q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16, sm_scale=scale)

        def step():
            for i in range(w.layers):
                wrapper.run(w.q[i], (w.k[i].unsqueeze(1), w.v[i].unsqueeze(1)), out=w.out[i])
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
        layer_ms = ms / w.layers
        peak, peak_kind = measured_peaks()
        gbs = w.bytes_per_layer() / (layer_ms / 1e3) / 1e9
        print(json.dumps({"impl": "flashinfer-fa2-native", "metric": METRIC, "value": round(w.B / (ms / 1e3), 2),
                          "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
                          "ms_per_step": round(ms, 4), "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
                          "config": {"workload": f"{base} inputs, native FlashInfer {flashinfer.__version__} FA2 "
                                                 f"BatchDecode(use_tensor_cores=True), all-local",
                                     "batch": w.B, "sum_kv_tokens": w.T, "layers": w.layers},
                          "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                                       "frac": round(gbs / peak, 4), "layer_ms": round(layer_ms, 4),
                                       "peak_source": f"{peak_kind} hbm_gbs"},
                          "clocks": clk}), flush=True)
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
    """The reference's CPU attention math (fp32 torch restatement of check_attention_output,
    oracle port) on this host's cores, same workload definition; bounded sample per step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle.attention import attend
    B, lmin, lmax, C, layers = WORKLOADS[args.workload]
    lengths, seed_used = draw_lengths(B, lmin, lmax, C, args.seed)
    T = int(lengths.sum())
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(args.seed)
    order = np.argsort(lengths)
    b = int(order[len(order) // 2])
    L = int(lengths[b])
    # sample: one request of the batch, one layer, gathered from a scattered pool of 4L slots
    pool_k = torch.randn((4 * L, 8, 128), generator=g).to(torch.bfloat16)
    pool_v = torch.randn((4 * L, 8, 128), generator=g).to(torch.bfloat16)
    slots = torch.randperm(4 * L, generator=g)[:L]
    q = torch.randn((1, 32, 128), generator=g).to(torch.bfloat16)

    def one():
        attend(q, pool_k.index_select(0, slots), pool_v.index_select(0, slots), L - 1, 128 ** -0.5)

    for _ in range(max(args.warmup, 1)):
        one()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    dt = (time.perf_counter() - t0) / args.steps
    step_s = dt / L * T * layers
    value = B / step_s
    sample = f"1 of {B} requests (L={L}), 1 layer per step; scaled by sum(L)={T} and {layers} layers"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": 0,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_s * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.workload}: CPU fp32 reference attention math", "batch": B,
                   "sum_kv_tokens": T, "length_seed": seed_used, "layers": layers},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    args = parse()
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
