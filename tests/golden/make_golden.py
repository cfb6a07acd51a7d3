"""Generate the golden fixtures in tests/golden/ by running the REFERENCE's own code on the CPU.

Usage (only where the reference checkout is available; the fixtures are committed):

    python tests/golden/make_golden.py --reference <path to Eyan-L/Dual checkout>

What is executed, all from the reference checkout, unmodified:
  * ``history_order``            final/cooperative_4gpu/code/peer/layout.py:5-22 (plain torch)
  * ``packing.prepare``          peer/packing.py:6-36              (Triton, CPU interpreter)
  * ``_count_remote``/``_pack_indices`` peer/backend.py:22-58       (Triton, CPU interpreter;
                                  the two functions are lifted out of the module with ``ast`` because
                                  importing backend.py pulls in SGLang)
  * ``_write_prefill_layout``     peer/page_ops.py:6-18             (Triton, CPU interpreter)
  * ``copy_pages``/``restore``    peer/fused_copy.py:24-33          (Triton, CPU interpreter)
  * ``check_attention_output``   V/nvlink_short_serving/.../backend.py:261-286 (fp32 torch; lifted
                                  with ``ast`` and run on SimpleNamespace fakes, the reference's own
                                  method in check_bookkeeping.py:9-27), with the reference's
                                  ``RemoteBank`` (peer/remote_bank.py) for 3-bank striping
  * ``limit_pages``               V/nvlink_migration_latency/.../backend.py:23-25
  * ``budget`` / ``repair_active_ratio`` count   peer/policy.py:42-46,107-110
"""
from __future__ import annotations

import argparse
import ast
import hashlib
import importlib.util
import json
import os
import sys
import tempfile
import types
from pathlib import Path
from types import SimpleNamespace as NS

os.environ["TRITON_INTERPRET"] = "1"  # must precede the first triton import

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases as C  # noqa: E402


def load_module(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def lift_functions(path: Path, names, tmpdir: Path, header: str, cls: str = None):
    """Copy the named top-level (or class-level) functions of ``path`` into an importable temp module."""
    tree = ast.parse(path.read_text())
    body = tree.body
    if cls is not None:
        body = next(n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == cls).body
    chunks = [header]
    src = path.read_text()
    for node in body:
        if isinstance(node, ast.FunctionDef) and node.name in names:
            seg = ast.get_source_segment(src, node, padded=False)
            deco = "".join("@" + ast.get_source_segment(src, d) + "\n" for d in node.decorator_list)
            chunks.append(deco + seg if not seg.lstrip().startswith("@") else seg)
    out = tmpdir / f"lifted_{path.stem}_{abs(hash(tuple(names))) % 10**8}.py"
    out.write_text("\n\n".join(chunks) + "\n")
    return load_module(out.stem, out)


class _Indexer:
    """``obj[layer, plane]`` -> fn((layer, plane))."""

    def __init__(self, fn):
        self.fn = fn

    def __getitem__(self, key):
        return self.fn(key)


class TorchProxy(types.ModuleType):
    """``torch`` with ``testing.assert_close`` replaced by a recorder (to read the oracle's expected)."""

    def __init__(self):
        super().__init__("torch_proxy")
        self.captured = []
        rec = self.captured
        self.testing = NS(assert_close=lambda actual, expected, **kw: rec.append(expected.clone()))

    def __getattr__(self, name):
        return getattr(torch, name)


# ------------------------------------------------------------------ generators
def gen_history_order(layout, rng) -> dict:
    out = []
    known = dict(encoded=list(range(40)), far=[True] * 7 + [False] * 33, prefix=40, rn=5, tn=32)
    for rn, tn in [(5, 32), (8, 128), (3, 8), (1, 2), (0, 32), (31, 32)]:
        for trial in range(12):
            n = int(rng.integers(0, 300))
            prefix = int(rng.integers(0, n + 1))
            p_remote = float(rng.choice([0.0, 0.05, 0.18, 0.5, 0.95, 1.0]))
            far = np.zeros(n, bool)
            far[:prefix] = rng.random(prefix) < p_remote
            if trial % 3 == 0:  # FIFO remote prefix (what migration produces)
                r = int(far[:prefix].sum())
                far[:prefix] = False
                far[:r] = True
            encoded = rng.integers(0, 10**6, n).astype(np.int32)
            out.append(dict(encoded=encoded.tolist(), far=far.tolist(), prefix=prefix, rn=rn, tn=tn))
    out.append(known)
    for c in out:
        res = layout.history_order(torch.tensor(c["encoded"], dtype=torch.int32), torch.tensor(c["far"]),
                                   c["prefix"], c["rn"], c["tn"])
        c["expected"] = res.tolist()
    return dict(cases=out)


def random_tables(rng, B, max_len, cap, remote_prefix: bool, p_remote: float, prefix_frac=None):
    rows = B + 2
    tier = np.full((rows, max_len), -1, np.int32)
    slot = np.zeros((rows, max_len), np.int32)
    req = rng.permutation(rows)[:B].astype(np.int32)
    seq = rng.integers(1, max_len + 1, B).astype(np.int32)
    prefix = (seq if prefix_frac is None else
              np.minimum(seq, (seq * rng.uniform(0, prefix_frac, B)).astype(np.int32))).astype(np.int32)
    local = rng.permutation(cap)[: int(seq.sum())] + 1
    o = 0
    rid_next = 0
    for b in range(B):
        n, p = int(seq[b]), int(prefix[b])
        far = np.zeros(n, bool)
        far[:p] = rng.random(p) < p_remote
        if remote_prefix:
            r = int(far.sum())
            far[:] = False
            far[:r] = True
        t = far.astype(np.int32)
        s = local[o:o + n].astype(np.int32)
        o += n
        nr = int(far.sum())
        s[far] = np.arange(rid_next, rid_next + nr)
        rid_next += nr
        tier[req[b], :n] = t
        slot[req[b], :n] = s
    return tier, slot, req, seq, prefix


def gen_packers(peer_dir: Path, tmp: Path, rng) -> dict:
    import triton
    packing = load_module("ref_packing", peer_dir / "packing.py")
    page_ops_dir = str(peer_dir)
    sys.path.insert(0, page_ops_dir)
    page_ops = load_module("ref_page_ops", peer_dir / "page_ops.py")
    lifted = lift_functions(peer_dir / "backend.py", ["_count_remote", "_pack_indices"], tmp,
                            "import triton\nimport triton.language as tl\n")
    out = {}
    k = 0
    # decode packer: remote-prefix tables (its documented precondition)
    for rn, tn in [(5, 32), (8, 128), (0, 32)]:
        for trial in range(3):
            B, L, cap = int(rng.integers(1, 7)), int(rng.integers(1, 700)), 5000
            tier, slot, req, seq, _ = random_tables(rng, B, L, cap, True, float(rng.choice([0.06, 0.18, 0.6, 1.0])))
            T = torch.from_numpy
            remote = torch.zeros(B, dtype=torch.int32)
            indices = torch.full((int(seq.sum()) + 8,), -7, dtype=torch.int32)
            pad = triton.next_power_of_2(int(seq.max()))
            lifted._count_remote[(B,)](T(tier), T(req), T(seq), remote, tier.shape[1], pad, num_warps=4)
            lifted._pack_indices[(B, triton.cdiv(int(seq.max()), 256))](
                T(tier), T(slot), T(req), T(seq), remote, indices, tier.shape[1], cap, B,
                triton.next_power_of_2(B), 256, rn, tn, num_warps=4)
            out[f"decode{k}"] = dict(tier=tier, slot=slot, req=req, seq=seq, cap=np.int64(cap), rn=np.int64(rn),
                                     tn=np.int64(tn), remote=remote.numpy(), full=indices.numpy())
            k += 1
    # prefill packer: arbitrary tier maps inside the prefix, local query suffix
    k = 0
    for rn, tn in [(5, 32), (8, 128), (3, 8), (0, 32)]:
        for trial in range(3):
            B, L, cap = int(rng.integers(1, 7)), int(rng.integers(1, 700)), 5000
            tier, slot, req, seq, prefix = random_tables(rng, B, L, cap, trial == 2,
                                                         float(rng.choice([0.05, 0.18, 0.5, 0.95])), prefix_frac=1.0)
            T = torch.from_numpy
            full = torch.full((int(seq.sum()) + 8,), -7, dtype=torch.int32)
            hist = torch.full((int(prefix.sum()) + 8,), -7, dtype=torch.int32)
            packing.prepare[(B,)](T(tier), T(slot), T(req), T(seq), T(prefix), full, hist, tier.shape[1], cap, B,
                                  triton.next_power_of_2(B), triton.next_power_of_2(int(seq.max())), rn, tn,
                                  num_warps=8)
            out[f"prefill{k}"] = dict(tier=tier, slot=slot, req=req, seq=seq, prefix=prefix, cap=np.int64(cap),
                                      rn=np.int64(rn), tn=np.int64(tn), full=full.numpy(), history=hist.numpy())
            k += 1
    # layout writer
    for k in range(3):
        B, L = int(rng.integers(1, 6)), 300
        tier = np.full((B + 2, L), -1, np.int32)
        slot = np.zeros_like(tier)
        req = rng.permutation(B + 2)[:B].astype(np.int32)
        length = rng.integers(1, 100, B).astype(np.int32)
        prefix = rng.integers(0, L - 100, B).astype(np.int32)
        start = np.concatenate([[0], np.cumsum(length)[:-1]]).astype(np.int32)
        loc = rng.integers(1, 10**6, int(length.sum())).astype(np.int64)
        t2, s2 = torch.from_numpy(tier.copy()), torch.from_numpy(slot.copy())
        page_ops.write_prefill_layout(t2, s2, torch.from_numpy(req), torch.from_numpy(start),
                                      torch.from_numpy(length), torch.from_numpy(prefix), torch.from_numpy(loc),
                                      int(length.max()))
        out[f"layout{k}"] = dict(tier=tier, slot=slot, req=req, start=start, length=length, prefix=prefix, loc=loc,
                                 tier_out=t2.numpy(), slot_out=s2.numpy())
    return out


def gen_copy(peer_dir: Path) -> dict:
    fc = load_module("ref_fused_copy", peer_dir / "fused_copy.py")
    sys.path.insert(0, str(peer_dir))
    rb = load_module("ref_remote_bank", peer_dir / "remote_bank.py")
    out = {}
    layers, local_slots, bank_slots = 36, 40, 12
    for case, (n, seed) in enumerate([(2, 1), (17, 2), (30, 3)]):
        g = torch.Generator().manual_seed(seed)
        local = [torch.zeros((local_slots, 8, 128), dtype=torch.bfloat16) for _ in range(layers * 2)]
        source = (torch.randperm(local_slots - 1, generator=g)[:n] + 1).long()
        target = torch.randperm(3 * bank_slots, generator=g)[:n].long()
        for i in range(layers):
            for plane in range(2):
                value = ((torch.arange(n * 1024).reshape(n, 8, 128) % 127) / 64 + i / 16 + plane / 8).to(torch.bfloat16)
                local[2 * i + plane].index_copy_(0, source, value)
        banks = [torch.zeros((layers, 2, bank_slots, 8, 128), dtype=torch.bfloat16) for _ in range(3)]
        bank = rb.RemoteBank(banks)
        pointers = torch.tensor([t.data_ptr() for t in local], dtype=torch.int64)
        fc.copy_pages(pointers, bank, source, target)
        fwd = [hashlib.sha256(b.view(torch.int16).numpy().tobytes()).hexdigest() for b in banks]
        # reverse: bring the remote ids back into fresh local slots
        back = [torch.zeros_like(t) for t in local]
        back_ptr = torch.tensor([t.data_ptr() for t in back], dtype=torch.int64)
        dest = (torch.randperm(local_slots - 1, generator=g)[:n] + 1).long()
        fc.restore(back_ptr, bank, target, dest)
        rev = hashlib.sha256(b"".join(t.view(torch.int16).numpy().tobytes() for t in back)).hexdigest()
        out[f"copy{case}"] = dict(n=n, source=source.tolist(), target=target.tolist(), dest=dest.tolist(),
                                  layers=layers, local_slots=local_slots, bank_slots=bank_slots,
                                  forward_bank_sha256=fwd, reverse_local_sha256=rev)
    return out


def gen_attention(short_backend: Path, peer_dir: Path, tmp: Path) -> dict:
    sys.path.insert(0, str(peer_dir))
    rb = load_module("ref_remote_bank2", peer_dir / "remote_bank.py")
    tree = ast.parse(short_backend.read_text())
    cls = next(n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == "ReplayBackend")
    fn = next(n for n in cls.body if isinstance(n, ast.FunctionDef) and n.name == "check_attention_output")
    module = ast.fix_missing_locations(ast.Module(body=[fn], type_ignores=[]))
    proxy = TorchProxy()
    ns = dict(torch=proxy)
    exec(compile(module, "reference-check_attention_output", "exec"), ns)
    check = ns["check_attention_output"]
    out = {}
    for banks in (1, 3):
        for case in C.all_cases(banks=banks):
            if banks == 3:
                # The reference RemoteBank striping (g % 3, g // 3) through its own Plane.index_select;
                # one layer ([1, 2, slots, 8, 128] per bank) is all the oracle reads.
                bank = object.__new__(rb.RemoteBank)
                bank.banks = [torch.stack([k, v]).unsqueeze(0) for k, v in zip(case.peer_k, case.peer_v)]
                peer = _Indexer(lambda key, bank=bank: rb.Plane(bank, 0, key[1]))
            else:
                # 2-GPU layout: one donor tensor, physical slot = g (short_serving backend.py:276)
                peer = _Indexer(lambda key, case=case: (case.peer_k[0], case.peer_v[0])[key[1]])
            for mode in ("decode", "prefill"):
                if mode == "decode":
                    q = case.decode_q()
                    fb = NS(seq_lens_cpu=torch.tensor(case.lengths), forward_mode=NS(is_extend=lambda: False),
                            batch_size=len(case.lengths))
                else:
                    q = case.q
                    fb = NS(seq_lens_cpu=torch.tensor(case.lengths), forward_mode=NS(is_extend=lambda: True),
                            extend_seq_lens_cpu=case.qlens, extend_prefix_lens_cpu=case.prefixes,
                            batch_size=len(case.lengths))
                raw = NS(token_to_kv_pool=NS(get_kv_buffer=lambda layer: (case.k_local, case.v_local)))
                state = NS(enabled=True, slot=case.slot, tier=case.tier, raw=raw, peer=peer,
                           req_objects=[NS(kv=NS(req_pool_idx=r)) for r in case.requests],
                           cfg=dict(reference_atol=0.01, reference_rtol=0.02), layer_checks=[], frames=[],
                           remote_active=0)
                proxy.captured.clear()
                check(state, q, torch.zeros(q.shape, dtype=torch.float32), 0, fb)
                expected = proxy.captured[0].float()
                if mode == "prefill":
                    # keep first / middle / last query row of every request (fixture size)
                    rows, o = [], 0
                    for ql in case.qlens:
                        rows += sorted({o, o + ql // 2, o + ql - 1})
                        o += ql
                    out[f"{case.name}_b{banks}_{mode}_rows"] = np.array(rows, np.int64)
                    expected = expected[rows]
                out[f"{case.name}_b{banks}_{mode}"] = expected.numpy()
    return out


def gen_policy(mig_backend: Path, peer_dir: Path, tmp: Path, rng) -> dict:
    lifted = lift_functions(mig_backend, ["limit_pages"], tmp, "")
    sys.path.insert(0, str(peer_dir))
    policy = load_module("ref_policy", peer_dir / "policy.py")
    rows = []
    for _ in range(300):
        local = int(rng.integers(0, 200000))
        remote = int(rng.integers(0, 40000))
        a, b = [(599, 10000), (1797, 10000)][int(rng.integers(0, 2))]
        free = int(rng.integers(0, 20000))
        residents = int(rng.integers(0, 20000))
        lim = lifted.limit_pages(local, remote, a, b)
        st = NS(cfg=dict(kv_capacity_tokens=10**7, remote_ratio_numerator=a, remote_ratio_denominator=b),
                physical_allocator=NS(available_size=lambda local=local: 10**7 - local), committed_remote=remote,
                peer_free=[0] * free, residents=[0] * residents)
        bud = policy.budget(st)
        # repair count as computed inside repair_active_ratio (peer/policy.py:109-110)
        rep = 0 if (not remote or b * remote < a * local) else (b * remote - a * local) // (a + b) + 1
        rows.append(dict(local=local, remote=remote, a=a, b=b, peer_free=free, residents=residents, limit=lim,
                         budget=list(bud), repair=rep))
    return dict(rows=rows)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    args = ap.parse_args()
    ref = args.reference
    peer_dir = ref / "final/cooperative_4gpu/code/peer"
    short_backend = ref / "final/vendor/nvlink_short_serving/launch_local_20261031_r2/code/backend.py"
    mig_backend = ref / "final/vendor/nvlink_migration_latency/launch_large_20261031_r2/code/backend.py"
    rng = np.random.default_rng(20261201)
    with tempfile.TemporaryDirectory() as td:
        tmp = Path(td)
        sys.path.insert(0, str(tmp))
        layout = load_module("ref_layout", peer_dir / "layout.py")
        (HERE / "history_order.json").write_text(json.dumps(gen_history_order(layout, rng)))
        np.savez_compressed(HERE / "packers.npz", **{f"{k}__{f}": v for k, d in gen_packers(peer_dir, tmp, rng).items()
                                                     for f, v in d.items()})
        (HERE / "copy.json").write_text(json.dumps(gen_copy(peer_dir), indent=1))
        np.savez_compressed(HERE / "attention.npz", **gen_attention(short_backend, peer_dir, tmp))
        (HERE / "policy.json").write_text(json.dumps(gen_policy(mig_backend, peer_dir, tmp, rng)))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
