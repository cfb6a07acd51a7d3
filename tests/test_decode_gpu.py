"""Parity of the tiered split-KV decode kernel (through the C ABI) against the pinned oracle.

Tolerance (the hot path's parity target): bf16 outputs within 2e-3 abs / 1e-2 rel of the fp32 reference;
LSE (base 2) within the same bound.
"""
import numpy as np
import pytest
import torch

import cases as C
from gpu_util import DEV, decode, pack_decode, to_dev
from oracle import attention as OA
from oracle import layout as OL
from dual_b200 import ops
from dual_b200.wrapper import BatchDecodeWithPagedKVCacheWrapper

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2


def _status(ws):
    return int(ws[:4].view(torch.int32).item())


@pytest.mark.parametrize("banks", [1, 3])
def test_decode_matches_reference_golden(golden_dir, banks):
    gold = np.load(golden_dir / "attention.npz")
    for case in C.all_cases(banks=banks):
        dev = to_dev(case)
        indptr, idx, st = pack_decode(dev, case.requests, case.lengths, case.local_capacity)
        out, lse, ws = decode(case.decode_q(), dev, indptr, idx, case.local_capacity)
        torch.cuda.synchronize()
        ref = torch.from_numpy(gold[f"{case.name}_b{banks}_decode"])
        torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL, msg=case.name)
        _, ref_lse = OA.decode_from_indices(case.decode_q(), case.k_local, case.v_local, case.peer_k, case.peer_v,
                                            indptr.cpu().tolist(), idx.cpu(), case.local_capacity)
        torch.testing.assert_close(lse.cpu(), ref_lse, atol=ATOL, rtol=RTOL, msg=case.name)
        assert _status(ws) == 0 and int(st.item()) == 0


@pytest.mark.parametrize("num_ctas", [1, 2, 5, 37, 300])
def test_decode_split_counts(num_ctas):
    """Any CTA count (one CTA per head group .. more CTAs than tokens) gives the same answer."""
    case = C.validate_case(4)  # empty_decode_splits: lengths 1 and 3
    case2 = C.config1(banks=3)
    for c in (case, case2):
        dev = to_dev(c)
        indptr, idx, _ = pack_decode(dev, c.requests, c.lengths, c.local_capacity)
        out, lse, ws = decode(c.decode_q(), dev, indptr, idx, c.local_capacity, num_ctas=num_ctas)
        ref, ref_lse = OA.decode_from_indices(c.decode_q(), c.k_local, c.v_local, c.peer_k, c.peer_v,
                                              indptr.cpu().tolist(), idx.cpu(), c.local_capacity)
        torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(lse.cpu(), ref_lse, atol=ATOL, rtol=RTOL)
        assert _status(ws) == 0


def test_decode_empty_request_and_deterministic():
    case = C.config1()
    dev = to_dev(case)
    lengths = [case.lengths[0], 0, case.lengths[2], 0]
    indptr, idx, _ = pack_decode(dev, case.requests, lengths, case.local_capacity)
    q = case.decode_q()
    out1, lse1, _ = decode(q, dev, indptr, idx, case.local_capacity)
    out2, lse2, _ = decode(q, dev, indptr, idx, case.local_capacity)
    assert torch.equal(out1, out2) and torch.equal(lse1, lse2)
    assert (out1[1] == 0).all() and (out1[3] == 0).all()
    assert torch.isinf(lse1[1]).all() and (lse1[1] < 0).all()
    ref, _ = OA.decode_from_indices(q, case.k_local, case.v_local, case.peer_k, case.peer_v, indptr.cpu().tolist(),
                                    idx.cpu(), case.local_capacity)
    torch.testing.assert_close(out1.float().cpu(), ref, atol=ATOL, rtol=RTOL)


def test_remote_value_perturbation_and_exact_restore():
    """V/nvlink_prefill/.../validate_kernel.py:61-68: +0.5 on supplier V shifts a remote-only output
    by 0.5; restoring the exact source restores the output bit for bit."""
    case = C.validate_case(2, banks=3)  # remote_only
    dev = to_dev(case)
    indptr, idx, _ = pack_decode(dev, case.requests, case.lengths, case.local_capacity)
    base, _, _ = decode(case.decode_q(), dev, indptr, idx, case.local_capacity)
    saved = [v.clone() for v in dev["peer_v"]]
    for v in dev["peer_v"]:
        v.add_(0.5)
    shifted, _, _ = decode(case.decode_q(), dev, indptr, idx, case.local_capacity)
    torch.testing.assert_close(shifted.float() - base.float(), torch.full_like(base.float(), 0.5), atol=0.012,
                               rtol=0.02)
    for v, s in zip(dev["peer_v"], saved):
        v.copy_(s)
    restored, _, _ = decode(case.decode_q(), dev, indptr, idx, case.local_capacity)
    assert torch.equal(restored, base)


def test_lse_merge_of_split_requests():
    """Decode a request as two disjoint index lists and merge with the base-2 LSEs (cascade rule)."""
    case = C.config1(banks=3)
    dev = to_dev(case)
    L = case.lengths[3]
    indptr, idx, _ = pack_decode(dev, [3], [L], case.local_capacity)
    cut = 1234
    q = case.decode_q()[3:4].repeat(2, 1, 1)
    indptr2 = torch.tensor([0, cut, L], dtype=torch.int32, device=DEV)
    out2, lse2, _ = decode(q, dev, indptr2, idx, case.local_capacity)
    full, lse_full, _ = decode(q[:1], dev, indptr, idx, case.local_capacity)
    om, lm = OA.merge_states(out2[0:1].float().cpu(), lse2[0:1].cpu(), out2[1:2].float().cpu(), lse2[1:2].cpu())
    torch.testing.assert_close(om, full.float().cpu(), atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lm, lse_full.cpu(), atol=ATOL, rtol=RTOL)


def test_bad_page_ids_set_status_not_fault():
    case = C.validate_case(0)
    dev = to_dev(case)
    indptr, idx, _ = pack_decode(dev, case.requests, case.lengths, case.local_capacity)
    bad = idx.clone()
    bad[0] = case.local_capacity + 1 + 10**6  # remote id far beyond the supplier bank
    out, _, ws = decode(case.decode_q(), dev, indptr, bad, case.local_capacity)
    torch.cuda.synchronize()
    assert _status(ws) & 0x2


def test_wrapper_reference_calling_convention():
    """plan() once, run(q, paged_kv, *peers, unified_indices, local_capacity, sm_scale) per layer,
    exactly as the reference hook passes them (peer/backend.py:132-138)."""
    case = C.config1(banks=3)
    dev = to_dev(case)
    indptr, idx, _ = pack_decode(dev, case.requests, case.lengths, case.local_capacity)
    ws = torch.empty(128 * 1024 * 1024, dtype=torch.uint8, device=DEV)
    w = BatchDecodeWithPagedKVCacheWrapper(ws, "NHD", use_tensor_cores=True)
    w.plan(indptr, idx, torch.ones(4, dtype=torch.int32), 32, 8, 128, 1, q_data_type=torch.bfloat16,
           sm_scale=128 ** -0.5)
    peers = [t for pair in zip(dev["peer_k"], dev["peer_v"]) for t in pair]
    q = case.decode_q().to(DEV)
    paged = (dev["k_local"].unsqueeze(1), dev["v_local"].unsqueeze(1))
    out, lse = w.run_return_lse(q, paged, *peers, idx, case.local_capacity, 128 ** -0.5)
    ref, ref_lse = OA.decode_from_indices(case.decode_q(), case.k_local, case.v_local, case.peer_k, case.peer_v,
                                          indptr.cpu().tolist(), idx.cpu(), case.local_capacity)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse.cpu(), ref_lse, atol=ATOL, rtol=RTOL)
    # native (all-local) mode: indices from plan()
    case1 = C.validate_case(0)
    dev1 = to_dev(case1)
    indptr1, idx1, _ = pack_decode(dev1, case1.requests, case1.lengths, case1.local_capacity)
    w.plan(indptr1, idx1, torch.ones(3, dtype=torch.int32), 32, 8, 128, 1)
    o1 = w.run(case1.decode_q().to(DEV), (dev1["k_local"], dev1["v_local"]))
    ref1, _ = OA.decode_from_indices(case1.decode_q(), case1.k_local, case1.v_local, [], [],
                                     indptr1.cpu().tolist(), idx1.cpu(), case1.local_capacity)
    torch.testing.assert_close(o1.float().cpu(), ref1, atol=ATOL, rtol=RTOL)


def test_decode_cuda_graph_replay():
    """The run is capturable: replay with new q / indices in the same buffers matches eager."""
    case = C.config1(banks=3)
    dev = to_dev(case)
    indptr, idx, _ = pack_decode(dev, case.requests, case.lengths, case.local_capacity)
    q = case.decode_q().to(DEV)
    B = q.shape[0]
    out = torch.empty((B, 32, 128), dtype=torch.bfloat16, device=DEV)
    lse = torch.empty((B, 32), dtype=torch.float32, device=DEV)
    ws = torch.zeros(ops.decode_workspace_size(B, ops.default_ctas(0)), dtype=torch.uint8, device=DEV)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ops.tiered_decode(q, dev["k_local"], dev["v_local"], case.local_capacity, dev["peer_k"], dev["peer_v"],
                          indptr, idx, 128 ** -0.5, out, lse, ws)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        ops.tiered_decode(q, dev["k_local"], dev["v_local"], case.local_capacity, dev["peer_k"], dev["peer_v"],
                          indptr, idx, 128 ** -0.5, out, lse, ws)
    q.copy_(torch.randn_like(q))
    g.replay()
    torch.cuda.synchronize()
    ref, _ = OA.decode_from_indices(q.cpu(), case.k_local, case.v_local, case.peer_k, case.peer_v,
                                    indptr.cpu().tolist(), idx.cpu(), case.local_capacity)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)


def test_decode_long_contexts_against_oracle():
    """Config-2 shaped requests (L up to 32K, 1M-slot-style scattered pages) on a sampled subset."""
    g = torch.Generator().manual_seed(7)
    lengths = [32768, 2048, 17000, 9001, 30000, 4096]
    pool = sum(lengths) + 1000
    perm = (torch.randperm(pool, generator=g) + 1)[: sum(lengths)].int()
    k = torch.randn((pool + 1, 8, 128), generator=g).to(torch.bfloat16)
    v = torch.randn((pool + 1, 8, 128), generator=g).to(torch.bfloat16)
    q = torch.randn((len(lengths), 32, 128), generator=g).to(torch.bfloat16)
    indptr = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32)
    dev = dict(k_local=k.to(DEV), v_local=v.to(DEV), peer_k=[], peer_v=[])
    out, lse, ws = decode(q, dev, indptr.to(DEV), perm.to(DEV), pool)
    ref, ref_lse = OA.decode_from_indices(q, k, v, [], [], indptr.tolist(), perm, pool)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse.cpu(), ref_lse, atol=ATOL, rtol=RTOL)


def test_decode_eight_supplier_banks():
    """The most supplier banks the ABI takes (8): striping g % 8 over every case's remote rows."""
    for case in C.all_cases(banks=8):
        dev = to_dev(case)
        indptr, idx, st = pack_decode(dev, case.requests, case.lengths, case.local_capacity)
        out, lse, ws = decode(case.decode_q(), dev, indptr, idx, case.local_capacity)
        ref, ref_lse = OA.decode_from_indices(case.decode_q(), case.k_local, case.v_local, case.peer_k, case.peer_v,
                                              indptr.cpu().tolist(), idx.cpu(), case.local_capacity)
        torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL, msg=case.name)
        torch.testing.assert_close(lse.cpu(), ref_lse, atol=ATOL, rtol=RTOL, msg=case.name)
        assert _status(ws) == 0 and int(st.item()) == 0


def _growing_scores(lengths, pool, seed):
    """K rows whose scores with q climb along the list (by ~40 in the log2 domain over a request),
    so the running maximum keeps moving past the lazy-rescale threshold (2^8) inside a segment."""
    g = torch.Generator().manual_seed(seed)
    B = len(lengths)
    q = torch.randn((B, 32, 128), generator=g)
    q = (q / q.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    k = torch.randn((pool + 1, 8, 128), generator=g) * 0.3
    v = torch.randn((pool + 1, 8, 128), generator=g).to(torch.bfloat16)
    perm = (torch.randperm(pool, generator=g) + 1)[: sum(lengths)]
    off = 0
    for b, L in enumerate(lengths):
        ramp = torch.linspace(0.0, 330.0, L)  # x 128^-0.5 x log2(e) ~ 42 in the log2 domain
        direction = q[b].float().view(8, 4, 128).mean(dim=1)  # shared by the GQA group of each kv head
        k[perm[off:off + L]] += ramp[:, None, None] * direction[None] / direction.norm(dim=-1, keepdim=True)[None]
        off += L
    return q, k.to(torch.bfloat16), v, perm.int()


def test_decode_rescales_when_the_max_keeps_growing():
    lengths = [5000, 300, 17, 2600]
    pool = sum(lengths) + 10
    q, k, v, perm = _growing_scores(lengths, pool, 3)
    indptr = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32)
    dev = dict(k_local=k.to(DEV), v_local=v.to(DEV), peer_k=[], peer_v=[])
    for num_ctas in (0, 7):
        out, lse, ws = decode(q, dev, indptr.to(DEV), perm.to(DEV), pool, num_ctas=num_ctas)
        ref, ref_lse = OA.decode_from_indices(q, k, v, [], [], indptr.tolist(), perm, pool)
        torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(lse.cpu(), ref_lse, atol=ATOL, rtol=RTOL)
        assert _status(ws) == 0


def test_decode_strided_views_and_other_scale():
    """q as a view of a fused qkv projection (token stride 6144), out as a view into a wider buffer,
    a scale other than 128^-0.5 and no LSE: the strides go through the ABI as given."""
    case = C.config1(banks=3)
    dev = to_dev(case)
    indptr, idx, _ = pack_decode(dev, case.requests, case.lengths, case.local_capacity)
    B = len(case.lengths)
    qkv = torch.zeros((B, 6144), dtype=torch.bfloat16, device=DEV)
    qkv[:, :4096] = case.decode_q().to(DEV).view(B, 4096)
    q = qkv[:, :4096].view(B, 32, 128)
    wide = torch.full((B, 40, 128), 3.0, dtype=torch.bfloat16, device=DEV)
    out = wide[:, 4:36]
    ws = torch.zeros(ops.decode_workspace_size(B, ops.default_ctas(0)), dtype=torch.uint8, device=DEV)
    scale = 0.05
    ops.tiered_decode(q, dev["k_local"], dev["v_local"], case.local_capacity, dev["peer_k"], dev["peer_v"], indptr,
                      idx, scale, out, None, ws)
    torch.cuda.synchronize()
    ref, _ = OA.decode_from_indices(case.decode_q(), case.k_local, case.v_local, case.peer_k, case.peer_v,
                                    indptr.cpu().tolist(), idx.cpu(), case.local_capacity, sm_scale=scale)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    assert bool((wide[:, :4] == 3.0).all()) and bool((wide[:, 36:] == 3.0).all())  # nothing outside the view
    assert _status(ws) == 0


def test_one_workspace_many_launches_counters_return_to_zero():
    """Requests split across CTAs are merged inside the decode kernel: the last CTA to finish a
    (request, kv head) merges, found through an arrival counter in the workspace that it resets.  One
    workspace, zeroed once, then serves launches of different batches and CTA counts (which change
    which requests are split, whole or empty), and every counter is back at zero after each."""
    runs = []
    for case in (C.config1(banks=3), C.validate_case(4), C.validate_case(3, banks=3)):
        dev = to_dev(case)
        lengths = list(case.lengths)
        if len(lengths) == 4:
            lengths[1] = 0  # an empty request between split ones
        indptr, idx, _ = pack_decode(dev, case.requests, lengths, case.local_capacity)
        ref, ref_lse = OA.decode_from_indices(case.decode_q(), case.k_local, case.v_local, case.peer_k,
                                              case.peer_v, indptr.cpu().tolist(), idx.cpu(), case.local_capacity)
        runs.append((case, dev, indptr, idx, ref, ref_lse))
    ws = torch.full((ops.decode_workspace_size(4, 300),), 0xA5, dtype=torch.uint8, device=DEV)
    ops.decode_workspace_reset(ws, 4)
    for rep in range(2):
        for case, dev, indptr, idx, ref, ref_lse in runs:
            for num_ctas in (1, 7, 148, 300):
                B = len(case.lengths)
                out = torch.full((B, 32, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
                lse = torch.full((B, 32), float("nan"), dtype=torch.float32, device=DEV)
                ops.tiered_decode(case.decode_q().to(DEV), dev["k_local"], dev["v_local"], case.local_capacity,
                                  dev["peer_k"], dev["peer_v"], indptr, idx, 128 ** -0.5, out, lse, ws, num_ctas)
                torch.cuda.synchronize()
                msg = f"{case.name} ctas={num_ctas} rep={rep}"
                torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL, msg=msg)
                torch.testing.assert_close(lse.cpu(), ref_lse, atol=ATOL, rtol=RTOL, msg=msg)
                assert _status(ws) == 0
                assert int(ws[256:256 + 4 * 8 * 4].view(torch.int32).abs().sum().item()) == 0, msg
