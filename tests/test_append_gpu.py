"""Parity of the tcgen05 causal append / prefill kernel (through the C ABI) against the pinned oracle:
the reference's own fp32 check in extend mode (golden), random append batches shaped like the
4-GPU configuration (long prefixes, skewed remote share, remote only in the history), the
non-causal history + causal chunk cascade merged by LSE, and the FlashInfer-style wrapper."""
import numpy as np
import pytest
import torch

import cases as C
from dual_b200 import ops
from dual_b200.wrapper import BatchPrefillWithPagedKVCacheWrapper
from oracle import attention as OA

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ATOL, RTOL = 2e-3, 1e-2


def _dev(case):
    d = torch.device(DEV)
    return (case.k_local.to(d), case.v_local.to(d), [t.to(d) for t in case.peer_k], [t.to(d) for t in case.peer_v],
            case.tier.to(d), case.slot.to(d))


def _full_list(tier, slot, requests, lengths, prefixes, capacity, rn=5, tn=32, history=False):
    d = torch.device(DEV)
    req = torch.tensor(requests, dtype=torch.int32, device=d)
    seq = torch.tensor(lengths, dtype=torch.int32, device=d)
    pre = torch.tensor(prefixes, dtype=torch.int32, device=d)
    full = torch.empty(sum(lengths), dtype=torch.int32, device=d)
    hist = torch.empty(max(sum(prefixes), 1), dtype=torch.int32, device=d)
    ops.pack_read_order(tier, slot, req, seq, capacity, rn, tn, full, prefix_lens=pre, history_out=hist)
    return full, hist


def _append(q, k, v, pk, pv, qlens, kvlens, indices, capacity, causal=True):
    d = torch.device(DEV)
    qo = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    kv = np.concatenate([[0], np.cumsum(kvlens)]).astype(np.int32)
    work = ops.append_plan(qo, kv, causal).to(d)
    out = torch.empty((int(qo[-1]), 32, 128), dtype=torch.bfloat16, device=d)
    lse = torch.empty((int(qo[-1]), 32), dtype=torch.float32, device=d)
    status = torch.zeros(1, dtype=torch.int32, device=d)
    ops.tiered_append(q.to(d), k, v, capacity, pk, pv, torch.from_numpy(qo).to(d), torch.from_numpy(kv).to(d),
                      indices, causal, 128 ** -0.5, work, out, lse, status)
    torch.cuda.synchronize()
    return out, lse, int(status.item())


@pytest.mark.parametrize("banks", [1, 3])
def test_append_matches_reference_golden(golden_dir, banks):
    gold = np.load(golden_dir / "attention.npz")
    for case in C.all_cases(banks=banks):
        k, v, pk, pv, tier, slot = _dev(case)
        full, _ = _full_list(tier, slot, case.requests, case.lengths, case.prefixes, case.local_capacity)
        out, lse, st = _append(case.q, k, v, pk, pv, case.qlens, case.lengths, full, case.local_capacity)
        assert st == 0, case.name
        rows = torch.from_numpy(gold[f"{case.name}_b{banks}_prefill_rows"])
        ref = torch.from_numpy(gold[f"{case.name}_b{banks}_prefill"])
        torch.testing.assert_close(out.float().cpu()[rows], ref, atol=ATOL, rtol=RTOL, msg=case.name)
        _, ref_lse = OA.tiered_attention(case.q, case.k_local, case.v_local, case.peer_k, case.peer_v, case.tier,
                                         case.slot, case.requests, case.lengths, case.qlens, case.prefixes)
        torch.testing.assert_close(lse.cpu(), ref_lse, atol=ATOL, rtol=RTOL, msg=case.name)


def _random_batch(seed, B=6, pmax=3000, qmax=300, banks=3, skew=True):
    """Append batch like the 4-GPU configuration, scaled down: prefix ~ U[100, pmax], query
    ~ logU[1, qmax], ~18% remote in the history with one request ~95% remote, remote ids striped."""
    g = torch.Generator().manual_seed(seed)
    rng = np.random.default_rng(seed)
    prefixes = rng.integers(100, pmax + 1, B).tolist()
    qlens = np.exp(rng.uniform(0, np.log(qmax), B)).astype(int).clip(1).tolist()
    lengths = [p + q for p, q in zip(prefixes, qlens)]
    total = sum(lengths)
    k_local = torch.randn((total + 1, 8, 128), generator=g).to(torch.bfloat16)
    v_local = torch.randn((total + 1, 8, 128), generator=g).to(torch.bfloat16)
    per_bank = total // banks + 2
    peer_k = [torch.randn((per_bank, 8, 128), generator=g).to(torch.bfloat16) for _ in range(banks)]
    peer_v = [torch.randn((per_bank, 8, 128), generator=g).to(torch.bfloat16) for _ in range(banks)]
    tier = torch.full((B + 1, max(lengths)), -1, dtype=torch.int32)
    slot = torch.zeros_like(tier)
    perm = torch.randperm(total, generator=g) + 1
    off, rid = 0, 0
    requests = list(rng.permutation(B + 1)[:B])
    for b, (L, p) in enumerate(zip(lengths, prefixes)):
        frac = 0.95 if (skew and b == 0) else 0.15
        far = np.zeros(L, bool)
        far[:p] = rng.random(p) < frac
        r = requests[b]
        s = perm[off:off + L].int().clone()
        off += L
        nr = int(far.sum())
        s[torch.from_numpy(far)] = torch.arange(rid, rid + nr, dtype=torch.int32)
        rid += nr
        tier[r, :L] = torch.from_numpy(far.astype(np.int32))
        slot[r, :L] = s
    q = torch.randn((sum(qlens), 32, 128), generator=g).to(torch.bfloat16)
    return C.TieredCase(f"rand{seed}", q, k_local, v_local, peer_k, peer_v, tier, slot, [int(x) for x in requests],
                        lengths, qlens, prefixes, total)


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_append_random_batches_against_oracle(seed):
    case = _random_batch(seed)
    k, v, pk, pv, tier, slot = _dev(case)
    full, _ = _full_list(tier, slot, case.requests, case.lengths, case.prefixes, case.local_capacity)
    out, lse, st = _append(case.q, k, v, pk, pv, case.qlens, case.lengths, full, case.local_capacity)
    assert st == 0
    ref, ref_lse = OA.tiered_attention(case.q, case.k_local, case.v_local, case.peer_k, case.peer_v, case.tier,
                                       case.slot, case.requests, case.lengths, case.qlens, case.prefixes)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse.cpu(), ref_lse, atol=ATOL, rtol=RTOL)


def test_cascade_history_plus_chunk_merge_equals_full_causal():
    """SGLang's ragged cascade (peer/cascade_oracle.py): non-causal attention over the (re-ordered)
    history + causal attention of the chunk over itself, merged by base-2 LSE, equals the full
    causal append over the Full list."""
    case = _random_batch(7, B=4)
    k, v, pk, pv, tier, slot = _dev(case)
    full, hist = _full_list(tier, slot, case.requests, case.lengths, case.prefixes, case.local_capacity)
    out_full, lse_full, _ = _append(case.q, k, v, pk, pv, case.qlens, case.lengths, full, case.local_capacity)
    out_h, lse_h, _ = _append(case.q, k, v, pk, pv, case.qlens, case.prefixes, hist, case.local_capacity,
                              causal=False)
    # chunk-only list: the query suffix of every request (local slots, in order)
    chunk = torch.cat([full[sum(case.lengths[:b]) + case.prefixes[b]: sum(case.lengths[:b + 1])]
                       for b in range(len(case.lengths))])
    out_c, lse_c, _ = _append(case.q, k, v, pk, pv, case.qlens, case.qlens, chunk, case.local_capacity, causal=True)
    om, lm = OA.merge_states(out_h.float().cpu(), lse_h.cpu(), out_c.float().cpu(), lse_c.cpu())
    torch.testing.assert_close(om, out_full.float().cpu(), atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lm, lse_full.cpu(), atol=ATOL, rtol=RTOL)


def test_append_edges_single_token_and_exact_tiles():
    """q_len 1 (decode-shaped), q_len a multiple of 32, kv length a multiple of 128."""
    g = torch.Generator().manual_seed(11)
    lengths, qlens = [128, 256 + 32, 1, 128 * 3], [1, 32, 1, 64]
    prefixes = [L - q for L, q in zip(lengths, qlens)]
    total = sum(lengths)
    k = torch.randn((total + 1, 8, 128), generator=g).to(torch.bfloat16)
    v = torch.randn((total + 1, 8, 128), generator=g).to(torch.bfloat16)
    q = torch.randn((sum(qlens), 32, 128), generator=g).to(torch.bfloat16)
    idx = (torch.randperm(total, generator=g) + 1).int()
    out, lse, st = _append(q, k.to(DEV), v.to(DEV), [], [], qlens, lengths, idx.to(DEV), total)
    assert st == 0
    # oracle: every request reads its own slice of idx, history first then the suffix, all local
    tier = torch.zeros((4, max(lengths)), dtype=torch.int32)
    slot = torch.zeros_like(tier)
    o = 0
    for b, L in enumerate(lengths):
        slot[b, :L] = idx[o:o + L]
        o += L
    ref, ref_lse = OA.tiered_attention(q, k, v, [], [], tier, slot, [0, 1, 2, 3], lengths, qlens, prefixes)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse.cpu(), ref_lse, atol=ATOL, rtol=RTOL)


def test_prefill_wrapper_reference_convention():
    case = _random_batch(5, B=3)
    k, v, pk, pv, tier, slot = _dev(case)
    full, _ = _full_list(tier, slot, case.requests, case.lengths, case.prefixes, case.local_capacity)
    w = BatchPrefillWithPagedKVCacheWrapper(torch.empty(1 << 20, dtype=torch.uint8, device=DEV), "NHD")
    qo = torch.tensor(np.concatenate([[0], np.cumsum(case.qlens)]), dtype=torch.int32)
    kv = torch.tensor(np.concatenate([[0], np.cumsum(case.lengths)]), dtype=torch.int32)
    w.plan(qo, kv, full, torch.ones(3, dtype=torch.int32), 32, 8, 128, 1, causal=True, q_data_type=torch.bfloat16)
    peers = [t for pair in zip(pk, pv) for t in pair]
    out, lse = w.run_return_lse(case.q.to(DEV), (k.unsqueeze(1), v.unsqueeze(1)), *peers, full,
                                case.local_capacity, 128 ** -0.5)
    ref, ref_lse = OA.tiered_attention(case.q, case.k_local, case.v_local, case.peer_k, case.peer_v, case.tier,
                                       case.slot, case.requests, case.lengths, case.qlens, case.prefixes)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse.cpu(), ref_lse, atol=ATOL, rtol=RTOL)
    assert w.status() == 0


def test_prefill_wrapper_cuda_graph_replay():
    """plan() builds the work list on the host, so run() is capturable: a graph replayed with new
    queries in the same buffers matches the oracle."""
    case = _random_batch(9, B=3)
    k, v, pk, pv, tier, slot = _dev(case)
    full, _ = _full_list(tier, slot, case.requests, case.lengths, case.prefixes, case.local_capacity)
    w = BatchPrefillWithPagedKVCacheWrapper(torch.empty(1 << 20, dtype=torch.uint8, device=DEV), "NHD")
    qo = torch.tensor(np.concatenate([[0], np.cumsum(case.qlens)]), dtype=torch.int32)
    kv = torch.tensor(np.concatenate([[0], np.cumsum(case.lengths)]), dtype=torch.int32)
    w.plan(qo, kv, full, torch.ones(3, dtype=torch.int32), 32, 8, 128, 1, causal=True, q_data_type=torch.bfloat16)
    peers = [t for pair in zip(pk, pv) for t in pair]
    q = case.q.to(DEV)
    out = torch.empty_like(q)
    lse = torch.empty((q.shape[0], 32), dtype=torch.float32, device=DEV)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        w.run(q, (k.unsqueeze(1), v.unsqueeze(1)), *peers, full, case.local_capacity, 128 ** -0.5, out=out, lse=lse,
              return_lse=True)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        w.run(q, (k.unsqueeze(1), v.unsqueeze(1)), *peers, full, case.local_capacity, 128 ** -0.5, out=out, lse=lse,
              return_lse=True)
    q2 = torch.randn(q.shape, generator=torch.Generator().manual_seed(99)).to(torch.bfloat16)
    q.copy_(q2)
    g.replay()
    torch.cuda.synchronize()
    ref, ref_lse = OA.tiered_attention(q2, case.k_local, case.v_local, case.peer_k, case.peer_v, case.tier,
                                       case.slot, case.requests, case.lengths, case.qlens, case.prefixes)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse.cpu(), ref_lse, atol=ATOL, rtol=RTOL)
    assert w.status() == 0


def test_stale_work_list_is_a_status_error_not_a_fault():
    """A work list planned for more requests than the launch has: the out-of-range items are
    rejected by the kernel's own check (DUAL_STATUS_BAD_LENGTH), the rest still compute."""
    d = torch.device(DEV)
    g = torch.Generator().manual_seed(3)
    lengths, qlens = [300, 200, 150, 100], [40, 30, 20, 10]
    total = sum(lengths)
    k = torch.randn((total + 1, 8, 128), generator=g).to(torch.bfloat16).to(d)
    v = torch.randn((total + 1, 8, 128), generator=g).to(torch.bfloat16).to(d)
    idx = (torch.randperm(total, generator=g) + 1).int().to(d)
    qo4 = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    kv4 = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    work = ops.append_plan(qo4, kv4, True).to(d)  # items for 4 requests
    qo2, kv2 = torch.from_numpy(qo4[:3].copy()).to(d), torch.from_numpy(kv4[:3].copy()).to(d)  # launch has 2
    q = torch.randn((int(qo4[2]), 32, 128), generator=g).to(torch.bfloat16).to(d)
    out = torch.zeros_like(q)
    lse = torch.zeros((q.shape[0], 32), dtype=torch.float32, device=d)
    status = torch.zeros(1, dtype=torch.int32, device=d)
    ops.tiered_append(q, k, v, total, [], [], qo2, kv2, idx, True, 128 ** -0.5, work, out, lse, status)
    torch.cuda.synchronize()
    assert int(status.item()) & 0x10  # DUAL_STATUS_BAD_LENGTH


def test_append_eight_supplier_banks():
    case = _random_batch(41, B=4, banks=8)
    k, v, pk, pv, tier, slot = _dev(case)
    full, _ = _full_list(tier, slot, case.requests, case.lengths, case.prefixes, case.local_capacity)
    out, lse, st = _append(case.q, k, v, pk, pv, case.qlens, case.lengths, full, case.local_capacity)
    assert st == 0
    ref, ref_lse = OA.tiered_attention(case.q, case.k_local, case.v_local, case.peer_k, case.peer_v, case.tier,
                                       case.slot, case.requests, case.lengths, case.qlens, case.prefixes)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse.cpu(), ref_lse, atol=ATOL, rtol=RTOL)


def test_append_rescales_when_the_max_keeps_growing():
    """History rows whose scores climb along the list: the running maximum moves past the lazy
    rescale threshold again and again, and the output in TMEM is rescaled in place each time."""
    g = torch.Generator().manual_seed(5)
    prefixes, qlens = [3000, 700], [40, 130]
    lengths = [p + q for p, q in zip(prefixes, qlens)]
    total = sum(lengths)
    # queries of kv head h all lean towards one direction u_h; the history's keys climb along u_h
    direction = torch.randn((8, 128), generator=g)
    direction = direction / direction.norm(dim=-1, keepdim=True)
    q = direction.repeat_interleave(4, 0)[None] + 0.5 * torch.randn((sum(qlens), 32, 128), generator=g) / 128 ** 0.5
    q = q / q.norm(dim=-1, keepdim=True)
    k = torch.randn((total + 1, 8, 128), generator=g) * 0.3
    v = torch.randn((total + 1, 8, 128), generator=g).to(torch.bfloat16)
    slots, off = [], 1
    for L in lengths:
        ramp = torch.linspace(0.0, 330.0, L)
        k[off:off + L] += ramp[:, None, None] * direction[None]
        slots.append(torch.arange(off, off + L, dtype=torch.int32))
        off += L
    q, k = q.to(torch.bfloat16), k.to(torch.bfloat16)
    tier = torch.zeros((2, max(lengths)), dtype=torch.int32)
    slot = torch.zeros_like(tier)
    for b, L in enumerate(lengths):
        slot[b, :L] = slots[b]
    d = torch.device(DEV)
    full, _ = _full_list(tier.to(d), slot.to(d), [0, 1], lengths, prefixes, total)
    out, lse, st = _append(q, k.to(d), v.to(d), [], [], qlens, lengths, full, total)
    assert st == 0
    ref, ref_lse = OA.tiered_attention(q, k, v, [], [], tier, slot, [0, 1], lengths, qlens, prefixes)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse.cpu(), ref_lse, atol=ATOL, rtol=RTOL)


def test_append_strided_views_and_other_scale():
    """q as a view of a fused qkv projection and out inside a wider buffer, scale 0.07."""
    case = _random_batch(43, B=3)
    k, v, pk, pv, tier, slot = _dev(case)
    full, _ = _full_list(tier, slot, case.requests, case.lengths, case.prefixes, case.local_capacity)
    d = torch.device(DEV)
    n = case.q.shape[0]
    qkv = torch.zeros((n, 6144), dtype=torch.bfloat16, device=d)
    qkv[:, :4096] = case.q.to(d).view(n, 4096)
    q = qkv[:, :4096].view(n, 32, 128)
    wide = torch.full((n, 40, 128), 3.0, dtype=torch.bfloat16, device=d)
    out = wide[:, 8:]
    qo = np.concatenate([[0], np.cumsum(case.qlens)]).astype(np.int32)
    kv = np.concatenate([[0], np.cumsum(case.lengths)]).astype(np.int32)
    work = ops.append_plan(qo, kv, True).to(d)
    lse = torch.empty((n, 32), dtype=torch.float32, device=d)
    status = torch.zeros(1, dtype=torch.int32, device=d)
    ops.tiered_append(q, k, v, case.local_capacity, pk, pv, torch.from_numpy(qo).to(d), torch.from_numpy(kv).to(d),
                      full, True, 0.07, work, out, lse, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref, ref_lse = OA.tiered_attention(case.q, case.k_local, case.v_local, case.peer_k, case.peer_v, case.tier,
                                       case.slot, case.requests, case.lengths, case.qlens, case.prefixes, sm_scale=0.07)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse.cpu(), ref_lse, atol=ATOL, rtol=RTOL)
    assert bool((wide[:, :8] == 3.0).all())
