"""Host-side logic without a GPU: the append work list (coverage, grouping, order, costs), the
wrapper's reading of the reference's positional tail, the paged-KV forms it accepts, and the
plan-time rejection of what the kernels do not implement."""
import numpy as np
import pytest
import torch

from dual_b200 import ops
from dual_b200.wrapper import BatchPrefillWithPagedKVCacheWrapper, _unpack_paged_kv, split_tiered_args

PAIR, TILE = 64, 128


def _plan(qlens, kvlens, causal=True):
    qo = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    kv = np.concatenate([[0], np.cumsum(kvlens)]).astype(np.int32)
    return ops.append_plan(qo, kv, causal).numpy()


@pytest.mark.parametrize("causal", [True, False])
def test_append_plan_covers_every_item_once_grouped_longest_first(causal):
    rng = np.random.default_rng(5)
    qlens = rng.integers(0, 700, 12).tolist()
    kvlens = [q + int(rng.integers(0, 5000)) for q in qlens]
    w = _plan(qlens, kvlens, causal)
    items = [tuple(x) for x in w[:, :3]]
    expect = {(b, h, t) for b, q in enumerate(qlens) for h in range(8) for t in range((q + PAIR - 1) // PAIR)}
    assert len(items) == len(set(items)) and set(items) == expect
    # costs: kv tiles the item's query pair can see
    for b, h, t, cost in w:
        q, L = qlens[b], kvlens[b]
        end = min(L, L - q + min(q, (t + 1) * PAIR)) if causal else L
        assert cost == (end + TILE - 1) // TILE
    # each (request, kv head) group is contiguous, groups by descending total length, pairs descending
    groups = [(b, h) for b, h, _, _ in w]
    change = [i for i in range(1, len(groups)) if groups[i] != groups[i - 1]]
    starts = [0] + change
    seen = [groups[i] for i in starts]
    assert len(seen) == len(set(seen)), "a group is split"
    glen = [(kvlens[g[0]] + TILE - 1) // TILE for g in seen]
    assert glen == sorted(glen, reverse=True)
    for s, e in zip(starts, starts[1:] + [len(w)]):
        assert list(w[s:e, 2]) == sorted(w[s:e, 2], reverse=True)


def test_append_plan_rejects_short_causal_lists():
    with pytest.raises(Exception):
        _plan([10], [5], causal=True)
    assert _plan([0, 0], [3, 4]).shape[0] == 0


def test_split_tiered_args_reads_the_reference_tail():
    t = [torch.empty(1) for _ in range(8)]
    idx = torch.empty(3, dtype=torch.int32)
    for pairs in range(0, 4):
        pk, pv, i, cap, scale = split_tiered_args(t[:2 * pairs] + [idx, 99, 0.125])
        assert pk == t[0:2 * pairs:2] and pv == t[1:2 * pairs:2] and i is idx and cap == 99 and scale == 0.125
    with pytest.raises(ValueError):
        split_tiered_args([t[0], idx, 99, 0.125])  # odd number of peer tensors
    with pytest.raises(ValueError):
        split_tiered_args([idx, 99])


def test_paged_kv_forms():
    k, v = torch.empty(5, 1, 8, 128), torch.empty(5, 1, 8, 128)
    k1, v1 = _unpack_paged_kv((k, v))
    assert k1 is k and v1 is v
    both = torch.randn(5, 2, 1, 8, 128)
    k2, v2 = _unpack_paged_kv(both)
    assert k2.shape == (5, 1, 8, 128) and torch.equal(v2, both[:, 1])
    with pytest.raises(ValueError):
        _unpack_paged_kv(torch.empty(5, 8, 128))


def test_prefill_plan_on_the_host_and_its_refusals():
    w = BatchPrefillWithPagedKVCacheWrapper(torch.empty(16, dtype=torch.uint8), "NHD")
    qo = torch.tensor([0, 70, 71], dtype=torch.int32)
    kv = torch.tensor([0, 500, 600], dtype=torch.int32)
    idx = torch.arange(1, 601, dtype=torch.int32)
    last = torch.ones(2, dtype=torch.int32)
    w.plan(qo, kv, idx, last, 32, 8, 128, 1, causal=True)
    assert w._plan["total_q"] == 71 and w._plan["work"].shape[0] == 8 * (2 + 1)
    bad = [dict(num_qo_heads=16), dict(page_size=16), dict(window_left=128), dict(logits_soft_cap=30.0),
           dict(pos_encoding_mode="ROPE_LLAMA"), dict(custom_mask=torch.ones(4, dtype=torch.bool)),
           dict(head_dim_vo=64)]
    base = dict(num_qo_heads=32, num_kv_heads=8, head_dim_qk=128, page_size=1)
    for kw in bad:
        args = {**base, **kw}
        with pytest.raises(ValueError):
            w.plan(qo, kv, idx, last, args.pop("num_qo_heads"), args.pop("num_kv_heads"), args.pop("head_dim_qk"),
                   args.pop("page_size"), causal=True, **args)
    with pytest.raises(ValueError):
        BatchPrefillWithPagedKVCacheWrapper(torch.empty(16, dtype=torch.uint8), "HND")


def test_append_plan_spreads_mostly_remote_requests():
    """With per-request remote counts, the items of requests more than half remote are spread evenly
    over the first 90 % of the launch, longest first; every item still appears exactly once and the
    others keep the grouped, longest-first order."""
    rng = np.random.default_rng(9)
    qlens = rng.integers(64, 700, 16).tolist()
    kvlens = [q + int(rng.integers(1000, 8000)) for q in qlens]
    remote = [int(0.95 * (L - q)) if b % 8 == 0 else int(0.03 * (L - q)) for b, (q, L) in
              enumerate(zip(qlens, kvlens))]
    qo = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    kv = np.concatenate([[0], np.cumsum(kvlens)]).astype(np.int32)
    grouped = ops.append_plan(qo, kv, True).numpy()
    spread = ops.append_plan(qo, kv, True, remote).numpy()
    assert sorted(map(tuple, grouped)) == sorted(map(tuple, spread))
    heavy = np.isin(spread[:, 0], [0, 8])
    pos = np.nonzero(heavy)[0]
    n, k = len(spread), len(pos)
    assert k == int(np.isin(grouped[:, 0], [0, 8]).sum()) > 0
    gaps = np.diff(pos)
    assert pos[0] == 0 and pos[-1] < 0.9 * n + 2 and gaps.min() >= 1
    assert gaps.max() - gaps.min() <= 1  # even spacing
    assert list(spread[heavy][:, 3]) == sorted(spread[heavy][:, 3], reverse=True)
    light = [tuple(x) for x in spread[~heavy]]
    assert light == [tuple(x) for x in grouped if x[0] not in (0, 8)]
    with pytest.raises(Exception):
        ops.append_plan(qo, kv, True, [-1] * 16)
