"""Migration state machine (dual_b200.migration.TierManager): budget arithmetic, FIFO victims,
submit/poll/commit, release + ratio repair, page-table audit.  CPU tests drive it with the
oracle copy on host arrays; the GPU test uses the CUDA copy kernel on the async side stream."""
import numpy as np
import pytest
import torch

from dual_b200.migration import LocalAllocator, TierManager, limit_pages
from oracle import copy as OC
from oracle import policy as OP


class HostPools:
    """Local pool planes and supplier banks as uint16 arrays; the oracle copy moves bits."""

    def __init__(self, planes, local_slots, banks, bank_slots, seed=0):
        rng = np.random.default_rng(seed)
        self.local = [rng.integers(0, 2 ** 16, (local_slots + 1, 64), dtype=np.uint16) for _ in range(planes)]
        self.banks = [[np.zeros((bank_slots, 64), np.uint16) for _ in range(planes)] for _ in range(banks)]

    def copier(self, source, target, reverse):
        OC.migrate_copy(self.local, self.banks, source.tolist(), target.tolist(), reverse)

    def row(self, tier, slot, plane):
        if tier == 1:
            n = len(self.banks)
            return self.banks[slot % n][plane][slot // n]
        return self.local[plane][slot]


def _manager(local_cap=200, banks=3, bank_slots=20, a=1797, b=10000, tokens=16, rows=8, ctx=256, cap=None):
    pools = HostPools(4, local_cap, banks, bank_slots)
    tier = torch.full((rows, ctx), -1, dtype=torch.int32)
    slot = torch.zeros_like(tier)
    rtt = torch.zeros_like(tier)
    m = TierManager(tier, slot, local_cap, banks * bank_slots, a, b, pools.copier, migration_tokens=tokens,
                    req_to_token=rtt, remote_cap=cap)
    return m, pools


def _snapshot(m, pools):
    """Logical content of every live position (bits of plane 0 and 3), wherever it lives."""
    out = {}
    for rid, n in m.live.items():
        for p in range(n):
            t, s = int(m.tier[rid, p]), int(m.slot[rid, p])
            out[(rid, p)] = (pools.row(t, s, 0).copy(), pools.row(t, s, 3).copy())
    return out


def test_limit_matches_oracle_exhaustively():
    for local in range(0, 400, 7):
        for remote in range(0, 80, 3):
            for a, b in ((599, 10000), (1797, 10000)):
                assert limit_pages(local, remote, a, b) == OP.limit_pages(local, remote, a, b)


def test_allocator_free_list():
    al = LocalAllocator(5)
    assert al.alloc(3) == [1, 2, 3] and al.available_size() == 2
    assert al.alloc(3) is None
    al.free([2])
    assert al.available_size() == 3


def test_fifo_migration_preserves_every_position_and_invariants():
    m, pools = _manager()
    for rid in range(4):
        m.begin_forward()
        m.append(rid, 40)
    before = _snapshot(m, pools)
    m.begin_forward()
    rec = m.submit(needed=0, asynchronous=True)
    assert rec is not None and m.poll() == "ready"  # host copies complete synchronously
    assert m.audit()["remote_active_tokens"] == 0  # not switched before commit (pinned + reserved)
    m.commit()
    assert m.poll() == "idle"
    info = m.audit()
    assert info["remote_active_tokens"] == 16 and info["local_active_tokens"] == 160 - 16
    # FIFO victims: the oldest 16 positions (request 0, positions 0..15) became remote
    assert (m.tier[0, :16] == 1).all() and (m.tier[0, 16:40] == 0).all()
    assert (m.req_to_token[0, :16] == 0).all()
    after = _snapshot(m, pools)
    assert after.keys() == before.keys()
    for k, v in before.items():
        assert np.array_equal(after[k][0], v[0]) and np.array_equal(after[k][1], v[1]), k


def test_remote_row_ranges_cover_every_committed_remote_position():
    m, pools = _manager()
    assert m.remote_row_ranges(3) == [(0, 0)] * 3
    for rid in range(4):
        m.begin_forward()
        m.append(rid, 40)
    m.begin_forward()
    m.submit(needed=0, asynchronous=True)
    assert m.remote_row_ranges(3) == [(0, 0)] * 3  # nothing committed yet
    m.commit()
    ranges = m.remote_row_ranges(3)
    for (rid, pos), g in m.remote_positions.items():
        lo, hi = ranges[g % 3]
        assert lo <= g // 3 < hi
        assert int(m.tier[rid, pos]) == 1 and int(m.slot[rid, pos]) == g
    assert sum(hi - lo for lo, hi in ranges) >= len(m.remote_positions)
    with pytest.raises(ValueError):
        m.remote_row_ranges(0)


def test_remote_row_ranges_follow_releases():
    """After the requests that own every remote row are released, no bank has a range left to stage."""
    m, pools = _manager()
    for rid in range(4):
        m.begin_forward()
        m.append(rid, 40)
    m.begin_forward()
    m.submit(needed=0, asynchronous=True)
    m.commit()
    owners = {rid for rid, _ in m.remote_positions}
    assert owners and any(hi > lo for lo, hi in m.remote_row_ranges(3))
    m.release(sorted(owners))
    assert not m.remote_positions
    assert m.remote_row_ranges(3) == [(0, 0)] * 3
    m.audit()


def test_strict_bound_is_never_crossed():
    m, pools = _manager(local_cap=400, tokens=2048, ctx=400)
    m.begin_forward()
    m.append(0, 300)
    m.begin_forward()
    m.submit(asynchronous=False)
    m.commit()
    local, remote, _ = m.budget()
    assert 10000 * remote < 1797 * local
    assert limit_pages(local, remote, 1797, 10000) == 0 or remote == 60  # capacity-capped at 3*20 slots
    m.audit()


def test_headroom_and_prefetch_cycle_with_audit_every_step():
    m, pools = _manager(local_cap=120, bank_slots=30, tokens=8, rows=6, ctx=200)
    m.begin_forward()
    for rid in range(4):
        m.append(rid, 25)
    ref = _snapshot(m, pools)
    for step in range(8):  # 100 + 4*8 tokens: needs remote slots, stays inside L + R with R/L < 17.97%
        m.ensure_headroom(4)
        m.begin_forward()
        for rid in range(4):
            m.append(rid, 1)
        new = _snapshot(m, pools)
        for k, v in ref.items():  # old positions keep their bytes across migrations
            assert np.array_equal(new[k][0], v[0]) and np.array_equal(new[k][1], v[1])
        ref = new
        m.prefetch_next(4)
        m.audit()
    assert m.migrations, "local pressure must have triggered migrations"


def test_release_and_ratio_repair_restore_bytes():
    m, pools = _manager(local_cap=300, tokens=40)
    m.begin_forward()
    m.append(0, 150)
    m.append(1, 120)
    m.begin_forward()
    m.submit(asynchronous=False)
    m.commit()
    assert m.committed_remote == 40
    snap = _snapshot(m, pools)
    m.release([1])  # local shrinks to 110: 40 remote now breaks 10000*R < 1797*L
    local, remote, _ = m.budget()
    assert 10000 * remote < 1797 * local and m.restorations
    after = _snapshot(m, pools)
    for k, v in after.items():
        assert np.array_equal(v[0], snap[k][0]) and np.array_equal(v[1], snap[k][1])
    m.audit()
    r = m.restorations[0]
    assert r["tokens"] == OP.repair_count(r["local_before"], r["remote_before"], 1797, 10000)


@pytest.mark.parametrize("local,remote,pending", [(0, 0, 0), (240, 0, 0), (240, 10, 0), (240, 10, 5), (255, 0, 14)])
def test_bookkeeping_states_like_reference(local, remote, pending):
    """The reference's CPU bookkeeping regression states (check_bookkeeping.py:15): empty, native,
    committed-peer and in-flight-peer reservations."""
    m, pools = _manager(local_cap=256 + 64, banks=1, bank_slots=64, tokens=max(pending, 1), a=1797, b=1000,
                        rows=2, ctx=400)
    m.begin_forward()
    if local + remote:
        m.append(1, local + remote)
    if remote:
        m.migration_tokens = remote
        m.begin_forward()
        m.submit(asynchronous=False)
        m.commit()
    if pending:
        m.migration_tokens = pending
        m.begin_forward()
        m.submit(asynchronous=False)
    info = m.audit()
    assert (info["local_active_tokens"], info["remote_active_tokens"]) == (local, remote)


def test_victims_must_predate_current_forward():
    m, pools = _manager(tokens=50)
    m.begin_forward()
    m.append(0, 30)
    with pytest.raises(RuntimeError, match="predate"):
        m.submit()  # the 30 tokens were written by the current forward
    m.begin_forward()
    m.submit()
    m.commit()
    m.audit()


@pytest.mark.gpu
def test_cuda_migration_async_bit_exact_and_decode_unchanged():
    from dual_b200 import ops
    from dual_b200.migration import CudaCopier
    from dual_b200.remote_bank import RemoteBank, local_plane_pointers
    dev = torch.device("cuda:0")
    layers, local_cap, bank_slots, banks = 4, 4096, 1024, 3
    g = torch.Generator(device=dev).manual_seed(1)
    kv = [(torch.randn((local_cap + 1, 8, 128), generator=g, device=dev).to(torch.bfloat16),
           torch.randn((local_cap + 1, 8, 128), generator=g, device=dev).to(torch.bfloat16)) for _ in range(layers)]
    bank = RemoteBank([torch.zeros((layers, 2, bank_slots, 8, 128), dtype=torch.bfloat16, device=dev)
                       for _ in range(banks)], layers=layers)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    copier = CudaCopier(local_plane_pointers(kv, dev), bank.pointers, 2 * layers, banks, local_cap + 1, bank_slots,
                        status)
    tier = torch.full((4, 3000), -1, dtype=torch.int32, device=dev)
    slot = torch.zeros_like(tier)
    m = TierManager(tier, slot, local_cap, banks * bank_slots, 1797, 10000, copier, migration_tokens=512)
    m.begin_forward()
    lengths = [1000, 700, 1500, 300]
    for rid, n in enumerate(lengths):
        m.append(rid, n)
    q = torch.randn((4, 32, 128), generator=g, device=dev).to(torch.bfloat16)

    def run_decode(layer):
        req = torch.arange(4, dtype=torch.int32, device=dev)
        seq = torch.tensor(lengths, dtype=torch.int32, device=dev)
        idx = torch.empty(sum(lengths), dtype=torch.int32, device=dev)
        ops.pack_read_order(tier, slot, req, seq, local_cap, 5, 32, idx)
        indptr = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=dev)
        out = torch.empty_like(q)
        ws = torch.zeros(ops.decode_workspace_size(4, ops.default_ctas(0)), dtype=torch.uint8, device=dev)
        pk, pv = bank.layer_kv(layer)
        ops.tiered_decode(q, kv[layer][0], kv[layer][1], local_cap, pk, pv, indptr, idx, 128 ** -0.5, out, None, ws)
        return out

    before = [run_decode(i) for i in range(layers)]
    m.begin_forward()
    p = m.submit(asynchronous=True)
    assert p is not None
    assert m.wait(10.0)
    src, tgt = p.source.clone(), p.target.clone()
    m.commit()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    for layer in range(layers):
        for plane in range(2):
            got = bank.gather(layer, plane, tgt)
            want = kv[layer][plane].index_select(0, src)
            assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    info = m.audit()
    assert info["remote_active_tokens"] == 512
    for layer in range(layers):
        after = run_decode(layer)
        torch.testing.assert_close(after.float(), before[layer].float(), atol=2e-3, rtol=1e-2)


def _skewed_run(cap):
    """One old long request and four newer short ones under local pressure (the reference's FIFO
    pushed its oldest requests to ~95 % remote); migrate until the global budget is used."""
    m, pools = _manager(local_cap=400, banks=3, bank_slots=40, a=1797, b=10000, tokens=8, rows=6, ctx=400, cap=cap)
    m.begin_forward()
    m.append(0, 160)
    m.begin_forward()
    for rid in range(1, 5):
        m.append(rid, 40)
    before = _snapshot(m, pools)
    for _ in range(12):
        m.begin_forward()
        if m.submit(asynchronous=True) is None:
            break
        assert m.poll() == "ready"
        m.commit()
        m.audit()
    after = _snapshot(m, pools)
    for k, v in before.items():
        assert np.array_equal(after[k][0], v[0]) and np.array_equal(after[k][1], v[1]), k
    return m


def test_fifo_victims_concentrate_remote_share_on_the_oldest_request():
    m = _skewed_run(None)
    info = m.audit()
    assert info["remote_active_tokens"] > 0
    shares = {r["request"]: r["remote"] / r["context"] for r in info["per_request"]}
    assert shares[0] == info["max_request_remote_share"] and all(shares[r] == 0 for r in range(1, 5))


def test_remote_cap_spreads_remote_share_and_keeps_every_invariant():
    fifo = _skewed_run(None).audit()
    m = _skewed_run(0.15)
    info = m.audit()
    assert info["max_request_remote_share"] <= 0.15 + 1e-9
    assert info["remote_active_tokens"] > 0
    assert sum(r["remote"] > 0 for r in info["per_request"]) > 1  # more than the oldest request holds remote KV
    assert info["max_request_remote_share"] < fifo["max_request_remote_share"]
    local, remote, _ = m.budget()
    assert 10000 * remote < 1797 * local


def test_remote_cap_is_soft_when_local_slots_must_be_freed():
    m, pools = _manager(local_cap=100, banks=3, bank_slots=40, tokens=16, rows=4, ctx=200, cap=0.05)
    m.begin_forward()
    m.append(0, 100)  # local pool full; the cap allows 5 remote positions of request 0
    before = _snapshot(m, pools)
    m.begin_forward()
    m.ensure_headroom(8)  # must free 8 slots: the cap yields to the headroom requirement
    assert m.allocator.available_size() >= 8
    info = m.audit()
    assert info["remote_active_tokens"] >= 8
    after = _snapshot(m, pools)
    for k, v in before.items():
        assert np.array_equal(after[k][0], v[0]) and np.array_equal(after[k][1], v[1]), k


def test_remote_cap_rejects_out_of_range_values():
    with pytest.raises(ValueError):
        _manager(cap=0.0)
    with pytest.raises(ValueError):
        _manager(cap=1.5)


class FakeSGLangAllocator:
    """SGLang's token_to_kv_pool_allocator interface: a free-page tensor, alloc slices, free concatenates."""

    def __init__(self, size):
        self.free_pages = torch.arange(1, size + 1, dtype=torch.int64)

    def available_size(self):
        return len(self.free_pages)

    def alloc(self, need_size):
        if need_size > len(self.free_pages):
            return None
        out, self.free_pages = self.free_pages[:need_size], self.free_pages[need_size:]
        return out

    def free(self, free_index):
        self.free_pages = torch.cat((self.free_pages, free_index.to(torch.int64)))


def test_tier_manager_drives_sglangs_allocator():
    from dual_b200.migration import SGLangAllocatorAdapter
    pools = HostPools(4, 200, 3, 20)
    tier = torch.full((8, 256), -1, dtype=torch.int32)
    slot = torch.zeros_like(tier)
    rtt = torch.zeros_like(tier)
    fake = FakeSGLangAllocator(200)
    m = TierManager(tier, slot, 200, 60, 1797, 10000, pools.copier, migration_tokens=16, req_to_token=rtt,
                    allocator=SGLangAllocatorAdapter(fake))
    for rid in range(4):
        m.begin_forward()
        m.append(rid, 40)
    assert fake.available_size() == 40
    before = _snapshot(m, pools)
    m.begin_forward()
    m.submit()
    m.commit()
    assert fake.available_size() == 56  # migrated-out local slots went back to SGLang's allocator
    info = m.audit()
    assert info["remote_active_tokens"] == 16
    after = _snapshot(m, pools)
    for k, v in before.items():
        assert np.array_equal(after[k][0], v[0]) and np.array_equal(after[k][1], v[1]), k
    m.release([0])
    assert fake.available_size() == 56 + 24  # request 0's remaining local slots
    m.audit()
    m.reset()
    assert m.allocator.inner is fake  # SGLang's allocator is not replaced
