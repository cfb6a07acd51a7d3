"""Per-layer staging of supplier rows (the reference's LayerStager, peer/staging.py) through the C ABI:
the row kernel copies exactly the rows the index list names and the copy-engine path exactly the
given row ranges, bit-exact, nothing else written; the append kernel over the stage buffers gives
bit-identical outputs to the append over the banks; the LayerStager in both modes over a
multi-layer RemoteBank matches per-layer in-place reads; a remote id beyond the banks is skipped
and reported."""
import pytest
import torch

from dual_b200 import ops
from dual_b200.remote_bank import RemoteBank
from dual_b200.staging import LayerStager
from test_append_gpu import _append, _dev, _full_list, _random_batch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
SENTINEL = 7.0


def _stage_buffers(pk):
    return ([torch.full_like(t, SENTINEL) for t in pk], [torch.full_like(t, SENTINEL) for t in pk])


def _remote_ids(full, capacity):
    f = full.cpu().long()
    return (f[f > capacity] - capacity - 1).unique()


@pytest.mark.parametrize("banks", [1, 3])
def test_stage_copies_exactly_the_named_rows(banks):
    case = _random_batch(21, banks=banks)
    k, v, pk, pv, tier, slot = _dev(case)
    full, _ = _full_list(tier, slot, case.requests, case.lengths, case.prefixes, case.local_capacity)
    sk, sv = _stage_buffers(pk)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.stage_remote_rows(pk, pv, sk, sv, full, case.local_capacity, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    g = _remote_ids(full, case.local_capacity)
    assert g.numel() > 0
    for b in range(banks):
        rows = g[g % banks == b] // banks
        named = torch.zeros(pk[b].shape[0], dtype=torch.bool)
        named[rows] = True
        for src, dst in ((pk[b], sk[b]), (pv[b], sv[b])):
            s, d = src.cpu(), dst.cpu()
            assert torch.equal(d[named].view(torch.int16), s[named].view(torch.int16))
            assert bool((d[~named] == SENTINEL).all())


def test_stage_honours_num_indices_and_ignores_local_entries():
    case = _random_batch(22, banks=2)
    k, v, pk, pv, tier, slot = _dev(case)
    full, _ = _full_list(tier, slot, case.requests, case.lengths, case.prefixes, case.local_capacity)
    n = full.numel() // 3
    sk, sv = _stage_buffers(pk)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.stage_remote_rows(pk, pv, sk, sv, full, case.local_capacity, status, num_indices=n, max_ctas=3)
    torch.cuda.synchronize()
    staged = sum(int((t.cpu() != SENTINEL).any(dim=(1, 2)).sum()) for t in sk)
    assert staged == _remote_ids(full[:n], case.local_capacity).numel()


@pytest.mark.parametrize("seed", [23, 24])
def test_append_over_stage_buffers_is_bit_identical(seed):
    case = _random_batch(seed, banks=3)
    k, v, pk, pv, tier, slot = _dev(case)
    full, _ = _full_list(tier, slot, case.requests, case.lengths, case.prefixes, case.local_capacity)
    out0, lse0, st0 = _append(case.q, k, v, pk, pv, case.qlens, case.lengths, full, case.local_capacity)
    sk, sv = _stage_buffers(pk)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.stage_remote_rows(pk, pv, sk, sv, full, case.local_capacity, status)
    out1, lse1, st1 = _append(case.q, k, v, sk, sv, case.qlens, case.lengths, full, case.local_capacity)
    assert st0 == 0 and st1 == 0 and int(status.item()) == 0
    assert torch.equal(out0, out1)
    assert torch.equal(lse0, lse1)


@pytest.mark.parametrize("banks", [1, 3])
def test_stage_bank_range_copies_exactly_the_range(banks):
    d = torch.device(DEV)
    pk = [torch.randn((50, 8, 128), device=d).to(torch.bfloat16) for _ in range(banks)]
    pv = [torch.randn((50, 8, 128), device=d).to(torch.bfloat16) for _ in range(banks)]
    sk, sv = _stage_buffers(pk)
    ranges = [(3, 17), (0, 0), (49, 50)][:banks]
    streams = [torch.cuda.Stream(d) for _ in range(banks)]
    ops.stage_bank_range(pk, pv, sk, sv, ranges, streams)
    torch.cuda.synchronize()
    for b, (lo, hi) in enumerate(ranges):
        inside = torch.zeros(50, dtype=torch.bool)
        inside[lo:hi] = True
        for src, dst in ((pk[b], sk[b]), (pv[b], sv[b])):
            s_, d_ = src.cpu(), dst.cpu()
            assert torch.equal(d_[inside].view(torch.int16), s_[inside].view(torch.int16))
            assert bool((d_[~inside] == SENTINEL).all())
    with pytest.raises(Exception):
        ops.stage_bank_range(pk, pv, sk, sv, [(0, 51)] * banks, streams)


@pytest.mark.parametrize("mode", ["range", "rows"])
def test_layer_stager_pipeline_matches_in_place_reads(mode):
    """Three layers with different supplier data: copy-engine ranges on per-bank streams (depth 2)
    or the row kernel on the caller's stream."""
    layers = 3
    case = _random_batch(25, banks=2)
    k, v, pk, pv, tier, slot = _dev(case)
    full, _ = _full_list(tier, slot, case.requests, case.lengths, case.prefixes, case.local_capacity)
    g = torch.Generator(device=DEV).manual_seed(5)
    banks = [torch.empty((layers, 2) + tuple(t.shape), dtype=torch.bfloat16, device=DEV).normal_(generator=g)
             for t in pk]
    bank = RemoteBank(banks, layers=layers)
    stager = LayerStager.from_bank(bank, DEV, depth=2, mode=mode, max_ctas=8)
    assert stager.bytes == (2 if mode == "range" else 1) * 2 * sum(t.numel() * 2 for t in pk)
    outs = []
    # the range mode copies the rows the list names: here the whole span each bank uses
    g = _remote_ids(full, case.local_capacity)
    ranges = [(int((g[g % 2 == b] // 2).min()), int((g[g % 2 == b] // 2).max()) + 1) for b in range(2)]
    stager.start(full, case.local_capacity, row_ranges=ranges)
    for i in range(layers):
        tail = stager.tail(i)
        outs.append(_append(case.q, k, v, tail[0::2], tail[1::2], case.qlens, case.lengths, full,
                            case.local_capacity))
        stager.next(i)
    torch.cuda.synchronize()
    assert stager.status() == 0
    for i in range(layers):
        ks, vs = bank.layer_kv(i)
        ref = _append(case.q, k, v, ks, vs, case.qlens, case.lengths, full, case.local_capacity)
        assert outs[i][2] == 0 and ref[2] == 0
        assert torch.equal(outs[i][0], ref[0]), i
        assert torch.equal(outs[i][1], ref[1]), i
    with pytest.raises(RuntimeError):
        LayerStager.from_bank(bank, DEV).wait(0)


def test_remote_id_beyond_banks_is_skipped_and_reported():
    d = torch.device(DEV)
    pk = [torch.randn((16, 8, 128), device=d).to(torch.bfloat16) for _ in range(2)]
    pv = [torch.randn((16, 8, 128), device=d).to(torch.bfloat16) for _ in range(2)]
    C = 100
    # remote ids 3 (bank 1, row 1) and 40 (bank 0, row 20 >= 16: beyond the bank), one local entry
    idx = torch.tensor([5, C + 1 + 3, C + 1 + 40], dtype=torch.int32, device=d)
    sk, sv = _stage_buffers(pk)
    status = torch.zeros(1, dtype=torch.int32, device=d)
    ops.stage_remote_rows(pk, pv, sk, sv, idx, C, status)
    torch.cuda.synchronize()
    assert int(status.item()) & 0x2
    assert torch.equal(sk[1][1].cpu().view(torch.int16), pk[1][1].cpu().view(torch.int16))
    assert bool((sk[0].cpu() == SENTINEL).all()) and bool((sv[0].cpu() == SENTINEL).all())
    changed = (sk[1].cpu() != SENTINEL).any(dim=(1, 2))
    assert changed.nonzero().flatten().tolist() == [1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_stage_from_peer_gpu_banks():
    from dual_b200 import topology
    n = torch.cuda.device_count()
    for dd in range(1, n):
        topology.enable_peer(0, dd)
    case = _random_batch(26, banks=3)
    k, v, pk, pv, tier, slot = _dev(case)
    owners = [torch.device(f"cuda:{1 + i % (n - 1)}") for i in range(3)]
    rk = [t.to(o) for t, o in zip(pk, owners)]
    rv = [t.to(o) for t, o in zip(pv, owners)]
    full, _ = _full_list(tier, slot, case.requests, case.lengths, case.prefixes, case.local_capacity)
    sk, sv = _stage_buffers(pk)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.stage_remote_rows(rk, rv, sk, sv, full, case.local_capacity, status)
    out1, lse1, st1 = _append(case.q, k, v, sk, sv, case.qlens, case.lengths, full, case.local_capacity)
    out0, lse0, st0 = _append(case.q, k, v, rk, rv, case.qlens, case.lengths, full, case.local_capacity)
    assert st0 == 0 and st1 == 0 and int(status.item()) == 0
    assert torch.equal(out0, out1) and torch.equal(lse0, lse1)
    # copy engines from the peers, whole banks, one stream per bank
    rk2, rv2 = _stage_buffers(pk)
    streams = [torch.cuda.Stream(torch.device(DEV)) for _ in range(3)]
    ops.stage_bank_range(rk, rv, rk2, rv2, [(0, t.shape[0]) for t in rk], streams)
    torch.cuda.synchronize()
    for a_, b_ in zip(rk + rv, rk2 + rv2):
        assert torch.equal(a_.cpu().view(torch.int16), b_.cpu().view(torch.int16))
