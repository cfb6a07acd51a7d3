"""The KV writer in front of tiered attention (SGLang's set_kv_buffer as the reference calls it,
V/nvlink_prefill_timing/backend.py:34,42) through the C ABI: bit-exact against torch's index_put for
int64 and int32 locations, with k / v as strided views into a fused qkv buffer; a slot outside the
pool is skipped and reported while the other rows are written."""
import pytest
import torch

from dual_b200 import ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _pools(C, g):
    return (torch.empty((C + 1, 8, 128), dtype=torch.bfloat16, device=DEV).normal_(generator=g),
            torch.empty((C + 1, 8, 128), dtype=torch.bfloat16, device=DEV).normal_(generator=g))


@pytest.mark.parametrize("loc_dtype", [torch.int64, torch.int32])
@pytest.mark.parametrize("n", [1, 37, 4096])
def test_set_kv_buffer_matches_index_put(loc_dtype, n):
    g = torch.Generator(device=DEV).manual_seed(n)
    C = 8192
    kp, vp = _pools(C, g)
    qkv = torch.empty((n, 6144), dtype=torch.bfloat16, device=DEV).normal_(generator=g)  # q | k | v of n tokens
    k = qkv[:, 4096:5120].view(n, 8, 128)
    v = qkv[:, 5120:].view(n, 8, 128)
    loc = torch.randperm(C + 1, generator=g, device=DEV)[:n].to(loc_dtype)  # may include the dummy slot 0
    ref_k, ref_v = kp.clone(), vp.clone()
    ref_k[loc.long()] = k
    ref_v[loc.long()] = v
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.set_kv_buffer(kp, vp, loc, k, v, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(kp.view(torch.int16), ref_k.view(torch.int16))
    assert torch.equal(vp.view(torch.int16), ref_v.view(torch.int16))


def test_set_kv_buffer_skips_and_reports_a_bad_slot():
    g = torch.Generator(device=DEV).manual_seed(3)
    C = 100
    kp, vp = _pools(C, g)
    k = torch.empty((3, 8, 128), dtype=torch.bfloat16, device=DEV).normal_(generator=g)
    v = torch.empty((3, 8, 128), dtype=torch.bfloat16, device=DEV).normal_(generator=g)
    loc = torch.tensor([5, C + 1, 7], dtype=torch.int64, device=DEV)
    before_k = kp.clone()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.set_kv_buffer(kp, vp, loc, k, v, status)
    torch.cuda.synchronize()
    assert int(status.item()) & 0x1
    assert torch.equal(kp[5], k[0]) and torch.equal(kp[7], k[2]) and torch.equal(vp[7], v[2])
    untouched = torch.ones(C + 1, dtype=torch.bool)
    untouched[[5, 7]] = False
    assert torch.equal(kp[untouched].view(torch.int16), before_k[untouched].view(torch.int16))
