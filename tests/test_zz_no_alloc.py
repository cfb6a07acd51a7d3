"""The allocation-free decode entry point ``dual_tiered_decode_noalloc``.

Some callers cannot give this library device memory: a serving process whose
memory manager already owns nearly all of HBM and forbids out-of-band
cudaMalloc (which would also stall the device mid-decode), or a foreign-language
binding that only holds the attention tensors.  For them the decode keeps its
split-KV partial states in a fixed device array inside the library.  These tests
call that entry point through the C ABI and check it on two calls in a row: the
first with the larger batch and CTA count, so the shared array still holds stale
partial states of more segments than the second call uses, against the golden
vectors made from the reference's own check and against the workspace-based
``dual_tiered_decode`` run on a NaN-filled workspace (any read of a segment the
call did not write would show).  They also check the size limit, the status
word of callers that pass none (read back with ``dual_decode_noalloc_status``)
and ``device = -1``.  This file is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import cases
from dual_b200 import _lib, ops

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ATOL, RTOL = 2e-3, 1e-2
BAD_LENGTH = 0x10


def _inputs(case):
    d = torch.device(DEV)
    k, v = case.k_local.to(d), case.v_local.to(d)
    pk, pv = [t.to(d) for t in case.peer_k], [t.to(d) for t in case.peer_v]
    req = torch.tensor(case.requests, dtype=torch.int32, device=d)
    seq = torch.tensor(case.lengths, dtype=torch.int32, device=d)
    idx = torch.empty(sum(case.lengths), dtype=torch.int32, device=d)
    ops.pack_read_order(case.tier.to(d), case.slot.to(d), req, seq, case.local_capacity, 5, 32, idx)
    indptr = torch.tensor(np.concatenate([[0], np.cumsum(case.lengths)]), dtype=torch.int32, device=d)
    return case.decode_q().to(d), k, v, pk, pv, indptr, idx


def _noalloc(q, k, v, pk, pv, indptr, idx, capacity, status=None, num_ctas=0, batch=None, device=0,
             num_indices=None):
    lib = _lib.load()
    B = q.shape[0] if batch is None else batch
    out = torch.empty((q.shape[0], 32, 128), dtype=torch.bfloat16, device=DEV)
    lse = torch.empty((q.shape[0], 32), dtype=torch.float32, device=DEV)
    n = len(pk)
    arr_k = (C.c_void_p * max(n, 1))(*[t.data_ptr() for t in pk])
    arr_v = (C.c_void_p * max(n, 1))(*[t.data_ptr() for t in pv])
    rc = lib.dual_tiered_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), v.data_ptr(), k.stride(0) * 2, capacity,
        arr_k, arr_v, n, (pk[0].stride(0) * 2) if n else 0, pk[0].shape[0] if n else 0,
        indptr.data_ptr(), idx.data_ptr(), idx.numel() if num_indices is None else num_indices, B, 128 ** -0.5,
        out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(),
        None if status is None else status.data_ptr(), num_ctas, device, torch.cuda.current_stream().cuda_stream)
    return rc, out, lse


def _noalloc_status():
    lib = _lib.load()
    v = C.c_uint32(0xFFFFFFFF)
    rc = lib.dual_decode_noalloc_status(C.byref(v), 0, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.dual_last_error()
    return int(v.value)


def _with_workspace(q, k, v, pk, pv, indptr, idx, capacity, num_ctas):
    """The workspace entry point on a workspace whose partial-state area is NaN."""
    out = torch.empty((q.shape[0], 32, 128), dtype=torch.bfloat16, device=DEV)
    lse = torch.empty((q.shape[0], 32), dtype=torch.float32, device=DEV)
    nbytes = ops.decode_workspace_size(q.shape[0], num_ctas)
    ws = torch.full((nbytes // 4,), float("nan"), dtype=torch.float32, device=DEV).view(torch.uint8)
    ops.decode_workspace_reset(ws, q.shape[0])  # status word and arrival counters start cleared
    ops.tiered_decode(q, k, v, capacity, pk, pv, indptr, idx, 128 ** -0.5, out, lse, ws, num_ctas)
    return out, lse, ws


def test_noalloc_two_calls_in_a_row_match_golden_and_workspace_entry(golden_dir):
    gold = np.load(golden_dir / "attention.npz")
    default = ops.default_ctas(0)
    # first call: 4 requests over twice the default CTA count; second: 1 request over the default
    runs = [(cases.config1(banks=3), 2 * default, "config1_banks3_b3_decode"),
            (cases.validate_case(3, banks=1), default, "long_prefix_b1_decode")]
    for case, num_ctas, key in runs:
        args = _inputs(case)
        rc, out, lse = _noalloc(*args, case.local_capacity, num_ctas=num_ctas)
        assert rc == 0, _lib.load().dual_last_error()
        ref_out, ref_lse, ws = _with_workspace(*args, case.local_capacity, num_ctas)
        torch.cuda.synchronize()
        assert _noalloc_status() == 0
        assert int(ws[:4].view(torch.int32).item()) == 0
        torch.testing.assert_close(out.float().cpu(), torch.from_numpy(gold[key]), atol=ATOL, rtol=RTOL, msg=key)
        torch.testing.assert_close(out.float(), ref_out.float(), atol=ATOL, rtol=RTOL, msg=case.name)
        torch.testing.assert_close(lse, ref_lse, atol=ATOL, rtol=RTOL, msg=case.name)
        assert torch.isfinite(out.float()).all() and torch.isfinite(lse).all()


def test_noalloc_caller_status_word_and_size_limit():
    case = cases.config1(banks=3)
    args = _inputs(case)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc, out, _ = _noalloc(*args, case.local_capacity, status=status)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref_out, _, _ = _with_workspace(*args, case.local_capacity, ops.default_ctas(0))
    torch.testing.assert_close(out.float(), ref_out.float(), atol=ATOL, rtol=RTOL)
    # (num_ctas + batch) x 16896 B + the header and counters must fit in the 8 MiB array: 148 CTAs +
    # 400 requests do not.
    rc, _, _ = _noalloc(*args, case.local_capacity, batch=400)
    assert rc == 3
    assert b"num_ctas + batch" in _lib.load().dual_last_error()


def test_noalloc_without_status_word_reports_through_read_back():
    """status == NULL: a call whose index list is shorter than indptr says (bad length, tail skipped,
    no out-of-range read) is reported by dual_decode_noalloc_status; the next such call starts from a
    cleared word."""
    case = cases.config1(banks=3)
    args = _inputs(case)
    short = args[-1].numel() - 100
    rc, _, _ = _noalloc(*args, case.local_capacity, num_indices=short)
    assert rc == 0
    torch.cuda.synchronize()
    assert _noalloc_status() & BAD_LENGTH
    rc, out, _ = _noalloc(*args, case.local_capacity)
    assert rc == 0
    torch.cuda.synchronize()
    assert _noalloc_status() == 0
    ref_out, _, _ = _with_workspace(*args, case.local_capacity, ops.default_ctas(0))
    torch.testing.assert_close(out.float(), ref_out.float(), atol=ATOL, rtol=RTOL)


def test_noalloc_negative_device_means_current_device():
    case = cases.validate_case(4, banks=1)  # empty_decode_splits: lengths 1 and 3
    args = _inputs(case)
    rc, out, lse = _noalloc(*args, case.local_capacity, device=-1)
    assert rc == 0, _lib.load().dual_last_error()
    ref_out, ref_lse, _ = _with_workspace(*args, case.local_capacity, ops.default_ctas(0))
    torch.testing.assert_close(out.float(), ref_out.float(), atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse, ref_lse, atol=ATOL, rtol=RTOL)
    assert torch.cuda.current_device() == 0
