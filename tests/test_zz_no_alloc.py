"""The allocation-free decode entry point ``dual_tiered_decode_noalloc``.

Some callers cannot give this library device memory: a serving process whose
memory manager already owns nearly all of HBM and forbids out-of-band
cudaMalloc (which would also stall the device mid-decode), or a foreign-language
binding that only holds the attention tensors.  For them the decode keeps its
split-KV partial states in a fixed device array inside the library.  These tests
call that entry point through the C ABI and check its output against the
workspace-based ``dual_tiered_decode`` on two calls in a row (different shapes,
so the shared array holds the first call's data when the second one runs), plus
its size limit.  This file is named to be collected last.
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


def _noalloc(q, k, v, pk, pv, indptr, idx, capacity, status=None, num_ctas=0, batch=None):
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
        indptr.data_ptr(), idx.data_ptr(), idx.numel(), B, 128 ** -0.5,
        out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(),
        None if status is None else status.data_ptr(), num_ctas, 0, torch.cuda.current_stream().cuda_stream)
    return rc, out, lse


def _with_workspace(q, k, v, pk, pv, indptr, idx, capacity):
    out = torch.empty((q.shape[0], 32, 128), dtype=torch.bfloat16, device=DEV)
    lse = torch.empty((q.shape[0], 32), dtype=torch.float32, device=DEV)
    ws = torch.zeros(ops.decode_workspace_size(q.shape[0], ops.default_ctas(0)), dtype=torch.uint8, device=DEV)
    ops.tiered_decode(q, k, v, capacity, pk, pv, indptr, idx, 128 ** -0.5, out, lse, ws)
    return out, lse


def test_noalloc_matches_workspace_entry_two_calls_in_a_row():
    first = cases.config1(banks=3)
    second = cases.validate_case(3, banks=1)  # long_prefix: different batch, lengths and supplier count
    for case in (first, second):
        args = _inputs(case)
        rc, out, lse = _noalloc(*args, case.local_capacity)
        assert rc == 0, _lib.load().dual_last_error()
        ref_out, ref_lse = _with_workspace(*args, case.local_capacity)
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref_out.float(), atol=ATOL, rtol=RTOL, msg=case.name)
        torch.testing.assert_close(lse, ref_lse, atol=ATOL, rtol=RTOL, msg=case.name)


def test_noalloc_caller_status_word_and_size_limit():
    case = cases.config1(banks=3)
    args = _inputs(case)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc, out, _ = _noalloc(*args, case.local_capacity, status=status)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref_out, _ = _with_workspace(*args, case.local_capacity)
    torch.testing.assert_close(out.float(), ref_out.float(), atol=ATOL, rtol=RTOL)
    # (num_ctas + batch) x 16896 B + 256 B must fit in the 8 MiB array: 148 CTAs + 400 requests do not.
    rc, _, _ = _noalloc(*args, case.local_capacity, batch=400)
    assert rc == 3
    assert b"num_ctas + batch" in _lib.load().dual_last_error()
