"""ctypes binding of the C-ABI library ``libdual_b200.so`` (declared in include/dual_b200.h).

There is no CPU fallback: if the library is missing or fails to load, every
entry point raises.  Errors returned by the C ABI become ``DualError`` with the
library's thread-local message (the reference raised ``RuntimeError('CUDA n: ...')``
from its ctypes helper, V/nvlink_cooperation/cuda_ipc.py:48-50, and asserted
elsewhere).
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

_LIB = None
_LOCK = threading.Lock()

I32P = C.POINTER(C.c_int32)
I64P = C.POINTER(C.c_int64)
U32P = C.POINTER(C.c_uint32)
VP = C.c_void_p

# name -> (restype, argtypes): must mirror include/dual_b200.h exactly.
SIGNATURES = {
    "dual_last_error": (C.c_char_p, []),
    "dual_abi_version": (C.c_int, []),
    "dual_decode_workspace_size": (C.c_size_t, [C.c_int, C.c_int]),
    "dual_decode_default_ctas": (C.c_int, [C.c_int]),
    "dual_decode_workspace_reset": (C.c_int, [VP, C.c_size_t, C.c_int, C.c_int, VP]),
    "dual_tiered_decode": (C.c_int, [
        VP, C.c_int64, C.c_int64,              # q, strides
        VP, VP, C.c_int64, C.c_int64,          # k_local, v_local, local stride, capacity
        C.POINTER(VP), C.POINTER(VP), C.c_int,  # peer_k, peer_v, num_peers
        C.c_int64, C.c_int64,                  # peer stride, peer slots
        VP, VP, C.c_int64, C.c_int,            # indptr, indices, num_indices, batch
        C.c_double,                            # sm_scale
        VP, C.c_int64, C.c_int64, VP,          # out, strides, lse
        VP, C.c_size_t, C.c_int,               # workspace, bytes, num_ctas
        C.c_int, VP]),                         # device, stream
    "dual_tiered_decode_noalloc": (C.c_int, [
        VP, C.c_int64, C.c_int64,              # q, strides
        VP, VP, C.c_int64, C.c_int64,          # k_local, v_local, local stride, capacity
        C.POINTER(VP), C.POINTER(VP), C.c_int,  # peer_k, peer_v, num_peers
        C.c_int64, C.c_int64,                  # peer stride, peer slots
        VP, VP, C.c_int64, C.c_int,            # indptr, indices, num_indices, batch
        C.c_double,                            # sm_scale
        VP, C.c_int64, C.c_int64, VP,          # out, strides, lse
        VP, C.c_int,                           # status (nullable), num_ctas
        C.c_int, VP]),                         # device, stream
    "dual_decode_noalloc_status": (C.c_int, [U32P, C.c_int, VP]),
    "dual_append_plan": (C.c_int, [VP, VP, VP, C.c_int, C.c_int, VP, C.c_int64, C.POINTER(C.c_int64)]),
    "dual_tiered_append": (C.c_int, [
        VP, C.c_int64, C.c_int64,              # q, strides
        VP, VP, C.c_int64, C.c_int64,          # k_local, v_local, local stride, capacity
        C.POINTER(VP), C.POINTER(VP), C.c_int,  # peer_k, peer_v, num_peers
        C.c_int64, C.c_int64,                  # peer stride, peer slots
        VP, VP, VP, C.c_int64, C.c_int, C.c_int,  # qo_indptr, kv_indptr, indices, num_indices, batch, causal
        C.c_double, VP, C.c_int64,             # sm_scale, work, num_work
        VP, C.c_int64, C.c_int64, VP,          # out, strides, lse
        VP, C.c_int, VP]),                     # status, device, stream
    "dual_pack_read_order": (C.c_int, [
        VP, VP, C.c_int64, C.c_int64, VP, VP, VP, VP, C.c_int, C.c_int64, C.c_int, C.c_int, VP, VP, VP, C.c_int, VP]),
    "dual_write_prefill_layout": (C.c_int, [
        VP, VP, C.c_int64, C.c_int64, VP, VP, VP, VP, VP, C.c_int, C.c_int, C.c_int, VP, C.c_int, VP]),
    "dual_set_kv_buffer": (C.c_int, [
        VP, VP, C.c_int64, C.c_int64, VP, C.c_int64, VP, C.c_int64, VP, C.c_int, C.c_int64, VP, C.c_int, VP]),
    "dual_migrate_copy": (C.c_int, [
        VP, VP, C.c_int, C.c_int, VP, VP, C.c_int64, C.c_int, C.c_int64, C.c_int64, C.c_int64, VP, C.c_int,
        C.c_int, VP]),
    "dual_stage_remote_rows": (C.c_int, [
        VP, VP, VP, VP, C.c_int, C.c_int64, C.c_int64, C.c_int64, C.c_int64,  # banks, stages, n, strides, slots, row
        VP, C.c_int64, C.c_int64, VP, C.c_int, C.c_int, VP]),  # indices, n, C, status, max_ctas, device, stream
    "dual_stage_bank_range": (C.c_int, [
        VP, VP, VP, VP, C.c_int, C.c_int64, C.c_int64, C.c_int64, C.c_int64,  # banks, stages, n, strides, slots, row
        VP, VP, VP, C.c_int]),  # row_begin, row_end, streams, device
    "dual_debug_inject": (C.c_int, [C.c_uint32]),
    "dual_status_clear": (C.c_int, [VP, C.c_int, VP]),
    "dual_status_read": (C.c_int, [VP, U32P, C.c_int, VP]),
    "dual_supplier_alloc": (C.c_int, [C.c_int, C.c_size_t, C.POINTER(VP), C.POINTER(C.c_ubyte)]),
    "dual_supplier_free": (C.c_int, [C.c_int, VP]),
    "dual_ipc_open": (C.c_int, [C.c_int, C.POINTER(C.c_ubyte), C.POINTER(VP)]),
    "dual_ipc_close": (C.c_int, [C.c_int, VP]),
    "dual_enable_peer": (C.c_int, [C.c_int, C.c_int]),
    "dual_can_access_peer": (C.c_int, [C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "dual_p2p_attribute": (C.c_int, [C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "dual_pointer_info": (C.c_int, [VP, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "dual_device_count": (C.c_int, [C.POINTER(C.c_int)]),
}

STATUS_BITS = {
    0x1: "bad local slot",
    0x2: "bad remote slot",
    0x4: "wait timeout",
    0x8: "bad copy slot",
    0x10: "bad length",
    0x20: "bad tier value",
}


class DualError(RuntimeError):
    """A C-ABI call returned a nonzero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"dual_b200 error {code}: {message}")
        self.code = code


def library_path() -> Path:
    """The in-tree build, or the file named by DUAL_B200_LIBRARY (an alternative build of the same ABI)."""
    override = os.environ.get("DUAL_B200_LIBRARY")
    if override:
        return Path(override)
    return Path(__file__).resolve().parent / "lib" / "libdual_b200.so"


def load():
    """Load (once) and return the ctypes handle; raises if the library is absent."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        path = library_path()
        if not path.exists():
            raise RuntimeError(
                f"dual_b200 CUDA library not built ({path} missing); run `python -m dual_b200.build` "
                "or __graft_entry__.build() -- there is no CPU fallback")
        lib = C.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
        return lib


def check(rc: int) -> None:
    if rc != 0:
        msg = load().dual_last_error()
        raise DualError(rc, msg.decode() if msg else "")


def describe_status(value: int) -> str:
    return ", ".join(v for k, v in STATUS_BITS.items() if value & k) or "ok"
