"""The C-ABI library loads, exports every symbol include/dual_b200.h declares, and rejects bad
arguments with error codes + messages.  CPU only: no call here reaches a CUDA API."""
import ctypes as C
import re
from pathlib import Path

import pytest

from dual_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "dual_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(dual_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 19
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} missing from the ctypes signature table"
    assert set(_lib.SIGNATURES) == set(names)
    assert lib.dual_abi_version() == 200


def test_argument_errors_are_codes_not_crashes():
    lib = _lib.load()
    rc = lib.dual_tiered_decode(None, 0, 0, None, None, 0, 0, None, None, 0, 0, 0, None, None, 0, -1, 0.1,
                                None, 0, 0, None, None, 0, 0, -1, None)
    assert rc == 1 and b"batch" in lib.dual_last_error()
    rc = lib.dual_tiered_decode(None, 0, 0, None, None, 0, 0, None, None, 0, 0, 0, None, None, 0, 4, 0.1,
                                None, 0, 0, None, None, 0, 0, -1, None)
    assert rc == 1 and b"null" in lib.dual_last_error()
    rc = lib.dual_pack_read_order(1, 1, 4, 8, 1, 1, None, None, 2, 100, 32, 32, 1, None, None, -1, None)
    assert rc == 1 and b"remote_rows" in lib.dual_last_error()
    rc = lib.dual_migrate_copy(None, None, 72, 3, None, None, -5, 0, 2048, 10, 10, None, 0, -1, None)
    assert rc == 1
    rc = lib.dual_migrate_copy(1, 1, 72, 3, 1, 1, 4, 0, 2047, 10, 10, 1, 0, -1, None)
    assert rc == 1 and b"row_bytes" in lib.dual_last_error()
    with pytest.raises(_lib.DualError):
        _lib.check(lib.dual_write_prefill_layout(None, None, 1, 1, None, None, None, None, None, 1, 3, 5, None, -1, None))


def test_stage_arguments_are_checked_before_any_launch():
    lib = _lib.load()
    assert lib.dual_stage_remote_rows(None, None, None, None, 1, 2048, 2048, 4, 2048, None, 0, 10, None, 0, -1,
                                      None) == 0
    arr = (C.c_void_p * 1)(16)
    rc = lib.dual_stage_remote_rows(arr, arr, arr, arr, 0, 2048, 2048, 4, 2048, 16, 8, 10, 16, 0, -1, None)
    assert rc == 1 and b"num_banks" in lib.dual_last_error()
    rc = lib.dual_stage_remote_rows(arr, arr, arr, arr, 1, 2048, 2048, 4, 2047, 16, 8, 10, 16, 0, -1, None)
    assert rc == 1 and b"row_bytes" in lib.dual_last_error()
    rc = lib.dual_stage_remote_rows(arr, arr, arr, arr, 1, 1024, 2048, 4, 2048, 16, 8, 10, 16, 0, -1, None)
    assert rc == 1 and b"strides" in lib.dual_last_error()
    bad = (C.c_void_p * 1)(24)
    rc = lib.dual_stage_remote_rows(arr, arr, bad, arr, 1, 2048, 2048, 4, 2048, 16, 8, 10, 16, 0, -1, None)
    assert rc == 1 and b"aligned" in lib.dual_last_error()


def test_kv_writer_arguments_are_checked_before_any_launch():
    lib = _lib.load()
    assert lib.dual_set_kv_buffer(None, None, 2048, 10, None, 1024, None, 1024, None, 1, 0, None, -1, None) == 0
    rc = lib.dual_set_kv_buffer(16, 16, 2048, 10, 16, 1000, 16, 1024, 16, 1, 4, 16, -1, None)
    assert rc == 1 and b"token strides" in lib.dual_last_error()
    rc = lib.dual_set_kv_buffer(16, 16, 1024, 10, 16, 1024, 16, 1024, 16, 1, 4, 16, -1, None)
    assert rc == 1 and b"slot stride" in lib.dual_last_error()
    rc = lib.dual_set_kv_buffer(None, 16, 2048, 10, 16, 1024, 16, 1024, 16, 1, 4, 16, -1, None)
    assert rc == 1 and b"null" in lib.dual_last_error()


def test_fault_injection_mask_is_validated():
    """The test-only injection hook accepts its known bit and 0, refuses anything else (no GPU)."""
    lib = _lib.load()
    assert lib.dual_debug_inject(0x80) == 1
    assert b"injection" in lib.dual_last_error()
    assert lib.dual_debug_inject(0x1) == 0
    assert lib.dual_debug_inject(0) == 0


def test_workspace_size_formula():
    lib = _lib.load()
    # 256 B header + B x 8 arrival counters (rounded up to 256 B) + (G + B) segments x 32 q heads x 132 floats
    assert lib.dual_decode_workspace_size(64, 148) == 256 + 2048 + (148 + 64) * 32 * 132 * 4
    assert lib.dual_decode_workspace_size(1, 1) == 256 + 256 + 2 * 32 * 132 * 4
    assert lib.dual_decode_workspace_size(9, 4) == 256 + 512 + 13 * 32 * 132 * 4


def test_workspace_reset_checks_size_before_any_launch():
    lib = _lib.load()
    assert lib.dual_decode_workspace_reset(None, 4096, 4, -1, None) == 1
    assert lib.dual_decode_workspace_reset(256, 300, 64, -1, None) == 3
    assert b"too small" in lib.dual_last_error()


def test_no_cpu_fallback(monkeypatch, tmp_path):
    """The product path fails loudly when the CUDA library is missing."""
    monkeypatch.setattr(_lib, "_LIB", None)
    monkeypatch.setattr(_lib, "library_path", lambda: tmp_path / "missing.so")
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.load()
