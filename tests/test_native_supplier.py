"""The native supplier process (dual_b200/lib/dual_supplier, supplier_service.cpp) against the
Python compute side of the handshake (ipc.open_suppliers / close_suppliers), on the CPU with
file-backed banks: allocation, two-way probe, close, free; and its failure modes (no compute
process, a layout mismatch, an allocation failure) end both sides with errors, never a hang."""
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

from dual_b200 import ipc
from test_topology_ipc import FileBackend


def _spawn(tmp_path, role, layers=2, slots=16, timeout=20.0, directory=None):
    return ipc.spawn_native_supplier(tmp_path / f"s{role}.sock", role, 7, layers, slots, backend="file",
                                     directory=directory or tmp_path, timeout=timeout)


def test_native_supplier_handshake_and_release(tmp_path):
    procs, chans = zip(*[_spawn(tmp_path, r) for r in range(2)])
    backend = FileBackend(tmp_path)
    try:
        bank, ptrs = ipc.open_suppliers(list(chans), 0, 2, 16, backend, timeout=20.0)
        assert len(bank.banks) == 2 and tuple(bank.banks[0].shape) == (2, 2, 16, 8, 128)
        bank.banks[1][1, 0, 5].fill_(3.0)  # written by the compute side into supplier 1's memory
        name = backend.maps[ptrs[1]][1]
        seen = torch.from_numpy(np.array(np.memmap(tmp_path / name, dtype=np.uint8, mode="r"))).view(torch.bfloat16)
        assert float(seen.view(2, 2, 16, 8, 128)[1, 0, 5, 0, 0]) == 3.0
        ipc.close_suppliers(list(chans), 0, ptrs, backend, timeout=20.0)
        assert [p.wait(timeout=20) for p in procs] == [0, 0]
        assert not list(tmp_path.glob("bank_*.bin"))  # the suppliers freed their banks
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
                p.wait()


def test_native_supplier_gives_up_without_a_compute_process(tmp_path):
    exe = Path(ipc.__file__).resolve().parent / "lib" / "dual_supplier"
    proc = subprocess.Popen([str(exe), "--socket", str(tmp_path / "x.sock"), "--role", "0", "--device", "0",
                             "--layers", "1", "--slots", "4", "--backend", "file", "--dir", str(tmp_path),
                             "--timeout", "1"], stderr=subprocess.PIPE)
    try:
        assert proc.wait(timeout=30) == 1
        assert b"no compute process" in proc.stderr.read()
        assert not list(tmp_path.glob("bank_*.bin"))
    finally:
        if proc.poll() is None:
            proc.kill()
            proc.wait()


def test_layout_mismatch_fails_both_sides(tmp_path):
    proc, ch = _spawn(tmp_path, 0, slots=16)
    try:
        with pytest.raises(RuntimeError, match="expected"):
            ipc.open_suppliers([ch], 0, 2, 32, FileBackend(tmp_path), timeout=20.0)
        ch.close()  # the compute side gives up: the supplier sees the connection go and frees its bank
        assert proc.wait(timeout=30) == 1
        assert not list(tmp_path.glob("bank_*.bin"))
    finally:
        if proc.poll() is None:
            proc.kill()
            proc.wait()


def test_allocation_failure_is_reported_before_listening(tmp_path):
    with pytest.raises(RuntimeError, match="exited"):
        _spawn(tmp_path, 0, directory=tmp_path / "missing", timeout=20.0)
