"""Supplier-bank lifecycle across processes: allocate, export, import, probe, close, free.

Restates the reference's donor/compute handshake (final/cooperative_4gpu/code/peer/host4.py:47-96,
V/nvlink_cooperation/.../cuda_ipc.py:18-88, measure.py:20-34):

supplier (owner of the bank)            compute GPU process
  cudaMalloc + IPC handle ------------>  allocation {handle, slots, bytes}
  bank := 0, bank[0] := role + 1.5        enable peer, open handle, zero-copy view,
                                          check bank[0] == role + 1.5, write role + 2.25
                         <------------   probe_written
  check bank[0] == role + 2.25 -------->  verified
                         <------------   closed       (after cudaIpcCloseMemHandle)
  cudaFree ---------------------------->  freed

Any exception on the supplier side is sent as ``{"type": "failure"}`` and
re-raised by the compute side; every receive has a timeout, so a supplier
that dies or never answers fails the compute side with ``TimeoutError``
instead of blocking it forever.

The memory backend is pluggable: ``CudaIpcBackend`` (C ABI: cudaMalloc /
cudaIpcGetMemHandle / cudaIpcOpenMemHandle / cudaDeviceEnablePeerAccess) is the
product path; tests run the same protocol on CPU with file-backed shared memory.
"""
from __future__ import annotations

import ctypes as C
import json
import socket
import subprocess
import time
import traceback
from pathlib import Path
from typing import List, Optional, Sequence, Tuple

import torch

from .remote_bank import RemoteBank

SLOT_BYTES_PER_LAYER = 2 * 8 * 128 * 2  # K + V, 8 kv heads x 128 x bf16


def bank_bytes(layers: int, slots: int) -> int:
    return layers * slots * SLOT_BYTES_PER_LAYER


class _Borrowed:
    """Zero-copy device view of memory this process does not own (measure.py:20-24)."""

    def __init__(self, address: int, nbytes: int):
        self.__cuda_array_interface__ = dict(shape=(nbytes,), typestr="|u1", data=(address, False), version=3)


class CudaIpcBackend:
    def __init__(self):
        from . import _lib
        self._lib = _lib
        self.lib = _lib.load()

    def allocate(self, device: int, nbytes: int) -> Tuple[int, bytes]:
        ptr = C.c_void_p()
        handle = (C.c_ubyte * 64)()
        self._lib.check(self.lib.dual_supplier_alloc(device, nbytes, C.byref(ptr), handle))
        return int(ptr.value), bytes(handle)

    def view(self, ptr: int, device: int, layers: int, slots: int) -> torch.Tensor:
        raw = torch.as_tensor(_Borrowed(ptr, bank_bytes(layers, slots)), device=f"cuda:{device}")
        assert raw.data_ptr() == ptr, "IPC import must be a zero-copy view"
        return raw.view(torch.bfloat16).view(layers, 2, slots, 8, 128)

    def open(self, device: int, handle: bytes) -> int:
        assert len(handle) == 64
        ptr = C.c_void_p()
        buf = (C.c_ubyte * 64).from_buffer_copy(handle)
        self._lib.check(self.lib.dual_ipc_open(device, buf, C.byref(ptr)))
        return int(ptr.value)

    def close(self, device: int, ptr: int) -> None:
        self._lib.check(self.lib.dual_ipc_close(device, C.c_void_p(ptr)))

    def free(self, device: int, ptr: int) -> None:
        self._lib.check(self.lib.dual_supplier_free(device, C.c_void_p(ptr)))

    def enable_peer(self, device: int, owner: int) -> None:
        if device != owner:
            self._lib.check(self.lib.dual_enable_peer(device, owner))

    def sync(self, device: int) -> None:
        torch.cuda.synchronize(device)


# ------------------------------------------------------------------ channels
class PipeChannel:
    """multiprocessing Connection with receive timeouts (the reference's Pipe + stop-flag polling)."""

    def __init__(self, conn, stop_event=None):
        self.conn, self.stop = conn, stop_event

    def send(self, obj) -> None:
        self.conn.send(obj)

    def recv(self, timeout: Optional[float]):
        waited = 0.0
        step = 0.2
        while not self.conn.poll(step):
            waited += step
            if self.stop is not None and self.stop.is_set():
                raise RuntimeError("peer process stopped before the handshake completed")
            if timeout is not None and waited >= timeout:
                raise TimeoutError(f"no message from the peer process within {timeout:.1f} s")
        return self.conn.recv()


class DistChannel:
    """torch.distributed point-to-point object channel (gloo or nccl process group)."""

    def __init__(self, peer: int, group=None):
        self.peer, self.group = peer, group

    def send(self, obj) -> None:
        import torch.distributed as dist
        dist.send_object_list([obj], dst=self.peer, group=self.group)

    def recv(self, timeout: Optional[float]):
        import torch.distributed as dist
        buf = [None]
        dist.recv_object_list(buf, src=self.peer, group=self.group)  # bounded by the group's timeout
        return buf[0]


class SocketChannel:
    """One JSON object per line over a Unix-domain socket: the channel of the native supplier
    process (``dual_b200/lib/dual_supplier``, supplier_service.cpp).  The 64-byte handle travels
    as hex.  Connecting retries until the supplier listens (bounded), and fails early if the
    supplier process has already exited."""

    def __init__(self, path, connect_timeout: float = 60.0, process=None):
        deadline = time.monotonic() + connect_timeout
        while True:
            s = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
            try:
                s.connect(str(path))
                break
            except (FileNotFoundError, ConnectionRefusedError):
                s.close()
                if process is not None and process.poll() is not None:
                    err = process.stderr.read().decode(errors="replace") if process.stderr else ""
                    raise RuntimeError(f"supplier process exited ({process.returncode}) before listening: {err}")
                if time.monotonic() > deadline:
                    raise TimeoutError(f"no supplier listening on {path} within {connect_timeout:.1f} s")
                time.sleep(0.02)
        self.sock, self.buf = s, b""

    def send(self, obj) -> None:
        self.sock.sendall((json.dumps(obj) + "\n").encode())

    def recv(self, timeout: Optional[float]):
        deadline = None if timeout is None else time.monotonic() + timeout
        while b"\n" not in self.buf:
            left = None if deadline is None else deadline - time.monotonic()
            if left is not None and left <= 0:
                raise TimeoutError(f"no message from the supplier within {timeout:.1f} s")
            self.sock.settimeout(left)
            try:
                data = self.sock.recv(65536)
            except socket.timeout:
                raise TimeoutError(f"no message from the supplier within {timeout:.1f} s") from None
            if not data:
                raise RuntimeError("the supplier closed the connection")
            self.buf += data
        line, self.buf = self.buf.split(b"\n", 1)
        msg = json.loads(line)
        if isinstance(msg.get("handle"), str):
            msg["handle"] = bytes.fromhex(msg["handle"])
        return msg

    def close(self) -> None:
        self.sock.close()


def spawn_native_supplier(socket_path, role: int, device: int, layers: int, slots: int, backend: str = "cuda",
                          directory=None, timeout: float = 120.0, close_timeout: Optional[float] = None):
    """Start the native supplier process for one bank and connect to it: (process, SocketChannel).
    The caller waits for the process after ``close_suppliers`` (it exits 0 once it has freed the
    bank) or kills that exact process on failure."""
    exe = Path(__file__).resolve().parent / "lib" / "dual_supplier"
    if not exe.exists():
        raise RuntimeError(f"{exe} is not built (python -m dual_b200.build)")
    cmd = [str(exe), "--socket", str(socket_path), "--role", str(role), "--device", str(device),
           "--layers", str(layers), "--slots", str(slots), "--backend", backend, "--timeout", str(timeout)]
    if directory is not None:
        cmd += ["--dir", str(directory)]
    if close_timeout is not None:
        cmd += ["--close-timeout", str(close_timeout)]
    proc = subprocess.Popen(cmd, stdout=subprocess.DEVNULL, stderr=subprocess.PIPE)
    try:
        return proc, SocketChannel(socket_path, connect_timeout=timeout, process=proc)
    except BaseException:
        proc.kill()
        proc.wait()
        raise


def _expect(msg, kind: str):
    if not isinstance(msg, dict):
        raise RuntimeError(f"malformed handshake message {msg!r}")
    if msg.get("type") == "failure":
        raise RuntimeError(f"supplier failed: {msg.get('error', '')}")
    if msg.get("type") != kind:
        raise RuntimeError(f"expected {kind!r}, got {msg.get('type')!r}")
    return msg


# --------------------------------------------------------------- the protocol
def serve_supplier(channel, role: int, device: int, layers: int, slots: int, backend=None,
                   timeout: float = 120.0, close_timeout: Optional[float] = None) -> dict:
    """Supplier side: own one bank for the life of the compute process, then free it."""
    backend = backend or CudaIpcBackend()
    ptr = None
    try:
        nbytes = bank_bytes(layers, slots)
        ptr, handle = backend.allocate(device, nbytes)
        bank = backend.view(ptr, device, layers, slots)
        bank.zero_()
        bank.view(-1)[0] = role + 1.5
        backend.sync(device)
        channel.send(dict(type="allocation", role=role, owner_device=device, layers=layers, slots=slots,
                          bytes=nbytes, handle=handle))
        _expect(channel.recv(timeout), "probe_written")
        backend.sync(device)
        seen = float(bank.view(-1)[0].item())
        if seen != role + 2.25:
            raise RuntimeError(f"probe write not visible on the supplier (read {seen}, want {role + 2.25})")
        channel.send(dict(type="verified"))
        _expect(channel.recv(close_timeout), "closed")
        backend.free(device, ptr)
        ptr = None
        channel.send(dict(type="freed"))
        return dict(role=role, owner=device, bidirectional_probe=True, released=True)
    except BaseException:
        try:
            channel.send(dict(type="failure", role=role, error=traceback.format_exc()))
        except Exception:
            pass
        if ptr is not None:
            try:
                backend.free(device, ptr)
            except Exception:
                pass
        raise


def open_suppliers(channels: Sequence, device: int, layers: int, slots: int, backend=None,
                   timeout: float = 120.0) -> Tuple[RemoteBank, List[int]]:
    """Compute side: import every supplier's bank (role = channel index), probe both directions."""
    backend = backend or CudaIpcBackend()
    banks, ptrs = [], []
    try:
        for role, ch in enumerate(channels):
            alloc = _expect(ch.recv(timeout), "allocation")
            if alloc["slots"] != slots or alloc["layers"] != layers or alloc["role"] != role:
                raise RuntimeError(f"supplier {role} announced {alloc['layers']}x{alloc['slots']} slots, "
                                   f"expected {layers}x{slots}")
            backend.enable_peer(device, alloc["owner_device"])
            ptr = backend.open(device, alloc["handle"])
            ptrs.append(ptr)
            bank = backend.view(ptr, device, layers, slots)
            seen = float(bank.view(-1)[0].item())
            if seen != role + 1.5:
                raise RuntimeError(f"supplier {role} probe value {seen} != {role + 1.5}: wrong mapping")
            bank.view(-1)[0] = role + 2.25
            backend.sync(device)
            ch.send(dict(type="probe_written"))
            _expect(ch.recv(timeout), "verified")
            bank.view(-1)[0] = 0  # leave the bank zeroed for use
            banks.append(bank)
        backend.sync(device)
        return RemoteBank(banks, layers=layers), ptrs
    except BaseException:
        for ptr in ptrs:
            try:
                backend.close(device, ptr)
            except Exception:
                pass
        raise


def close_suppliers(channels: Sequence, device: int, ptrs: Sequence[int], backend=None,
                    timeout: float = 120.0) -> None:
    """Compute side: unmap every bank, tell its supplier, wait until it has freed the memory."""
    backend = backend or CudaIpcBackend()
    backend.sync(device)
    for ch, ptr in zip(channels, ptrs):
        backend.close(device, ptr)
        ch.send(dict(type="closed"))
        _expect(ch.recv(timeout), "freed")
