"""Host-side supplier plumbing on the CPU: topology checks against a fake NVML / fake CUDA
runtime, and the supplier <-> compute handshake (dual_b200.ipc) run as two gloo ranks and as
piped processes with file-backed shared memory standing in for device memory.  Failures are
made on the host (a supplier that raises, a supplier that exits without answering)."""
import ctypes as C
import multiprocessing as mp
import os
import socket
from pathlib import Path
from types import SimpleNamespace as NS

import numpy as np
import pytest
import torch

from dual_b200 import ipc, topology


# ----------------------------------------------------------------- topology
class FakeNvml:
    NVML_NVLINK_MAX_LINKS = 4
    NVML_NVLINK_DEVICE_TYPE_GPU = 0
    NVML_NVLINK_DEVICE_TYPE_SWITCH = 2
    NVML_P2P_CAPS_INDEX_NVLINK = 3
    NVML_P2P_STATUS_OK = 0
    NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX = 138
    NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_RX = 139

    def __init__(self, n=4, links_down=(), no_nvlink_pairs=()):
        self.n, self.links_down, self.no_nvlink = n, set(links_down), set(no_nvlink_pairs)
        self.inits = 0

    def nvmlInit(self): self.inits += 1
    def nvmlShutdown(self): self.inits -= 1
    def nvmlDeviceGetCount(self): return self.n
    def nvmlDeviceGetHandleByIndex(self, i): return i
    def nvmlDeviceGetName(self, h): return b"NVIDIA B200"
    def nvmlDeviceGetUUID(self, h): return f"GPU-{h:04d}"
    def nvmlDeviceGetPciInfo(self, h): return NS(busId=f"0000:{h:02x}:00.0".encode())
    def nvmlDeviceGetNvLinkState(self, h, link): return 0 if (h, link) in self.links_down else 1
    def nvmlDeviceGetNvLinkRemoteDeviceType(self, h, link): return self.NVML_NVLINK_DEVICE_TYPE_SWITCH
    def nvmlDeviceGetP2PStatus(self, a, b, idx): return 1 if (a, b) in self.no_nvlink else 0

    def nvmlDeviceGetFieldValues(self, h, fields):
        return [NS(fieldId=f, scopeId=l, nvmlReturn=0, value=NS(ullVal=1000 * l + f)) for f, l in fields]


class FakeLib:
    def __init__(self, no_peer=()):
        self.no_peer = set(no_peer)
        self.enabled = []

    def dual_can_access_peer(self, a, b, out):
        out._obj.value = 0 if (a, b) in self.no_peer else 1
        return 0

    def dual_p2p_attribute(self, a, b, attr, out):
        out._obj.value = 0
        return 0

    def dual_enable_peer(self, a, b):
        self.enabled.append((a, b))
        return 0


def test_topology_nvswitch_uniform_and_supplier_check():
    topo = topology.discover(nvml=FakeNvml(), lib=FakeLib())
    assert [g.name for g in topo.gpus] == ["NVIDIA B200"] * 4
    assert topo.switched(0) and topo.uniform([0, 1, 2, 3])
    topo.check_suppliers(0, [1, 2, 3])  # 1 + 3 layout
    with pytest.raises(RuntimeError, match="is the compute GPU"):
        topo.check_suppliers(0, [0])


def test_topology_rejects_missing_peer_or_nvlink():
    topo = topology.discover(nvml=FakeNvml(no_nvlink_pairs={(0, 2)}), lib=FakeLib(no_peer={(0, 3)}))
    with pytest.raises(RuntimeError) as e:
        topo.check_suppliers(0, [1, 2, 3])
    assert "GPU 0 cannot access peer GPU 3" in str(e.value) and "GPU 0 -> GPU 2" in str(e.value)
    assert not topo.uniform([0, 1, 2, 3])


def test_nvlink_snapshot_reads_counters_only():
    nv = FakeNvml(n=1, links_down={(0, 3)})
    snap = topology.nvlink_snapshot(0, nvml=nv)
    assert snap["active_links"] == [0, 1, 2] and len(snap["fields"]) == 6 and nv.inits == 0


# ------------------------------------------------------------------ IPC protocol
class FileBackend:
    """Shared files as 'device memory': handles are file names, views map the same pages."""

    def __init__(self, root, fail_on_allocate=False):
        self.root = Path(root)
        self.maps, self.fail = {}, fail_on_allocate
        self.peers = []

    def allocate(self, device, nbytes):
        if self.fail:
            raise MemoryError("injected supplier allocation failure")
        name = f"bank_{os.getpid()}_{len(self.maps)}.bin"
        mm = np.memmap(self.root / name, dtype=np.uint8, mode="w+", shape=(nbytes,))
        key = id(mm)
        self.maps[key] = (mm, name)
        return key, name.encode().ljust(64, b"\0")

    def view(self, ptr, device, layers, slots):
        mm, _ = self.maps[ptr]
        return torch.from_numpy(mm).view(torch.bfloat16).view(layers, 2, slots, 8, 128)

    def open(self, device, handle):
        name = handle.rstrip(b"\0").decode()
        mm = np.memmap(self.root / name, dtype=np.uint8, mode="r+")
        self.maps[id(mm)] = (mm, name)
        return id(mm)

    def close(self, device, ptr):
        self.maps.pop(ptr)

    def free(self, device, ptr):
        mm, name = self.maps.pop(ptr)
        del mm
        (self.root / name).unlink()

    def enable_peer(self, device, owner):
        self.peers.append((device, owner))

    def sync(self, device):
        pass


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, port, root, q):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", world_size=2, rank=rank)
    try:
        backend = FileBackend(root)
        if rank == 1:
            q.put(("supplier", ipc.serve_supplier(ipc.DistChannel(0), 0, 7, 2, 16, backend)))
        else:
            bank, ptrs = ipc.open_suppliers([ipc.DistChannel(1)], 0, 2, 16, backend)
            bank.banks[0][1, 0, 5].fill_(3.0)  # a write that the supplier's memory must hold
            seen = float(torch.from_numpy(np.memmap(Path(root) / backend.maps[ptrs[0]][1], dtype=np.uint8,
                                                    mode="r")).view(torch.bfloat16).view(2, 2, 16, 8, 128)[1, 0, 5, 0, 0])
            ipc.close_suppliers([ipc.DistChannel(1)], 0, ptrs, backend)
            q.put(("compute", dict(peers=backend.peers, seen=seen, shape=tuple(bank.shape))))
    finally:
        dist.destroy_process_group()


def test_handshake_over_two_gloo_ranks(tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, port, str(tmp_path), q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = dict(q.get(timeout=5) for _ in range(2))
    assert got["supplier"]["bidirectional_probe"] and got["supplier"]["released"]
    assert got["compute"]["peers"] == [(0, 7)] and got["compute"]["seen"] == 3.0
    assert got["compute"]["shape"] == (2, 2, 16, 8, 128)
    assert not list(tmp_path.glob("bank_*.bin")), "supplier must free its bank after close"


def _piped_supplier(conn, root, mode):
    ch = ipc.PipeChannel(conn)
    if mode == "exit_silently":
        os._exit(0)  # a supplier that dies before the handshake
    try:
        ipc.serve_supplier(ch, 0, 1, 1, 8, FileBackend(root, fail_on_allocate=(mode == "fail")), timeout=10)
    except BaseException:
        pass


@pytest.mark.parametrize("mode,error", [("fail", RuntimeError), ("exit_silently", TimeoutError)])
def test_supplier_failures_end_the_compute_side(tmp_path, mode, error):
    ctx = mp.get_context("spawn")
    a, b = ctx.Pipe()
    p = ctx.Process(target=_piped_supplier, args=(b, str(tmp_path), mode))
    p.start()
    # a failing supplier answers (slowly: the child imports torch); a dead one never does
    with pytest.raises(error) as e:
        ipc.open_suppliers([ipc.PipeChannel(a)], 0, 1, 8, FileBackend(tmp_path),
                           timeout=120.0 if mode == "fail" else 3.0)
    p.join(30)
    if mode == "fail":
        assert "injected supplier allocation failure" in str(e.value)


def test_probe_mismatch_is_detected(tmp_path):
    """A handle that maps the wrong memory (probe value absent) is refused."""
    backend = FileBackend(tmp_path)
    ptr, handle = backend.allocate(0, ipc.bank_bytes(1, 8))

    class Chan:
        def __init__(self):
            self.sent = []

        def send(self, m):
            self.sent.append(m)

        def recv(self, timeout):
            return dict(type="allocation", role=0, owner_device=1, layers=1, slots=8, bytes=0, handle=handle)

    with pytest.raises(RuntimeError, match="wrong mapping"):
        ipc.open_suppliers([Chan()], 0, 1, 8, backend)
