"""Supplier-GPU topology discovery over NVLink / NVSwitch (read-only).

Replaces the reference's checks: ``topology`` parses ``nvidia-smi topo -m`` and
asserts an ``NV*`` link between the compute GPU and every donor
(final/cooperative_4gpu/code/peer/host4.py:27-44); ``nvlink_snapshot`` reads NVML
NVLink TX/RX throughput counters (V/nvlink_cooperation/.../prototype.py:52-70);
``Cuda.enable_peer`` asserts cudaDeviceCanAccessPeer (cuda_ipc.py:55-64).

Here the same facts come from NVML (link state, remote device type: GPU or
NVSwitch, NVLink P2P status) and the CUDA runtime through the C ABI (peer access,
P2P performance rank).  Nothing is written to any GPU setting.  ``nvml`` and the
library handle can be injected (tests use fakes; no GPU needed).
"""
from __future__ import annotations

import ctypes as C
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence


def _nvml():
    import pynvml
    return pynvml


@dataclass
class GpuInfo:
    index: int
    uuid: str
    pci_bus_id: str
    name: str
    nvlinks_active: List[int] = field(default_factory=list)
    nvlink_remote: Dict[int, str] = field(default_factory=dict)  # link -> "gpu" | "switch" | "other"


@dataclass
class Topology:
    gpus: List[GpuInfo]
    peer_access: Dict[tuple, bool]          # (src, dst) -> cudaDeviceCanAccessPeer
    performance_rank: Dict[tuple, int]      # (src, dst) -> cudaDevP2PAttrPerformanceRank
    nvlink_p2p: Dict[tuple, bool]           # (src, dst) -> NVML NVLink P2P status OK

    def switched(self, index: int) -> bool:
        """True when every active NVLink of GPU ``index`` ends at an NVSwitch (uniform peers)."""
        g = self.gpus[index]
        return bool(g.nvlinks_active) and all(v == "switch" for v in g.nvlink_remote.values())

    def check_suppliers(self, compute: int, suppliers: Sequence[int]) -> None:
        """Raise unless every supplier is peer-accessible from ``compute`` and reached over NVLink."""
        problems = []
        for s in suppliers:
            if s == compute:
                problems.append(f"supplier {s} is the compute GPU")
                continue
            if not self.peer_access.get((compute, s), False):
                problems.append(f"GPU {compute} cannot access peer GPU {s}")
            if self.nvlink_p2p and not self.nvlink_p2p.get((compute, s), False):
                problems.append(f"GPU {compute} -> GPU {s} is not an NVLink P2P path")
        if problems:
            raise RuntimeError("supplier topology check failed: " + "; ".join(problems))

    def uniform(self, devices: Sequence[int]) -> bool:
        """All pairs peer-accessible with one performance rank (NVSwitch: every peer at full bandwidth)."""
        ranks = {self.performance_rank.get((a, b)) for a in devices for b in devices if a != b}
        return all(self.peer_access.get((a, b), False) for a in devices for b in devices if a != b) and len(ranks) <= 1


def discover(nvml=None, lib=None, max_links: Optional[int] = None) -> Topology:
    """Inventory + NVLink state (NVML) and peer access / P2P rank (CUDA runtime via the C ABI)."""
    nvml = nvml or _nvml()
    if lib is None:
        from . import _lib
        lib = _lib.load()
    nvml.nvmlInit()
    try:
        count = nvml.nvmlDeviceGetCount()
        links = max_links if max_links is not None else getattr(nvml, "NVML_NVLINK_MAX_LINKS", 18)
        switch_t = getattr(nvml, "NVML_NVLINK_DEVICE_TYPE_SWITCH", 2)
        gpu_t = getattr(nvml, "NVML_NVLINK_DEVICE_TYPE_GPU", 0)
        gpus, handles = [], []
        for i in range(count):
            h = nvml.nvmlDeviceGetHandleByIndex(i)
            handles.append(h)
            name = nvml.nvmlDeviceGetName(h)
            uuid = nvml.nvmlDeviceGetUUID(h)
            pci = nvml.nvmlDeviceGetPciInfo(h).busId
            decode = lambda x: x.decode() if isinstance(x, bytes) else str(x)
            info = GpuInfo(i, decode(uuid), decode(pci), decode(name))
            for link in range(links):
                try:
                    if nvml.nvmlDeviceGetNvLinkState(h, link):
                        info.nvlinks_active.append(link)
                        try:
                            t = nvml.nvmlDeviceGetNvLinkRemoteDeviceType(h, link)
                            info.nvlink_remote[link] = "switch" if t == switch_t else ("gpu" if t == gpu_t else "other")
                        except Exception:
                            info.nvlink_remote[link] = "other"
                except Exception:
                    continue
            gpus.append(info)
        nvlink_p2p = {}
        idx = getattr(nvml, "NVML_P2P_CAPS_INDEX_NVLINK", 3)
        ok = getattr(nvml, "NVML_P2P_STATUS_OK", 0)
        for a in range(count):
            for b in range(count):
                if a != b:
                    try:
                        nvlink_p2p[(a, b)] = nvml.nvmlDeviceGetP2PStatus(handles[a], handles[b], idx) == ok
                    except Exception:
                        pass
    finally:
        nvml.nvmlShutdown()
    peer, rank = {}, {}
    n = len(gpus)
    for a in range(n):
        for b in range(n):
            if a == b:
                continue
            v = C.c_int(0)
            if lib.dual_can_access_peer(a, b, C.byref(v)) == 0:
                peer[(a, b)] = bool(v.value)
            r = C.c_int(0)
            if lib.dual_p2p_attribute(a, b, 0, C.byref(r)) == 0:
                rank[(a, b)] = int(r.value)
    return Topology(gpus, peer, rank, nvlink_p2p)


def nvlink_snapshot(index: int, nvml=None) -> dict:
    """NVLink TX/RX data-throughput counters of one GPU (for measuring peer traffic)."""
    nvml = nvml or _nvml()
    out = dict(cpu_unix_ns=time.time_ns(), fields=[], active_links=[])
    nvml.nvmlInit()
    try:
        h = nvml.nvmlDeviceGetHandleByIndex(index)
        for link in range(getattr(nvml, "NVML_NVLINK_MAX_LINKS", 18)):
            try:
                if nvml.nvmlDeviceGetNvLinkState(h, link):
                    out["active_links"].append(link)
            except Exception:
                continue
        fields = [(f, link) for link in out["active_links"]
                  for f in (nvml.NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX, nvml.NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_RX)]
        if fields:
            for f in nvml.nvmlDeviceGetFieldValues(h, fields):
                out["fields"].append(dict(field_id=f.fieldId, link=f.scopeId, status=f.nvmlReturn,
                                          value=int(f.value.ullVal)))
    finally:
        nvml.nvmlShutdown()
    return out


def enable_peer(device: int, peer: int, lib=None) -> None:
    """cudaDeviceEnablePeerAccess(device -> peer); already-enabled is fine."""
    if lib is None:
        from . import _lib
        lib = _lib.load()
        _lib.check(lib.dual_enable_peer(int(device), int(peer)))
    else:
        rc = lib.dual_enable_peer(int(device), int(peer))
        if rc != 0:
            raise RuntimeError(f"enable_peer({device}, {peer}) failed with {rc}")
