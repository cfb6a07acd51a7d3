"""Torch-tensor front end of the C-ABI kernels (device pointers + current stream).

PyTorch only supplies device memory and streams here; every computation is a
kernel from libdual_b200.so.  Functions validate shapes/dtypes on the host and
launch asynchronously on ``torch.cuda.current_stream()``; all of them are safe
inside CUDA-graph capture (no host synchronisation, no allocation) except
``status`` which reads the device status word back.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import torch

from . import _lib

NUM_QO_HEADS = 32
NUM_KV_HEADS = 8
HEAD_DIM = 128
SLOT_BYTES = NUM_KV_HEADS * HEAD_DIM * 2  # one token slot of one plane (K or V) of one layer


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _dev(t: torch.Tensor) -> int:
    if t.device.type != "cuda":
        raise ValueError(f"expected a CUDA tensor, got {t.device}")
    return t.device.index


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def decode_workspace_size(batch: int, num_ctas: int = 0) -> int:
    return int(_lib.load().dual_decode_workspace_size(int(batch), int(num_ctas)))


def decode_workspace_reset(workspace: torch.Tensor, batch: int) -> None:
    """Zero a decode workspace's status word and arrival counters (once before first use; again after
    a launch that reported a timeout or a bad length)."""
    lib = _lib.load()
    _lib.check(lib.dual_decode_workspace_reset(workspace.data_ptr(), workspace.numel() * workspace.element_size(),
                                               int(batch), _dev(workspace), _stream(workspace.device)))


def default_ctas(device: int = 0) -> int:
    return int(_lib.load().dual_decode_default_ctas(int(device)))


def _pool_stride(pool: torch.Tensor, name: str) -> int:
    """Byte stride between consecutive token slots of an NHD page_size-1 plane."""
    _check(pool.dtype == torch.bfloat16, f"{name} must be bf16")
    if pool.dim() == 4:  # [pages, page_size=1, heads, dim]
        _check(pool.shape[1] == 1, f"{name}: page_size must be 1")
        _check(pool.stride(3) == 1 and pool.stride(2) == HEAD_DIM, f"{name}: heads x dim must be contiguous")
        _check(tuple(pool.shape[2:]) == (NUM_KV_HEADS, HEAD_DIM), f"{name}: expected 8 kv heads x 128")
    else:
        _check(pool.dim() == 3 and tuple(pool.shape[1:]) == (NUM_KV_HEADS, HEAD_DIM),
               f"{name}: expected [slots, 8, 128] or [slots, 1, 8, 128]")
        _check(pool.stride(2) == 1 and pool.stride(1) == HEAD_DIM, f"{name}: heads x dim must be contiguous")
    return pool.stride(0) * 2


def tiered_decode(q: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor, local_capacity: int,
                  peer_k: Sequence[torch.Tensor], peer_v: Sequence[torch.Tensor],
                  kv_indptr: torch.Tensor, unified_indices: torch.Tensor, sm_scale: float,
                  out: torch.Tensor, lse: Optional[torch.Tensor], workspace: torch.Tensor,
                  num_ctas: int = 0, batch: Optional[int] = None) -> None:
    """One decode layer over the tiered pool (local HBM + supplier banks)."""
    dev = _dev(q)
    B = q.shape[0] if batch is None else int(batch)
    _check(q.dtype == torch.bfloat16 and q.dim() == 3 and tuple(q.shape[1:]) == (NUM_QO_HEADS, HEAD_DIM)
           and q.stride(2) == 1, "q must be bf16 [B, 32, 128] with contiguous head_dim")
    _check(out.dtype == torch.bfloat16 and out.dim() == 3 and out.stride(2) == 1, "out must be bf16 [B, 32, 128]")
    _check(kv_indptr.dtype == torch.int32 and unified_indices.dtype == torch.int32, "indptr/indices must be int32")
    _check(kv_indptr.numel() >= B + 1, "kv_indptr too short")
    if lse is not None:
        _check(lse.dtype == torch.float32 and lse.is_contiguous() and lse.numel() >= B * NUM_QO_HEADS,
               "lse must be contiguous fp32 [B, 32]")
    ls = _pool_stride(k_local, "k_local")
    _check(_pool_stride(v_local, "v_local") == ls, "k/v local pools must share a slot stride")
    n = len(peer_k)
    _check(len(peer_v) == n, "peer_k / peer_v count mismatch")
    pk = (C.c_void_p * max(n, 1))(*[p.data_ptr() for p in peer_k])
    pv = (C.c_void_p * max(n, 1))(*[p.data_ptr() for p in peer_v])
    ps, slots = 0, 0
    if n:
        ps = _pool_stride(peer_k[0], "peer_k0")
        slots = peer_k[0].shape[0]
        for i in range(n):
            _check(_pool_stride(peer_k[i], f"peer_k{i}") == ps and _pool_stride(peer_v[i], f"peer_v{i}") == ps,
                   "all supplier banks must share a slot stride")
            _check(peer_k[i].shape[0] == slots and peer_v[i].shape[0] == slots, "supplier banks differ in size")
    lib = _lib.load()
    _lib.check(lib.dual_tiered_decode(
        q.data_ptr(), q.stride(0), q.stride(1),
        k_local.data_ptr(), v_local.data_ptr(), ls, int(local_capacity),
        pk, pv, n, ps, slots,
        kv_indptr.data_ptr(), unified_indices.data_ptr(), unified_indices.numel(), B,
        float(sm_scale),
        out.data_ptr(), out.stride(0), out.stride(1), _ptr(lse),
        workspace.data_ptr(), workspace.numel() * workspace.element_size(), int(num_ctas),
        dev, _stream(q.device)))


def append_plan(qo_indptr, kv_indptr, causal: bool, remote_counts=None) -> torch.Tensor:
    """Host-side work list (request, kv head, 64-token query pair, kv tiles it sees), grouped by
    (request, kv head), longest groups first and pairs longest first, as an int32 CPU tensor [n, 4].
    ``qo_indptr`` / ``kv_indptr``: host sequences or CPU tensors.  ``remote_counts`` (optional, per
    request: list entries on suppliers) spreads the items of mostly-remote requests over the launch."""
    qo = torch.as_tensor(qo_indptr, dtype=torch.int32).cpu().contiguous()
    kv = torch.as_tensor(kv_indptr, dtype=torch.int32).cpu().contiguous()
    B = qo.numel() - 1
    rc = None
    if remote_counts is not None:
        rc = torch.as_tensor(remote_counts, dtype=torch.int32).cpu().contiguous()
        _check(rc.numel() == B, "remote_counts needs one count per request")
    lib = _lib.load()
    n = C.c_int64(0)
    _lib.check(lib.dual_append_plan(qo.data_ptr(), kv.data_ptr(), _ptr(rc), B, int(bool(causal)), None, 0,
                                    C.byref(n)))
    work = torch.empty((max(n.value, 1), 4), dtype=torch.int32)
    _lib.check(lib.dual_append_plan(qo.data_ptr(), kv.data_ptr(), _ptr(rc), B, int(bool(causal)), work.data_ptr(),
                                    n.value, C.byref(n)))
    return work[: n.value]


def tiered_append(q: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor, local_capacity: int,
                  peer_k: Sequence[torch.Tensor], peer_v: Sequence[torch.Tensor], qo_indptr: torch.Tensor,
                  kv_indptr: torch.Tensor, unified_indices: torch.Tensor, causal: bool, sm_scale: float,
                  work: torch.Tensor, out: torch.Tensor, lse: Optional[torch.Tensor], status: torch.Tensor) -> None:
    """Causal (or non-causal) append attention over the tiered pool; ``work`` from ``append_plan`` on the device."""
    dev = _dev(q)
    _check(q.dtype == torch.bfloat16 and q.dim() == 3 and tuple(q.shape[1:]) == (NUM_QO_HEADS, HEAD_DIM)
           and q.stride(2) == 1, "q must be bf16 [sum q, 32, 128]")
    _check(out.dtype == torch.bfloat16 and out.shape == q.shape and out.stride(2) == 1, "out must match q")
    _check(qo_indptr.dtype == torch.int32 and kv_indptr.dtype == torch.int32 and unified_indices.dtype == torch.int32,
           "indptrs / indices must be int32")
    _check(work.dtype == torch.int32 and work.is_contiguous() and work.device == q.device, "work must be int32 on the device")
    if lse is not None:
        _check(lse.dtype == torch.float32 and lse.is_contiguous(), "lse must be contiguous fp32 [sum q, 32]")
    ls = _pool_stride(k_local, "k_local")
    _check(_pool_stride(v_local, "v_local") == ls, "k/v local pools must share a slot stride")
    n = len(peer_k)
    pk = (C.c_void_p * max(n, 1))(*[t.data_ptr() for t in peer_k])
    pv = (C.c_void_p * max(n, 1))(*[t.data_ptr() for t in peer_v])
    ps = _pool_stride(peer_k[0], "peer_k0") if n else 0
    slots = peer_k[0].shape[0] if n else 0
    lib = _lib.load()
    _lib.check(lib.dual_tiered_append(
        q.data_ptr(), q.stride(0), q.stride(1), k_local.data_ptr(), v_local.data_ptr(), ls, int(local_capacity),
        pk, pv, n, ps, slots, qo_indptr.data_ptr(), kv_indptr.data_ptr(), unified_indices.data_ptr(),
        unified_indices.numel(), qo_indptr.numel() - 1, int(bool(causal)), float(sm_scale), work.data_ptr(),
        work.shape[0], out.data_ptr(), out.stride(0), out.stride(1), _ptr(lse), status.data_ptr(), dev,
        _stream(q.device)))


def pack_read_order(tier: torch.Tensor, slot: torch.Tensor, req_pool_indices: torch.Tensor,
                    seq_lens: torch.Tensor, local_capacity: int, remote_rows: int, tile_rows: int,
                    full_out: torch.Tensor, prefix_lens: Optional[torch.Tensor] = None,
                    history_out: Optional[torch.Tensor] = None, new_loc: Optional[torch.Tensor] = None,
                    status: Optional[torch.Tensor] = None) -> None:
    """Unified index list in the interleaved read order (decode: prefix_lens=None)."""
    dev = _dev(tier)
    for name, t in (("tier", tier), ("slot", slot), ("req_pool_indices", req_pool_indices),
                    ("seq_lens", seq_lens), ("full_out", full_out)):
        _check(t.dtype == torch.int32, f"{name} must be int32")
    _check(tier.shape == slot.shape and tier.stride() == slot.stride() and tier.stride(1) == 1,
           "tier/slot must be row-major tables of one shape")
    if prefix_lens is not None:
        _check(prefix_lens.dtype == torch.int32, "prefix_lens must be int32")
    if new_loc is not None:
        _check(new_loc.dtype == torch.int64, "new_loc must be int64 (out_cache_loc)")
    B = req_pool_indices.numel()
    lib = _lib.load()
    _lib.check(lib.dual_pack_read_order(
        tier.data_ptr(), slot.data_ptr(), tier.shape[0], tier.stride(0), req_pool_indices.data_ptr(), seq_lens.data_ptr(),
        _ptr(prefix_lens), _ptr(new_loc), B, int(local_capacity), int(remote_rows), int(tile_rows),
        full_out.data_ptr(), _ptr(history_out), _ptr(status), dev, _stream(tier.device)))


def write_prefill_layout(tier: torch.Tensor, slot: torch.Tensor, req_pool_indices: torch.Tensor,
                         start: torch.Tensor, length: torch.Tensor, prefix: torch.Tensor,
                         locations: torch.Tensor, max_length: int, status: Optional[torch.Tensor] = None) -> None:
    """tier=0, slot=locations for the newly appended positions of every request."""
    dev = _dev(tier)
    _check(locations.dtype in (torch.int64, torch.int32), "locations must be int32 or int64")
    for name, t in (("req", req_pool_indices), ("start", start), ("length", length), ("prefix", prefix)):
        _check(t.dtype == torch.int32, f"{name} must be int32")
    lib = _lib.load()
    _lib.check(lib.dual_write_prefill_layout(
        tier.data_ptr(), slot.data_ptr(), tier.shape[0], tier.stride(0), req_pool_indices.data_ptr(),
        start.data_ptr(), length.data_ptr(), prefix.data_ptr(), locations.data_ptr(),
        int(locations.dtype == torch.int64), req_pool_indices.numel(), int(max_length), _ptr(status), dev,
        _stream(tier.device)))


def set_kv_buffer(k_local: torch.Tensor, v_local: torch.Tensor, locations: torch.Tensor, k: torch.Tensor,
                  v: torch.Tensor, status: torch.Tensor) -> None:
    """New tokens' K / V rows ``[n, 8, 128]`` (token stride free) into local slots ``locations``
    (SGLang ``out_cache_loc``, int64 or int32) of one layer's pools; bad slots are skipped and recorded."""
    ls = _pool_stride(k_local, "k_local")
    _check(_pool_stride(v_local, "v_local") == ls, "k/v local pools must share a slot stride")
    n = locations.numel()
    for t, name in ((k, "k"), (v, "v")):
        _check(t.dtype == torch.bfloat16 and t.dim() == 3 and tuple(t.shape[1:]) == (NUM_KV_HEADS, HEAD_DIM)
               and t.stride(2) == 1 and t.stride(1) == HEAD_DIM and t.shape[0] == n,
               f"{name} must be bf16 [n, 8, 128] with heads x dims contiguous")
    _check(locations.dtype in (torch.int64, torch.int32) and locations.is_contiguous(), "locations must be int64/int32")
    _check(status.dtype in (torch.int32, torch.uint32) and status.numel() >= 1, "status must be a 32-bit word")
    lib = _lib.load()
    _lib.check(lib.dual_set_kv_buffer(
        k_local.data_ptr(), v_local.data_ptr(), ls, k_local.shape[0] - 1, k.data_ptr(), k.stride(0), v.data_ptr(),
        v.stride(0), locations.data_ptr(), int(locations.dtype == torch.int64), n, status.data_ptr(), _dev(k_local),
        _stream(k_local.device)))


def migrate_copy(local_planes: torch.Tensor, remote_planes: torch.Tensor, num_planes: int, num_banks: int,
                 source: torch.Tensor, target: torch.Tensor, reverse: bool, local_slots: int,
                 remote_slots: int, status: torch.Tensor, row_bytes: int = SLOT_BYTES, max_ctas: int = 0) -> None:
    """Byte-exact copy of token slots across all planes between the local pool and supplier banks."""
    dev = _dev(source)
    _check(local_planes.dtype == torch.int64 and remote_planes.dtype == torch.int64, "pointer tables must be int64")
    _check(local_planes.numel() >= num_planes and remote_planes.numel() >= num_banks * num_planes,
           "pointer tables too short")
    _check(source.dtype == torch.int64 and target.dtype == torch.int64 and source.numel() == target.numel(),
           "source/target must be int64 of equal length")
    _check(status.dtype in (torch.int32, torch.uint32) and status.numel() >= 1, "status must be a 32-bit word")
    lib = _lib.load()
    _lib.check(lib.dual_migrate_copy(
        local_planes.data_ptr(), remote_planes.data_ptr(), int(num_planes), int(num_banks), source.data_ptr(),
        target.data_ptr(), source.numel(), int(bool(reverse)), int(row_bytes), int(local_slots), int(remote_slots),
        status.data_ptr(), int(max_ctas), dev, _stream(source.device)))


def stage_remote_rows(peer_k: Sequence[torch.Tensor], peer_v: Sequence[torch.Tensor],
                      stage_k: Sequence[torch.Tensor], stage_v: Sequence[torch.Tensor],
                      unified_indices: torch.Tensor, local_capacity: int, status: torch.Tensor,
                      num_indices: Optional[int] = None, max_ctas: int = 0) -> None:
    """Copy the supplier rows the index list names (both planes) into the same rows of local stage
    buffers, which then replace the banks in ``tiered_append`` with the index list unchanged."""
    _check(unified_indices.dtype == torch.int32 and unified_indices.is_contiguous(), "indices must be contiguous int32")
    _check(status.dtype in (torch.int32, torch.uint32) and status.numel() >= 1, "status must be a 32-bit word")
    n, slots, ps, ss = _stage_shapes(peer_k, peer_v, stage_k, stage_v, unified_indices.device)
    count = unified_indices.numel() if num_indices is None else int(num_indices)
    _check(0 <= count <= unified_indices.numel(), "num_indices out of range")
    lib = _lib.load()
    _lib.check(lib.dual_stage_remote_rows(
        _ptrs(peer_k), _ptrs(peer_v), _ptrs(stage_k), _ptrs(stage_v), n, ps, ss, slots, SLOT_BYTES,
        unified_indices.data_ptr(), count, int(local_capacity), status.data_ptr(), int(max_ctas),
        _dev(unified_indices), _stream(unified_indices.device)))


def stage_bank_range(peer_k: Sequence[torch.Tensor], peer_v: Sequence[torch.Tensor],
                     stage_k: Sequence[torch.Tensor], stage_v: Sequence[torch.Tensor],
                     row_ranges: Sequence[Sequence[int]], streams: Sequence[torch.cuda.Stream]) -> None:
    """Copy rows [begin, end) of both planes of every bank into the same rows of its stage buffers
    on the copy engines, bank b on ``streams[b]`` (no SM work)."""
    n, slots, ps, ss = _stage_shapes(peer_k, peer_v, stage_k, stage_v, stage_k[0].device)
    _check(len(row_ranges) == n and len(streams) == n, "need one row range and one stream per bank")
    begin = (C.c_int64 * n)(*[int(r[0]) for r in row_ranges])
    end = (C.c_int64 * n)(*[int(r[1]) for r in row_ranges])
    handles = (C.c_void_p * n)(*[s.cuda_stream for s in streams])
    lib = _lib.load()
    _lib.check(lib.dual_stage_bank_range(
        _ptrs(peer_k), _ptrs(peer_v), _ptrs(stage_k), _ptrs(stage_v), n, ps, ss, slots, SLOT_BYTES, begin, end,
        handles, _dev(stage_k[0])))


def _ptrs(ts: Sequence[torch.Tensor]):
    return (C.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _stage_shapes(peer_k, peer_v, stage_k, stage_v, device):
    """(banks, rows, bank stride, stage stride) after checking every bank / stage plane."""
    n = len(peer_k)
    _check(n >= 1 and len(peer_v) == n and len(stage_k) == n and len(stage_v) == n,
           "need one (k, v) bank and one (k, v) stage buffer per supplier")
    slots = peer_k[0].shape[0]
    ps = _pool_stride(peer_k[0], "peer_k0")
    ss = _pool_stride(stage_k[0], "stage_k0")
    for i in range(n):
        for t, name, stride in ((peer_k[i], "peer_k", ps), (peer_v[i], "peer_v", ps), (stage_k[i], "stage_k", ss),
                                (stage_v[i], "stage_v", ss)):
            _check(t.shape[0] == slots and _pool_stride(t, f"{name}{i}") == stride,
                   f"{name}{i}: every bank and stage buffer needs the same rows and stride")
        _check(stage_k[i].device == device and stage_v[i].device == device,
               "stage buffers must be on the index list's device")
    return n, slots, ps, ss


def debug_inject(mask: int) -> None:
    """Test hook: DUAL_INJECT_* bits for the following launches (0 disables; see dual_b200.h)."""
    _lib.check(_lib.load().dual_debug_inject(int(mask)))


INJECT_APPEND_WITHHOLD_K0 = 0x1
STATUS_WAIT_TIMEOUT = 0x4


def status_clear(status: torch.Tensor) -> None:
    lib = _lib.load()
    _lib.check(lib.dual_status_clear(status.data_ptr(), _dev(status), _stream(status.device)))


def status_read(status: torch.Tensor) -> int:
    lib = _lib.load()
    v = C.c_uint32(0)
    _lib.check(lib.dual_status_read(status.data_ptr(), C.byref(v), _dev(status), _stream(status.device)))
    return int(v.value)
