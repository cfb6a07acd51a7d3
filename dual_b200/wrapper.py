"""FlashInfer-compatible attention wrappers backed by the dual_b200 kernels.

The reference keeps FlashInfer's wrapper API and swaps the kernel underneath:
``activate(wrapper)`` installs a custom JIT module whose ``run`` takes, after
``paged_kv``, the supplier tensors ``peer_k0, peer_v0, peer_k1, peer_v1, peer_k2,
peer_v2``, then ``unified_indices`` and the scalars ``local_capacity, sm_scale``
(final/cooperative_4gpu/code/peer/flashinfer_peer.py:16-19,145-150; the 2-GPU
twin passes one ``peer_k, peer_v`` pair,
V/nvlink_flashinfer_interleaved_decode/flashinfer_peer.py:16-19).  SGLang's
attention backend calls ``plan`` once per step and ``run`` once per layer
(peer/backend.py:124-149).  These classes accept exactly that convention:

* ``run(q, paged_kv)``                      -- native all-local decode over the planned indices;
* ``run(q, paged_kv, *peers, unified_indices, local_capacity, sm_scale)`` -- tiered decode,
  any number (0..8) of (peer_k, peer_v) pairs.

No CPU path exists: the wrappers raise if the CUDA library is not built.
"""
from __future__ import annotations

import functools
import math
from typing import Optional, Sequence, Tuple, Union

import torch

from . import ops

TENSORS = ["peer_k0", "peer_v0", "peer_k1", "peer_v1", "peer_k2", "peer_v2", "unified_indices"]
SCALARS = ["local_capacity", "sm_scale"]


def _unpack_paged_kv(paged_kv: Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]):
    if isinstance(paged_kv, (tuple, list)):
        k, v = paged_kv
        return k, v
    if paged_kv.dim() == 5:  # [pages, 2, page_size, heads, dim] (NHD)
        return paged_kv[:, 0], paged_kv[:, 1]
    raise ValueError("paged_kv must be (k_cache, v_cache) or a [pages, 2, 1, 8, 128] tensor")


def split_tiered_args(args: Sequence) -> Tuple[list, list, torch.Tensor, int, float]:
    """Split the reference's positional tail into (peer_k list, peer_v list, indices, C, sm_scale)."""
    if len(args) < 3 or (len(args) - 3) % 2:
        raise ValueError("tiered run expects (*[peer_k_i, peer_v_i], unified_indices, local_capacity, sm_scale)")
    peers = list(args[:-3])
    indices, capacity, scale = args[-3], args[-2], args[-1]
    return peers[0::2], peers[1::2], indices, int(capacity), float(scale)


class BatchDecodeWithPagedKVCacheWrapper:
    """Paged GQA decode (32 q / 8 kv heads, head_dim 128, bf16, page_size 1, NHD)."""

    def __init__(self, float_workspace_buffer: torch.Tensor, kv_layout: str = "NHD",
                 use_cuda_graph: bool = False, use_tensor_cores: bool = True,
                 paged_kv_indptr_buffer: Optional[torch.Tensor] = None,
                 paged_kv_indices_buffer: Optional[torch.Tensor] = None,
                 paged_kv_last_page_len_buffer: Optional[torch.Tensor] = None,
                 backend: str = "auto", jit_args=None, num_ctas: int = 0, max_batch_size: int = 0):
        if kv_layout != "NHD":
            raise ValueError("only the NHD layout is supported")
        self._kv_layout = kv_layout
        self.use_tensor_cores = use_tensor_cores
        self._use_cuda_graph = use_cuda_graph
        self.device = float_workspace_buffer.device
        self._float_workspace = float_workspace_buffer
        self._num_ctas = num_ctas or ops.default_ctas(self.device.index or 0)
        self._indptr_buf = paged_kv_indptr_buffer
        self._indices_buf = paged_kv_indices_buffer
        self._last_page_len_buf = paged_kv_last_page_len_buffer
        self._max_batch = max_batch_size
        self._batch = None
        self._sm_scale = None
        self._jit_additional_tensor_names = list(TENSORS)
        self._jit_additional_scalar_names = list(SCALARS)

    @property
    def is_cuda_graph_enabled(self) -> bool:
        return self._use_cuda_graph

    def plan(self, indptr: torch.Tensor, indices: torch.Tensor, last_page_len: torch.Tensor,
             num_qo_heads: int, num_kv_heads: int, head_dim: int, page_size: int,
             pos_encoding_mode: str = "NONE", window_left: int = -1,
             logits_soft_cap: Optional[float] = None, q_data_type="bfloat16", kv_data_type=None,
             data_type=None, sm_scale: Optional[float] = None, rope_scale=None, rope_theta=None,
             non_blocking: bool = True, **kwargs) -> None:
        if (num_qo_heads, num_kv_heads, head_dim, page_size) != (ops.NUM_QO_HEADS, ops.NUM_KV_HEADS,
                                                                 ops.HEAD_DIM, 1):
            raise ValueError("dual_b200 decode is built for 32 q heads, 8 kv heads, head_dim 128, page_size 1")
        if pos_encoding_mode != "NONE" or window_left != -1 or logits_soft_cap not in (None, 0, 0.0):
            raise ValueError("only DefaultAttention (no RoPE fusion, window or soft cap) is supported")
        batch = indptr.numel() - 1
        if self._indptr_buf is None or self._indptr_buf.numel() < batch + 1:
            if self._use_cuda_graph and self._indptr_buf is not None:
                raise ValueError("batch exceeds the CUDA-graph indptr buffer")
            self._indptr_buf = torch.empty(max(batch + 1, self._max_batch + 1), dtype=torch.int32,
                                           device=self.device)
        self._indptr_buf[: batch + 1].copy_(indptr.to(torch.int32), non_blocking=non_blocking)
        n = indices.numel()
        if self._indices_buf is None or self._indices_buf.numel() < n:
            if self._use_cuda_graph and self._indices_buf is not None:
                raise ValueError("indices exceed the CUDA-graph indices buffer")
            self._indices_buf = torch.empty(max(n, 1), dtype=torch.int32, device=self.device)
        self._indices_buf[:n].copy_(indices.to(torch.int32), non_blocking=non_blocking)
        need = ops.decode_workspace_size(max(batch, self._max_batch), self._num_ctas)
        if self._float_workspace.numel() * self._float_workspace.element_size() < need:
            raise ValueError(f"float_workspace_buffer too small: need {need} bytes")
        # the caller's buffer may hold anything (FlashInfer's wrappers take torch.empty workspaces):
        # zero the status word and the per-(request, kv head) arrival counters the kernel merges by
        ops.decode_workspace_reset(self._float_workspace, max(batch, self._max_batch))
        self._batch = batch
        self._sm_scale = float(sm_scale) if sm_scale is not None else 1.0 / math.sqrt(head_dim)

    def run(self, q: torch.Tensor, paged_kv_cache, *args, q_scale=None, k_scale=None, v_scale=None,
            out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None, return_lse: bool = False,
            enable_pdl=None, window_left=None, **kwargs):
        if self._batch is None:
            raise RuntimeError("plan() must be called before run()")
        if q_scale not in (None, 1.0) or k_scale not in (None, 1.0) or v_scale not in (None, 1.0):
            raise ValueError("fp8 scales are not supported (bf16 KV only)")
        k, v = _unpack_paged_kv(paged_kv_cache)
        if args:
            peer_k, peer_v, indices, capacity, scale = split_tiered_args(args)
        else:
            peer_k, peer_v, indices, capacity, scale = [], [], self._indices_buf, k.shape[0] - 1, self._sm_scale
        B = self._batch
        if q.shape[0] != B:
            raise ValueError(f"q has {q.shape[0]} rows but plan() was for batch {B}")
        if out is None:
            out = torch.empty_like(q)
        if return_lse and lse is None:
            lse = torch.empty((B, ops.NUM_QO_HEADS), dtype=torch.float32, device=q.device)
        ops.tiered_decode(q, k, v, capacity, peer_k, peer_v, self._indptr_buf, indices, scale, out,
                          lse if return_lse else None, self._float_workspace, self._num_ctas, batch=B)
        return (out, lse) if return_lse else out

    run_return_lse = functools.partialmethod(run, return_lse=True)


class BatchPrefillWithPagedKVCacheWrapper:
    """Paged append / prefill attention (page_size 1, NHD), FlashInfer's plan/run convention.

    ``plan`` takes the (host or device) ``qo_indptr`` / ``paged_kv_indptr`` like FlashInfer's planner,
    builds the work list on the host (one item per request x kv head x 64 query tokens, grouped by
    request and kv head, longest first) and uploads it; ``run`` launches the tcgen05 append kernel.  The reference passes the same tiered tail as for decode
    (peer/prefill_backend.py:25-37): ``run(q, paged_kv, *peers, indices, local_capacity, sm_scale)``,
    where ``indices`` is the packer's Full list (causal, non-ragged) or History list (ragged cascade).
    """

    def __init__(self, float_workspace_buffer: torch.Tensor, kv_layout: str = "NHD", use_cuda_graph: bool = False,
                 qo_indptr_buf=None, paged_kv_indptr_buf=None, paged_kv_indices_buf=None,
                 paged_kv_last_page_len_buf=None, custom_mask_buf=None, mask_indptr_buf=None,
                 backend: str = "auto", jit_args=None):
        if kv_layout != "NHD":
            raise ValueError("only the NHD layout is supported")
        self.device = float_workspace_buffer.device
        self._float_workspace = float_workspace_buffer
        self._status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._plan = None
        self._custom_mask_buf = None
        self._window_left = -1
        self._jit_module = None
        self._jit_additional_tensor_names = list(TENSORS)
        self._jit_additional_scalar_names = list(SCALARS)

    def plan(self, qo_indptr, paged_kv_indptr, paged_kv_indices, paged_kv_last_page_len, num_qo_heads: int,
             num_kv_heads: int, head_dim_qk: int, page_size: int, head_dim_vo: Optional[int] = None,
             custom_mask=None, packed_custom_mask=None, causal: bool = False, pos_encoding_mode: str = "NONE",
             use_fp16_qk_reduction: bool = False, sm_scale: Optional[float] = None, window_left: int = -1,
             logits_soft_cap: Optional[float] = None, rope_scale=None, rope_theta=None, q_data_type="bfloat16",
             kv_data_type=None, non_blocking: bool = True, remote_counts=None, **kwargs) -> None:
        """FlashInfer's plan.  ``remote_counts`` (dual_b200 extension, optional): per request, how many
        of its list entries are on suppliers (``TierManager.remote_counts``); mostly-remote requests'
        work items are then spread over the launch so their NVLink reads overlap compute."""
        if (num_qo_heads, num_kv_heads, head_dim_qk, page_size) != (ops.NUM_QO_HEADS, ops.NUM_KV_HEADS,
                                                                    ops.HEAD_DIM, 1):
            raise ValueError("dual_b200 append is built for 32 q heads, 8 kv heads, head_dim 128, page_size 1")
        if head_dim_vo not in (None, head_dim_qk):
            raise ValueError("head_dim_vo must equal head_dim_qk")
        if custom_mask is not None or packed_custom_mask is not None or window_left != -1 or \
                logits_soft_cap not in (None, 0, 0.0) or pos_encoding_mode != "NONE":
            raise ValueError("only DefaultAttention (causal or not; no custom mask, window, soft cap, RoPE fusion)")
        qo_h = torch.as_tensor(qo_indptr).to("cpu", torch.int32)
        kv_h = torch.as_tensor(paged_kv_indptr).to("cpu", torch.int32)
        work = ops.append_plan(qo_h, kv_h, causal, remote_counts)
        self._plan = dict(qo=qo_h.to(self.device, non_blocking=non_blocking),
                          kv=kv_h.to(self.device, non_blocking=non_blocking),
                          indices=torch.as_tensor(paged_kv_indices).to(self.device, torch.int32),
                          work=work.to(self.device, non_blocking=non_blocking), causal=bool(causal),
                          total_q=int(qo_h[-1]), batch=qo_h.numel() - 1,
                          sm_scale=float(sm_scale) if sm_scale is not None else 1.0 / math.sqrt(head_dim_qk))

    def run(self, q: torch.Tensor, paged_kv_cache, *args, q_scale=None, k_scale=None, v_scale=None,
            out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None, return_lse: bool = False,
            enable_pdl=None, window_left=None, **kwargs):
        if self._plan is None:
            raise RuntimeError("plan() must be called before run()")
        pl = self._plan
        k, v = _unpack_paged_kv(paged_kv_cache)
        if args:
            peer_k, peer_v, indices, capacity, scale = split_tiered_args(args)
        else:
            peer_k, peer_v, indices, capacity, scale = [], [], pl["indices"], k.shape[0] - 1, pl["sm_scale"]
        if q.shape[0] != pl["total_q"]:
            raise ValueError(f"q has {q.shape[0]} rows, plan() was for {pl['total_q']}")
        if out is None:
            out = torch.empty_like(q)
        if return_lse and lse is None:
            lse = torch.empty((q.shape[0], ops.NUM_QO_HEADS), dtype=torch.float32, device=q.device)
        ops.tiered_append(q, k, v, capacity, peer_k, peer_v, pl["qo"], pl["kv"], indices, pl["causal"], scale,
                          pl["work"], out, lse if return_lse else None, self._status)
        return (out, lse) if return_lse else out

    run_return_lse = functools.partialmethod(run, return_lse=True)

    def status(self) -> int:
        """Device status bits accumulated by this wrapper's launches (synchronous read)."""
        return ops.status_read(self._status)


def activate(wrapper):
    """Compatibility shim for the reference's ``flashinfer_peer.activate`` (peer/flashinfer_peer.py:145-150).

    dual_b200 wrappers are natively tiered; this only records the extra-argument names.
    """
    wrapper._jit_additional_tensor_names = list(TENSORS)
    wrapper._jit_additional_scalar_names = list(SCALARS)
    return wrapper
