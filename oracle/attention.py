"""fp32 attention oracle over a tiered (local + supplier) paged KV cache.

Restates the reference's explicit-math check
``ReplayBackend.check_attention_output``
(final/vendor/nvlink_short_serving/launch_local_20261031_r2/code/backend.py:261-286):
gather K/V per logical position by tier (local pool for tier 0, supplier pool
for tier 1), upcast bf16 -> fp32, expand GQA by ``repeat_interleave(4)``,
scores * 128**-0.5, causal visibility ``pos <= prefix + i``, softmax, @ V.
The reference function returns no LSE; this oracle adds
``lse = logsumexp(scaled scores)`` and reports it in base 2, the convention of
FlashInfer's returned ``lse`` (its kernels write ``log2(d) + m`` with ``m`` in
the log2-scaled domain, flashinfer/attention/prefill.cuh in the pinned
flashinfer-python 0.6.x).

Supplier striping follows ``RemoteBank`` (peer/remote_bank.py:8-23): global
remote id g lives in bank ``g % n``, physical slot ``g // n``.
TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).
"""
from __future__ import annotations

import math
from typing import List, Sequence, Tuple

import torch

LOG2E = 1.0 / math.log(2.0)
GQA = 4


def gather_remote(banks: Sequence[torch.Tensor], gids: torch.Tensor) -> torch.Tensor:
    """Rows of the striped supplier pool for global remote ids ``gids`` (RemoteBank.Plane.index_select)."""
    n = len(banks)
    out = torch.empty((gids.numel(),) + tuple(banks[0].shape[1:]), dtype=banks[0].dtype)
    for d in range(n):
        mask = gids % n == d
        if mask.any():
            out[mask] = banks[d].index_select(0, gids[mask] // n)
    return out


def resolve_pages(pages: torch.Tensor, local_capacity: int, local: torch.Tensor,
                  banks: Sequence[torch.Tensor]) -> torch.Tensor:
    """Rows addressed by unified page ids (peer/flashinfer_peer.py:44-54 tiered_address)."""
    pages = pages.long()
    far = pages > local_capacity
    out = torch.empty((pages.numel(),) + tuple(local.shape[1:]), dtype=local.dtype)
    out[~far] = local.index_select(0, pages[~far])
    if far.any():
        out[far] = gather_remote(banks, pages[far] - local_capacity - 1)
    return out


def attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, prefix: int, sm_scale: float
           ) -> Tuple[torch.Tensor, torch.Tensor]:
    """One request: q [qlen, 32, 128], k/v [L, 8, 128] (bf16) -> (out fp32 [qlen,32,128], lse2 fp32 [qlen,32])."""
    qlen, L = q.shape[0], k.shape[0]
    query = q.float().transpose(0, 1)                                  # [32, qlen, 128]
    key = k.float().repeat_interleave(GQA, 1).transpose(0, 1)          # [32, L, 128]
    value = v.float().repeat_interleave(GQA, 1).transpose(0, 1)
    score = (query @ key.transpose(1, 2)) * sm_scale                   # [32, qlen, L]
    visible = torch.arange(L)[None, :] <= prefix + torch.arange(qlen)[:, None]
    score = score.masked_fill(~visible[None, :, :], float("-inf"))
    out = (score.softmax(-1) @ value).transpose(0, 1)                  # [qlen, 32, 128]
    lse = torch.logsumexp(score, -1).transpose(0, 1) * LOG2E           # [qlen, 32], base 2
    return out, lse


def tiered_attention(q: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor,
                     peer_k: Sequence[torch.Tensor], peer_v: Sequence[torch.Tensor],
                     tier: torch.Tensor, slot: torch.Tensor, requests: Sequence[int],
                     lengths: Sequence[int], qlens: Sequence[int], prefixes: Sequence[int],
                     sm_scale: float = 128 ** -0.5) -> Tuple[torch.Tensor, torch.Tensor]:
    """The reference check over the tier/slot tables (decode: qlens=1, prefix=L-1)."""
    outs: List[torch.Tensor] = []
    lses: List[torch.Tensor] = []
    offset = 0
    for rid, L, ql, p in zip(requests, lengths, qlens, prefixes):
        slots = slot[rid, :L].long()
        remote = tier[rid, :L] == 1
        kv = []
        for local, banks in ((k_local, peer_k), (v_local, peer_v)):
            value = torch.empty((L,) + tuple(local.shape[1:]), dtype=local.dtype)
            value[~remote] = local.index_select(0, slots[~remote])
            if remote.any():
                value[remote] = gather_remote(banks, slots[remote])
            kv.append(value)
        o, l = attend(q[offset:offset + ql], kv[0], kv[1], p, sm_scale)
        outs.append(o)
        lses.append(l)
        offset += ql
    return torch.cat(outs), torch.cat(lses)


def decode_from_indices(q: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor,
                        peer_k: Sequence[torch.Tensor], peer_v: Sequence[torch.Tensor],
                        indptr: Sequence[int], indices: torch.Tensor, local_capacity: int,
                        sm_scale: float = 128 ** -0.5) -> Tuple[torch.Tensor, torch.Tensor]:
    """Decode over a unified index list (what ``run`` receives): q [B,32,128] -> (out, lse2).

    Decode is order-independent in exact arithmetic, so the read order of the
    unified list only changes rounding; requests with no KV give out 0, lse -inf.
    """
    B = q.shape[0]
    out = torch.zeros((B, 32, 128), dtype=torch.float32)
    lse = torch.full((B, 32), float("-inf"), dtype=torch.float32)
    for b in range(B):
        s, e = int(indptr[b]), int(indptr[b + 1])
        if e <= s:
            continue
        pages = indices[s:e]
        k = resolve_pages(pages, local_capacity, k_local, peer_k)
        v = resolve_pages(pages, local_capacity, v_local, peer_v)
        o, l = attend(q[b:b + 1], k, v, e - s - 1, sm_scale)
        out[b] = o[0]
        lse[b] = l[0]
    return out, lse


def merge_states(o_a: torch.Tensor, lse_a: torch.Tensor, o_b: torch.Tensor, lse_b: torch.Tensor
                 ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Merge two partial attention states with base-2 LSEs (FlashInfer merge_state / SGLang
    ``_safe_merge_state`` semantics, used by the reference cascade, peer/cascade_oracle.py:28)."""
    m = torch.maximum(lse_a, lse_b)
    m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    wa = torch.exp2(lse_a - m)
    wb = torch.exp2(lse_b - m)
    s = wa + wb
    o = (o_a.float() * wa[..., None] + o_b.float() * wb[..., None]) / s[..., None]
    return o, m + torch.log2(s)
