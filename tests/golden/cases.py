"""Seeded input builders shared by the golden-fixture generator and the tests.

All tensors are generated on the CPU with explicit ``torch.Generator`` seeds so
the generator script (run where the reference is mounted) and the tests (run
here and on the GPU box, same torch build) see bit-identical inputs.

Cases:
  * ``config1`` -- the CPU reference config 1: one Qwen3-8B-shaped decode layer, 4 requests
    with L = 512/1024/2048/4096, slots from a seeded permutation of a 16,384-slot
    pool, the last floor(0.1 L) positions of each request remote, stored in a
    second (supplier) pool; Q, K, V ~ N(0, 1) in bf16.
  * ``validate`` -- the five shapes of the reference's kernel check
    (V/nvlink_prefill/launch_20261031_r5/code/validate_kernel.py:10-36): local_tail,
    mixed_ragged (alternating tiers), remote_only, long_prefix (every 20th position
    remote), empty_decode_splits; requests in reversed table rows, local slots from
    1 upward, remote ids from 0 upward.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List

import torch

BF16 = torch.bfloat16
HEADS_KV, HEADS_Q, DIM = 8, 32, 128


@dataclass
class TieredCase:
    name: str
    q: torch.Tensor                 # [sum(qlens), 32, 128] bf16
    k_local: torch.Tensor           # [C+1, 8, 128]
    v_local: torch.Tensor
    peer_k: List[torch.Tensor]      # supplier banks, striped g % n
    peer_v: List[torch.Tensor]
    tier: torch.Tensor              # [rows, max_len] int32
    slot: torch.Tensor
    requests: List[int]
    lengths: List[int]
    qlens: List[int]
    prefixes: List[int]
    local_capacity: int
    extra: dict = field(default_factory=dict)

    def decode_q(self) -> torch.Tensor:
        """Query of the last token of every request (decode view of the case)."""
        starts = [sum(self.qlens[:i]) for i in range(len(self.qlens))]
        return torch.stack([self.q[s + n - 1] for s, n in zip(starts, self.qlens)])


def config1(seed: int = 20261029, banks: int = 1) -> TieredCase:
    g = torch.Generator().manual_seed(seed)
    lengths = [512, 1024, 2048, 4096]
    pool = 16384
    perm = torch.randperm(pool, generator=g) + 1          # local pages 1..16384 (page 0 = dummy)
    k_local = torch.randn((pool + 1, HEADS_KV, DIM), generator=g).to(BF16)
    v_local = torch.randn((pool + 1, HEADS_KV, DIM), generator=g).to(BF16)
    n_remote = sum(L // 10 for L in lengths)              # 766
    per_bank = (n_remote + banks - 1) // banks + 3
    peer_k = [torch.randn((per_bank, HEADS_KV, DIM), generator=g).to(BF16) for _ in range(banks)]
    peer_v = [torch.randn((per_bank, HEADS_KV, DIM), generator=g).to(BF16) for _ in range(banks)]
    q = torch.randn((len(lengths), HEADS_Q, DIM), generator=g).to(BF16)
    tier = torch.full((len(lengths), max(lengths)), -1, dtype=torch.int32)
    slot = torch.zeros_like(tier)
    off, rid_next = 0, 0
    for b, L in enumerate(lengths):
        tier[b, :L] = 0
        slot[b, :L] = perm[off:off + L].int()
        off += L
        r = L // 10
        tier[b, L - r:L] = 1
        slot[b, L - r:L] = torch.arange(rid_next, rid_next + r, dtype=torch.int32)
        rid_next += r
    return TieredCase("config1" if banks == 1 else f"config1_banks{banks}", q, k_local, v_local, peer_k, peer_v,
                      tier, slot, list(range(len(lengths))), lengths, [1] * len(lengths),
                      [L - 1 for L in lengths], pool)


VALIDATE_SHAPES = [
    ("local_tail", [0, 0, 0], [1, 37, 63], "local"),
    ("mixed_ragged", [65, 7], [33, 5], "alternating"),
    ("remote_only", [31], [17], "remote"),
    ("long_prefix", [4096], [79], "sparse"),
    ("empty_decode_splits", [0, 2], [1, 1], "local"),
]


def validate_case(index: int, seed: int = 20261031, banks: int = 1) -> TieredCase:
    name, prefixes, qlens, placement = VALIDATE_SHAPES[index]
    g = torch.Generator().manual_seed(seed + index)
    lengths = [p + q for p, q in zip(prefixes, qlens)]
    total, batch = sum(lengths), len(lengths)
    k_local = torch.randn((total + 1, HEADS_KV, DIM), generator=g).to(BF16)
    v_local = torch.randn((total + 1, HEADS_KV, DIM), generator=g).to(BF16)
    per_bank = (total + banks - 1) // banks + 1
    peer_k = [torch.randn((per_bank, HEADS_KV, DIM), generator=g).to(BF16) for _ in range(banks)]
    peer_v = [torch.randn((per_bank, HEADS_KV, DIM), generator=g).to(BF16) for _ in range(banks)]
    tier = torch.zeros((batch + 1, max(lengths)), dtype=torch.int32)
    slot = torch.zeros_like(tier)
    requests = list(range(batch - 1, -1, -1))
    local_next, remote_next = 1, 0
    for b, L in enumerate(lengths):
        ar = torch.arange(L)
        if placement == "alternating":
            remote = ar % 2 == 0
        elif placement == "sparse":
            remote = ar % 20 == 0
        else:
            remote = torch.full((L,), placement == "remote")
        nr = int(remote.sum())
        nl = L - nr
        row = slot[requests[b], :L]
        row[remote] = torch.arange(remote_next, remote_next + nr, dtype=torch.int32)
        row[~remote] = torch.arange(local_next, local_next + nl, dtype=torch.int32)
        slot[requests[b], :L] = row
        tier[requests[b], :L] = remote.int()
        local_next += nl
        remote_next += nr
    q = torch.randn((sum(qlens), HEADS_Q, DIM), generator=g).to(BF16)
    return TieredCase(name, q, k_local, v_local, peer_k, peer_v, tier, slot, requests, lengths, qlens,
                      prefixes, total)


def all_cases(banks: int = 1) -> List[TieredCase]:
    return [config1(banks=banks)] + [validate_case(i, banks=banks) for i in range(len(VALIDATE_SHAPES))]


def decode_view(case: TieredCase):
    """(q [B,32,128], requests, lengths) for a decode step over each request's full KV."""
    return case.decode_q(), case.requests, case.lengths
