"""Supplier banks of the remote KV tier and their pointer tables.

Restates ``RemoteBank`` (final/cooperative_4gpu/code/peer/remote_bank.py:18-38)
for any number of suppliers: global remote id ``g`` lives in bank ``g % n`` at
physical slot ``g // n``; each bank is a ``[layers, 2, slots, 8, 128]`` bf16
tensor (an IPC-mapped or peer-accessible view of a supplier GPU's memory); the
device pointer table is bank-major, ``pointers[bank * 2L + 2 * layer + plane]``
(the reference's ``bank[layer, plane].data_ptr()`` order), which is what the
migration kernel consumes.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import torch


class RemoteBank:
    def __init__(self, banks: Sequence[torch.Tensor], layers: int = 36):
        if not banks:
            raise ValueError("at least one supplier bank is required")
        shape = tuple(banks[0].shape)
        if len(shape) != 5 or shape[0] != layers or shape[1] != 2 or shape[3:] != (8, 128):
            raise ValueError(f"supplier bank must be [{layers}, 2, slots, 8, 128], got {shape}")
        if any(tuple(b.shape) != shape or b.dtype != torch.bfloat16 for b in banks):
            raise ValueError("all supplier banks must share shape and be bf16")
        self.banks: List[torch.Tensor] = list(banks)
        self.layers = layers
        self.slots_per_bank = shape[2]
        self.shape = (layers, 2, len(banks) * shape[2], 8, 128)
        self.device = banks[0].device
        self.pointers = torch.tensor([b[layer, plane].data_ptr() for b in self.banks for layer in range(layers)
                                      for plane in range(2)], dtype=torch.int64, device=self.device)

    @property
    def num_banks(self) -> int:
        return len(self.banks)

    @property
    def capacity(self) -> int:
        return len(self.banks) * self.slots_per_bank

    def layer(self, i: int) -> List[torch.Tensor]:
        """Positional tail for ``run``: peer_k0, peer_v0, peer_k1, peer_v1, ... of layer ``i``."""
        return [t for b in self.banks for t in (b[i, 0], b[i, 1])]

    def layer_kv(self, i: int) -> Tuple[List[torch.Tensor], List[torch.Tensor]]:
        return [b[i, 0] for b in self.banks], [b[i, 1] for b in self.banks]

    def gather(self, layer: int, plane: int, gids: torch.Tensor) -> torch.Tensor:
        """Rows for global remote ids (audit / numerics only; the kernels resolve ids themselves)."""
        n = len(self.banks)
        out = torch.empty((gids.numel(), 8, 128), dtype=torch.bfloat16, device=gids.device)
        for d, b in enumerate(self.banks):
            mask = gids % n == d
            if bool(mask.any()):
                out[mask] = b[layer, plane].index_select(0, (gids[mask] // n).to(b.device)).to(gids.device)
        return out


def local_plane_pointers(kv_buffers: Sequence[Tuple[torch.Tensor, torch.Tensor]], device) -> torch.Tensor:
    """Pointer table of the local pool planes, ``[2 * layer + plane]`` (policy.py:116-117 order)."""
    return torch.tensor([t.data_ptr() for k, v in kv_buffers for t in (k, v)], dtype=torch.int64, device=device)
