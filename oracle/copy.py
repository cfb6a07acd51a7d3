"""Migration-copy oracle: byte-exact slot copy across all planes.

Restates the addressing of the reference's Triton ``_copy``
(final/cooperative_4gpu/code/peer/fused_copy.py:6-21): for every plane and
every pair (source[i], target[i]), forward copies local slot ``source[i]`` to
global remote id ``target[i]`` = bank ``target[i] % banks``, physical slot
``target[i] // banks``; reverse copies remote id ``source[i]`` to local slot
``target[i]``.  Planes are uint16/bf16 arrays of shape [slots, elems]; the copy
is done on raw bits, so results compare with ``np.array_equal``.
TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).
"""
from __future__ import annotations

from typing import Sequence

import numpy as np


def migrate_copy(local_planes: Sequence[np.ndarray], remote_banks: Sequence[Sequence[np.ndarray]],
                 source: Sequence[int], target: Sequence[int], reverse: bool) -> None:
    """In place.  ``remote_banks[bank][plane]``; ``local_planes[plane]``."""
    banks = len(remote_banks)
    for s, t in zip(source, target):
        g, loc = (int(s), int(t)) if reverse else (int(t), int(s))
        bank, phys = g % banks, g // banks
        for pl, lp in enumerate(local_planes):
            rp = remote_banks[bank][pl]
            if reverse:
                lp[loc] = rp[phys]
            else:
                rp[phys] = lp[loc]


def pattern(n: int, layer: int, plane: int, elems: int = 1024) -> np.ndarray:
    """The reference's deterministic payload ``(arange%127)/64 + layer/16 + plane/8`` as bf16 bits
    (V/nvlink_migration_latency/.../fused_copy.py:35), rounded to nearest even like torch's cast."""
    x = (np.arange(n * elems, dtype=np.float32).reshape(n, elems) % 127) / 64 + layer / 16 + plane / 8
    x = x.astype(np.float32)
    bits = x.view(np.uint32)
    rounded = bits + 0x7FFF + ((bits >> 16) & 1)
    return (rounded >> 16).astype(np.uint16)
