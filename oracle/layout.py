"""Read-order oracle: history_order and the page-table packers on the CPU.

``history_order`` restates the reference's CPU specification of the read
order (final/cooperative_4gpu/code/peer/layout.py:5-22): the fully visible
prefix is stably split into remote and local entries and re-emitted as tiles
of TN rows, each RN remote rows then TN-RN local rows; a tile that cannot be
filled regularly takes extra local rows first, then extra remote rows; the
query suffix stays in place.  ``read_order`` is the same permutation in the
closed form the reference's Triton packer uses (peer/packing.py:19-34), in
numpy.  ``pack_tables`` restates ``packing.prepare`` (peer/packing.py:6-36)
and, with prefix == length, the decode packer ``_count_remote`` +
``_pack_indices`` (peer/backend.py:22-58; identical on remote-prefix maps).
``write_layout`` restates ``_write_prefill_layout`` (peer/page_ops.py:6-18).
TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import numpy as np


def history_order(encoded: Sequence[int], far: Sequence[bool], prefix: int, remote_rows: int,
                  tile_rows: int = 128) -> List[int]:
    """Loop form (small inputs): permutation of the first ``prefix`` entries, suffix unchanged."""
    encoded = list(encoded)
    far = [bool(x) for x in far]
    assert len(encoded) == len(far) and 0 <= prefix <= len(encoded)
    assert not any(far[prefix:]), "current input KV must stay local and ordered"
    if remote_rows == 0:
        return encoded
    assert 0 < remote_rows < tile_rows
    remote = [e for e, f in zip(encoded[:prefix], far[:prefix]) if f]
    local = [e for e, f in zip(encoded[:prefix], far[:prefix]) if not f]
    out: List[int] = []
    ri = li = 0
    while ri < len(remote) or li < len(local):
        rr = remote[ri:ri + remote_rows]
        ll = local[li:li + tile_rows - remote_rows]
        ri += len(rr)
        li += len(ll)
        missing = tile_rows - len(rr) - len(ll)
        extra = local[li:li + missing]
        ll += extra
        li += len(extra)
        missing -= len(extra)
        extra = remote[ri:ri + missing]
        rr += extra
        ri += len(extra)
        out.extend(rr + ll)
    return out + encoded[prefix:]


def read_order_destinations(far: np.ndarray, prefix: int, remote_rows: int, tile_rows: int) -> np.ndarray:
    """Destination index of every position 0..n-1 (closed form of history_order)."""
    n = far.shape[0]
    pos = np.arange(n, dtype=np.int64)
    if remote_rows == 0:
        return pos
    RN, TN = remote_rows, tile_rows
    LN = TN - RN
    old = pos < prefix
    fr = old & far
    nr = old & ~far
    r = int(fr.sum())
    l = prefix - r
    rr = np.cumsum(fr) - 1
    ll = np.cumsum(nr) - 1
    groups = min(r // RN, l // LN)
    base = groups * TN
    rleft, lleft = r - groups * RN, l - groups * LN
    tail_r, tail_l = min(rleft, RN), min(lleft, LN)
    extra_l = min(TN - tail_r - tail_l, lleft - tail_l)
    tail_l += extra_l
    tail_r += min(TN - tail_r - tail_l, rleft - tail_r)
    tail = tail_r + tail_l
    rpos = np.where(rr < groups * RN, (rr // RN) * TN + rr % RN,
                    np.where(rr < groups * RN + tail_r, base + rr - groups * RN,
                             base + tail + rr - groups * RN - tail_r))
    lpos = np.where(ll < groups * LN, (ll // LN) * TN + RN + ll % LN,
                    np.where(ll < groups * LN + tail_l, base + tail_r + ll - groups * LN,
                             base + tail + ll - groups * LN - tail_l))
    return np.where(old, np.where(fr, rpos, lpos), pos)


def read_order(encoded: np.ndarray, far: np.ndarray, prefix: int, remote_rows: int, tile_rows: int
               ) -> np.ndarray:
    dest = read_order_destinations(np.asarray(far, dtype=bool), prefix, remote_rows, tile_rows)
    out = np.empty_like(np.asarray(encoded))
    out[dest] = encoded
    return out


def encode(tier_row: np.ndarray, slot_row: np.ndarray, local_capacity: int) -> np.ndarray:
    """Unified page id: slot for local, slot + C + 1 for remote (int32 arithmetic)."""
    return (slot_row.astype(np.int64) + np.where(tier_row == 1, local_capacity + 1, 0)).astype(np.int32)


def pack_tables(tier: np.ndarray, slot: np.ndarray, requests: Sequence[int], lengths: Sequence[int],
                prefixes: Optional[Sequence[int]], local_capacity: int, remote_rows: int, tile_rows: int
                ) -> Tuple[np.ndarray, Optional[np.ndarray]]:
    """Full (and History when ``prefixes`` is given) unified index lists for a batch."""
    full, hist = [], []
    for i, (rid, n) in enumerate(zip(requests, lengths)):
        p = n if prefixes is None else int(prefixes[i])
        t = tier[rid, :n]
        enc = encode(t, slot[rid, :n], local_capacity)
        order = read_order(enc, t == 1, p, remote_rows, tile_rows)
        full.append(order)
        hist.append(order[:p])
    cat = lambda xs: np.concatenate(xs).astype(np.int32) if xs else np.zeros(0, np.int32)
    return cat(full), (cat(hist) if prefixes is not None else None)


def write_layout(tier: np.ndarray, slot: np.ndarray, requests, starts, lengths, prefixes, locations) -> None:
    """In place: tier=0, slot=locations[start+j] at positions prefix+j, j < length."""
    for rid, s, n, p in zip(requests, starts, lengths, prefixes):
        slot[rid, p:p + n] = np.asarray(locations[s:s + n]).astype(np.int32)
        tier[rid, p:p + n] = 0
