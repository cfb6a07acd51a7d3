"""Helpers shared by the GPU tests: move a golden case to the device and run the product path."""
from __future__ import annotations

import numpy as np
import torch

from dual_b200 import ops

DEV = "cuda:0"


def to_dev(case):
    d = torch.device(DEV)
    return dict(k_local=case.k_local.to(d), v_local=case.v_local.to(d),
                peer_k=[p.to(d) for p in case.peer_k], peer_v=[p.to(d) for p in case.peer_v],
                tier=case.tier.to(d), slot=case.slot.to(d))


def pack_decode(dev, requests, lengths, capacity, rn=5, tn=32):
    req = torch.tensor(requests, dtype=torch.int32, device=DEV)
    seq = torch.tensor(lengths, dtype=torch.int32, device=DEV)
    full = torch.full((max(sum(lengths), 1),), -7, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.pack_read_order(dev["tier"], dev["slot"], req, seq, capacity, rn, tn, full, status=status)
    indptr = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=DEV)
    return indptr, full, status


def decode(q, dev, indptr, indices, capacity, num_ctas=0, sm_scale=128 ** -0.5, lse=True):
    B = q.shape[0]
    out = torch.empty((B, 32, 128), dtype=torch.bfloat16, device=DEV)
    l = torch.empty((B, 32), dtype=torch.float32, device=DEV) if lse else None
    ws = torch.zeros(ops.decode_workspace_size(B, num_ctas or ops.default_ctas(0)), dtype=torch.uint8, device=DEV)
    ops.tiered_decode(q.to(DEV), dev["k_local"], dev["v_local"], capacity, dev["peer_k"], dev["peer_v"],
                      indptr, indices, sm_scale, out, l, ws, num_ctas)
    return out, l, ws
