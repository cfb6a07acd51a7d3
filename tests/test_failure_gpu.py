"""Failure detection on the GPU without a fault: a device-side wait is made to run out (the append
loaders withhold the arrival on their first K tile, a flag nothing else sets), and the kernel must
turn it into DUAL_STATUS_WAIT_TIMEOUT within its bounded wait, unwind every role, free its tensor
memory and leave the context usable for the next, correct launch."""
import time

import numpy as np
import pytest
import torch

import cases as C
from dual_b200 import ops
from oracle import attention as OA

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _run(case, full):
    d = torch.device(DEV)
    qo = np.concatenate([[0], np.cumsum(case.qlens)]).astype(np.int32)
    kv = np.concatenate([[0], np.cumsum(case.lengths)]).astype(np.int32)
    work = ops.append_plan(qo, kv, True).to(d)
    out = torch.zeros((int(qo[-1]), 32, 128), dtype=torch.bfloat16, device=d)
    lse = torch.zeros((int(qo[-1]), 32), dtype=torch.float32, device=d)
    status = torch.zeros(1, dtype=torch.int32, device=d)
    ops.tiered_append(case.q.to(d), case.k_local.to(d), case.v_local.to(d), case.local_capacity,
                      [t.to(d) for t in case.peer_k], [t.to(d) for t in case.peer_v], torch.from_numpy(qo).to(d),
                      torch.from_numpy(kv).to(d), full, True, 128 ** -0.5, work, out, lse, status)
    torch.cuda.synchronize()
    return out, lse, int(status.item())


def test_append_wait_expires_to_status_and_context_survives():
    d = torch.device(DEV)
    case = next(c for c in C.all_cases(banks=3) if c.name == "long_prefix")
    full = torch.empty(sum(case.lengths), dtype=torch.int32, device=d)
    ops.pack_read_order(case.tier.to(d), case.slot.to(d), torch.tensor(case.requests, dtype=torch.int32, device=d),
                        torch.tensor(case.lengths, dtype=torch.int32, device=d), case.local_capacity, 5, 32, full,
                        prefix_lens=torch.tensor(case.prefixes, dtype=torch.int32, device=d))
    ops.debug_inject(ops.INJECT_APPEND_WITHHOLD_K0)
    try:
        t0 = time.monotonic()
        _, _, st = _run(case, full)
        elapsed = time.monotonic() - t0
    finally:
        ops.debug_inject(0)
    assert st & ops.STATUS_WAIT_TIMEOUT, f"status {st:#x}"
    assert elapsed < 30.0
    # same launch without the injection: the context is intact and the result is right
    out, lse, st = _run(case, full)
    assert st == 0
    ref, ref_lse = OA.tiered_attention(case.q, case.k_local, case.v_local, case.peer_k, case.peer_v, case.tier,
                                       case.slot, case.requests, case.lengths, case.qlens, case.prefixes)
    torch.testing.assert_close(out.float().cpu(), ref, atol=2e-3, rtol=1e-2)
    torch.testing.assert_close(lse.cpu(), ref_lse, atol=2e-3, rtol=1e-2)
