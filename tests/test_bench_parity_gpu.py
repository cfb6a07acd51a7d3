"""bench.py's sampled parity check (the "parity" key of its JSON lines) on the GPU, at reduced sizes:
the decode sampler on the all-local "small" workload, the tiered sampler on a one-GPU config-5 map
(R/L 17.97 %, remote prefix, read order RN/TN 5/32, the supplier bank in this GPU's memory) with
its 302 MB 72-plane migration step, and the append sampler on "append-small".  Each must pass the
2e-3 / 1e-2 bar against the fp32 oracle, and the migrated rows must be bit-exact."""
import types

import pytest
import torch

import bench

pytestmark = pytest.mark.gpu


def _args(workload, **kw):
    return types.SimpleNamespace(workload=workload, seed=20261101, mig_ctas=64, warmup=1, steps=1, stage=None,
                                 no_e2e=True, no_cpu_baseline=True, **kw)


def test_decode_sampler_on_small_workload():
    w = bench.DecodeWorkload(_args("small"), torch.device("cuda:0"))
    w.step()
    torch.cuda.synchronize()
    par = w.parity()
    assert par["pass"], par
    assert len(par["samples"]) >= 4
    assert int(w.ws[:4].view(torch.int32).item()) == 0


def test_tiered_sampler_on_reduced_config5_map(monkeypatch):
    # config 5's ratios and read order, 16 requests, one resident layer, the bank on the same GPU
    monkeypatch.setitem(bench.TIERED, "parity-c5", (16, 4096, 32768, 0.1797, "prefix", 5, 32, 1, True))
    w = bench.TieredWorkload(_args("parity-c5"), compute=0, supplier=0)
    for _ in range(3):  # three steps: two migration batches committed, one in flight
        w.step()
    torch.cuda.synchronize()
    par = w.parity()
    assert par["pass"], par
    assert any("remote=" in s and not s.endswith("remote=0") for s in par["samples"])
    assert w.migrated_bit_exact()
    assert int(w.mig_status.item()) == 0 and int(w.status.item()) == 0


def test_append_sampler_on_append_small():
    from dual_b200 import ops
    S = bench.append_setup(_args("append-small"), "append-small")
    ops.tiered_append(S.q, S.k, S.v, S.C, S.pk, S.pv, S.qo_d, S.kv_d, S.full, True, 128 ** -0.5, S.work, S.out,
                      S.lse, S.status)
    torch.cuda.synchronize()
    par = bench.append_parity(S)
    assert par["pass"], par
    assert int(S.status.item()) == 0
