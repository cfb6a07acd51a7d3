"""Migration copy kernel (CUDA, through the C ABI): bit-exact against the reference's Triton fused copy
(golden hashes) and the oracle; forward (local -> supplier) and reverse (restore)."""
import hashlib
import json

import numpy as np
import pytest
import torch

from dual_b200 import ops
from dual_b200.remote_bank import RemoteBank, local_plane_pointers
from oracle import copy as OC

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _pattern_pool(layers, slots, source, n):
    local = [torch.zeros((slots, 8, 128), dtype=torch.bfloat16, device=DEV) for _ in range(2 * layers)]
    for i in range(layers):
        for plane in range(2):
            bits = torch.from_numpy(OC.pattern(n, i, plane).view(np.int16)).view(torch.bfloat16).reshape(n, 8, 128)
            local[2 * i + plane].index_copy_(0, torch.tensor(source, device=DEV), bits.to(DEV))
    return local


def test_copy_matches_reference_triton(golden_dir):
    for name, c in json.loads((golden_dir / "copy.json").read_text()).items():
        layers = c["layers"]
        local = _pattern_pool(layers, c["local_slots"], c["source"], c["n"])
        banks = [torch.zeros((layers, 2, c["bank_slots"], 8, 128), dtype=torch.bfloat16, device=DEV)
                 for _ in range(3)]
        bank = RemoteBank(banks)
        lp = local_plane_pointers([(local[2 * i], local[2 * i + 1]) for i in range(layers)], DEV)
        status = torch.zeros(1, dtype=torch.int32, device=DEV)
        src = torch.tensor(c["source"], dtype=torch.int64, device=DEV)
        dst = torch.tensor(c["target"], dtype=torch.int64, device=DEV)
        ops.migrate_copy(lp, bank.pointers, 2 * layers, 3, src, dst, False, c["local_slots"], c["bank_slots"], status)
        torch.cuda.synchronize()
        for b in range(3):
            digest = hashlib.sha256(banks[b].view(torch.int16).cpu().numpy().tobytes()).hexdigest()
            assert digest == c["forward_bank_sha256"][b], (name, b)
        back = [torch.zeros_like(t) for t in local]
        bp = local_plane_pointers([(back[2 * i], back[2 * i + 1]) for i in range(layers)], DEV)
        dest = torch.tensor(c["dest"], dtype=torch.int64, device=DEV)
        ops.migrate_copy(bp, bank.pointers, 2 * layers, 3, dst, dest, True, c["local_slots"], c["bank_slots"], status)
        torch.cuda.synchronize()
        digest = hashlib.sha256(b"".join(t.view(torch.int16).cpu().numpy().tobytes() for t in back)).hexdigest()
        assert digest == c["reverse_local_sha256"], name
        assert int(status.item()) == 0


@pytest.mark.parametrize("n,banks", [(1, 1), (2048, 3), (777, 2)])
def test_copy_random_bit_exact(n, banks):
    layers, lslots = 36, 4096
    bslots = (n + banks - 1) // banks + 5
    g = torch.Generator(device=DEV).manual_seed(n)
    local = [torch.randn((lslots, 8, 128), generator=g, device=DEV).to(torch.bfloat16) for _ in range(2 * layers)]
    bank_t = [torch.zeros((layers, 2, bslots, 8, 128), dtype=torch.bfloat16, device=DEV) for _ in range(banks)]
    bank = RemoteBank(bank_t)
    lp = local_plane_pointers([(local[2 * i], local[2 * i + 1]) for i in range(layers)], DEV)
    src = (torch.randperm(lslots - 1, device=DEV)[:n] + 1).long()
    dst = torch.randperm(banks * bslots - 4, device=DEV)[:n].long()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.migrate_copy(lp, bank.pointers, 2 * layers, banks, src, dst, False, lslots, bslots, status)
    torch.cuda.synchronize()
    for pl in range(2 * layers):
        got = bank.gather(pl // 2, pl % 2, dst)
        assert torch.equal(got.view(torch.int16), local[pl].index_select(0, src).view(torch.int16)), pl
    assert int(status.item()) == 0


def test_copy_out_of_range_sets_status():
    layers, lslots, bslots = 2, 16, 4
    local = [torch.zeros((lslots, 8, 128), dtype=torch.bfloat16, device=DEV) for _ in range(2 * layers)]
    bank_t = [torch.zeros((layers, 2, bslots, 8, 128), dtype=torch.bfloat16, device=DEV)]
    bank = RemoteBank(bank_t, layers=layers)
    lp = local_plane_pointers([(local[2 * i], local[2 * i + 1]) for i in range(layers)], DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    src = torch.tensor([3, 99], dtype=torch.int64, device=DEV)
    dst = torch.tensor([1, 2], dtype=torch.int64, device=DEV)
    ops.migrate_copy(lp, bank.pointers, 2 * layers, 1, src, dst, False, lslots, bslots, status)
    torch.cuda.synchronize()
    assert int(status.item()) & 0x8
