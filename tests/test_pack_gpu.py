"""Read-order packer and layout writer (CUDA, through the C ABI): bit-exact against the reference's
own Triton kernels (golden fixtures) and against the oracle at full sizes."""
import numpy as np
import pytest
import torch

from dual_b200 import ops
from oracle import layout as OL

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _groups(path):
    data = np.load(path)
    out = {}
    for key in data.files:
        g, f = key.split("__")
        out.setdefault(g, {})[f] = data[key]
    return out


def _t(x, dtype=torch.int32):
    return torch.as_tensor(np.ascontiguousarray(x)).to(dtype).to(DEV)


def test_decode_packer_matches_reference_triton(golden_dir):
    for name, g in _groups(golden_dir / "packers.npz").items():
        if not name.startswith("decode"):
            continue
        T = int(g["seq"].sum())
        full = torch.full((T + 8,), -7, dtype=torch.int32, device=DEV)
        ops.pack_read_order(_t(g["tier"]), _t(g["slot"]), _t(g["req"]), _t(g["seq"]), int(g["cap"]), int(g["rn"]),
                            int(g["tn"]), full)
        assert np.array_equal(full.cpu().numpy(), g["full"]), name


def test_prefill_packer_matches_reference_triton(golden_dir):
    for name, g in _groups(golden_dir / "packers.npz").items():
        if not name.startswith("prefill"):
            continue
        T, P = int(g["seq"].sum()), int(g["prefix"].sum())
        full = torch.full((T + 8,), -7, dtype=torch.int32, device=DEV)
        hist = torch.full((P + 8,), -7, dtype=torch.int32, device=DEV)
        ops.pack_read_order(_t(g["tier"]), _t(g["slot"]), _t(g["req"]), _t(g["seq"]), int(g["cap"]), int(g["rn"]),
                            int(g["tn"]), full, prefix_lens=_t(g["prefix"]), history_out=hist)
        assert np.array_equal(full.cpu().numpy(), g["full"]), name
        assert np.array_equal(hist.cpu().numpy(), g["history"]), name


def test_layout_writer_matches_reference_triton(golden_dir):
    for name, g in _groups(golden_dir / "packers.npz").items():
        if not name.startswith("layout"):
            continue
        tier, slot = _t(g["tier"]), _t(g["slot"])
        ops.write_prefill_layout(tier, slot, _t(g["req"]), _t(g["start"]), _t(g["length"]), _t(g["prefix"]),
                                 _t(g["loc"], torch.int64), int(g["length"].max()))
        assert np.array_equal(tier.cpu().numpy(), g["tier_out"]), name
        assert np.array_equal(slot.cpu().numpy(), g["slot_out"]), name


@pytest.mark.parametrize("rn,tn,p_remote,prefix_mode", [(5, 32, 0.18, "fifo"), (8, 128, 0.06, "tail"),
                                                          (5, 32, 0.95, "random"), (0, 32, 0.3, "random"),
                                                          (31, 32, 0.5, "random")])
def test_packer_full_size_against_oracle(rn, tn, p_remote, prefix_mode):
    rng = np.random.default_rng(11)
    B, maxL, cap = 64, 32768, 1 << 20
    lengths = rng.integers(2048, maxL + 1, B).astype(np.int32)
    rows = B + 3
    tier = np.full((rows, maxL), -1, np.int32)
    slot = np.zeros((rows, maxL), np.int32)
    req = rng.permutation(rows)[:B].astype(np.int32)
    for b in range(B):
        n = int(lengths[b])
        far = rng.random(n) < p_remote
        if prefix_mode == "fifo":
            r = int(far.sum()); far[:] = False; far[:r] = True
        elif prefix_mode == "tail":
            r = int(far.sum()); far[:] = False; far[n - r:] = True
        tier[req[b], :n] = far
        slot[req[b], :n] = rng.integers(1, cap, n)
    full = torch.empty(int(lengths.sum()), dtype=torch.int32, device=DEV)
    ops.pack_read_order(_t(tier), _t(slot), _t(req), _t(lengths), cap, rn, tn, full)
    ref, _ = OL.pack_tables(tier, slot, req, lengths, None, cap, rn, tn)
    assert np.array_equal(full.cpu().numpy(), ref)
    # prefill form with a local query suffix
    prefix = (lengths * rng.uniform(0.5, 1.0, B)).astype(np.int32)
    for b in range(B):
        tier[req[b], prefix[b]:lengths[b]] = 0
    full2 = torch.empty(int(lengths.sum()), dtype=torch.int32, device=DEV)
    hist2 = torch.empty(int(prefix.sum()), dtype=torch.int32, device=DEV)
    ops.pack_read_order(_t(tier), _t(slot), _t(req), _t(lengths), cap, rn, tn, full2, prefix_lens=_t(prefix),
                        history_out=hist2)
    ref_f, ref_h = OL.pack_tables(tier, slot, req, lengths, prefix, cap, rn, tn)
    assert np.array_equal(full2.cpu().numpy(), ref_f) and np.array_equal(hist2.cpu().numpy(), ref_h)


def test_fused_decode_step_write():
    """new_loc writes slot[req, seq-1] (tier 0) before packing, like the decode-step table write."""
    rng = np.random.default_rng(5)
    B, L = 5, 300
    tier = np.zeros((B, L), np.int32)
    slot = rng.integers(1, 1000, (B, L)).astype(np.int32)
    tier[:, :20] = 1
    seq = rng.integers(30, L, B).astype(np.int32)
    req = np.arange(B, dtype=np.int32)
    loc = rng.integers(1, 1000, B).astype(np.int64)
    t, s = _t(tier), _t(slot)
    full = torch.empty(int(seq.sum()), dtype=torch.int32, device=DEV)
    ops.pack_read_order(t, s, _t(req), _t(seq), 5000, 5, 32, full, new_loc=_t(loc, torch.int64))
    for b in range(B):
        slot[b, seq[b] - 1] = loc[b]
        tier[b, seq[b] - 1] = 0
    ref, _ = OL.pack_tables(tier, slot, req, seq, None, 5000, 5, 32)
    assert np.array_equal(full.cpu().numpy(), ref)
    assert np.array_equal(s.cpu().numpy(), slot) and np.array_equal(t.cpu().numpy(), tier)


def test_packer_empty_and_bad_lengths():
    tier = torch.zeros((2, 8), dtype=torch.int32, device=DEV)
    slot = torch.zeros_like(tier)
    full = torch.full((4,), -7, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.pack_read_order(tier, slot, _t([0, 1]), _t([0, 3]), 100, 5, 32, full, status=status)
    assert full.cpu().tolist() == [0, 0, 0, -7] and int(status.item()) == 0
    ops.pack_read_order(tier, slot, _t([0]), _t([4]), 100, 5, 32, full, prefix_lens=_t([6]), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 0x10
