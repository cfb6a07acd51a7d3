"""Pin the CPU oracle to the reference: every restatement against fixtures produced by the
reference's own code (tests/golden/make_golden.py).  CPU only."""
import hashlib
import json

import numpy as np
import pytest
import torch

import cases as C
from oracle import attention as OA
from oracle import copy as OC
from oracle import layout as OL
from oracle import policy as OP


def _npz_groups(path):
    data = np.load(path)
    groups = {}
    for key in data.files:
        g, f = key.split("__")
        groups.setdefault(g, {})[f] = data[key]
    return groups


def test_history_order_matches_reference(golden_dir):
    cases = json.loads((golden_dir / "history_order.json").read_text())["cases"]
    assert len(cases) > 50
    for c in cases:
        got = OL.history_order(c["encoded"], c["far"], c["prefix"], c["rn"], c["tn"])
        assert got == c["expected"], (c["rn"], c["tn"], c["prefix"])
        closed = OL.read_order(np.array(c["encoded"], np.int32), np.array(c["far"], bool), c["prefix"], c["rn"],
                               c["tn"])
        assert closed.tolist() == c["expected"]


def test_history_order_known_answer():
    # 7 remote + 33 local, RN/TN = 5/32 (the reference's own worked example)
    got = OL.history_order(list(range(40)), [True] * 7 + [False] * 33, 40, 5, 32)
    assert got == list(range(5)) + list(range(7, 34)) + [5, 6] + list(range(34, 40))


def test_decode_packer_matches_reference_triton(golden_dir):
    groups = _npz_groups(golden_dir / "packers.npz")
    n = 0
    for name, g in groups.items():
        if not name.startswith("decode"):
            continue
        full, _ = OL.pack_tables(g["tier"], g["slot"], g["req"], g["seq"], None, int(g["cap"]), int(g["rn"]),
                                 int(g["tn"]))
        T = int(g["seq"].sum())
        assert np.array_equal(full, g["full"][:T]), name
        assert (g["full"][T:] == -7).all()
        n += 1
    assert n >= 9


def test_prefill_packer_matches_reference_triton(golden_dir):
    groups = _npz_groups(golden_dir / "packers.npz")
    n = 0
    for name, g in groups.items():
        if not name.startswith("prefill"):
            continue
        full, hist = OL.pack_tables(g["tier"], g["slot"], g["req"], g["seq"], g["prefix"], int(g["cap"]),
                                    int(g["rn"]), int(g["tn"]))
        T, P = int(g["seq"].sum()), int(g["prefix"].sum())
        assert np.array_equal(full, g["full"][:T]), name
        assert np.array_equal(hist, g["history"][:P]), name
        n += 1
    assert n >= 12


def test_layout_writer_matches_reference_triton(golden_dir):
    groups = _npz_groups(golden_dir / "packers.npz")
    for name, g in groups.items():
        if not name.startswith("layout"):
            continue
        tier, slot = g["tier"].copy(), g["slot"].copy()
        OL.write_layout(tier, slot, g["req"], g["start"], g["length"], g["prefix"], g["loc"])
        assert np.array_equal(tier, g["tier_out"]) and np.array_equal(slot, g["slot_out"]), name


def _copy_case(c):
    layers, ls, bs = c["layers"], c["local_slots"], c["bank_slots"]
    local = [np.zeros((ls, 1024), np.uint16) for _ in range(2 * layers)]
    for i in range(layers):
        for plane in range(2):
            local[2 * i + plane][c["source"]] = OC.pattern(c["n"], i, plane)
    banks = [[np.zeros((bs, 1024), np.uint16) for _ in range(2 * layers)] for _ in range(3)]
    return local, banks


def test_copy_matches_reference_triton(golden_dir):
    cases = json.loads((golden_dir / "copy.json").read_text())
    for name, c in cases.items():
        local, banks = _copy_case(c)
        OC.migrate_copy(local, banks, c["source"], c["target"], reverse=False)
        for b in range(3):
            digest = hashlib.sha256(np.stack(banks[b]).tobytes()).hexdigest()
            assert digest == c["forward_bank_sha256"][b], (name, b)
        back = [np.zeros_like(x) for x in local]
        OC.migrate_copy(back, banks, c["target"], c["dest"], reverse=True)
        assert hashlib.sha256(b"".join(x.tobytes() for x in back)).hexdigest() == c["reverse_local_sha256"], name


@pytest.mark.parametrize("banks", [1, 3])
def test_attention_oracle_matches_reference_fp32(golden_dir, banks):
    gold = np.load(golden_dir / "attention.npz")
    for case in C.all_cases(banks=banks):
        q = case.decode_q()
        out, lse = OA.tiered_attention(q, case.k_local, case.v_local, case.peer_k, case.peer_v, case.tier,
                                       case.slot, case.requests, case.lengths, [1] * len(case.lengths),
                                       [L - 1 for L in case.lengths])
        ref = torch.from_numpy(gold[f"{case.name}_b{banks}_decode"])
        torch.testing.assert_close(out, ref, atol=1e-5, rtol=1e-5)
        assert torch.isfinite(lse).all()
        outp, _ = OA.tiered_attention(case.q, case.k_local, case.v_local, case.peer_k, case.peer_v, case.tier,
                                      case.slot, case.requests, case.lengths, case.qlens, case.prefixes)
        rows = torch.from_numpy(gold[f"{case.name}_b{banks}_prefill_rows"])
        refp = torch.from_numpy(gold[f"{case.name}_b{banks}_prefill"])
        torch.testing.assert_close(outp[rows], refp, atol=1e-5, rtol=1e-5)


def test_decode_from_indices_equals_table_oracle():
    case = C.config1(banks=3)
    q = case.decode_q()
    tier, slot = case.tier.numpy(), case.slot.numpy()
    full, _ = OL.pack_tables(tier, slot, case.requests, case.lengths, None, case.local_capacity, 5, 32)
    indptr = np.concatenate([[0], np.cumsum(case.lengths)])
    out_i, lse_i = OA.decode_from_indices(q, case.k_local, case.v_local, case.peer_k, case.peer_v, indptr,
                                          torch.from_numpy(full), case.local_capacity)
    out_t, lse_t = OA.tiered_attention(q, case.k_local, case.v_local, case.peer_k, case.peer_v, case.tier,
                                       case.slot, case.requests, case.lengths, [1] * 4,
                                       [L - 1 for L in case.lengths])
    torch.testing.assert_close(out_i, out_t, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(lse_i, lse_t, atol=1e-5, rtol=1e-5)


def test_lse_merge_property():
    """Two disjoint halves merged with base-2 LSEs reproduce the whole (cascade semantics)."""
    g = torch.Generator().manual_seed(3)
    k = torch.randn(300, 8, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(300, 8, 128, generator=g).to(torch.bfloat16)
    q = torch.randn(1, 32, 128, generator=g).to(torch.bfloat16)
    o, l = OA.attend(q, k, v, 299, 128 ** -0.5)
    o1, l1 = OA.attend(q, k[:120], v[:120], 119, 128 ** -0.5)
    o2, l2 = OA.attend(q, k[120:], v[120:], 179, 128 ** -0.5)
    om, lm = OA.merge_states(o1, l1, o2, l2)
    torch.testing.assert_close(om, o, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(lm, l, atol=1e-5, rtol=1e-5)


def test_policy_matches_reference(golden_dir):
    rows = json.loads((golden_dir / "policy.json").read_text())["rows"]
    for r in rows:
        assert OP.limit_pages(r["local"], r["remote"], r["a"], r["b"]) == r["limit"]
        assert OP.budget(r["local"], r["remote"], r["peer_free"], r["residents"], r["a"], r["b"]) == r["budget"][2]
        assert OP.repair_count(r["local"], r["remote"], r["a"], r["b"]) == r["repair"]
        m = r["limit"]
        if m:
            assert r["b"] * (r["remote"] + m) < r["a"] * (r["local"] - m)
        assert not (r["b"] * (r["remote"] + m + 1) < r["a"] * (r["local"] - m - 1))
