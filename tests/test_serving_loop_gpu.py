"""A small serving loop through the public pieces, driven the way the reference's backend drives them
(peer/backend.py, peer/prefill_backend.py, peer/policy.py, peer/staging.py): a prefill of three
requests (K/V written by the native KV writer); FIFO migration of their oldest positions to two
supplier banks (TierManager + CudaCopier), launched early and left in flight across an extend
forward; a second extend whose
history is partly remote, read both in place and through the LayerStager (copy-engine ranges from
TierManager.remote_row_ranges); then a decode step.  Every attention output is checked against the
fp32 oracle over the logical K/V the loop wrote, the staged and in-place appends are bit-identical,
and the manager's audit holds after every step."""
import numpy as np
import pytest
import torch

from dual_b200 import ops
from dual_b200.migration import CudaCopier, TierManager
from dual_b200.remote_bank import RemoteBank, local_plane_pointers
from dual_b200.staging import LayerStager
from dual_b200.wrapper import BatchDecodeWithPagedKVCacheWrapper, BatchPrefillWithPagedKVCacheWrapper
from oracle import attention as OA

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2
LAYERS, CAP, BANKS, BANK_SLOTS, MAXCTX = 2, 4096, 2, 1024, 2048
SCALE = 128 ** -0.5


class Loop:
    def __init__(self):
        self.dev = torch.device("cuda:0")
        self.g = torch.Generator(device=self.dev).manual_seed(31)
        d = self.dev
        self.kv = [(torch.zeros((CAP + 1, 8, 128), dtype=torch.bfloat16, device=d),
                    torch.zeros((CAP + 1, 8, 128), dtype=torch.bfloat16, device=d)) for _ in range(LAYERS)]
        self.bank = RemoteBank([torch.zeros((LAYERS, 2, BANK_SLOTS, 8, 128), dtype=torch.bfloat16, device=d)
                                for _ in range(BANKS)], layers=LAYERS)
        self.status = torch.zeros(1, dtype=torch.int32, device=d)
        copier = CudaCopier(local_plane_pointers(self.kv, d), self.bank.pointers, 2 * LAYERS, BANKS, CAP + 1,
                            BANK_SLOTS, self.status)
        self.tier = torch.full((4, MAXCTX), -1, dtype=torch.int32, device=d)
        self.slot = torch.zeros_like(self.tier)
        self.m = TierManager(self.tier, self.slot, CAP, BANKS * BANK_SLOTS, 1797, 10000, copier,
                             migration_tokens=512)
        # logical K/V of every (request, position), wherever it lives
        self.logical = [[torch.zeros((4, MAXCTX, 8, 128), dtype=torch.bfloat16, device=d) for _ in range(2)]
                        for _ in range(LAYERS)]

    def write(self, rid, n):
        """A forward's new positions: local slots from the manager, K/V written by the native writer
        (SGLang's set_kv_buffer in the reference) from a fused qkv buffer, as the model would."""
        start = self.m.live.get(rid, 0)
        s = torch.tensor(self.m.append(rid, n), dtype=torch.long, device=self.dev)
        for layer in range(LAYERS):
            qkv = torch.empty((n, 6144), dtype=torch.bfloat16, device=self.dev).normal_(generator=self.g)
            k, v = qkv[:, 4096:5120].view(n, 8, 128), qkv[:, 5120:].view(n, 8, 128)
            ops.set_kv_buffer(self.kv[layer][0], self.kv[layer][1], s, k, v, self.status)
            self.logical[layer][0][rid, start:start + n] = k
            self.logical[layer][1][rid, start:start + n] = v

    def full_list(self, rids, lengths, prefixes=None):
        d = self.dev
        full = torch.empty(sum(lengths), dtype=torch.int32, device=d)
        pre = None if prefixes is None else torch.tensor(prefixes, dtype=torch.int32, device=d)
        ops.pack_read_order(self.tier, self.slot, torch.tensor(rids, dtype=torch.int32, device=d),
                            torch.tensor(lengths, dtype=torch.int32, device=d), CAP, 5, 32, full, prefix_lens=pre)
        return full

    def queries(self, n):
        return torch.empty((n, 32, 128), dtype=torch.bfloat16, device=self.dev).normal_(generator=self.g)

    def check(self, layer, out, lse, q, rids, lengths, qlens):
        off = 0
        for rid, L, ql in zip(rids, lengths, qlens):
            ref, ref_lse = OA.attend(q[off:off + ql].cpu(), self.logical[layer][0][rid, :L].cpu(),
                                     self.logical[layer][1][rid, :L].cpu(), L - ql, SCALE)
            torch.testing.assert_close(out[off:off + ql].float().cpu(), ref, atol=ATOL, rtol=RTOL)
            torch.testing.assert_close(lse[off:off + ql].cpu(), ref_lse, atol=ATOL, rtol=RTOL)
            off += ql

    def prefill(self, rids, qlens, stager=None):
        """One extend forward of every layer through the prefill wrapper; returns [(out, lse)] per layer."""
        lengths = [self.m.live[r] for r in rids]
        prefixes = [L - q for L, q in zip(lengths, qlens)]
        full = self.full_list(rids, lengths, prefixes)
        q = self.queries(sum(qlens))
        w = BatchPrefillWithPagedKVCacheWrapper(torch.empty(1 << 20, dtype=torch.uint8, device=self.dev), "NHD")
        qo = torch.tensor(np.concatenate([[0], np.cumsum(qlens)]), dtype=torch.int32)
        kvp = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32)
        w.plan(qo, kvp, full, torch.ones(len(rids), dtype=torch.int32), 32, 8, 128, 1, causal=True,
               q_data_type=torch.bfloat16)
        results = []
        if stager is not None:
            stager.start(full, CAP, row_ranges=self.m.remote_row_ranges(BANKS))
        for layer in range(LAYERS):
            tail = self.bank.layer(layer) if stager is None else stager.tail(layer)
            k, v = self.kv[layer]
            results.append(w.run_return_lse(q, (k.unsqueeze(1), v.unsqueeze(1)), *tail, full, CAP, SCALE))
            if stager is not None:
                stager.next(layer)
        torch.cuda.synchronize()
        assert w.status() == 0
        for layer, (out, lse) in enumerate(results):
            self.check(layer, out, lse, q, rids, lengths, qlens)
        return results


def test_prefill_migrate_extend_staged_and_decode():
    lp = Loop()
    m, rids = lp.m, [0, 1, 2]

    # forward 1: prompts, all local
    m.begin_forward()
    for rid, n in zip(rids, (1200, 800, 500)):
        lp.write(rid, n)
    lp.prefill(rids, [1200, 800, 500])
    m.audit()

    # forward 2: the forward's slots are allocated first, then the migration of older positions is
    # launched (peer/policy.py launch) and stays in flight during the extend's attention
    m.begin_forward()
    for rid, n in zip(rids, (100, 64, 32)):
        lp.write(rid, n)
    pending = m.submit(asynchronous=True)
    assert pending is not None
    lp.prefill(rids, [100, 64, 32])

    # step boundary: commit before the next forward allocates (the reference's transport order);
    # the history of request 0 is now partly remote
    assert m.wait(10.0)
    m.commit()
    m.begin_forward()
    info = m.audit()
    assert info["remote_active_tokens"] > 0 and int(lp.status.item()) == 0
    assert int((lp.tier[0] == 1).sum()) > 0
    for rid, n in zip(rids, (48, 16, 80)):
        lp.write(rid, n)
    in_place = lp.prefill(rids, [48, 16, 80])
    # the same forward again (same q: re-seed), history staged into local buffers by the copy engines
    lp.g.manual_seed(99)
    stager = LayerStager.from_bank(lp.bank, lp.dev, depth=2, mode="range")
    staged = lp.prefill(rids, [48, 16, 80], stager=stager)
    lp.g.manual_seed(99)
    again = lp.prefill(rids, [48, 16, 80])
    for (o1, l1), (o2, l2) in zip(staged, again):
        assert torch.equal(o1, o2) and torch.equal(l1, l2)
    assert len(in_place) == LAYERS
    m.audit()

    # forward 4: one decode token per request
    m.begin_forward()
    for rid in rids:
        lp.write(rid, 1)
    lengths = [m.live[r] for r in rids]
    idx = lp.full_list(rids, lengths)
    q = lp.queries(len(rids))
    w = BatchDecodeWithPagedKVCacheWrapper(torch.empty(64 << 20, dtype=torch.uint8, device=lp.dev), "NHD",
                                           use_tensor_cores=True)
    indptr = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32)
    w.plan(indptr, idx, torch.ones(len(rids), dtype=torch.int32), 32, 8, 128, 1)
    for layer in range(LAYERS):
        k, v = lp.kv[layer]
        out, lse = w.run_return_lse(q, (k.unsqueeze(1), v.unsqueeze(1)), *lp.bank.layer(layer), idx, CAP, SCALE)
        torch.cuda.synchronize()
        lp.check(layer, out, lse, q, rids, lengths, [1] * len(rids))
    m.audit()
