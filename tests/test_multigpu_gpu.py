"""Remote tier across GPUs: supplier banks in another GPU's HBM, read by the decode kernel with
peer loads, written by the migration kernel with peer stores, mapped in-process (peer access)
or across processes (CUDA IPC handshake).  Needs >= 2 GPUs; skipped otherwise."""
import multiprocessing as mp

import numpy as np
import pytest
import torch

import cases as C
from dual_b200 import ipc, ops, topology
from dual_b200.migration import CudaCopier, TierManager
from dual_b200.remote_bank import RemoteBank, local_plane_pointers
from oracle import attention as OA

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]
ATOL, RTOL = 2e-3, 1e-2


def _decode(q, k, v, pk, pv, lengths, tier, slot, requests, capacity):
    dev = q.device
    req = torch.tensor(requests, dtype=torch.int32, device=dev)
    seq = torch.tensor(lengths, dtype=torch.int32, device=dev)
    idx = torch.empty(sum(lengths), dtype=torch.int32, device=dev)
    ops.pack_read_order(tier, slot, req, seq, capacity, 5, 32, idx)
    indptr = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    lse = torch.empty((q.shape[0], 32), dtype=torch.float32, device=dev)
    ws = torch.zeros(ops.decode_workspace_size(q.shape[0], ops.default_ctas(dev.index)), dtype=torch.uint8,
                     device=dev)
    ops.tiered_decode(q, k, v, capacity, pk, pv, indptr, idx, 128 ** -0.5, out, lse, ws)
    torch.cuda.synchronize(dev)
    return out, lse, indptr, idx, ws


def test_topology_of_this_box():
    topo = topology.discover()
    n = torch.cuda.device_count()
    assert len(topo.gpus) >= n
    topo.check_suppliers(0, list(range(1, n)))


@pytest.mark.parametrize("banks", [1, 3])
def test_decode_reads_supplier_banks_on_peer_gpus(banks):
    n = torch.cuda.device_count()
    for d in range(1, n):
        topology.enable_peer(0, d)
    case = C.config1(banks=banks)
    d0 = torch.device("cuda:0")
    owners = [torch.device(f"cuda:{1 + (i % (n - 1))}") for i in range(banks)]
    pk = [t.to(o) for t, o in zip(case.peer_k, owners)]
    pv = [t.to(o) for t, o in zip(case.peer_v, owners)]
    out, lse, indptr, idx, ws = _decode(case.decode_q().to(d0), case.k_local.to(d0), case.v_local.to(d0), pk, pv,
                                        case.lengths, case.tier.to(d0), case.slot.to(d0), case.requests,
                                        case.local_capacity)
    ref, ref_lse = OA.decode_from_indices(case.decode_q(), case.k_local, case.v_local, case.peer_k, case.peer_v,
                                          indptr.cpu().tolist(), idx.cpu(), case.local_capacity)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse.cpu(), ref_lse, atol=ATOL, rtol=RTOL)
    assert int(ws[:4].view(torch.int32).item()) == 0


def test_migration_to_peer_gpu_async_bit_exact():
    topology.enable_peer(0, 1)
    d0, d1 = torch.device("cuda:0"), torch.device("cuda:1")
    layers, cap, bank_slots = 4, 8192, 2048
    g = torch.Generator(device=d0).manual_seed(5)
    kv = [(torch.randn((cap + 1, 8, 128), generator=g, device=d0).to(torch.bfloat16),
           torch.randn((cap + 1, 8, 128), generator=g, device=d0).to(torch.bfloat16)) for _ in range(layers)]
    bank = RemoteBank([torch.zeros((layers, 2, bank_slots, 8, 128), dtype=torch.bfloat16, device=d1)], layers=layers)
    ptrs = bank.pointers.to(d0)
    status = torch.zeros(1, dtype=torch.int32, device=d0)
    copier = CudaCopier(local_plane_pointers(kv, d0), ptrs, 2 * layers, 1, cap + 1, bank_slots, status)
    tier = torch.full((2, 6000), -1, dtype=torch.int32, device=d0)
    slot = torch.zeros_like(tier)
    m = TierManager(tier, slot, cap, bank_slots, 1797, 10000, copier, migration_tokens=1024)
    m.begin_forward()
    m.append(0, 5000)
    m.append(1, 2000)
    m.begin_forward()
    p = m.submit(asynchronous=True)
    assert m.wait(10.0)
    src, tgt = p.source.clone(), p.target.clone()
    m.commit()
    torch.cuda.synchronize(d0)
    assert int(status.item()) == 0
    for layer in range(layers):
        for plane in range(2):
            got = bank.banks[0][layer, plane].index_select(0, tgt.to(d1)).to(d0)
            assert torch.equal(got.view(torch.int16), kv[layer][plane].index_select(0, src).view(torch.int16))
    m.audit()


def _ipc_supplier(conn, device, layers, slots):
    torch.cuda.set_device(device)
    ipc.serve_supplier(ipc.PipeChannel(conn), 0, device, layers, slots, timeout=120, close_timeout=300)


def test_ipc_supplier_process_decode_and_migrate():
    """A separate supplier process owns the bank on GPU 1; the compute side imports it by CUDA IPC
    (probe handshake), writes remote rows through the mapping, decodes against the oracle, and
    migrates local slots into it with the copy kernel."""
    ctx = mp.get_context("spawn")
    a, b = ctx.Pipe()
    layers, slots = 2, 4096
    proc = ctx.Process(target=_ipc_supplier, args=(b, 1, layers, slots))
    proc.start()
    try:
        bank, ptrs = ipc.open_suppliers([ipc.PipeChannel(a)], 0, layers, slots, timeout=180)
        case = C.config1(banks=1)
        d0 = torch.device("cuda:0")
        n_remote = case.peer_k[0].shape[0]
        bank.banks[0][0, 0, :n_remote].copy_(case.peer_k[0].to(d0))
        bank.banks[0][0, 1, :n_remote].copy_(case.peer_v[0].to(d0))
        out, lse, indptr, idx, ws = _decode(case.decode_q().to(d0), case.k_local.to(d0), case.v_local.to(d0),
                                            [bank.banks[0][0, 0]], [bank.banks[0][0, 1]], case.lengths,
                                            case.tier.to(d0), case.slot.to(d0), case.requests, case.local_capacity)
        ref, _ = OA.decode_from_indices(case.decode_q(), case.k_local, case.v_local, case.peer_k, case.peer_v,
                                        indptr.cpu().tolist(), idx.cpu(), case.local_capacity)
        torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
        # migration into the imported bank
        kv = [(case.k_local.to(d0), case.v_local.to(d0)) for _ in range(layers)]
        status = torch.zeros(1, dtype=torch.int32, device=d0)
        src = torch.arange(1, 301, dtype=torch.int64, device=d0)
        dst = torch.arange(1000, 1300, dtype=torch.int64, device=d0)
        ops.migrate_copy(local_plane_pointers(kv, d0), bank.pointers, 2 * layers, 1, src, dst, False,
                         case.local_capacity + 1, slots, status)
        torch.cuda.synchronize(d0)
        assert int(status.item()) == 0
        assert torch.equal(bank.banks[0][1, 0, 1000:1300].view(torch.int16),
                           kv[1][0][1:301].view(torch.int16))
        ipc.close_suppliers([ipc.PipeChannel(a)], 0, ptrs, timeout=120)
    finally:
        proc.join(180)
        if proc.is_alive():
            proc.kill()
    assert proc.exitcode == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_kernels_launch_on_every_device_of_one_process():
    """Kernel attributes (the large dynamic shared-memory limit) belong to each device's context:
    decode and append must launch on a second GPU after the first, in the same process."""
    case = C.config1(banks=3)
    for dev_i in (0, 1):
        d = torch.device(f"cuda:{dev_i}")
        with torch.cuda.device(d):
            tier, slot = case.tier.to(d), case.slot.to(d)
            req = torch.tensor(case.requests, dtype=torch.int32, device=d)
            seq = torch.tensor(case.lengths, dtype=torch.int32, device=d)
            idx = torch.empty(sum(case.lengths), dtype=torch.int32, device=d)
            ops.pack_read_order(tier, slot, req, seq, case.local_capacity, 5, 32, idx)
            indptr = torch.tensor(np.concatenate([[0], np.cumsum(case.lengths)]), dtype=torch.int32, device=d)
            k, v = case.k_local.to(d), case.v_local.to(d)
            pk, pv = [t.to(d) for t in case.peer_k], [t.to(d) for t in case.peer_v]
            q = case.decode_q().to(d)
            out = torch.empty((4, 32, 128), dtype=torch.bfloat16, device=d)
            lse = torch.empty((4, 32), dtype=torch.float32, device=d)
            ws = torch.zeros(ops.decode_workspace_size(4, ops.default_ctas(dev_i)), dtype=torch.uint8, device=d)
            ops.tiered_decode(q, k, v, case.local_capacity, pk, pv, indptr, idx, 128 ** -0.5, out, lse, ws)
            qo = np.arange(5, dtype=np.int32)
            kv = np.concatenate([[0], np.cumsum(case.lengths)]).astype(np.int32)
            work = ops.append_plan(qo, kv, True).to(d)
            out_a = torch.empty_like(q)
            lse_a = torch.empty((4, 32), dtype=torch.float32, device=d)
            status = torch.zeros(1, dtype=torch.int32, device=d)
            ops.tiered_append(q, k, v, case.local_capacity, pk, pv, torch.from_numpy(qo).to(d),
                              torch.from_numpy(kv).to(d), idx, True, 128 ** -0.5, work, out_a, lse_a, status)
            torch.cuda.synchronize(d)
        ref, ref_lse = OA.decode_from_indices(case.decode_q(), case.k_local, case.v_local, case.peer_k, case.peer_v,
                                              indptr.cpu().tolist(), idx.cpu(), case.local_capacity)
        torch.testing.assert_close(out.float().cpu(), ref, atol=2e-3, rtol=1e-2)
        # one query token per request with the whole list visible: the append equals the decode
        torch.testing.assert_close(out_a.float().cpu(), ref, atol=2e-3, rtol=1e-2)
        torch.testing.assert_close(lse_a.cpu(), ref_lse, atol=2e-3, rtol=1e-2)
        assert int(status.item()) == 0 and int(ws[:4].view(torch.int32).item()) == 0


def test_native_supplier_process_decode(tmp_path):
    """The native supplier executable owns the bank on GPU 1 (cudaMalloc + cudaIpcGetMemHandle);
    the compute side imports it through the same handshake, decodes against the oracle, and the
    supplier frees the bank and exits 0 after close."""
    layers, slots = 1, 4096
    proc, ch = ipc.spawn_native_supplier(tmp_path / "sup.sock", 0, 1, layers, slots, backend="cuda", timeout=120.0)
    try:
        bank, ptrs = ipc.open_suppliers([ch], 0, layers, slots, timeout=120)
        case = C.config1(banks=1)
        d0 = torch.device("cuda:0")
        n_remote = case.peer_k[0].shape[0]
        bank.banks[0][0, 0, :n_remote].copy_(case.peer_k[0].to(d0))
        bank.banks[0][0, 1, :n_remote].copy_(case.peer_v[0].to(d0))
        out, lse, indptr, idx, ws = _decode(case.decode_q().to(d0), case.k_local.to(d0), case.v_local.to(d0),
                                            [bank.banks[0][0, 0]], [bank.banks[0][0, 1]], case.lengths,
                                            case.tier.to(d0), case.slot.to(d0), case.requests, case.local_capacity)
        ref, _ = OA.decode_from_indices(case.decode_q(), case.k_local, case.v_local, case.peer_k, case.peer_v,
                                        indptr.cpu().tolist(), idx.cpu(), case.local_capacity)
        torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
        ipc.close_suppliers([ch], 0, ptrs, timeout=120)
        assert proc.wait(timeout=120) == 0
    finally:
        if proc.poll() is None:
            proc.kill()
            proc.wait()
