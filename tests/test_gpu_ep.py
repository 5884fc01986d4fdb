"""Expert-parallel block on GPUs: the segment GEMM entry point on one GPU,
and the NCCL expert-parallel block on two GPUs against the single-GPU block."""

import os
import socket

import numpy as np
import pytest
import torch

import oracle
from nki_moe_b200 import _lib, ops
from nki_moe_b200.workloads import WORKLOADS, make_moe_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda_env():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    old = os.environ.get("NKIMOE_SYNC_CHECK")
    os.environ["NKIMOE_SYNC_CHECK"] = "1"
    _lib.load()
    yield
    if old is None:
        os.environ.pop("NKIMOE_SYNC_CHECK", None)
    else:
        os.environ["NKIMOE_SYNC_CHECK"] = old


@pytest.mark.parametrize("schedule", [0, 1, 2])
def test_segment_experts_matches_oracle(schedule):
    """Segments ordered (source rank, local expert), expert = segment % E_local,
    as an all-to-all delivers them; some segments empty."""
    _lib.set_option("gemm_schedule", schedule)
    try:
        g = torch.Generator().manual_seed(3)
        H, I, El, P = 256, 128, 4, 3
        counts = torch.randint(0, 90, (P * El,), generator=g)
        counts[1] = 0
        counts[7] = 0
        R = int(counts.sum())
        a = torch.randn(R, H, generator=g).to(torch.bfloat16)
        rw = torch.rand(R, generator=g)
        gu = (torch.randn(El, H, 2 * I, generator=g) * 0.05).to(torch.bfloat16)
        dn = (torch.randn(El, I, H, generator=g) * 0.05).to(torch.bfloat16)
        pe = ops.packed_experts(gu.cuda(), dn.cuda(), "nxd")
        y = ops.segment_experts(a.cuda(), rw.cuda(), counts.to(torch.int32).cuda(), pe).float().cpu().numpy()
        ref = np.zeros((R, H), np.float32)
        o = 0
        for s, c in enumerate(counts.tolist()):
            if c:
                e = s % El
                ref[o:o + c] = rw[o:o + c, None].numpy() * oracle.expert_ffn(
                    a[o:o + c].float().numpy(), gu[e].float().numpy(), dn[e].float().numpy())
            o += c
        assert oracle.normwise_rel_err(y, ref) < 2e-2 and oracle.cosine(y, ref) > 0.999
    finally:
        _lib.set_option("gemm_schedule", 0)


def test_route_dispatch_combine_roundtrip():
    """dispatch then combine with unit rows weights reproduces sum_k x[t] (a
    size-independent property of the permutation pair)."""
    g = torch.Generator().manual_seed(5)
    T, H, E, K = 1000, 256, 16, 4
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).cuda()
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32).cuda()
    w = torch.ones(T, K, device="cuda")
    x_perm, row_w, slot_row, counts = ops.dispatch(x, idx, w, E)
    assert int(counts.sum()) == T * K
    out = ops.combine(x_perm, slot_row, T, K).float()
    np.testing.assert_allclose(out.cpu().numpy(), (K * x.float()).cpu().numpy(), rtol=1e-2, atol=1e-2)
    assert torch.equal(x_perm[slot_row.long()].view(T, K, H)[:, 0], x)


def test_ep_dispatch_matches_oracle():
    g = torch.Generator().manual_seed(9)
    T, H, E, K, P = 300, 256, 32, 8, 4
    el = E // P
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32)
    w = torch.rand(T, K, generator=g)
    xs, slots, wts, counts, slot_row = ops.ep_dispatch(x.cuda(), idx.cuda(), w.cuda(), P, el)
    dest = np.full((T, P), -1, np.int32)
    for t in range(T):
        for e in idx[t].tolist():
            dest[t, e // el] = e // el
    row_t, row_slot, offsets, ref_slot_row = oracle.permute(dest, P)
    n = int(offsets[-1])
    assert np.array_equal(counts.cpu().numpy(), np.diff(offsets))
    assert np.array_equal(slot_row.cpu().numpy().ravel(), ref_slot_row)
    assert torch.equal(xs[:n].cpu(), x[torch.from_numpy(row_t).long()])
    d_of = row_slot % P
    ids = idx.numpy()[row_t]
    local = (ids // el) == d_of[:, None]
    assert np.array_equal(slots[:n].cpu().numpy(), np.where(local, ids - d_of[:, None] * el, -1))
    assert np.array_equal(wts[:n].cpu().numpy(), np.where(local, w.numpy()[row_t], 0.0).astype(np.float32))


def test_given_routing_block_skips_empty_slots():
    g = torch.Generator().manual_seed(13)
    T, H, I, E, K = 200, 256, 128, 8, 4
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32)
    idx[torch.rand(T, K, generator=g) < 0.4] = -1
    w = torch.rand(T, K, generator=g)
    gu = (torch.randn(E, H, 2 * I, generator=g) * 0.05).to(torch.bfloat16)
    dn = (torch.randn(E, I, H, generator=g) * 0.05).to(torch.bfloat16)
    pe = ops.packed_experts(gu.cuda(), dn.cuda(), "nxd")
    out = ops.moe_experts(x.cuda(), pe, idx.cuda(), w.cuda()).float().cpu().numpy()
    ref = oracle.experts_forward(x.float().numpy(), gu.float().numpy(), dn.float().numpy(), idx.numpy(), w.numpy())
    assert oracle.normwise_rel_err(out, ref) < 2e-2 and oracle.cosine(out, ref) > 0.999


@pytest.mark.parametrize("overlap", [1, 0, 2])
def test_peer_ep_single_rank_equals_block(overlap):
    """The peer-memory EP block as a single rank equals the single-GPU block bit
    for bit, step after step: in the overlapped schedule (its own tokens'
    block straight from x) and in the one-block schedule (rows sent to itself,
    epoch flags, masking of rows left from an earlier, larger step)."""
    _lib.set_option("ep_overlap", overlap)
    from nki_moe_b200.ep_peer import PeerExpertParallelMoE
    from nki_moe_b200.nki_moe_integrated import NKIMoESimple

    wl = WORKLOADS["c3"]
    inp = make_moe_inputs(wl, device="cuda", tokens=1024)
    moe = NKIMoESimple(wl.hidden, wl.intermediate, wl.experts, wl.top_k, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        moe.router.weight.copy_(inp["router"])
        moe.gate_up_proj.copy_(inp["gate_up"].to(torch.bfloat16))
        moe.down_proj.copy_(inp["down"].to(torch.bfloat16))
    peer = PeerExpertParallelMoE.from_dense(moe, max_tokens=1024)
    try:
        for step, T in enumerate((1024, 600, 1024)):
            x = torch.randn(T, wl.hidden, generator=torch.Generator(device="cuda").manual_seed(70 + step),
                            device="cuda").to(torch.bfloat16)
            y = peer(x)
            assert ops.read_status(ops.workspace(x.device, 1)) == 0  # no bounded wait ran out
            ref = ops.moe_block(x, moe.router.weight, moe.packed(), wl.top_k)
            assert torch.equal(y, ref), f"step {step}: max diff {(y.float() - ref.float()).abs().max().item()}"
    finally:
        peer.close()
        _lib.set_option("ep_overlap", -1)


@pytest.mark.parametrize("overlap", [0, 2])
def test_peer_ep_single_rank_with_replica_slots_equals_block(overlap):
    """Hot-expert replica slots through the mapped exchange on a single rank:
    the rank holds two extra slots with copies of the two busiest experts of a
    routing sample, and the remap sends every other token of those experts to
    the copy (t mod 2).  Each (token, slot) row is the same arithmetic whichever
    slot computes it and the rank's sum runs over a token's slots in k order,
    so the output equals the single-GPU block bit for bit."""
    _lib.set_option("ep_overlap", overlap)
    from nki_moe_b200.ep_peer import PeerExpertParallelMoE, expert_load
    from nki_moe_b200.nki_moe_integrated import NKIMoESimple

    wl = WORKLOADS["c3"]
    inp = make_moe_inputs(wl, device="cuda", tokens=1024)
    moe = NKIMoESimple(wl.hidden, wl.intermediate, wl.experts, wl.top_k, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        moe.router.weight.copy_(inp["router"])
        moe.gate_up_proj.copy_(inp["gate_up"].to(torch.bfloat16))
        moe.down_proj.copy_(inp["down"].to(torch.bfloat16))
    E = wl.experts
    _, idx0, _ = ops.moe_block(inp["x"].to(torch.bfloat16), moe.router.weight, moe.packed(), wl.top_k,
                               return_routing=True)
    load = expert_load(idx0, E)
    hot = sorted(range(E), key=lambda e: (-load[e], e))[:2]
    slot_experts = [list(range(E)) + hot]
    holders = [[e] for e in range(E)]
    holders[hot[0]].append(E)
    holders[hot[1]].append(E + 1)
    sel = torch.tensor(slot_experts[0], dtype=torch.long, device="cuda")
    peer = PeerExpertParallelMoE(moe.router.weight, moe.gate_up_proj.detach().index_select(0, sel).contiguous(),
                                 moe.down_proj.detach().index_select(0, sel).contiguous(), E, wl.top_k, 1024,
                                 replicas=(slot_experts, holders))
    try:
        for step, T in enumerate((1024, 600)):
            x = torch.randn(T, wl.hidden, generator=torch.Generator(device="cuda").manual_seed(80 + step),
                            device="cuda").to(torch.bfloat16)
            y, idx, _ = peer(x, return_routing=True)
            assert ops.read_status(ops.workspace(x.device, 1)) == 0
            ref, ridx, _ = ops.moe_block(x, moe.router.weight, moe.packed(), wl.top_k, return_routing=True)
            assert torch.equal(idx, ridx)  # the real expert ids come back
            assert bool((idx == hot[0]).any()) and bool((idx == hot[1]).any())
            assert torch.equal(y, ref), f"step {step}: max diff {(y.float() - ref.float()).abs().max().item()}"
    finally:
        peer.close()
        _lib.set_option("ep_overlap", -1)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ep_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    from nki_moe_b200.ep import ExpertParallelMoE
    from nki_moe_b200.nki_moe_integrated import NKIMoESimple
    from nki_moe_b200.workloads import WORKLOADS, make_moe_inputs
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    wl = WORKLOADS["c3"]
    inp = make_moe_inputs(wl, device="cuda", tokens=1024)
    moe = NKIMoESimple(wl.hidden, wl.intermediate, wl.experts, wl.top_k, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        moe.router.weight.copy_(inp["router"])
        moe.gate_up_proj.copy_(inp["gate_up"].to(torch.bfloat16))
        moe.down_proj.copy_(inp["down"].to(torch.bfloat16))
    x = (torch.randn(1024, wl.hidden, generator=torch.Generator(device="cuda").manual_seed(50 + rank),
                     device="cuda")).to(torch.bfloat16)
    y_dedup = ExpertParallelMoE.from_dense(moe, dedup=True)(x)
    y_ep = ExpertParallelMoE.from_dense(moe, dedup=False)(x)
    y_one = ops.moe_block(x, moe.router.weight, moe.packed(), wl.top_k)
    # peer-memory exchange: two steps (the second with fewer tokens on rank 1)
    from nki_moe_b200.ep_peer import PeerExpertParallelMoE
    peer = PeerExpertParallelMoE.from_dense(moe, max_tokens=1024)
    x2 = x[: 1024 if rank == 0 else 700].flip(0).contiguous()
    y_peer1 = peer(x)
    y_peer2 = peer(x2)
    assert ops.read_status(ops.workspace(x.device, 1)) == 0  # no bounded wait ran out
    # the one-block schedule, then back to the overlapped one; a rank may take
    # either schedule whatever the other takes
    _lib.set_option("ep_overlap", 0)
    y_peer1b = peer(x)
    _lib.set_option("ep_overlap", 2 * (rank % 2))
    y_peer2b = peer(x2)
    _lib.set_option("ep_overlap", 2)
    y_peer2c = peer(x2)
    _lib.set_option("ep_overlap", -1)
    assert ops.read_status(ops.workspace(x.device, 1)) == 0
    y_dedup2 = ExpertParallelMoE.from_dense(moe, dedup=True)(x2)
    torch.cuda.synchronize()
    # rank 1 leaves a step (host side, between steps): rank 0's waits run out
    # after a short budget and its step raises; after a resync both ranks'
    # next step is correct again
    timed_out = 0
    if rank == 0:
        _lib.set_option("peer_wait_cycles", 4_000_000)
        try:
            peer(x)
            ops.read_status(ops.workspace(x.device, 1))
        except _lib.NKIMoEError as e:
            timed_out = int(e.code == _lib.ERR_DEVICE and "0x1" in str(e))
        finally:
            _lib.set_option("peer_wait_cycles", 20_000_000_000)
    torch.cuda.synchronize()
    dist.barrier()
    peer.resync()
    y_peer3 = peer(x2)
    assert ops.read_status(ops.workspace(x.device, 1)) == 0
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"peer3_{rank}.npy"), y_peer3.float().cpu().numpy())
    np.save(os.path.join(out_dir, f"peer1b_{rank}.npy"), y_peer1b.float().cpu().numpy())
    np.save(os.path.join(out_dir, f"peer2b_{rank}.npy"), y_peer2b.float().cpu().numpy())
    np.save(os.path.join(out_dir, f"peer2c_{rank}.npy"), y_peer2c.float().cpu().numpy())
    np.save(os.path.join(out_dir, f"timeout{rank}.npy"), np.array([timed_out]))
    peer.close()
    np.save(os.path.join(out_dir, f"peer{rank}.npy"), y_peer1.float().cpu().numpy())
    np.save(os.path.join(out_dir, f"peer2_{rank}.npy"), y_peer2.float().cpu().numpy())
    np.save(os.path.join(out_dir, f"dedup2_{rank}.npy"), y_dedup2.float().cpu().numpy())
    np.save(os.path.join(out_dir, f"dedup{rank}.npy"), y_dedup.float().cpu().numpy())
    np.save(os.path.join(out_dir, f"ep{rank}.npy"), y_ep.float().cpu().numpy())
    np.save(os.path.join(out_dir, f"one{rank}.npy"), y_one.float().cpu().numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_expert_parallel_two_gpus_matches_single_gpu(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_ep_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        a = np.load(tmp_path / f"ep{r}.npy")
        b = np.load(tmp_path / f"one{r}.npy")
        # one row per (token, slot): every output row is the same per-row
        # arithmetic as on one GPU
        assert np.array_equal(a, b), f"rank {r}: max diff {np.abs(a - b).max()}"
        # de-duplicated: per-rank partial sums are rounded to bf16 before the
        # final sum, so the block-output tolerance applies
        d = np.load(tmp_path / f"dedup{r}.npy")
        assert oracle.normwise_rel_err(d, b) < 2e-2 and oracle.cosine(d, b) > 0.999
        # the peer-memory exchange computes exactly what the NCCL de-duplicated
        # exchange computes (same rows, same order, same sums)
        assert np.array_equal(np.load(tmp_path / f"peer{r}.npy"), d), f"rank {r}: peer != dedup"
        assert np.array_equal(np.load(tmp_path / f"peer2_{r}.npy"), np.load(tmp_path / f"dedup2_{r}.npy"))
        # the one-block schedule and a mix of schedules across the ranks
        assert np.array_equal(np.load(tmp_path / f"peer1b_{r}.npy"), d)
        assert np.array_equal(np.load(tmp_path / f"peer2b_{r}.npy"), np.load(tmp_path / f"dedup2_{r}.npy"))
        assert np.array_equal(np.load(tmp_path / f"peer2c_{r}.npy"), np.load(tmp_path / f"dedup2_{r}.npy"))
        # after rank 1 left a step and the ranks resynchronised
        assert np.array_equal(np.load(tmp_path / f"peer3_{r}.npy"), np.load(tmp_path / f"dedup2_{r}.npy"))
    assert int(np.load(tmp_path / "timeout0.npy")[0]) == 1  # rank 0's step raised the wait timeout


def _replica_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    from nki_moe_b200.ep_peer import PeerExpertParallelMoE, expert_load
    from nki_moe_b200.nki_moe_integrated import NKIMoESimple
    from nki_moe_b200.workloads import WORKLOADS, make_moe_inputs
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    wl = WORKLOADS["c4"]  # Zipf(1.2) router bias: a few experts take most rows
    inp = make_moe_inputs(wl, device="cuda", tokens=2048)
    moe = NKIMoESimple(wl.hidden, wl.intermediate, wl.experts, wl.top_k, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        moe.router.weight.copy_(inp["router"])
        moe.gate_up_proj.copy_(inp["gate_up"].to(torch.bfloat16))
        moe.down_proj.copy_(inp["down"].to(torch.bfloat16))
    moe.router_bias = inp["router_bias"]
    rw, rb, pe = moe.router.weight, moe.router_bias, moe.packed()
    x_cal = torch.randn(1024, wl.hidden, generator=torch.Generator(device="cuda").manual_seed(90 + rank),
                        device="cuda").to(torch.bfloat16)
    _, idx_cal, _ = ops.moe_block(x_cal, rw, pe, wl.top_k, bias=rb, return_routing=True)
    load = expert_load(idx_cal, wl.experts)
    peer = PeerExpertParallelMoE.from_dense(moe, max_tokens=1024, extra_slots=2, expected_load=load)
    x = inp["x"].to(torch.bfloat16).view(world, 1024, wl.hidden)[rank].contiguous()
    ref, ridx, _ = ops.moe_block(x, rw, pe, wl.top_k, bias=rb, return_routing=True)
    outs = []
    for overlap in (0, 2, -1):
        _lib.set_option("ep_overlap", overlap)
        y, idx, _ = peer(x, return_routing=True)
        outs.append(y)
        assert torch.equal(idx, ridx)
    _lib.set_option("ep_overlap", -1)
    status = ops.read_status(ops.workspace(x.device, 1))
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"rep_ref{rank}.npy"), ref.float().cpu().numpy())
    for i, y in enumerate(outs):
        np.save(os.path.join(out_dir, f"rep{i}_{rank}.npy"), y.float().cpu().numpy())
    np.save(os.path.join(out_dir, f"rep_meta{rank}.npy"),
            np.array([status, sum(len(h) - 1 for h in peer.replicas[1]), peer.local_slots]))
    peer.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_expert_parallel_two_gpus_with_hot_expert_replicas(tmp_path):
    """Skewed routing (Zipf router bias) over two ranks with two replica slots
    each, planned from a calibration batch: the one-block and copy-engine
    schedules give the same output, which meets the block bar against the
    single-GPU block with identical routing (the real expert ids)."""
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_replica_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        status, copies, local_slots = np.load(tmp_path / f"rep_meta{r}.npy")
        assert status == 0 and copies >= 1 and local_slots == 64 + 2
        ref = np.load(tmp_path / f"rep_ref{r}.npy")
        ys = [np.load(tmp_path / f"rep{i}_{r}.npy") for i in range(3)]
        for y in ys:
            assert oracle.normwise_rel_err(y, ref) < 2e-2 and oracle.cosine(y, ref) > 0.999
            assert np.array_equal(y, ys[0])  # every schedule computes the same sums


def test_peer_wait_runs_out_when_a_peer_never_joins():
    """Rank 0 of two whose peer never reaches the step (host-side fault: the
    second rank's buffer is a local buffer that nobody serves).  Both of rank
    0's bounded waits run out after the short budget set here; the kernels
    return, the timeout bit lands in the status word and the host raises.  The
    next step on the same workspace (a single rank, sending to itself) then
    runs clean and equals the single-GPU block."""
    import ctypes

    from nki_moe_b200.ep_peer import PeerExpertParallelMoE
    from nki_moe_b200.nki_moe_integrated import NKIMoESimple

    wl = WORKLOADS["c3"]
    T, P, El = 256, 2, wl.experts // 2
    inp = make_moe_inputs(wl, device="cuda", tokens=T)
    moe = NKIMoESimple(wl.hidden, wl.intermediate, wl.experts, wl.top_k, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        moe.router.weight.copy_(inp["router"])
        moe.gate_up_proj.copy_(inp["gate_up"].to(torch.bfloat16))
        moe.down_proj.copy_(inp["down"].to(torch.bfloat16))
    x = inp["x"].to(torch.bfloat16)
    rw = moe.router.weight.detach().float().contiguous()
    pe_local = ops.packed_experts(moe.gate_up_proj.detach()[:El].contiguous(),
                                  moe.down_proj.detach()[:El].contiguous(), "nxd")
    H, I, E, K = wl.hidden, wl.intermediate, wl.experts, wl.top_k
    nbuf = _lib.size_call("nkimoe_ep_peer_buffer_bytes", P, T, H, K)
    bufs = []
    for _ in range(P):
        p = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        _lib.call("nkimoe_peer_alloc", nbuf, ctypes.byref(p), handle)
        bufs.append(p.value)
    ws = ops.workspace(x.device, _lib.size_call("nkimoe_ep_peer_workspace_bytes", T, H, I, E, K, P, T))
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    _lib.set_option("peer_wait_cycles", 2_000_000)  # ~1 ms
    try:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        _lib.call("nkimoe_ep_peer_forward", ops._p(x), ops._p(rw), None, None, ops._p(pe_local.w13),
                  ops._p(pe_local.w2), ops._p(out), None, None, T, H, I, E, K, P, 0, T, (ctypes.c_void_p * P)(*bufs), 1,
                  ops._p(ws), ws.numel(), ops._s(x))
        t1.record()
        with pytest.raises(_lib.NKIMoEError) as ei:
            ops.read_status(ws)
        assert ei.value.code == _lib.ERR_DEVICE
        assert "0x1" in str(ei.value)  # NKIMOE_DEV_TIMEOUT
        assert t0.elapsed_time(t1) < 1000.0  # the budget, not the ~10 s default, ended the waits
    finally:
        _lib.set_option("peer_wait_cycles", 20_000_000_000)
        torch.cuda.synchronize()
        for b in bufs:
            _lib.call("nkimoe_peer_free", ctypes.c_void_p(b))
    # the status word was cleared by the read; the next step is clean
    peer = PeerExpertParallelMoE.from_dense(moe, max_tokens=T)
    try:
        y = peer(x)
        assert ops.read_status(ops.workspace(x.device, 1)) == 0
        assert torch.equal(y, ops.moe_block(x, moe.router.weight, moe.packed(), wl.top_k))
    finally:
        peer.close()


def test_peer_ep_host_batches_equal_device_batches():
    """The expert-parallel block on host batches (two staging slots, copies on
    side streams, completion events so that neighbouring calls overlap) equals
    the device call on the same batch bit for bit, over calls of changing
    size."""
    from nki_moe_b200.ep_peer import PeerExpertParallelMoE
    from nki_moe_b200.nki_moe_integrated import NKIMoESimple

    wl = WORKLOADS["c3"]
    inp = make_moe_inputs(wl, device="cuda", tokens=1024)
    moe = NKIMoESimple(wl.hidden, wl.intermediate, wl.experts, wl.top_k, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        moe.router.weight.copy_(inp["router"])
        moe.gate_up_proj.copy_(inp["gate_up"].to(torch.bfloat16))
        moe.down_proj.copy_(inp["down"].to(torch.bfloat16))
    peer = PeerExpertParallelMoE.from_dense(moe, max_tokens=1024)
    g = torch.Generator().manual_seed(31)
    sizes = (1024, 700, 1024, 300)
    xs = [torch.randn(T, wl.hidden, generator=g).bfloat16().pin_memory() for T in sizes]
    outs = [torch.empty(T, wl.hidden, dtype=torch.bfloat16).pin_memory() for T in sizes]
    dones = [torch.cuda.Event() for _ in sizes]
    old = os.environ.get("NKIMOE_SYNC_CHECK")
    os.environ["NKIMOE_SYNC_CHECK"] = "0"
    try:
        for x, o, d in zip(xs, outs, dones):
            peer.forward_host(x, out=o, done=d)
        for x, o, d in zip(xs, outs, dones):
            d.synchronize()
            ref = peer(x.cuda()).cpu()
            assert torch.equal(o.view(torch.int16), ref.view(torch.int16)), f"{x.shape[0]} tokens"
        assert ops.read_status(ops.workspace(torch.device("cuda", 0), 1)) == 0
    finally:
        os.environ["NKIMOE_SYNC_CHECK"] = old if old is not None else "1"
        peer.close()
