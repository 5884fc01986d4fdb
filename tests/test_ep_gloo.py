"""Expert-parallel exchange logic on CPU: world-size-2 gloo ranks running the
block's orchestration (nki_moe_b200.ep) with the oracle as the compute
backend, checked against the single-process oracle block."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from nki_moe_b200.ep import ExpertParallelMoE

H, I, E, K, T = 256, 128, 8, 2, 24


class OracleKernels:
    """CPU stand-ins for the four compute steps (test infrastructure)."""

    def route(self, x, router_w, top_k, bias):
        lg = oracle.router_logits(x.numpy(), router_w.numpy())
        if bias is not None:
            lg = lg + bias.numpy()
        idx, w = oracle.topk_softmax(lg, top_k)
        return torch.from_numpy(idx), torch.from_numpy(w)

    def dispatch(self, x, idx, w, num_experts):
        row_t, row_slot, offsets, slot_row = oracle.permute(idx.numpy(), num_experts)
        x_perm = x[torch.from_numpy(row_t).long()]
        row_w = w.reshape(-1)[torch.from_numpy(row_slot).long()]
        counts = torch.from_numpy(np.diff(offsets).astype(np.int32))
        return x_perm, row_w, torch.from_numpy(slot_row), counts

    def experts(self, recv_x, recv_w, segment_counts, module):
        el = module.local_experts
        out = torch.zeros_like(recv_x)
        o = 0
        for s, c in enumerate(segment_counts.tolist()):
            if c:
                e = s % el
                y = oracle.expert_ffn(recv_x[o:o + c].numpy(), module.gate_up_local[e].numpy(),
                                      module.down_local[e].numpy())
                out[o:o + c] = torch.from_numpy(y) * recv_w[o:o + c, None]
            o += c
        return out

    def ep_dispatch(self, x, idx, w, num_ranks, el):
        T, K = idx.shape
        dest = np.full((T, num_ranks), -1, np.int32)
        for t in range(T):
            for e in idx[t].tolist():
                dest[t, e // el] = e // el
        row_t, row_slot, offsets, slot_row = oracle.permute(dest, num_ranks)
        d_of = row_slot % num_ranks
        ids = idx.numpy()[row_t]
        local = (ids // el) == d_of[:, None]
        slots = np.where(local, ids - d_of[:, None] * el, -1).astype(np.int32)
        wts = np.where(local, w.numpy()[row_t], 0.0).astype(np.float32)
        return (x[torch.from_numpy(row_t).long()], torch.from_numpy(slots), torch.from_numpy(wts),
                torch.from_numpy(np.diff(offsets).astype(np.int32)), torch.from_numpy(slot_row.reshape(T, num_ranks)))

    def routed_experts(self, recv_x, recv_slots, recv_w, module):
        out = torch.zeros_like(recv_x)
        for r in range(recv_x.shape[0]):
            for k in range(recv_slots.shape[1]):
                e = int(recv_slots[r, k])
                if e >= 0:
                    y = oracle.expert_ffn(recv_x[r:r + 1].numpy(), module.gate_up_local[e].numpy(),
                                          module.down_local[e].numpy())[0]
                    out[r] += float(recv_w[r, k]) * torch.from_numpy(y)
        return out

    def combine(self, y, slot_row, tokens, top_k):
        rows = slot_row.reshape(tokens, top_k).long()
        out = torch.zeros(tokens, y.shape[1])
        for k in range(top_k):
            ok = rows[:, k] >= 0
            out[ok] += y[rows[ok, k]]
        return out


def weights(skew):
    g = torch.Generator().manual_seed(11)
    router = torch.randn(E, H, generator=g) * 0.02
    gate_up = torch.randn(E, H, 2 * I, generator=g) * 0.02
    down = torch.randn(E, I, H, generator=g) * 0.02
    bias = None
    if skew:  # route almost everything to the experts of rank 0
        bias = torch.tensor([6.0] * (E // 2) + [-6.0] * (E // 2))
    return router, gate_up, down, bias


def worker(rank, world, port, skew, result_dir, fail_rank, dedup=True):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=15))
    router, gate_up, down, bias = weights(skew)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(100 + rank))
    el = E // world
    ep = ExpertParallelMoE(router, gate_up[rank * el:(rank + 1) * el], down[rank * el:(rank + 1) * el], E, K,
                           router_bias=bias, kernels=OracleKernels(), dedup=dedup)
    if rank == fail_rank:
        os._exit(3)  # this rank dies before the exchange
    try:
        out = ep(x)
        np.save(os.path.join(result_dir, f"out{rank}.npy"), out.numpy())
        np.save(os.path.join(result_dir, f"x{rank}.npy"), x.numpy())
    except Exception as exc:  # the surviving rank must see an error, not hang
        open(os.path.join(result_dir, f"err{rank}.txt"), "w").write(repr(exc))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("dedup", [True, False])
@pytest.mark.parametrize("skew", [False, True])
def test_ep_matches_single_process_oracle(tmp_path, skew, dedup):
    world = 2
    mp.start_processes(worker, args=(world, free_port(), skew, str(tmp_path), -1, dedup), nprocs=world, join=True,
                       start_method="spawn")
    router, gate_up, down, bias = weights(skew)
    for r in range(world):
        x = np.load(tmp_path / f"x{r}.npy")
        out = np.load(tmp_path / f"out{r}.npy")
        lg = oracle.router_logits(x, router.numpy())
        if bias is not None:
            lg = lg + bias.numpy()
        idx, w = oracle.topk_softmax(lg, K)
        ref = oracle.experts_forward(x, gate_up.numpy(), down.numpy(), idx, w)
        assert oracle.normwise_rel_err(out, ref) < 1e-5


def test_ep_rank_failure_surfaces_as_error(tmp_path):
    """Rank 1 exits before the first collective: rank 0's exchange must end
    with an error within the process-group timeout instead of hanging."""
    world = 2
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, False, str(tmp_path), 1)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung instead of failing"
    assert procs[1].exitcode == 3
    assert (tmp_path / "err0.txt").exists()
    assert not (tmp_path / "out0.npy").exists()
