"""Expert-parallel sparse-MoE block over ``torch.distributed`` (NCCL).

P ranks, one GPU each.  Rank r owns experts ``[r*E/P, (r+1)*E/P)`` and keeps
its own batch of tokens (tokens are sharded data-parallel before the block).
One forward:

  1. route        router GEMM + softmax/top-k/renormalise on the local tokens
  2. dispatch     one send row per (token, rank) pair that has at least one of
                  the token's experts ("dedup", default): the token's hidden
                  row plus its K slots as that rank sees them (local expert id
                  or -1, routing weight); rows grouped by rank, tokens ascending
  3. exchange     all-to-all of per-rank row counts (the block's one host
                  synchronisation, for the split sizes), then of rows, slots
                  and weights
  4. experts      the single-GPU given-routing block on the received rows with
                  the rank's local experts (permute, grouped GEMMs, combine):
                  one partial sum per received row
  5. return       all-to-all of the partial sums back to their senders
  6. combine      per token, sum of its per-rank partial sums in fp32

Each token crosses the network at most min(P, K) times each way instead of K
times (4x less traffic at P=2 with top-8, 1.5x at P=8).  ``dedup=False``
keeps one row per (token, slot): permute by global expert, exchange, grouped
GEMMs on the received (source rank, local expert) segments, and the
single-GPU combine, which is bit-identical to the single-GPU block.

The reference leaves expert parallelism to NxDI (``moe_ep_degree``,
qwen.py:272, :515); this is the B200 counterpart.  The compute steps are the
CUDA entry points of ``libnkimoe.so``; ``kernels`` can be replaced (the CPU
tests of the exchange logic run it with the oracle over gloo).
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn

from . import ops


class CudaKernels:
    """The product compute path: the sm_100a kernels through the C ABI."""

    def route(self, x, router_w, top_k, bias):
        return ops.route(x, router_w, top_k, bias=bias)

    def ep_dispatch(self, x, idx, w, num_ranks, experts_per_rank):
        return ops.ep_dispatch(x, idx, w, num_ranks, experts_per_rank)

    def routed_experts(self, recv_x, recv_slots, recv_w, module):
        return ops.moe_experts(recv_x, module.packed(), recv_slots, recv_w)

    def dispatch(self, x, idx, w, num_experts):
        return ops.dispatch(x, idx, w, num_experts)

    def experts(self, recv_x, recv_w, segment_counts, module):
        return ops.segment_experts(recv_x, recv_w, segment_counts, module.packed())

    def combine(self, y, slot_row, tokens, top_k):
        return ops.combine(y, slot_row, tokens, top_k)


def local_expert_range(num_experts: int, world: int, rank: int):
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not split over {world} ranks")
    el = num_experts // world
    return rank * el, (rank + 1) * el


class ExpertParallelMoE(nn.Module):
    """``forward(x [T, H]) -> [T, H]``: this rank's tokens through the
    expert-parallel block.  ``router_w`` is the full fp32 router [E, H]
    (replicated); ``gate_up_local`` [E/P, H, 2I] and ``down_local`` [E/P, I, H]
    are this rank's experts in the reference layout (qwen.py:164-226)."""

    def __init__(self, router_w: torch.Tensor, gate_up_local: torch.Tensor, down_local: torch.Tensor,
                 num_experts: int, top_k: int, group=None, router_bias: torch.Tensor | None = None,
                 kernels=None, dedup: bool = True):
        super().__init__()
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.num_experts = num_experts
        self.top_k = top_k
        self.local_experts = num_experts // self.world
        if self.local_experts * self.world != num_experts or gate_up_local.shape[0] != self.local_experts:
            raise ValueError("local expert weights do not match num_experts / world size")
        self.router_w = router_w
        self.router_bias = router_bias
        self.gate_up_local = gate_up_local
        self.down_local = down_local
        self.kernels = kernels if kernels is not None else CudaKernels()
        self.dedup = dedup

    @classmethod
    def from_dense(cls, moe, group=None, kernels=None, dedup: bool = True):
        """Slice this rank's experts out of an ``NKIMoESimple`` holding all of them."""
        g = group if group is not None else dist.group.WORLD
        lo, hi = local_expert_range(moe.num_experts, dist.get_world_size(g), dist.get_rank(g))
        return cls(moe.router.weight.detach().float(), moe.gate_up_proj.detach()[lo:hi].contiguous(),
                   moe.down_proj.detach()[lo:hi].contiguous(), moe.num_experts, moe.top_k, group=g,
                   router_bias=moe.router_bias, kernels=kernels, dedup=dedup)

    def packed(self):
        """This rank's experts in the GEMM layout (packed once, cached)."""
        return ops.packed_experts(self.gate_up_local, self.down_local, "nxd")

    def exchange_plan(self, expert_counts: torch.Tensor):
        """All-to-all of row counts.  Returns (recv_counts [P, E/P] on the
        device, send_rows, recv_rows) with the per-rank row totals on the host
        (the one synchronisation of the block)."""
        P, El = self.world, self.local_experts
        send_counts = expert_counts.reshape(P, El).to(torch.int32).contiguous()
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        tot = torch.stack([send_counts.sum(1), recv_counts.sum(1)]).cpu()
        return recv_counts, tot[0].tolist(), tot[1].tolist()

    def _exchange_counts(self, send_counts: torch.Tensor):
        """All-to-all of per-rank row counts; host copies of both directions."""
        send_counts = send_counts.to(torch.int32).contiguous()
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        tot = torch.stack([send_counts, recv_counts]).cpu()
        return tot[0].tolist(), tot[1].tolist()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._forward_dedup(x) if self.dedup else self._forward_segments(x)

    def _forward_dedup(self, x: torch.Tensor) -> torch.Tensor:
        k = self.kernels
        T, H = x.shape
        K, P = self.top_k, self.world
        idx, w = k.route(x, self.router_w, K, self.router_bias)
        x_send, slots, wts, counts, slot_row = k.ep_dispatch(x, idx, w, P, self.local_experts)
        send_rows, recv_rows = self._exchange_counts(counts)
        S, R = sum(send_rows), sum(recv_rows)
        recv_x = x_send.new_empty(R, H)
        recv_slots = slots.new_empty(R, K)
        recv_w = wts.new_empty(R, K)
        g = self.group
        dist.all_to_all_single(recv_x, x_send[:S], recv_rows, send_rows, group=g)
        dist.all_to_all_single(recv_slots, slots[:S], recv_rows, send_rows, group=g)
        dist.all_to_all_single(recv_w, wts[:S], recv_rows, send_rows, group=g)
        partial = k.routed_experts(recv_x, recv_slots, recv_w, self)
        back = partial.new_empty(S, H)
        dist.all_to_all_single(back, partial, send_rows, recv_rows, group=g)
        return k.combine(back, slot_row, T, P)

    def _forward_segments(self, x: torch.Tensor) -> torch.Tensor:
        k = self.kernels
        T, H = x.shape
        K = self.top_k
        idx, w = k.route(x, self.router_w, K, self.router_bias)
        x_perm, row_w, slot_row, counts = k.dispatch(x, idx, w, self.num_experts)
        recv_counts, send_rows, recv_rows = self.exchange_plan(counts)
        R = sum(recv_rows)
        recv_x = x_perm.new_empty(R, H)
        recv_w = row_w.new_empty(R)
        dist.all_to_all_single(recv_x, x_perm, recv_rows, send_rows, group=self.group)
        dist.all_to_all_single(recv_w, row_w, recv_rows, send_rows, group=self.group)
        y = k.experts(recv_x, recv_w, recv_counts.reshape(-1), self)
        y_back = y.new_empty(T * K, H)
        dist.all_to_all_single(y_back, y, send_rows, recv_rows, group=self.group)
        return k.combine(y_back, slot_row, T, K)
