"""Drop-in for the reference's ``nki_moe_expert`` module (B200 kernels).

Mirrors ``nki_moe_expert.py``: ``nki_moe_expert_kernel`` (:21-208),
``nki_moe_expert_fused_kernel_v2`` (:211-355), ``NKIMoEExpertMLP``
(:358-463), ``nki_grouped_expert_gemm`` (:466-542) and
``create_nki_moe_config`` (:545-556).  ``nki_grouped_expert_gemm`` applies
each row's own expert (the reference uses one representative expert per
128-row tile, :520-522).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import ops
from .nki_moe_kernel import _routed_block

__all__ = [
    "nki_moe_expert_kernel",
    "nki_moe_expert_fused_kernel_v2",
    "NKIMoEExpertMLP",
    "nki_grouped_expert_gemm",
    "create_nki_moe_config",
]


def nki_moe_expert_kernel(hidden_states, gate_up_proj, down_proj, expert_indices, expert_weights):
    """``(x[T,H], gate_up[E,H,2I], down[E,I,H], idx[T,K], w[T,K]) -> [T,H]``."""
    return _routed_block(hidden_states, gate_up_proj, down_proj, expert_indices, expert_weights)


def nki_moe_expert_fused_kernel_v2(hidden_states, gate_up_proj, down_proj, expert_indices, expert_weights):
    """Same contract as ``nki_moe_expert_kernel``."""
    return _routed_block(hidden_states, gate_up_proj, down_proj, expert_indices, expert_weights)


class NKIMoEExpertMLP(nn.Module):
    def __init__(self, num_experts: int, hidden_size: int, intermediate_size: int, top_k: int = 8,
                 use_fused_kernel: bool = True):
        super().__init__()
        self.num_experts = num_experts
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.top_k = top_k
        self.use_fused_kernel = use_fused_kernel

    def forward(self, hidden_states, gate_up_proj, down_proj, expert_indices, expert_weights):
        return _routed_block(hidden_states, gate_up_proj, down_proj, expert_indices, expert_weights)


def nki_grouped_expert_gemm(input_tokens, expert_weights, expert_ids, num_experts):
    """``out[m] = input_tokens[m] @ expert_weights[expert_ids[m]]``:
    ``[M,H] x [E,H,N] -> [M,N]``."""
    M, H = input_tokens.shape
    E, _, N = expert_weights.shape
    ids = expert_ids.reshape(M, 1)
    # rows grouped by expert (library permutation + gather), one slot per row
    ones = torch.ones(M, 1, dtype=torch.float32, device=input_tokens.device)
    a_perm, _, slot_row, counts = ops.dispatch(input_tokens.to(torch.bfloat16), ids, ones, num_experts)
    offsets = torch.zeros(num_experts + 1, dtype=torch.int32, device=input_tokens.device)
    offsets[1:] = counts.cumsum(0)
    # [E, N, H] K-major copy, made once per weight tensor and cached
    w_packed = ops.kmajor_weights(expert_weights, k_multiple=64, n_multiple=128)
    out_perm = ops.grouped_gemm(a_perm, w_packed, offsets)
    # back to token order: a one-slot combine copies row slot_row[m] to m
    out = ops.combine(out_perm, slot_row, M, 1)[:, :N]
    dt = input_tokens.dtype if input_tokens.dtype in (torch.float32, torch.bfloat16, torch.float16) else torch.bfloat16
    return out.to(dt)


def create_nki_moe_config():
    """Tile configuration of the B200 kernels (the reference returns its
    Trainium tile sizes)."""
    return {
        "prefill_tile_rows": 128,
        "prefill_tile_features": 256,
        "decode_tile_features": 128,
        "decode_tile_rows": (16, 32, 64),
        "k_per_stage": 64,
        "stages_prefill": 4,
        "stages_decode": 8,
        "tmem_double_buffered": True,
        "fused_activation": True,
        "fused_routing_weight": True,
    }
