"""Drop-in for the reference's ``nki_moe_kernel`` module (B200 kernels).

Mirrors ``nki_moe_kernel.py``: ``nki_moe_single_expert_forward`` (:32-182),
``nki_moe_full_forward`` (:185-289), ``nki_moe_optimized`` (:292-423),
``NKIMoELayer`` (:426-508) and ``integrate_nki_moe_to_model`` (:511-544).
The whole-block functions share one implementation, the routed grouped-GEMM
block; the reference's versions are a placeholder (:264-280) and an
every-expert-for-every-token loop (:324-414), so only their signatures and
the arithmetic of their CPU path (:473-508) are kept.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import ops
from .nki_moe_integrated import NKIMoEWrapper, nki_moe_expert_compute

# Qwen3-30B-A3B dimensions.  (The reference file says 2816 for the
# intermediate size, :22; the model's moe_intermediate_size is 768.)
HIDDEN_SIZE = 2048
INTERMEDIATE_SIZE = 768
NUM_EXPERTS = 128
TOP_K = 8

# B200 tile shapes of the grouped GEMMs (rows of a prefill tile, features of a
# prefill tile, K per pipeline stage).
TOKEN_TILE = 128
HIDDEN_TILE = 256
INTERM_TILE = 64

__all__ = [
    "nki_moe_single_expert_forward",
    "nki_moe_full_forward",
    "nki_moe_optimized",
    "NKIMoELayer",
    "integrate_nki_moe_to_model",
]


def nki_moe_single_expert_forward(hidden_states, gate_up_weight, down_weight, expert_weight):
    """One expert: ``[T,H] x [H,2I] -> SwiGLU -> x [I,H] -> * expert_weight[T]``."""
    return nki_moe_expert_compute(hidden_states, gate_up_weight, down_weight, expert_weight)


def _routed_block(hidden_states, gate_up_proj, down_proj, expert_indices, expert_weights):
    pe = ops.packed_experts(gate_up_proj, down_proj, "nxd")
    out = ops.moe_experts(hidden_states, pe, expert_indices, expert_weights)
    dt = hidden_states.dtype if hidden_states.dtype in (torch.float32, torch.bfloat16, torch.float16) else torch.bfloat16
    return out.to(dt)


def nki_moe_full_forward(hidden_states, gate_up_proj, down_proj, expert_indices, expert_weights):
    """``(x[T,H], gate_up[E,H,2I], down[E,I,H], idx[T,K], w[T,K]) -> [T,H]``."""
    return _routed_block(hidden_states, gate_up_proj, down_proj, expert_indices, expert_weights)


def nki_moe_optimized(hidden_states, gate_up_proj, down_proj, expert_indices, expert_weights):
    """Same contract as ``nki_moe_full_forward``."""
    return _routed_block(hidden_states, gate_up_proj, down_proj, expert_indices, expert_weights)


class NKIMoELayer(nn.Module):
    """``NKIMoELayer(config)``; ``forward(h[B,S,H], gate_up_proj, down_proj,
    expert_indices[T,K], expert_weights[T,K]) -> [B,S,H]``."""

    def __init__(self, config):
        super().__init__()
        self.hidden_size = config.hidden_size
        self.intermediate_size = getattr(config, "moe_intermediate_size", INTERMEDIATE_SIZE)
        self.num_experts = getattr(config, "num_experts", NUM_EXPERTS)
        self.top_k = getattr(config, "num_experts_per_tok", TOP_K)

    def forward(self, hidden_states, gate_up_proj, down_proj, expert_indices, expert_weights):
        B, S, H = hidden_states.shape
        out = _routed_block(hidden_states.reshape(-1, H), gate_up_proj, down_proj, expert_indices, expert_weights)
        return out.view(B, S, H)


def integrate_nki_moe_to_model(model, enable_nki_moe=True):
    """Route every layer's MoE through the B200 block (``NKIMoEWrapper``)."""
    if not enable_nki_moe:
        return model
    for layer in model.model.layers:
        layer.mlp = NKIMoEWrapper(layer.mlp)
    return model
