"""Drop-in for the reference's ``nki_moe_integrated`` module (B200 kernels).

Mirrors ``nki_moe_integrated.py``: ``nki_matmul_tiled`` (:27-84),
``nki_swiglu`` (:87-139), ``nki_moe_expert_compute`` (:142-206),
``nki_moe_aggregate`` (:209-251), ``NKIMoEWrapper`` (:258-387),
``NKIMoESimple`` (:390-496), ``enable_nki_moe`` (:503-529) and
``replace_with_nki_moe`` (:532-565).

Differences from the reference, all deliberate:
* there is one code path (the CUDA one); the reference's try/except fallback
  to the wrapped module (:284-288) is not reproduced: failures raise;
* ``NKIMoEWrapper`` routes every token to its own experts (the reference's
  ``_nki_forward`` picks one "representative" expert per slot, :362-364);
* when the block sits in a decoder that indexes ``self.mlp(h, mask)[0]``
  (qwen_with_nki.py:453) the module returns a 1-tuple (``return_tuple``).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from . import ops

__all__ = [
    "NKIMoEWrapper",
    "NKIMoESimple",
    "enable_nki_moe",
    "replace_with_nki_moe",
    "nki_matmul_tiled",
    "nki_swiglu",
    "nki_moe_expert_compute",
    "nki_moe_aggregate",
]


def _out_dtype(t: torch.Tensor):
    return t.dtype if t.dtype in (torch.float32, torch.bfloat16, torch.float16) else torch.bfloat16


def nki_matmul_tiled(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a[M,K] @ b[K,N]`` with fp32 accumulation on the tensor cores (one
    expert segment of the grouped GEMM).  K and N are zero-padded to the
    kernel's 64 / 128 granularity when needed.  ``b`` is the weight operand:
    its K-major, padded bf16 copy is made once and cached while ``b`` lives
    unmodified (``ops.kmajor_weights``), so repeated calls with one weight
    re-lay it out once."""
    M, K = a.shape
    N = b.shape[1]
    Kp = -(-K // 64) * 64
    a16 = a.to(torch.bfloat16)
    if Kp != K:
        a16 = torch.nn.functional.pad(a16, (0, Kp - K))
    w = ops.kmajor_weights(b, k_multiple=64, n_multiple=128)
    offsets = torch.tensor([0, M], dtype=torch.int32, device=a.device)
    out = ops.grouped_gemm(a16.contiguous(), w, offsets)
    return out[:, :N].to(_out_dtype(a))


def nki_swiglu(gate_up: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` over ``[M, 2N]`` -> ``[M, N]``."""
    return ops.swiglu(gate_up).to(_out_dtype(gate_up))


def nki_moe_expert_compute(hidden_states, gate_up_weight, down_weight, token_weights):
    """One expert over its tokens, scaled per token:
    ``w[t] * (silu(x Gu[:, :I]) * (x Gu[:, I:])) @ D``."""
    T, H = hidden_states.shape
    pe = ops.packed_experts(gate_up_weight.reshape(1, *gate_up_weight.shape),
                            down_weight.reshape(1, *down_weight.shape), "nxd")
    idx = torch.zeros(T, 1, dtype=torch.int32, device=hidden_states.device)
    w = token_weights.reshape(T, 1).float()
    return ops.moe_experts(hidden_states, pe, idx, w).to(_out_dtype(hidden_states))


def nki_moe_aggregate(expert_outputs: torch.Tensor) -> torch.Tensor:
    """Sum over the leading top-k axis of ``[K, T, H]``."""
    return ops.aggregate(expert_outputs).to(_out_dtype(expert_outputs))


# =============================================================================
# Modules
# =============================================================================

def _find_router_weight(mlp: nn.Module) -> torch.Tensor:
    for path in ("router.linear_router.weight", "router.weight", "gate.weight", "gate.linear_router.weight"):
        obj = mlp
        try:
            for part in path.split("."):
                obj = getattr(obj, part)
        except AttributeError:
            continue
        if isinstance(obj, torch.Tensor):
            return obj
    raise AttributeError("cannot find the router weight (router.linear_router / router / gate)")


def _find_expert_weights(mlp: nn.Module):
    """Returns (gate_up, down, layout) from an NxDI MoE module
    (expert_mlps.mlp_op.{gate_up_proj,down_proj}.weight, qwen.py:202,226), an HF
    Qwen3MoeSparseMoeBlock (experts.gate_up_proj [E,2I,H], experts.down_proj
    [E,H,I]) or a module that owns gate_up_proj / down_proj itself (NKIMoESimple)."""
    em = getattr(mlp, "expert_mlps", None)
    if em is not None and hasattr(em, "mlp_op"):
        op = em.mlp_op
        return op.gate_up_proj.weight, op.down_proj.weight, "nxd"
    ex = getattr(mlp, "experts", None)
    if ex is not None and isinstance(getattr(ex, "gate_up_proj", None), torch.Tensor):
        return ex.gate_up_proj, ex.down_proj, "hf"
    if isinstance(getattr(mlp, "gate_up_proj", None), torch.Tensor):
        return mlp.gate_up_proj, mlp.down_proj, "nxd"
    raise AttributeError("cannot find expert weights (expert_mlps.mlp_op / experts / gate_up_proj)")


def _find_top_k(mlp: nn.Module, default: int = 8) -> int:
    for obj, name in ((mlp, "top_k"), (getattr(mlp, "gate", None), "top_k"), (getattr(mlp, "router", None), "top_k")):
        v = getattr(obj, name, None) if obj is not None else None
        if isinstance(v, int):
            return v
    return default


def _host_batch(x: torch.Tensor, router_w: torch.Tensor) -> bool:
    """A batch on the host for weights on a GPU (the reference's module test
    calls the block on host ``hidden_states``, test_nki_moe.py:146-151): the
    block runs on that GPU with the copies overlapped, the result comes back
    to the host."""
    return not x.is_cuda and router_w.is_cuda


class NKIMoEWrapper(nn.Module):
    """Runs a wrapped MoE module's weights through the B200 block.

    ``forward(hidden_states[B,S,H], padding_mask=None)``.  Returns ``(out,)``
    for NxDI-style modules (the decoder takes ``[0]``) and a bare tensor for
    an HF ``Qwen3MoeSparseMoeBlock`` (whose own forward returns a tensor).
    """

    def __init__(self, original_mlp_module):
        super().__init__()
        self.original_mlp = original_mlp_module
        self.use_nki = True
        self.num_experts = getattr(original_mlp_module, "num_experts", None)
        self.top_k = _find_top_k(original_mlp_module)
        _, down, layout = _find_expert_weights(original_mlp_module)
        if self.num_experts is None:
            self.num_experts = down.shape[0]
        self.return_tuple = layout == "nxd" and hasattr(original_mlp_module, "expert_mlps")

    def forward(self, hidden_states: torch.Tensor, padding_mask: Optional[torch.Tensor] = None):
        out = self._nki_forward(hidden_states, padding_mask)
        return (out,) if self.return_tuple else out

    def _nki_forward(self, hidden_states: torch.Tensor, padding_mask=None):
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1])
        rw = _find_router_weight(self.original_mlp)
        gate_up, down, layout = _find_expert_weights(self.original_mlp)
        pe = ops.packed_experts(gate_up, down, layout)
        if _host_batch(x, rw):
            out = ops.moe_block_host(x, rw, pe, self.top_k)
        else:
            out = ops.moe_block(x, rw, pe, self.top_k)
        return out.to(_out_dtype(hidden_states)).view(shape)


class NKIMoESimple(nn.Module):
    """Standalone sparse-MoE block with the reference's parameters:
    ``router`` (Linear H->E, no bias), ``gate_up_proj [E, H, 2I]``,
    ``down_proj [E, I, H]``."""

    def __init__(self, hidden_size: int, intermediate_size: int, num_experts: int, top_k: int = 8,
                 router_dtype: torch.dtype = torch.float32, return_tuple: bool = False, device=None, dtype=None):
        super().__init__()
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.num_experts = num_experts
        self.top_k = top_k
        self.router_dtype = router_dtype
        self.return_tuple = return_tuple
        self.router = nn.Linear(hidden_size, num_experts, bias=False, device=device, dtype=router_dtype)
        kw = dict(device=device, dtype=dtype)
        self.register_parameter("gate_up_proj",
                                nn.Parameter(torch.randn(num_experts, hidden_size, 2 * intermediate_size, **kw)))
        self.register_parameter("down_proj",
                                nn.Parameter(torch.randn(num_experts, intermediate_size, hidden_size, **kw)))
        # optional per-expert logit bias (synthetic skewed-routing workloads)
        self.router_bias: Optional[torch.Tensor] = None
        # optional post-attention RMSNorm run inside the block (fuse_rmsnorm)
        self.rmsnorm: Optional[nn.Module] = None

    def fuse_rmsnorm(self, norm: nn.Module):
        """Run ``norm`` (an ``NKIRMSNorm`` or any module with ``weight`` and
        ``eps``/``variance_epsilon``) inside the block, as the reference's
        fused MoE kernel takes ``post_attention_layernorm``
        (qwen_with_nki.py:379-382; the decoder then skips its own norm call,
        :451-452): ``forward(h)`` computes ``moe(norm(h))``.  Prefill batches
        run the norm and the router logits in one kernel."""
        self.rmsnorm = norm
        return self

    def packed(self) -> ops.PackedExperts:
        return ops.packed_experts(self.gate_up_proj, self.down_proj, "nxd")

    def forward(self, hidden_states: torch.Tensor, padding_mask: Optional[torch.Tensor] = None):
        B, S, H = hidden_states.shape
        x = hidden_states.reshape(-1, H)
        rw = self.router.weight.float()
        if self.rmsnorm is not None:
            eps = getattr(self.rmsnorm, "eps", getattr(self.rmsnorm, "variance_epsilon", 1e-6))
            out = ops.moe_block_rmsnorm(ops._cuda(x, "hidden_states"), self.rmsnorm.weight, rw, self.packed(),
                                        self.top_k, eps=float(eps), bias=self.router_bias)
            out = out.to(_out_dtype(hidden_states)).view(B, S, H)
            return (out,) if self.return_tuple else out
        if _host_batch(x, rw):
            out = ops.moe_block_host(x, rw, self.packed(), self.top_k, bias=self.router_bias)
        else:
            out = ops.moe_block(x, rw, self.packed(), self.top_k, bias=self.router_bias)
        out = out.to(_out_dtype(hidden_states)).view(B, S, H)
        return (out,) if self.return_tuple else out

    def forward_with_routing(self, hidden_states: torch.Tensor):
        """Same as forward, plus ``(idx int32 [T,K], weights fp32 [T,K])``."""
        B, S, H = hidden_states.shape
        out, idx, w = ops.moe_block(hidden_states.reshape(-1, H), self.router.weight.float(), self.packed(),
                                    self.top_k, bias=self.router_bias, return_routing=True)
        return out.to(_out_dtype(hidden_states)).view(B, S, H), idx, w


# =============================================================================
# Integration helpers
# =============================================================================

def enable_nki_moe(model):
    """Wrap every decoder layer's ``mlp`` with ``NKIMoEWrapper``."""
    count = 0
    for layer in model.model.layers:
        if hasattr(layer, "mlp"):
            layer.mlp = NKIMoEWrapper(layer.mlp)
            count += 1
    return model


def replace_with_nki_moe(model, config):
    """Replace every layer's MoE with ``NKIMoESimple`` carrying the same weights.

    Raises ``AttributeError`` (naming the layer) when a layer's MoE holds no
    weights this function can find: the reference (nki_moe_integrated.py:545-563)
    then silently leaves randomly initialised experts in place, which this
    package does not do.  No layer is replaced unless every layer's weights
    were found."""
    new_mlps = []
    for i, layer in enumerate(model.model.layers):
        original = layer.mlp
        try:
            gate_up, down, layout = _find_expert_weights(original)
            rw = _find_router_weight(original)
        except AttributeError as e:
            raise AttributeError(f"replace_with_nki_moe: layer {i}: {e}") from e
        moe = NKIMoESimple(hidden_size=config.hidden_size, intermediate_size=config.moe_intermediate_size,
                           num_experts=config.num_experts, top_k=config.num_experts_per_tok, return_tuple=True)
        with torch.no_grad():
            if layout == "hf":
                gate_up = gate_up.transpose(1, 2)
                down = down.transpose(1, 2)
            moe.gate_up_proj.data = gate_up.detach().contiguous()
            moe.down_proj.data = down.detach().contiguous()
            moe.router.weight.data = rw.detach().float().contiguous()
        new_mlps.append(moe)
    for layer, moe in zip(model.model.layers, new_mlps):
        layer.mlp = moe
    return model
