"""Seeded synthetic workloads for the Qwen3-30B-A3B sparse-MoE block.

The reference measures on real checkpoints and real prompts that are not
available here; these generators stand in for them with the shapes, sizes and
value distributions of the benchmark configurations:

* ``c1``: one MoE layer, fp32 on CPU, 128 tokens, seed 0 (the reference's
  CPU-runnable case);
* ``c2``: bf16 decode shape, 64 tokens, seed 1 (expert-weight bandwidth bound);
* ``c3``: bf16 prefill shape, 8192 tokens (4 x 2048), seed 2 (tensor-core bound);
* ``c4``: bf16 skewed routing, 16384 tokens, seed 3, router logits biased by
  ``log(p_k)`` with ``p_k ~ rank^-1.2`` (Zipf) over a random expert permutation.

Layer shape (``qwen.py:243-310`` config, ``qwen.py:164-226`` weight layout):
hidden 2048, 128 experts, top-8, moe_intermediate 768, SwiGLU;
``gate_up_proj[E, H, 2I]`` (gate columns first), ``down_proj[E, I, H]``,
router ``[E, H]`` fp32.  Activations ~ N(0, 1), all weights ~ N(0, 0.02).
Generation order: router, gate_up, down, then x (then the Zipf bias).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

HIDDEN = 2048
INTERMEDIATE = 768
EXPERTS = 128
TOP_K = 8


@dataclass(frozen=True)
class MoEWorkload:
    name: str
    tokens: int
    seed: int
    dtype: str  # arithmetic type of the product path: "fp32" (oracle) or "bf16"
    hidden: int = HIDDEN
    intermediate: int = INTERMEDIATE
    experts: int = EXPERTS
    top_k: int = TOP_K
    zipf_s: float | None = None

    @property
    def flops(self) -> float:
        """Algorithmic FLOPs of one block: router GEMM + K expert FFNs per token."""
        h, i, e, k = self.hidden, self.intermediate, self.experts, self.top_k
        return float(self.tokens) * (2 * h * e + k * (2 * h * 2 * i + 2 * i * h))

    @property
    def expert_bytes(self) -> int:
        """bf16 bytes of one expert's gate_up + down weights."""
        return 2 * (self.hidden * 2 * self.intermediate + self.intermediate * self.hidden)


WORKLOADS = {
    "c1": MoEWorkload("c1_moe_fp32_t128", 128, 0, "fp32"),
    "c2": MoEWorkload("c2_moe_decode_bf16_t64", 64, 1, "bf16"),
    "c3": MoEWorkload("c3_moe_prefill_bf16_t8192", 8192, 2, "bf16"),
    "c4": MoEWorkload("c4_moe_skewed_bf16_t16384", 16384, 3, "bf16", zipf_s=1.2),
}


def zipf_bias(experts: int, s: float, gen: torch.Generator, device="cpu") -> torch.Tensor:
    """Per-expert logit bias ``log(p_k)``, ``p_k = k^-s / sum_j j^-s`` over ranks
    1..E, assigned to experts through a random permutation."""
    ranks = torch.arange(1, experts + 1, dtype=torch.float64)
    p = ranks.pow(-s)
    p = p / p.sum()
    perm = torch.randperm(experts, generator=gen)
    bias = torch.empty(experts, dtype=torch.float64)
    bias[perm] = torch.log(p)
    return bias.to(torch.float32).to(device)


def make_moe_inputs(w: MoEWorkload, device="cpu", tokens: int | None = None):
    """Seeded fp32 tensors for workload ``w`` (values are then cast as needed).

    On CPU the values are reproducible across machines with the same torch
    version (the golden fixtures rely on that); ``device='cuda'`` uses the
    CUDA generator, same distributions, different values.
    Returns a dict with ``x [T,H]``, ``router [E,H]``, ``gate_up [E,H,2I]``,
    ``down [E,I,H]`` and ``router_bias [E]`` (zeros unless ``zipf_s``).
    """
    T = w.tokens if tokens is None else tokens
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(w.seed)
    kw = dict(generator=gen, device=dev, dtype=torch.float32)
    router = torch.randn(w.experts, w.hidden, **kw) * 0.02
    gate_up = torch.randn(w.experts, w.hidden, 2 * w.intermediate, **kw) * 0.02
    down = torch.randn(w.experts, w.intermediate, w.hidden, **kw) * 0.02
    x = torch.randn(T, w.hidden, **kw)
    if w.zipf_s is not None:
        cpu_gen = torch.Generator().manual_seed(w.seed + 1000)
        bias = zipf_bias(w.experts, w.zipf_s, cpu_gen, device=dev)
    else:
        bias = torch.zeros(w.experts, dtype=torch.float32, device=dev)
    return {"x": x, "router": router, "gate_up": gate_up, "down": down, "router_bias": bias}


def tensor_checksum(t: torch.Tensor) -> float:
    """Order-independent float64 checksum used to detect RNG drift in fixtures."""
    t = t.detach().to("cpu", torch.float64)
    return float(t.sum()) + 1e-3 * float(t.abs().sum()) + math.sqrt(float((t * t).sum()))
