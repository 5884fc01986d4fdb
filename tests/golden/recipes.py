"""Seeded input recipes for the small golden cases (shared by the fixture
generator and the tests; CPU torch RNG, reproducible for a fixed torch version)."""

from __future__ import annotations

import torch


def tiny_moe():
    """The reference test's module case (test_nki_moe.py:121-147): H=256, I=512,
    E=4, top-2, B=2, S=8, weights N(0, 0.02), activations N(0, 1), seed 42.
    The reference test seeds only before the activations; here the weights are
    drawn after the same seed so that the case is reproducible."""
    g = torch.Generator().manual_seed(42)
    H, I, E = 256, 512, 4
    router = torch.randn(E, H, generator=g) * 0.02
    gate_up = torch.randn(E, H, 2 * I, generator=g) * 0.02
    down = torch.randn(E, I, H, generator=g) * 0.02
    x = torch.randn(2 * 8, H, generator=g)
    return {"x": x, "router": router, "gate_up": gate_up, "down": down, "top_k": 2}


def rmsnorm_case():
    g = torch.Generator().manual_seed(5)
    x = torch.randn(16, 2048, generator=g) * 3.0
    w = 1.0 + 0.1 * torch.randn(2048, generator=g)
    return {"x": x, "w": w, "eps": 1e-6}


def qk_rope_case():
    """16 tokens of a fused QKV row (32 q heads, 4 kv heads, head_dim 128),
    positions in [0, 640), RoPE theta 1e6, eps 1e-6."""
    g = torch.Generator().manual_seed(7)
    nh, nkv, hd, T = 32, 4, 128, 16
    qkv = torch.randn(T, (nh + 2 * nkv) * hd, generator=g) * 2.0
    q_w = 1.0 + 0.1 * torch.randn(hd, generator=g)
    k_w = 1.0 + 0.1 * torch.randn(hd, generator=g)
    positions = torch.randint(0, 640, (T,), generator=g)
    return {"qkv": qkv, "q_w": q_w, "k_w": k_w, "positions": positions, "n_heads": nh,
            "n_kv_heads": nkv, "head_dim": hd, "theta": 1e6, "eps": 1e-6}


def matmul_case():
    """test_nki_moe.py:44-49: M, K, N = 128, 512, 256, bf16, seed 42."""
    g = torch.Generator().manual_seed(42)
    a = torch.randn(128, 512, generator=g).to(torch.bfloat16)
    b = torch.randn(512, 256, generator=g).to(torch.bfloat16)
    return a, b


def swiglu_case():
    """test_nki_moe.py:86-90: gate_up [64, 1024], bf16, seed 42."""
    g = torch.Generator().manual_seed(42)
    return torch.randn(64, 1024, generator=g).to(torch.bfloat16)
