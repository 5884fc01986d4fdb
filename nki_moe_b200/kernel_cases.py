"""Single launches of the bandwidth-bound kernels on the 8192-token prefill
shapes, for kernel profilers (one process, one GPU, a few GB of device
memory):

    python -m nki_moe_b200.kernel_cases [--case block|norms|all]

``block``: one MoE block on 8192 tokens (hidden 2048, 128 experts, top-8,
intermediate 768; random N(0, 1) tokens, N(0, 0.02) weights made directly in
the packed layout), which launches the router, top-k, the three permutation
kernels, the row gather, the two grouped GEMMs and the combine once each.
``norms``: one RMSNorm and one residual-add + RMSNorm over [8192, 2048] bf16
rows, and one QK-norm + RoPE over [8192, 5120] fused QKV rows (32 query and
4 key/value heads of 128).

Algorithmic bytes per launch (the traffic a kernel cannot avoid):
  rmsnorm        8192 x 2048 x 2 B read and written, + 2048 x 4 B weight  =  67.1 MB
  add_rmsnorm    two rows read, two written                               = 134.2 MB
  qk_norm_rope   8192 x 5120 x 2 B read and written                       = 167.8 MB
  gather         8192 x 2048 x 2 B read + 65536 x 2048 x 2 B written      = 302.0 MB
  combine        65536 x 2048 x 2 B read + 8192 x 2048 x 2 B written      = 302.0 MB
  permutation    65536 x 4 B of expert ids read, 4 x 65536 x 4 B written  =   1.3 MB
"""

from __future__ import annotations

import argparse

import torch

from . import _lib, ops


def run_block(device):
    T, H, I, E, K = 8192, 2048, 768, 128, 8
    g = torch.Generator(device=device).manual_seed(2)
    x = torch.randn(T, H, generator=g, device=device).to(torch.bfloat16)
    rw = torch.randn(E, H, generator=g, device=device) * 0.02
    w13 = (torch.randn(E, 2 * I, H, generator=g, device=device) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g, device=device) * 0.02).to(torch.bfloat16)
    pe = ops.PackedExperts(w13, w2, E, H, I)
    ops.moe_block(x, rw, pe, K)
    torch.cuda.synchronize()


def run_norms(device):
    T, H = 8192, 2048
    g = torch.Generator(device=device).manual_seed(4)
    x = torch.randn(T, H, generator=g, device=device).to(torch.bfloat16)
    r = torch.randn(T, H, generator=g, device=device).to(torch.bfloat16)
    w = torch.rand(H, generator=g, device=device) + 0.5
    ops.rmsnorm(x, w, 1e-6)
    ops.add_rmsnorm(x, r, w, 1e-6)
    nh, nkv, hd = 32, 4, 128
    qkv = torch.randn(T, (nh + 2 * nkv) * hd, generator=g, device=device).to(torch.bfloat16)
    qw = torch.rand(hd, generator=g, device=device) + 0.5
    kw = torch.rand(hd, generator=g, device=device) + 0.5
    pos = torch.arange(T, device=device, dtype=torch.int64)
    ops.qk_norm_rope(qkv, qw, kw, pos, nh, nkv, hd, 1e6, 1e-6)
    torch.cuda.synchronize()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="all", choices=["block", "norms", "all"])
    ap.add_argument("--router-fused", type=int, default=1, choices=[0, 1],
                    help="tensor-core router: the planes' summed logits in one kernel (1) or the GEMM's partials (0)")
    a = ap.parse_args()
    if not torch.cuda.is_available():
        raise SystemExit("needs a CUDA device")
    _lib.load()
    _lib.set_option("router_fused", a.router_fused)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if a.case in ("block", "all"):
        run_block(dev)
    if a.case in ("norms", "all"):
        run_norms(dev)
    print("kernel cases done")


if __name__ == "__main__":
    main()
