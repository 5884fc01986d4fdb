"""Generate the golden fixtures that pin the oracle to the reference.

Run in the development container (the reference sources must be importable):

    python tests/golden/make_golden.py --reference /root/reference

The reference's modules import ``neuronxcc.nki`` at module top and decorate
their kernels with ``@nki.jit``.  Neither the Neuron SDK nor a Trainium device
exists here, so a minimal stand-in package (``jit`` = identity, an empty
``language`` module) is placed in ``sys.modules`` before the import.  CPU
tensors then take the reference's own PyTorch paths (``is_xla`` is False):

* ``NKIMoESimple.forward`` -> ``_pytorch_forward`` (nki_moe_integrated.py:428-496)
* ``NKIMoEExpertMLP._fallback_forward`` (nki_moe_expert.py:428-463)
* ``NKIMoELayer._pytorch_forward`` (nki_moe_kernel.py:473-508)
* ``NKIRMSNorm._fallback_forward`` (nki_custom_rmsnorm.py:125-129)

RMSNorm and QK-norm + rotate-half RoPE are also taken from HF transformers
(``Qwen3MoeRMSNorm``, ``Qwen3MoeRotaryEmbedding``, ``apply_rotary_pos_emb``),
the CPU classes the reference's model file uses (qwen_with_nki.py:251-252).

Inputs are regenerated from seeds by the tests (``nki_moe_b200.workloads`` and
the small recipes below); the fixtures store outputs plus input checksums.
"""

from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from nki_moe_b200.workloads import WORKLOADS, make_moe_inputs, tensor_checksum  # noqa: E402
from tests.golden import recipes  # noqa: E402


def install_neuron_stub():
    nxc = types.ModuleType("neuronxcc")
    nki = types.ModuleType("neuronxcc.nki")
    lang = types.ModuleType("neuronxcc.nki.language")
    nki.jit = lambda f=None, **kw: f if f is not None else (lambda g: g)
    nki.language = lang
    nxc.nki = nki
    sys.modules.update({"neuronxcc": nxc, "neuronxcc.nki": nki, "neuronxcc.nki.language": lang})


def run_simple(mod, x, router, gate_up, down, top_k):
    """Run the reference NKIMoESimple on CPU and capture logits / routing."""
    E, H, I2 = gate_up.shape
    moe = mod.NKIMoESimple(hidden_size=H, intermediate_size=I2 // 2, num_experts=E, top_k=top_k)
    with torch.no_grad():
        moe.router.weight.copy_(router)
        moe.gate_up_proj.copy_(gate_up)
        moe.down_proj.copy_(down)
    cap = {}
    moe.router.register_forward_hook(lambda m, i, o: cap.__setitem__("logits", o.detach().clone()))
    orig = moe._pytorch_forward

    def spy(hidden_flat, routing_weights, selected_experts):
        cap["w"] = routing_weights.detach().clone()
        cap["idx"] = selected_experts.detach().clone()
        return orig(hidden_flat, routing_weights, selected_experts)

    moe._pytorch_forward = spy
    with torch.no_grad():
        out = moe(x.reshape(1, *x.shape) if x.dim() == 2 else x)
    return out.reshape(-1, H), cap["logits"], cap["idx"], cap["w"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="directory holding the reference sources")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    install_neuron_stub()
    sys.path.insert(0, args.reference)
    import nki_custom_rmsnorm as ref_norm
    import nki_moe_expert as ref_expert
    import nki_moe_integrated as ref_int
    import nki_moe_kernel as ref_kernel
    from transformers.models.qwen3_moe import modeling_qwen3_moe as hf
    from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig

    torch.set_num_threads(max(1, os.cpu_count() or 1))

    # ---- tiny: the reference test's module shapes (test_nki_moe.py:121-147)
    t = recipes.tiny_moe()
    out, lg, idx, w = run_simple(ref_int, t["x"], t["router"], t["gate_up"], t["down"], t["top_k"])
    np.savez_compressed(
        os.path.join(args.out, "moe_tiny.npz"),
        out=out.numpy(), logits=lg.numpy(), idx=idx.numpy().astype(np.int32), w=w.numpy(),
        checksums=np.array([tensor_checksum(t[k]) for k in ("x", "router", "gate_up", "down")]),
    )
    print("tiny", out.shape, float(out.abs().max()))

    # ---- c1: one full-size layer, fp32, 128 tokens, seed 0
    wl = WORKLOADS["c1"]
    inp = make_moe_inputs(wl)
    out, lg, idx, w = run_simple(ref_int, inp["x"], inp["router"], inp["gate_up"], inp["down"], wl.top_k)
    # given-routing CPU paths of the other two reference modules must agree
    mlp = ref_expert.NKIMoEExpertMLP(wl.experts, wl.hidden, wl.intermediate, top_k=wl.top_k)
    cfg = types.SimpleNamespace(hidden_size=wl.hidden, moe_intermediate_size=wl.intermediate,
                                num_experts=wl.experts, num_experts_per_tok=wl.top_k)
    layer = ref_kernel.NKIMoELayer(cfg)
    with torch.no_grad():
        out_mlp = mlp._fallback_forward(inp["x"], inp["gate_up"], inp["down"], idx, w)
        out_layer = layer._pytorch_forward(inp["x"].reshape(1, *inp["x"].shape), inp["gate_up"],
                                           inp["down"], idx, w).reshape(-1, wl.hidden)
    d_mlp = float((out_mlp - out).abs().max())
    d_layer = float((out_layer - out).abs().max())
    print("c1", out.shape, "given-routing deltas", d_mlp, d_layer)
    np.savez_compressed(
        os.path.join(args.out, "moe_c1.npz"),
        out=out.numpy(), given_routing_max_delta=np.array([d_mlp, d_layer]),
        logits=lg.numpy(), idx=idx.numpy().astype(np.int32), w=w.numpy(),
        checksums=np.array([tensor_checksum(inp[k]) for k in ("x", "router", "gate_up", "down")]),
    )

    # ---- RMSNorm: reference fallback and HF (fp32)
    r = recipes.rmsnorm_case()
    norm = ref_norm.NKIRMSNorm(r["x"].shape[-1], eps=r["eps"])
    hfn = hf.Qwen3MoeRMSNorm(r["x"].shape[-1], eps=r["eps"])
    with torch.no_grad():
        norm.weight.copy_(r["w"])
        hfn.weight.copy_(r["w"])
        y_ref = norm._fallback_forward(r["x"])
        y_hf = hfn(r["x"])
    np.savez_compressed(os.path.join(args.out, "rmsnorm.npz"), y_ref=y_ref.numpy(),
                        hf_max_delta=np.array([float((y_ref - y_hf).abs().max())]),
                        checksums=np.array([tensor_checksum(r["x"]), tensor_checksum(r["w"])]))
    print("rmsnorm", float((y_ref - y_hf).abs().max()))

    # ---- QK-norm + RoPE (HF order and rotate-half convention), fp32
    q = recipes.qk_rope_case()
    T, nh, nkv, hd = q["qkv"].shape[0], q["n_heads"], q["n_kv_heads"], q["head_dim"]
    conf = Qwen3MoeConfig(hidden_size=2048, num_attention_heads=nh, num_key_value_heads=nkv, head_dim=hd,
                          rope_theta=q["theta"], rms_norm_eps=q["eps"], max_position_embeddings=4096)
    rot = hf.Qwen3MoeRotaryEmbedding(conf)
    qn = hf.Qwen3MoeRMSNorm(hd, eps=q["eps"])
    kn = hf.Qwen3MoeRMSNorm(hd, eps=q["eps"])
    with torch.no_grad():
        qn.weight.copy_(q["q_w"])
        kn.weight.copy_(q["k_w"])
        qs = qn(q["qkv"][:, :nh * hd].reshape(1, T, nh, hd)).transpose(1, 2)
        ks = kn(q["qkv"][:, nh * hd:(nh + nkv) * hd].reshape(1, T, nkv, hd)).transpose(1, 2)
        cos, sin = rot(q["qkv"], q["positions"].reshape(1, T))
        qe, ke = hf.apply_rotary_pos_emb(qs, ks, cos, sin)
    out = q["qkv"].clone()
    out[:, :nh * hd] = qe.transpose(1, 2).reshape(T, nh * hd)
    out[:, nh * hd:(nh + nkv) * hd] = ke.transpose(1, 2).reshape(T, nkv * hd)
    np.savez_compressed(os.path.join(args.out, "qk_rope.npz"), out=out.numpy(),
                        cos=cos.reshape(T, hd).numpy(), sin=sin.reshape(T, hd).numpy(),
                        checksums=np.array([tensor_checksum(q["qkv"])]))
    print("qk_rope", out.shape)

    # ---- pieces: the reference test's GEMM and SwiGLU cases (test_nki_moe.py:44-67, 86-108);
    # their expected values are torch.matmul and F.silu(gate) * up on the bf16 inputs.
    a, b = recipes.matmul_case()
    g = recipes.swiglu_case()
    gate, up = g.float().chunk(2, dim=-1)
    np.savez_compressed(os.path.join(args.out, "pieces.npz"),
                        matmul=(a.float() @ b.float()).numpy(),
                        swiglu=(torch.nn.functional.silu(gate) * up).numpy())
    print("done")


if __name__ == "__main__":
    main()
