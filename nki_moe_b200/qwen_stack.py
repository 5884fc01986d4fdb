"""Qwen3-MoE decoder stack on this library's kernels, for end-to-end latency.

The decoder wiring of the reference's model file (``qwen_with_nki.py:402-460``,
``NeuronQwen3MoeDecoderLayer.forward``): per layer

    r = h;  h = attn(rmsnorm(h));  h = r + h
    r = h;  h = moe(rmsnorm(h));   h = r + h

with the attention of ``qwen_with_nki.py:330-350`` (fused QKV projection,
per-head q/k RMSNorm, rotate-half RoPE with theta 1e6, GQA, scale
head_dim^-0.5) and a final RMSNorm + LM head (``qwen_with_nki.py:495``).

Library kernels on the path: RMSNorm and the fused residual-add + RMSNorm
(``nkimoe_rmsnorm`` / ``nkimoe_add_rmsnorm``), q/k RMSNorm + RoPE on the fused
QKV rows (``nkimoe_qk_norm_rope``, prefill), the decode step's attention fused
with its q/k norms, RoPE and KV-cache store (``nkimoe_decode_attention``) and
the whole MoE block (``nkimoe_moe_block``).  The dense projections (QKV, O,
LM head) are plain cuBLAS GEMMs through torch and prefill attention is torch's
scaled-dot-product attention; neither is part of the MoE hot path.

Decode keeps every shape static (a KV cache of ``max_seq`` positions, the
current position in a device tensor that the attention kernel reads), so one
decode step over all layers is captured into a single CUDA graph.
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import ops


@dataclass
class Qwen3MoEConfig:
    """Qwen3-30B-A3B shape (the defaults) or any smaller one of the same kind."""

    vocab_size: int = 151936
    hidden_size: int = 2048
    num_hidden_layers: int = 48
    num_attention_heads: int = 32
    num_key_value_heads: int = 4
    head_dim: int = 128
    moe_intermediate_size: int = 768
    num_experts: int = 128
    num_experts_per_tok: int = 8
    rope_theta: float = 1e6
    rms_norm_eps: float = 1e-6

    @classmethod
    def from_hf(cls, c) -> "Qwen3MoEConfig":
        theta = getattr(c, "rope_theta", None)
        if theta is None:
            theta = (getattr(c, "rope_parameters", None) or {}).get("rope_theta", 1e6)
        return cls(vocab_size=c.vocab_size, hidden_size=c.hidden_size, num_hidden_layers=c.num_hidden_layers,
                   num_attention_heads=c.num_attention_heads, num_key_value_heads=c.num_key_value_heads,
                   head_dim=getattr(c, "head_dim", c.hidden_size // c.num_attention_heads),
                   moe_intermediate_size=c.moe_intermediate_size, num_experts=c.num_experts,
                   num_experts_per_tok=c.num_experts_per_tok, rope_theta=float(theta), rms_norm_eps=c.rms_norm_eps)


class _Layer:
    """One decoder layer's weights in the layouts the kernels take.  With
    ``ep`` (an expert-parallel block holding this rank's experts) the MoE runs
    through it; otherwise ``experts`` holds all experts."""

    def __init__(self, in_norm, qkv_w, q_norm, k_norm, o_w, post_norm, router_w, experts: ops.PackedExperts,
                 ep=None, ep_decode=None):
        self.in_norm, self.qkv_w, self.q_norm, self.k_norm = in_norm, qkv_w, q_norm, k_norm
        self.o_w, self.post_norm, self.router_w, self.experts = o_w, post_norm, router_w, experts
        # expert parallel: one exchange sized for prefill batches, one for a
        # decode step (the receiver's kernels cover every source's whole region)
        self.ep, self.ep_decode = ep, ep_decode
        self.router_split = (ops.router_split(router_w) if ep is None and router_w.shape[0] % 128 == 0 else None)


class Qwen3MoEStack:
    """bf16 Qwen3-MoE causal LM: prefill, static-shape decode, greedy generate."""

    def __init__(self, cfg: Qwen3MoEConfig, embed: torch.Tensor, layers: list[_Layer], final_norm: torch.Tensor,
                 lm_head: torch.Tensor, max_batch: int, max_seq: int):
        self.cfg = cfg
        self.embed, self.layers, self.final_norm, self.lm_head = embed, layers, final_norm, lm_head
        self.device = embed.device
        self.max_batch, self.max_seq = max_batch, max_seq
        kv = (cfg.num_hidden_layers, max_batch, cfg.num_key_value_heads, max_seq, cfg.head_dim)
        self.k_cache = torch.zeros(kv, dtype=torch.bfloat16, device=self.device)
        self.v_cache = torch.zeros(kv, dtype=torch.bfloat16, device=self.device)
        self.length = 0
        # decode-step state (static for graph capture)
        self._pos = torch.zeros(1, dtype=torch.int64, device=self.device)
        self._tokens = torch.zeros(max_batch, dtype=torch.int64, device=self.device)
        self._graph = None
        self._graph_batch = None
        self._graph_out = None
        # the skinny linear kernel takes N % 16 == 0 and K % 32 == 0
        H, hd = cfg.hidden_size, cfg.head_dim
        nq, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
        self._skinny_ok = (H % 32 == 0 and (nq * hd) % 32 == 0 and ((nq + 2 * nkv) * hd) % 16 == 0
                           and H % 16 == 0 and cfg.vocab_size % 16 == 0)

    # ------------------------------------------------------------ construction
    @classmethod
    def random_init(cls, cfg: Qwen3MoEConfig, seed: int = 0, device="cuda", max_batch: int = 8,
                    max_seq: int = 640, std: float = 0.02, expert_parallel: bool = False,
                    group=None) -> "Qwen3MoEStack":
        """Random N(0, std) weights (norm weights 1, router fp32), expert weights
        drawn in the reference's ``[E, H, 2I]`` / ``[E, I, H]`` layout and
        packed once.

        ``expert_parallel``: one rank of an expert-parallel stack over the
        initialised process group (``group``, default WORLD): every rank draws
        the same weights (same generator sequence as the single-GPU stack),
        keeps the attention, norms, router and embeddings whole and only its
        ``E / P`` experts, and runs each layer's MoE as a peer-memory
        expert-parallel block over its own sequences (``max_batch`` of them,
        up to ``max_seq`` tokens each).  Every rank must run the same calls
        (prefill, decode steps) in the same order."""
        dev = torch.device(device)
        g = torch.Generator(device=dev).manual_seed(seed)
        H, hd = cfg.hidden_size, cfg.head_dim
        nq, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
        E, I = cfg.num_experts, cfg.moe_intermediate_size
        P, r = 1, 0
        if expert_parallel:
            import torch.distributed as dist

            from .ep_peer import PeerExpertParallelMoE
            P, r = dist.get_world_size(group), dist.get_rank(group)
            if E % P:
                raise ValueError(f"{E} experts do not split over {P} ranks")
        El = E // P

        def rnd(*shape, dtype=torch.bfloat16):
            return (torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * std).to(dtype)

        ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=dev)  # noqa: E731
        layers = []
        for _ in range(cfg.num_hidden_layers):
            gate_up = rnd(E, H, 2 * I)
            w13 = ops.pack_gate_up(gate_up[r * El:(r + 1) * El].contiguous(), "nxd")
            del gate_up
            down = rnd(E, I, H)
            w2 = ops.pack_down(down[r * El:(r + 1) * El].contiguous(), "nxd")
            del down
            experts = ops.PackedExperts(w13, w2, El, H, I)
            attn = (ones(H), rnd((nq + 2 * nkv) * hd, H), ones(hd), ones(hd), rnd(H, nq * hd), ones(H))
            router_w = rnd(E, H, dtype=torch.float32)
            ep = ep_decode = None
            if expert_parallel:
                ep = PeerExpertParallelMoE(router_w, None, None, E, cfg.num_experts_per_tok, max_batch * max_seq,
                                           group=group, device_epochs=True, packed=experts)
                ep_decode = PeerExpertParallelMoE(router_w, None, None, E, cfg.num_experts_per_tok, max_batch,
                                                  group=group, device_epochs=True, packed=experts)
            layers.append(_Layer(*attn, router_w, experts, ep=ep, ep_decode=ep_decode))
        return cls(cfg, rnd(cfg.vocab_size, H), layers, ones(H), rnd(cfg.vocab_size, H), max_batch, max_seq)

    def close(self):
        """Release the expert-parallel exchange buffers (every rank together)."""
        self.release_graph()
        for lyr in self.layers:
            for blk in (lyr.ep, lyr.ep_decode):
                if blk is not None:
                    blk.close()

    @classmethod
    def from_hf(cls, model, device="cuda", max_batch: int = 8, max_seq: int = 640) -> "Qwen3MoEStack":
        """Copy the weights of an HF ``Qwen3MoeForCausalLM`` (bf16 on the GPU,
        router fp32), expert weights from the HF ``[E, 2I, H]`` / ``[E, H, I]``
        layout."""
        cfg = Qwen3MoEConfig.from_hf(model.config)
        dev = torch.device(device)
        bf = lambda t: t.detach().to(dev, torch.bfloat16).contiguous()  # noqa: E731
        layers = []
        for lyr in model.model.layers:
            a, m = lyr.self_attn, lyr.mlp
            qkv = torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0)
            w13 = ops.pack_gate_up(bf(m.experts.gate_up_proj), "hf")
            w2 = ops.pack_down(bf(m.experts.down_proj), "hf")
            layers.append(_Layer(bf(lyr.input_layernorm.weight), bf(qkv), bf(a.q_norm.weight), bf(a.k_norm.weight),
                                 bf(a.o_proj.weight), bf(lyr.post_attention_layernorm.weight),
                                 m.gate.weight.detach().to(dev, torch.float32).contiguous(),
                                 ops.PackedExperts(w13, w2, cfg.num_experts, cfg.hidden_size,
                                                   cfg.moe_intermediate_size)))
        return cls(cfg, bf(model.model.embed_tokens.weight), layers, bf(model.model.norm.weight),
                   bf(model.lm_head.weight), max_batch, max_seq)

    @classmethod
    def from_safetensors(cls, path: str, device="cuda", max_batch: int = 8,
                         max_seq: int = 640) -> "Qwen3MoEStack":
        """Load an HF Qwen3-MoE checkpoint directory (hub format, bf16 or FP8
        with block scales) tensor by tensor: each layer's experts are read in
        the HF fused layout and packed on the device (``hf_loader``)."""
        from .hf_loader import Qwen3MoECheckpoint

        ck = Qwen3MoECheckpoint(path, device=device)
        cfg = Qwen3MoEConfig.from_hf(ck.hf_config)
        pre = ck.reader.prefix
        layers = []
        for l in range(cfg.num_hidden_layers):  # noqa: E741
            t = lambda rest, dtype=None: ck.layer_tensor(l, rest, dtype)  # noqa: E731
            qkv = torch.cat([t("self_attn.q_proj.weight"), t("self_attn.k_proj.weight"),
                             t("self_attn.v_proj.weight")], 0).contiguous()
            gate_up, down = ck.experts(l)
            I = gate_up.shape[1] // 2
            experts = ops.PackedExperts(ops.pack_gate_up(gate_up, "hf"), ops.pack_down(down, "hf"),
                                        cfg.num_experts, cfg.hidden_size, I)
            del gate_up, down
            layers.append(_Layer(t("input_layernorm.weight"), qkv, t("self_attn.q_norm.weight"),
                                 t("self_attn.k_norm.weight"), t("self_attn.o_proj.weight"),
                                 t("post_attention_layernorm.weight"),
                                 t("mlp.gate.weight", torch.float32).contiguous(), experts))
        lm = "lm_head.weight"
        lm_head = ck.tensor(lm) if ck.reader.has(lm) else ck.tensor(f"{pre}embed_tokens.weight")
        return cls(cfg, ck.tensor(f"{pre}embed_tokens.weight"), layers, ck.tensor(f"{pre}norm.weight"), lm_head,
                   max_batch, max_seq)

    # ------------------------------------------------------------ layers
    def _moe_add_norm(self, lyr: _Layer, x: torch.Tensor, res: torch.Tensor, norm_w: torch.Tensor,
                      decode: bool):
        """The layer's MoE block on ``x``, then the residual add and the next
        RMSNorm (the next layer's input norm, or the final norm): returns
        ``(normed, residual)``."""
        eps = self.cfg.rms_norm_eps
        if lyr.ep is not None:
            h = lyr.ep_decode(x) if decode else lyr.ep(x)
            return ops.add_rmsnorm(h, res, norm_w, eps)
        return ops.moe_block_add_rmsnorm(x, lyr.router_w, lyr.experts, self.cfg.num_experts_per_tok, res, norm_w,
                                         eps, router_w_split=lyr.router_split)

    def _qkv(self, lyr: _Layer, xn: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        c = self.cfg
        qkv = F.linear(xn, lyr.qkv_w)
        return ops.qk_norm_rope(qkv, lyr.q_norm, lyr.k_norm, positions, c.num_attention_heads,
                                c.num_key_value_heads, c.head_dim, c.rope_theta, c.rms_norm_eps, out=qkv)

    def _split(self, qkv: torch.Tensor, B: int, S: int):
        c = self.cfg
        nq, nkv, hd = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        q = qkv[:, : nq * hd].view(B, S, nq, hd).transpose(1, 2)
        k = qkv[:, nq * hd:(nq + nkv) * hd].view(B, S, nkv, hd).transpose(1, 2)
        v = qkv[:, (nq + nkv) * hd:].view(B, S, nkv, hd).transpose(1, 2)
        return q, k, v

    def _layers(self, h: torch.Tensor, attention, linear=F.linear, decode: bool = False):
        """Run every layer on h [T, H]; ``attention(li, lyr, xn)`` returns the
        attention output [T, nq*hd] before the O projection (``linear``).
        Returns the final norm of the residual stream."""
        eps = self.cfg.rms_norm_eps
        res = h
        xn = ops.rmsnorm(h, self.layers[0].in_norm, eps)
        for li, lyr in enumerate(self.layers):
            a = linear(attention(li, lyr, xn), lyr.o_w)
            xn, res = ops.add_rmsnorm(a, res, lyr.post_norm, eps)
            # the MoE output joins the residual and feeds the next norm
            nxt = self.layers[li + 1].in_norm if li + 1 < len(self.layers) else self.final_norm
            xn, res = self._moe_add_norm(lyr, xn, res, nxt, decode)
        return xn

    # ------------------------------------------------------------ prefill
    @torch.inference_mode()
    def prefill(self, input_ids: torch.Tensor, all_logits: bool = False) -> torch.Tensor:
        """Causal forward over ``input_ids [B, S]`` from position 0; fills the KV
        cache.  Returns the last position's logits ``[B, V]`` (or all
        positions' ``[B, S, V]`` with ``all_logits``)."""
        B, S = input_ids.shape
        if B > self.max_batch or S > self.max_seq:
            raise ValueError(f"batch {B} x {S} exceeds the cache ({self.max_batch} x {self.max_seq})")
        ids = input_ids.to(self.device)
        h = F.embedding(ids.reshape(-1), self.embed)
        positions = torch.arange(S, device=self.device, dtype=torch.int64).repeat(B)
        c = self.cfg

        def attention(li, lyr, xn):
            q, k, v = self._split(self._qkv(lyr, xn, positions), B, S)
            self.k_cache[li, :B, :, :S].copy_(k)
            self.v_cache[li, :B, :, :S].copy_(v)
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)  # [B, nq, S, hd]
            return o.transpose(1, 2).reshape(B * S, c.num_attention_heads * c.head_dim)

        hn = self._layers(h, attention)
        self.length = S
        if all_logits:
            return F.linear(hn, self.lm_head).view(B, S, -1)
        last = hn.view(B, S, -1)[:, -1]
        return F.linear(last, self.lm_head)

    # ------------------------------------------------------------ decode
    def _decode_body(self, B: int) -> torch.Tensor:
        """One decode step for ``self._tokens[:B]`` at position ``self._pos``:
        per layer the QKV projection, then one library kernel for the q/k
        norms + RoPE, the KV-cache store and the attention over the cache
        (``ops.decode_attention``)."""
        c = self.cfg
        h = F.embedding(self._tokens[:B], self.embed)
        # the projections of a decode batch (<= 16 rows) stream their weights
        # through the library's skinny linear kernel
        linear = ops.skinny_linear if B <= 16 and self._skinny_ok else F.linear

        def attention(li, lyr, xn):
            qkv = linear(xn, lyr.qkv_w)
            return ops.decode_attention(qkv, lyr.q_norm, lyr.k_norm, self._pos, self.k_cache[li], self.v_cache[li],
                                        c.num_attention_heads, c.num_key_value_heads, c.rope_theta, c.rms_norm_eps)

        hn = self._layers(h, attention, linear, decode=True)
        return linear(hn, self.lm_head)

    @torch.inference_mode()
    def decode(self, tokens: torch.Tensor, graph: bool = True) -> torch.Tensor:
        """One decode step: ``tokens [B]`` at position ``self.length``; returns
        logits ``[B, V]`` (a tensor of its own) and advances the position."""
        out = self._step(tokens, graph)
        return out.clone() if graph else out

    def _step(self, tokens: torch.Tensor, graph: bool) -> torch.Tensor:
        """Decode step returning, with ``graph``, the captured graph's output
        buffer itself (overwritten by the next step)."""
        B = tokens.shape[0]
        if self.length >= self.max_seq:
            raise ValueError("KV cache full")
        self._tokens[:B].copy_(tokens.to(self.device).reshape(-1))
        self._pos.fill_(self.length)
        if graph:
            if self._graph is None or self._graph_batch != B:
                self._capture(B)
            self._graph.replay()
            out = self._graph_out
        else:
            out = self._decode_body(B)
        self.length += 1
        return out

    def _capture(self, B: int):
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        # warm up on the capture stream (workspaces sized outside the capture);
        # the cache slot written here is rewritten by every replay
        with torch.cuda.stream(s):
            self._decode_body(B)
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            out = self._decode_body(B)
        self._graph, self._graph_batch, self._graph_out = g, B, out

    def release_graph(self):
        self._graph = self._graph_out = None

    # ------------------------------------------------------------ generate
    @torch.inference_mode()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int, graph: bool = True):
        """Greedy generation.  Returns ``(tokens [B, max_new_tokens], timing)``
        with timing = {"ttft_ms", "decode_ms", "decode_tok_s"} measured with
        CUDA events (TTFT = prefill through the first token's argmax)."""
        B = input_ids.shape[0]
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        torch.cuda.synchronize(self.device)
        ev[0].record()
        logits = self.prefill(input_ids)
        tok = logits.argmax(-1)
        ev[1].record()
        out = [tok]
        for _ in range(max_new_tokens - 1):
            tok = self._step(tok, graph).argmax(-1)
            out.append(tok)
        ev[2].record()
        torch.cuda.synchronize(self.device)
        ttft = ev[0].elapsed_time(ev[1])
        dec = ev[1].elapsed_time(ev[2])
        n = max_new_tokens - 1
        timing = {"ttft_ms": ttft, "decode_ms": dec, "decode_steps": n,
                  "decode_tok_s": (B * n) / (dec * 1e-3) if n and dec > 0 else math.nan}
        return torch.stack(out, 1), timing


def wall_ms(fn) -> float:
    torch.cuda.synchronize()
    t = time.perf_counter()
    fn()
    torch.cuda.synchronize()
    return (time.perf_counter() - t) * 1e3
