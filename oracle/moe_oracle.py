"""numpy restatement of the reference's CPU arithmetic for the MoE hot path.

TEST INFRASTRUCTURE ONLY (the checker, never the thing measured or shipped).

Every function cites the reference file:line it follows (paths are within the
Goomelo/nki-moe project).  Arithmetic is fp32 like the reference's CPU paths
(``router_dtype=torch.float32``, ``qwen_with_nki.py:276``); bf16 workloads are
checked by running this oracle in fp32 on the bf16-rounded inputs.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "bf16_round",
    "rmsnorm",
    "router_logits",
    "topk_softmax",
    "router_topk",
    "permute",
    "silu",
    "expert_ffn",
    "experts_forward",
    "experts_forward_loop",
    "moe_block",
    "swiglu",
    "aggregate",
    "rope_cos_sin",
    "rotate_half",
    "qk_norm_rope",
    "near_tie_tokens",
    "normwise_rel_err",
    "cosine",
]


def bf16_round(a) -> np.ndarray:
    """Round to the nearest bf16 (ties to even) and return the value as fp32."""
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + bias) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32).reshape(a.shape)


def rmsnorm(x, w, eps: float = 1e-6) -> np.ndarray:
    """RMSNorm over the last axis: ``x * rsqrt(mean(x^2) + eps) * w``.

    Follows ``nki_custom_rmsnorm.py:45-64`` (square, sum over the row, divide
    by the hidden size, rsqrt of mean+eps, multiply by x, then by the weight)
    with the fp32 compute of HF ``Qwen3MoeRMSNorm`` used on CPU
    (``qwen_with_nki.py:251-252``).
    """
    x32 = np.asarray(x, dtype=np.float32)
    ms = np.mean(np.square(x32), axis=-1, keepdims=True, dtype=np.float32)
    r = (np.float32(1.0) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    return (x32 * r * np.asarray(w, dtype=np.float32)).astype(np.float32)


def router_logits(x, router_w) -> np.ndarray:
    """``logits = x @ Wr^T`` in fp32 (``nki_moe_integrated.py:437``, ``nn.Linear`` without bias)."""
    x32 = np.asarray(x, dtype=np.float32)
    return (x32 @ np.asarray(router_w, dtype=np.float32).T).astype(np.float32)


def topk_softmax(logits, top_k: int):
    """softmax -> top-k (descending) -> renormalise, ``nki_moe_integrated.py:438-443``.

    Selection is by logit, descending, ties to the lower expert id.  softmax is
    monotone, so this is the order ``torch.topk`` gives on the probabilities;
    the logit breaks exact probability ties deterministically.
    Returns ``idx`` int32 ``[T,K]`` and renormalised weights fp32 ``[T,K]``.
    """
    lg = np.asarray(logits, dtype=np.float32)
    m = lg.max(axis=-1, keepdims=True)
    e = np.exp(lg - m).astype(np.float32)
    p = (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    idx = np.argsort(-lg, axis=-1, kind="stable")[:, :top_k].astype(np.int32)
    wt = np.take_along_axis(p, idx.astype(np.int64), axis=-1)
    wt = (wt / wt.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return idx, wt


def router_topk(x, router_w, top_k: int):
    """Full router, ``nki_moe_integrated.py:436-443``: returns ``(logits, idx, w)``."""
    lg = router_logits(x, router_w)
    idx, wt = topk_softmax(lg, top_k)
    return lg, idx, wt


def near_tie_tokens(logits, top_k: int, gap: float = 1e-5) -> np.ndarray:
    """Boolean mask of tokens whose k-th and (k+1)-th softmax probabilities
    differ by at most ``gap``; routing of those tokens may legitimately flip
    between two fp32 GEMMs with different reduction orders."""
    lg = np.asarray(logits, dtype=np.float32)
    m = lg.max(axis=-1, keepdims=True)
    e = np.exp((lg - m).astype(np.float64))
    p = e / e.sum(axis=-1, keepdims=True)
    ps = -np.sort(-p, axis=-1)
    if top_k >= lg.shape[-1]:
        return np.zeros(lg.shape[0], dtype=bool)
    return (ps[:, top_k - 1] - ps[:, top_k]) <= gap


def permute(idx, num_experts: int):
    """Group the T*K (token, slot) assignments by expert.

    Order follows ``nki_moe_integrated.py:450-467``: slot k outer, expert e
    inner, tokens ascending through a boolean mask, so that inside expert e the
    rows are in (k, t) lexicographic order (the same order HF's
    ``torch.where(expert_mask[e])`` gives).

    A negative id marks an empty slot (no row; used for the per-rank slot
    lists of the expert-parallel dispatch); an id >= E is an error.

    Returns ``(row_token, row_slot, offsets, slot_row)``:
      row_token[r] = t of permuted row r; row_slot[r] = t*K + k;
      offsets[E+1] = exclusive prefix of per-expert counts;
      slot_row[t*K + k] = r (inverse permutation; -1 for an empty slot).
    """
    idx = np.asarray(idx)
    T, K = idx.shape
    flat = idx.T.reshape(-1).astype(np.int64)  # j = k*T + t
    if flat.size and flat.max() >= num_experts:
        raise ValueError("expert index out of range")
    valid = np.nonzero(flat >= 0)[0]
    order = valid[np.argsort(flat[valid], kind="stable")]
    row_k = order // max(T, 1)
    row_t = order % max(T, 1)
    counts = np.bincount(flat[valid], minlength=num_experts)
    offsets = np.zeros(num_experts + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    row_slot = (row_t * K + row_k).astype(np.int32)
    slot_row = np.full(T * K, -1, dtype=np.int32)
    slot_row[row_slot] = np.arange(row_slot.size, dtype=np.int32)
    return row_t.astype(np.int32), row_slot, offsets, slot_row


def silu(g):
    """``F.silu``: ``g * sigmoid(g)`` in fp32."""
    g = np.asarray(g, dtype=np.float32)
    return (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32)


def swiglu(gate_up) -> np.ndarray:
    """``silu(gate) * up`` over a ``[M, 2N]`` gate|up split, ``nki_moe_integrated.py:114-131``."""
    gu = np.asarray(gate_up, dtype=np.float32)
    n = gu.shape[-1] // 2
    return (silu(gu[..., :n]) * gu[..., n:]).astype(np.float32)


def expert_ffn(x_rows, gate_up_e, down_e) -> np.ndarray:
    """One expert on its rows: ``silu(X Gu[:, :I]) * (X Gu[:, I:]) @ D``.

    ``nki_moe_integrated.py:154-161`` (matmul -> SwiGLU -> matmul), weights in
    the ``gate_up_proj[H, 2I]`` / ``down_proj[I, H]`` layout of ``qwen.py:164-226``.
    """
    gu = np.asarray(x_rows, dtype=np.float32) @ np.asarray(gate_up_e, dtype=np.float32)
    return (swiglu(gu) @ np.asarray(down_e, dtype=np.float32)).astype(np.float32)


def experts_forward(x, gate_up, down, idx, wt) -> np.ndarray:
    """Whole MoE expert stage given routing, grouped by expert.

    Same arithmetic as the reference's given-routing CPU paths
    (``nki_moe_kernel.py:473-508``, ``nki_moe_expert.py:428-463``) and the
    grouped XLA branch of ``nki_moe_integrated.py:446-469``; the combine adds
    ``w[t,k] * y`` into a zero accumulator with k ascending (``:482-494``).
    """
    x = np.asarray(x, dtype=np.float32)
    T, H = x.shape
    idx = np.asarray(idx)
    wt = np.asarray(wt, dtype=np.float32)
    K = idx.shape[1]
    E = gate_up.shape[0]
    row_t, row_slot, offsets, slot_row = permute(idx, E)
    y = np.zeros((max(row_t.size, 1), H), dtype=np.float32)
    for e in range(E):
        s, f = int(offsets[e]), int(offsets[e + 1])
        if f > s:
            y[s:f] = expert_ffn(x[row_t[s:f]], gate_up[e], down[e])
    out = np.zeros((T, H), dtype=np.float32)
    rows = slot_row.reshape(T, K)
    for k in range(K):
        ok = rows[:, k] >= 0  # empty slots contribute nothing
        out[ok] += wt[ok, k:k + 1] * y[rows[ok, k]]
    return out


def experts_forward_loop(x, gate_up, down, idx, wt) -> np.ndarray:
    """Per-token, per-slot loop exactly as ``nki_moe_integrated.py:477-496``
    (pure-Python loops; small cases only)."""
    x = np.asarray(x, dtype=np.float32)
    T, H = x.shape
    out = np.zeros((T, H), dtype=np.float32)
    for t in range(T):
        for k in range(idx.shape[1]):
            e = int(idx[t, k])
            out[t] += np.float32(wt[t, k]) * expert_ffn(x[t:t + 1], gate_up[e], down[e])[0]
    return out


def moe_block(x, router_w, gate_up, down, top_k: int):
    """``NKIMoESimple.forward`` (``nki_moe_integrated.py:428-475``) on ``[T, H]``.

    Returns ``(out, logits, idx, w)``.
    """
    lg, idx, wt = router_topk(x, router_w, top_k)
    return experts_forward(x, gate_up, down, idx, wt), lg, idx, wt


def aggregate(expert_outputs) -> np.ndarray:
    """Sum over the leading top-k axis in fp32, ``nki_moe_integrated.py:236-243``."""
    eo = np.asarray(expert_outputs, dtype=np.float32)
    acc = np.zeros(eo.shape[1:], dtype=np.float32)
    for k in range(eo.shape[0]):
        acc += eo[k]
    return acc


def rope_cos_sin(positions, head_dim: int, theta: float):
    """Rotate-half RoPE tables as HF ``Qwen3MoeRotaryEmbedding`` builds them:
    ``inv_freq = 1 / theta^(2i/d)`` in fp32, ``freqs = pos * inv_freq``,
    ``emb = cat(freqs, freqs)``; returns fp32 ``cos, sin`` of shape ``[T, d]``.
    The RoPE base comes from ``qwen_with_nki.py:330-334`` (``rope_theta``)."""
    ar = np.arange(0, head_dim, 2, dtype=np.int64).astype(np.float32) / np.float32(head_dim)
    inv_freq = (np.float32(1.0) / np.power(np.float32(theta), ar, dtype=np.float32)).astype(np.float32)
    pos = np.asarray(positions).astype(np.float32)
    freqs = (pos[:, None] * inv_freq[None, :]).astype(np.float32)
    emb = np.concatenate([freqs, freqs], axis=-1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def rotate_half(x) -> np.ndarray:
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def qk_norm_rope(qkv, q_w, k_w, positions, n_heads: int, n_kv_heads: int,
                 head_dim: int, theta: float, eps: float = 1e-6) -> np.ndarray:
    """Per-head q/k RMSNorm followed by rotate-half RoPE on a fused QKV row.

    Order as in HF ``Qwen3MoeAttention`` (q_norm/k_norm on ``[.., heads, d]``,
    then ``apply_rotary_pos_emb``); the q/k norms are the
    ``NKIRMSNorm(head_dim)`` of ``qwen_with_nki.py:349-350``.  ``qkv`` is
    ``[T, (n_heads + 2*n_kv_heads)*head_dim]`` laid out ``[Q | K | V]``; the
    return value has the same layout with V unchanged.
    """
    qkv = np.asarray(qkv, dtype=np.float32)
    T = qkv.shape[0]
    qd, kd = n_heads * head_dim, n_kv_heads * head_dim
    q = rmsnorm(qkv[:, :qd].reshape(T, n_heads, head_dim), q_w, eps)
    k = rmsnorm(qkv[:, qd:qd + kd].reshape(T, n_kv_heads, head_dim), k_w, eps)
    cos, sin = rope_cos_sin(positions, head_dim, theta)
    q = q * cos[:, None, :] + rotate_half(q) * sin[:, None, :]
    k = k * cos[:, None, :] + rotate_half(k) * sin[:, None, :]
    out = qkv.copy()
    out[:, :qd] = q.reshape(T, qd)
    out[:, qd:qd + kd] = k.reshape(T, kd)
    return out.astype(np.float32)


def normwise_rel_err(y, y_ref) -> float:
    """``max|y - y_ref| / max|y_ref|`` (the bf16 block-output bar)."""
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    den = np.max(np.abs(y_ref))
    return float(np.max(np.abs(y - y_ref)) / den) if den > 0 else float(np.max(np.abs(y)))


def cosine(y, y_ref) -> float:
    a = np.asarray(y, dtype=np.float64).ravel()
    b = np.asarray(y_ref, dtype=np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / (na * nb))
