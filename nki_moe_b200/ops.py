"""Tensor-level entry points over the C ABI.

PyTorch is used here only as plumbing: device memory, the current CUDA
stream and dtype conversions at the boundary.  Every computation runs in
``libnkimoe.so``; CPU tensors are rejected (no CPU fallback), except as the
host buffers of :func:`moe_block_host`, whose block runs on the GPU.
"""

from __future__ import annotations

import ctypes
import os
import threading
import weakref
from collections import OrderedDict

import torch

from . import _lib
from ._lib import BF16, F32, I32, I64, LAYOUT_HF, LAYOUT_NXD, call, size_call

__all__ = [
    "rmsnorm", "add_rmsnorm", "qk_norm_rope", "router_logits", "topk_softmax", "permute",
    "pack_gate_up", "pack_down", "PackedExperts", "packed_experts", "moe_experts", "moe_block",
    "grouped_gemm", "swiglu", "aggregate", "read_status", "workspace", "sync_check_enabled", "router_split",
    "route", "dispatch", "segment_experts", "combine", "ep_dispatch", "decode_attention", "skinny_linear",
    "moe_block_add_rmsnorm", "moe_block_host", "kmajor_weights",
    "release_captured_workspaces", "moe_block_rmsnorm",
]

_DT = {torch.float32: F32, torch.bfloat16: BF16, torch.int32: I32, torch.int64: I64}


def sync_check_enabled() -> bool:
    """When NKIMOE_SYNC_CHECK=1, every block call synchronises and raises on a
    device-flagged fault (timeout, expert id out of range) -- except while a
    CUDA graph is being captured, where a synchronisation is not allowed."""
    return os.environ.get("NKIMOE_SYNC_CHECK", "0") == "1" and not torch.cuda.is_current_stream_capturing()


def _cuda(t: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (this package has no CPU path)")
    return t


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None and t.numel() > 0 else ctypes.c_void_p(0)


def _s(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _contig(t: torch.Tensor, dtype=None) -> torch.Tensor:
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t if t.is_contiguous() else t.contiguous()


# ---------------------------------------------------------------- workspace
_ws_lock = threading.Lock()
_ws: dict = {}
# Buffers that a CUDA graph captured and that a later, larger call replaced:
# the graph still writes them on every replay, so they stay alive until the
# caller says its graphs are gone (release_captured_workspaces).
_ws_retired: list = []


def _grow(table: dict, key, device: torch.device, nbytes: int, zero: bool) -> torch.Tensor:
    """The buffer of ``table[key]``, replaced by a larger one when it is
    smaller than ``nbytes``.  A buffer handed out while the current stream
    is being captured is marked, and a marked buffer that gets replaced is
    kept in ``_ws_retired`` instead of going back to the allocator."""
    capturing = torch.cuda.is_current_stream_capturing()
    with _ws_lock:
        buf = table.get(key)
        if buf is None or buf.numel() < nbytes:
            if buf is not None and getattr(buf, "_nkimoe_captured", False):
                _ws_retired.append(buf)
            n = max(nbytes, 1 << 20 if not zero else 1 << 16)
            buf = torch.zeros(n, dtype=torch.uint8, device=device) if zero else \
                torch.empty(n, dtype=torch.uint8, device=device)
            table[key] = buf
        if capturing:
            buf._nkimoe_captured = True
        return buf


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A per-(device, stream) scratch buffer from the torch caching allocator,
    grown on demand and reused by later calls on the same stream.  A buffer
    that a CUDA graph captured outlives its replacement by a larger call
    (streams from torch's pool reuse their handles), until
    :func:`release_captured_workspaces`."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    return _grow(_ws, key, device, nbytes, zero=False)


def release_captured_workspaces() -> int:
    """Drop the replaced workspaces kept for captured CUDA graphs (call after
    those graphs are destroyed).  Returns how many were released."""
    with _ws_lock:
        n = len(_ws_retired)
        _ws_retired.clear()
    return n


def read_status(ws: torch.Tensor) -> int:
    st = ctypes.c_int(0)
    call("nkimoe_read_status", _p(ws), _s(ws), ctypes.byref(st))
    return st.value


# ---------------------------------------------------------------- norms
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, out_dtype=None) -> torch.Tensor:
    """``x * rsqrt(mean(x^2) + eps) * weight`` over the last axis (K1)."""
    _cuda(x, "x")
    _cuda(weight, "weight")
    if x.dtype not in (torch.float32, torch.bfloat16):
        x = x.to(torch.bfloat16)
    if weight.dtype not in (torch.float32, torch.bfloat16):
        weight = weight.float()
    x = _contig(x)
    weight = _contig(weight)
    out_dtype = out_dtype or x.dtype
    out = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    H = x.shape[-1]
    rows = x.numel() // H if H else 0
    call("nkimoe_rmsnorm", _p(x), _DT[x.dtype], _p(weight), _DT[weight.dtype], _p(out), _DT[out_dtype],
         rows, H, float(eps), _s(x))
    return out


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
                residual_out: torch.Tensor | None = None):
    """``r = x + residual``; returns ``(rmsnorm(r), r)`` (bf16)."""
    x = _contig(_cuda(x, "x"), torch.bfloat16)
    residual = _contig(_cuda(residual, "residual"), torch.bfloat16)
    weight = _contig(_cuda(weight, "weight"))
    if weight.dtype not in (torch.float32, torch.bfloat16):
        weight = weight.float()
    if residual_out is None:
        residual_out = torch.empty_like(x)
    out = torch.empty_like(x)
    H = x.shape[-1]
    call("nkimoe_add_rmsnorm", _p(x), _p(residual), _p(residual_out), _p(weight), _DT[weight.dtype], _p(out),
         x.numel() // H, H, float(eps), _s(x))
    return out, residual_out


def qk_norm_rope(qkv: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor, positions: torch.Tensor,
                 n_heads: int, n_kv_heads: int, head_dim: int = 128, theta: float = 1e6, eps: float = 1e-6,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-head q/k RMSNorm + rotate-half RoPE on a fused ``[T, (nh+2nkv)*d]``
    bf16 QKV row (K6).  ``out`` may be ``qkv`` (in place)."""
    qkv = _contig(_cuda(qkv, "qkv"), torch.bfloat16)
    T = qkv.numel() // ((n_heads + 2 * n_kv_heads) * head_dim)
    wdt = torch.float32 if q_weight.dtype == torch.float32 else torch.bfloat16
    qw = _contig(_cuda(q_weight, "q_weight"), wdt)
    kw = _contig(_cuda(k_weight, "k_weight"), wdt)
    pos = _contig(_cuda(positions, "positions").reshape(-1), torch.int64)
    if pos.numel() != T:
        raise ValueError(f"positions has {pos.numel()} entries for {T} tokens")
    if out is None:
        out = torch.empty_like(qkv)
    call("nkimoe_qk_norm_rope", _p(qkv), _p(out), _p(qw), _p(kw), _DT[wdt], _p(pos), T, n_heads, n_kv_heads,
         head_dim, float(theta), float(eps), _s(qkv))
    return out


_attn_ws: dict = {}


def _attention_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Zero-filled per-(device, stream) workspace of the decode attention
    (its split counters must start at zero; every call leaves them at zero).
    Kept for captured graphs as :func:`workspace` is."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    return _grow(_attn_ws, key, device, nbytes, zero=True)


def decode_attention(qkv: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor, positions: torch.Tensor,
                     k_cache: torch.Tensor, v_cache: torch.Tensor, n_heads: int, n_kv_heads: int,
                     theta: float = 1e6, eps: float = 1e-6, scale: float | None = None,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """One decode step of grouped-query attention over a KV cache, fused with
    the q/k RMSNorm + RoPE of the step's token and the store of its key and
    value at its position.

    ``qkv``: ``[B, (n_heads + 2*n_kv_heads) * 128]`` bf16, the QKV projection
    before the norms; ``positions``: int64 ``[B]`` or ``[1]`` (one position for
    every sequence); ``k_cache``/``v_cache``: one layer's ``[B', n_kv_heads,
    max_seq, 128]`` bf16 caches (B' >= B, updated in place).  Returns
    ``[B, n_heads * 128]`` bf16."""
    hd = 128
    qkv = _cuda(qkv, "qkv")
    if qkv.dtype != torch.bfloat16 or not qkv.is_contiguous():
        raise ValueError("qkv must be a contiguous bf16 tensor")
    B = qkv.numel() // ((n_heads + 2 * n_kv_heads) * hd)
    for name, c in (("k_cache", k_cache), ("v_cache", v_cache)):
        _cuda(c, name)
        if c.dtype != torch.bfloat16 or c.dim() != 4 or c.shape[1] != n_kv_heads or c.shape[3] != hd:
            raise ValueError(f"{name} must be bf16 [B, {n_kv_heads}, max_seq, {hd}]")
        if c.shape[0] < B or not c[:B].is_contiguous():
            raise ValueError(f"{name} must hold {B} contiguous sequences")
    max_seq = k_cache.shape[2]
    if v_cache.shape != k_cache.shape:
        raise ValueError("k_cache and v_cache differ in shape")
    wdt = torch.float32 if q_weight.dtype == torch.float32 else torch.bfloat16
    qw = _contig(_cuda(q_weight, "q_weight"), wdt)
    kw = _contig(_cuda(k_weight, "k_weight"), wdt)
    pos = _cuda(positions, "positions").reshape(-1)
    if pos.dtype != torch.int64 or not pos.is_contiguous():
        raise ValueError("positions must be a contiguous int64 tensor")
    if pos.numel() not in (1, B):
        raise ValueError(f"positions has {pos.numel()} entries for {B} sequences")
    if out is None:
        out = torch.empty(B, n_heads * hd, dtype=torch.bfloat16, device=qkv.device)
    nbytes = size_call("nkimoe_decode_attention_workspace_bytes", B, n_heads, n_kv_heads, hd, max_seq)
    ws = _attention_workspace(qkv.device, nbytes)
    call("nkimoe_decode_attention", _p(qkv), _p(qw), _p(kw), _DT[wdt], _p(pos), 0 if pos.numel() == 1 else 1,
         _p(k_cache), _p(v_cache), _p(out), B, n_heads, n_kv_heads, hd, max_seq, float(theta), float(eps),
         float(scale if scale is not None else hd ** -0.5), _p(ws), ws.numel(), _s(qkv))
    if sync_check_enabled():
        read_status(ws)
    return out


def skinny_linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ w.T`` for at most 16 rows of ``x`` (bf16, fp32 accumulation):
    the decode step's projections, streaming ``w`` [N, K] once."""
    x = _cuda(x, "x")
    w = _cuda(w, "w")
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError("skinny_linear takes bf16 x and w")
    x = _contig(x)
    w = _contig(w)
    K = x.shape[-1]
    M = x.numel() // K if K else 0
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"w is {tuple(w.shape)}, x has {K} columns")
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=torch.bfloat16, device=x.device)
    call("nkimoe_skinny_linear", _p(x), _p(w), _p(out), M, N, K, _s(x))
    return out


# ---------------------------------------------------------------- router
def router_logits(x: torch.Tensor, router_w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    x = _contig(_cuda(x, "x"), torch.bfloat16)
    rw = _contig(_cuda(router_w, "router_w"), torch.float32)
    b = _contig(bias, torch.float32) if bias is not None else None
    T, H = x.shape
    E = rw.shape[0]
    out = torch.empty(T, E, dtype=torch.float32, device=x.device)
    call("nkimoe_router_logits", _p(x), _p(rw), _p(b), _p(out), T, H, E, _s(x))
    return out


def topk_softmax(logits: torch.Tensor, top_k: int):
    lg = _contig(_cuda(logits, "logits"), torch.float32)
    T, E = lg.shape
    idx = torch.empty(T, top_k, dtype=torch.int32, device=lg.device)
    w = torch.empty(T, top_k, dtype=torch.float32, device=lg.device)
    call("nkimoe_topk_softmax", _p(lg), T, E, top_k, _p(idx), _p(w), _s(lg))
    return idx, w


# ---------------------------------------------------------------- permutation
def permute(idx: torch.Tensor, num_experts: int):
    """Returns ``(row_token, row_slot, slot_row, expert_offsets)`` (int32)."""
    idx = _contig(_cuda(idx, "idx"))
    if idx.dtype not in (torch.int32, torch.int64):
        idx = idx.to(torch.int64)
    T, K = idx.shape
    dev = idx.device
    rt = torch.empty(T * K, dtype=torch.int32, device=dev)
    rs = torch.empty(T * K, dtype=torch.int32, device=dev)
    sr = torch.empty(T * K, dtype=torch.int32, device=dev)
    off = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    nbytes = size_call("nkimoe_permute_workspace_bytes", T, K, num_experts)
    ws = workspace(dev, nbytes)
    call("nkimoe_permute", _p(idx), _DT[idx.dtype], T, K, num_experts, _p(rt), _p(rs), _p(sr), _p(off), _p(ws),
         ws.numel(), _s(idx))
    if sync_check_enabled():
        read_status(ws)
    return rt, rs, sr, off


# ---------------------------------------------------------------- weights
class PackedExperts:
    """Expert weights in the GEMM layout: ``w13 [E, 2I, H]`` (K-major, 128-row
    blocks of [gate 64 | up 64]) and ``w2 [E, H, I]`` (K-major), bf16."""

    def __init__(self, w13: torch.Tensor, w2: torch.Tensor, num_experts: int, hidden: int, inter: int):
        self.w13, self.w2 = w13, w2
        self.num_experts, self.hidden, self.inter = num_experts, hidden, inter


def pack_gate_up(gate_up: torch.Tensor, layout: str = "nxd") -> torch.Tensor:
    g = _contig(_cuda(gate_up, "gate_up"), torch.bfloat16)
    if layout == "nxd":
        E, H, I2 = g.shape
        code = LAYOUT_NXD
    elif layout == "hf":
        E, I2, H = g.shape
        code = LAYOUT_HF
    else:
        raise ValueError(f"unknown layout {layout}")
    out = torch.empty(E, I2, H, dtype=torch.bfloat16, device=g.device)
    call("nkimoe_pack_gate_up", _p(g), code, _p(out), E, H, I2 // 2, _s(g))
    return out


def pack_down(down: torch.Tensor, layout: str = "nxd") -> torch.Tensor:
    d = _contig(_cuda(down, "down"), torch.bfloat16)
    if layout == "nxd":
        E, I, H = d.shape
        code = LAYOUT_NXD
    elif layout == "hf":
        E, H, I = d.shape
        code = LAYOUT_HF
    else:
        raise ValueError(f"unknown layout {layout}")
    out = torch.empty(E, H, I, dtype=torch.bfloat16, device=d.device)
    call("nkimoe_pack_down", _p(d), code, _p(out), E, H, I, _s(d))
    return out


_pack_lock = threading.Lock()
_pack_cache: "OrderedDict[tuple, tuple]" = OrderedDict()
_PACK_CACHE_MAX = int(os.environ.get("NKIMOE_PACK_CACHE", "4"))


def _stamp(t: torch.Tensor):
    return (t.data_ptr(), t._version, tuple(t.shape), t.dtype, t.device.index)


def packed_experts(gate_up: torch.Tensor, down: torch.Tensor, layout: str = "nxd") -> PackedExperts:
    """Pack (once) and cache.  An entry is reused only while the very same
    source tensors are alive and unmodified (weak references + pointer,
    version and shape stamps), so freed-and-reused memory never hits a stale
    entry."""
    key = (id(gate_up), id(down), layout)
    with _pack_lock:
        hit = _pack_cache.get(key)
        if hit is not None:
            wg, wd, sg, sd, pe = hit
            if wg() is gate_up and wd() is down and sg == _stamp(gate_up) and sd == _stamp(down):
                _pack_cache.move_to_end(key)
                return pe
            del _pack_cache[key]
    w13 = pack_gate_up(gate_up.detach(), layout)
    w2 = pack_down(down.detach(), layout)
    E, I2, H = w13.shape
    pe = PackedExperts(w13, w2, E, H, I2 // 2)
    with _pack_lock:
        for k in [k for k, v in _pack_cache.items() if v[0]() is None or v[1]() is None]:
            del _pack_cache[k]
        _pack_cache[key] = (weakref.ref(gate_up), weakref.ref(down), _stamp(gate_up), _stamp(down), pe)
        while len(_pack_cache) > _PACK_CACHE_MAX:
            _pack_cache.popitem(last=False)
    return pe


_kmajor_cache: "OrderedDict[int, tuple]" = OrderedDict()


def kmajor_weights(w: torch.Tensor, k_multiple: int = 64, n_multiple: int = 128) -> torch.Tensor:
    """Weights ``w [E, K, N]`` (or ``[K, N]``, taken as one expert) as the
    grouped GEMM's K-major bf16 operand ``[E, N', K']``, K and N zero-padded to
    the given multiples.  The transpose runs in the library (``nkimoe_pack_down``)
    once per weight tensor and is cached while ``w`` lives unmodified (weak
    reference + pointer/version stamp, as :func:`packed_experts`)."""
    key = id(w)
    with _pack_lock:
        hit = _kmajor_cache.get(key)
        if hit is not None and hit[0]() is w and hit[1] == _stamp(w) and hit[2] == (k_multiple, n_multiple):
            _kmajor_cache.move_to_end(key)
            return hit[3]
    src = _contig(_cuda(w, "w").detach(), torch.bfloat16)
    if src.dim() == 2:
        src = src.unsqueeze(0)
    E, K, N = src.shape
    Kp, Np = -(-K // k_multiple) * k_multiple, -(-N // n_multiple) * n_multiple
    if (Kp, Np) != (K, N):
        src = torch.nn.functional.pad(src, (0, Np - N, 0, Kp - K)).contiguous()
    out = torch.empty(E, Np, Kp, dtype=torch.bfloat16, device=src.device)
    # pack_down's plain transpose: [E, I, H] -> [E, H, I] with I = K', H = N'
    call("nkimoe_pack_down", _p(src), LAYOUT_NXD, _p(out), E, Np, Kp, _s(src))
    with _pack_lock:
        for k in [k for k, v in _kmajor_cache.items() if v[0]() is None]:
            del _kmajor_cache[k]
        _kmajor_cache[key] = (weakref.ref(w), _stamp(w), (k_multiple, n_multiple), out)
        while len(_kmajor_cache) > _PACK_CACHE_MAX:
            _kmajor_cache.popitem(last=False)
    return out


# ---------------------------------------------------------------- MoE block
def moe_experts(x: torch.Tensor, experts: PackedExperts, idx: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    """``out[t] = sum_k w[t,k] * FFN_{idx[t,k]}(x[t])`` (bf16 in/out)."""
    x = _contig(_cuda(x, "x"), torch.bfloat16)
    idx = _contig(_cuda(idx, "idx"))
    if idx.dtype not in (torch.int32, torch.int64):
        idx = idx.to(torch.int64)
    w = _contig(_cuda(weights, "weights"), torch.float32)
    T, H = x.shape
    K = idx.shape[1]
    E, I = experts.num_experts, experts.inter
    if H != experts.hidden or idx.shape[0] != T or w.shape != idx.shape:
        raise ValueError("shape mismatch between hidden states, routing and expert weights")
    out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
    nbytes = size_call("nkimoe_moe_workspace_bytes", T, H, I, E, K)
    ws = workspace(x.device, nbytes)
    call("nkimoe_moe_experts", _p(x), _p(experts.w13), _p(experts.w2), _p(idx), _DT[idx.dtype], _p(w), _p(out),
         T, H, I, E, K, _p(ws), ws.numel(), _s(x))
    if sync_check_enabled():
        read_status(ws)
    return out


_router_lock = threading.Lock()
_router_cache: "OrderedDict[int, tuple]" = OrderedDict()


def router_split(router_w: torch.Tensor) -> torch.Tensor:
    """fp32 router weights [E, H] -> bf16 planes [3, E, H] (hi, mid, lo; exact
    sum) for the tensor-core router; cached while the source tensor lives
    unmodified."""
    key = id(router_w)
    with _router_lock:
        hit = _router_cache.get(key)
        if hit is not None and hit[0]() is router_w and hit[1] == _stamp(router_w):
            return hit[2]
    rw = _contig(_cuda(router_w, "router_w").detach(), torch.float32)
    E, H = rw.shape
    out = torch.empty(3, E, H, dtype=torch.bfloat16, device=rw.device)
    call("nkimoe_router_split", _p(rw), _p(out), E, H, _s(rw))
    with _router_lock:
        for k in [k for k, v in _router_cache.items() if v[0]() is None]:
            del _router_cache[k]
        _router_cache[key] = (weakref.ref(router_w), _stamp(router_w), out)
        while len(_router_cache) > _PACK_CACHE_MAX:
            _router_cache.popitem(last=False)
    return out


def moe_block(x: torch.Tensor, router_w: torch.Tensor, experts: PackedExperts, top_k: int,
              bias: torch.Tensor | None = None, return_routing: bool = False, tensor_router: bool = True,
              router_w_split: torch.Tensor | None = None):
    """Router (fp32) + softmax/top-k/renormalise + experts (K2..K7).

    With ``tensor_router`` the fp32 router GEMM of large batches runs on the
    tensor cores over the exact three-plane bf16 split of ``router_w``
    (``router_w_split``, [3, E, H] from :func:`router_split`, when the caller
    keeps it; otherwise taken from a small cache)."""
    x = _contig(_cuda(x, "x"), torch.bfloat16)
    rsplit = None
    if tensor_router and router_w.shape[0] % 128 == 0:
        rsplit = router_w_split if router_w_split is not None else router_split(router_w)
    rw = _contig(_cuda(router_w, "router_w"), torch.float32)
    b = _contig(bias, torch.float32) if bias is not None else None
    T, H = x.shape
    E, I = experts.num_experts, experts.inter
    out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
    idx = w = None
    if return_routing:
        idx = torch.empty(T, top_k, dtype=torch.int32, device=x.device)
        w = torch.empty(T, top_k, dtype=torch.float32, device=x.device)
    nbytes = size_call("nkimoe_moe_workspace_bytes", T, H, I, E, top_k)
    ws = workspace(x.device, nbytes)
    call("nkimoe_moe_block", _p(x), _p(rw), _p(b), _p(rsplit), _p(experts.w13), _p(experts.w2), _p(out), _p(idx),
         _p(w), T, H, I, E, top_k, _p(ws), ws.numel(), _s(x))
    if sync_check_enabled():
        read_status(ws)
    return (out, idx, w) if return_routing else out


_host_ws: dict = {}


def _host_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Per-(device, stream) workspace of the host-batch block, kept apart from
    :func:`workspace`: with a completion event, the library's copy back still
    reads a call's staging rows after the stream has moved on, so no device
    entry point may write them meanwhile."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    with _ws_lock:
        buf = _host_ws.get(key)
        if buf is not None and buf.numel() >= nbytes:
            return buf
    # the copy streams may still use the buffer being replaced (its memory
    # goes back to this stream's pool)
    torch.cuda.synchronize(device)
    buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
    with _ws_lock:
        _host_ws[key] = buf
    return buf


def moe_block_host(x: torch.Tensor, router_w: torch.Tensor, experts: PackedExperts, top_k: int,
                   bias: torch.Tensor | None = None, out: torch.Tensor | None = None, chunk_tokens: int = 0,
                   return_routing: bool = False, router_w_split: torch.Tensor | None = None,
                   non_blocking: bool = False, done: torch.cuda.Event | None = None):
    """:func:`moe_block` on a HOST batch ``x [T, H]`` (bf16; page-locked for
    the copies to overlap): the tokens cross to the weights' GPU in chunks
    whose copies overlap the block on the chunk before, and the result comes
    back to ``out`` (a new page-locked host tensor when None).  Equal to
    :func:`moe_block` on the whole batch bit for bit (chunks are cut only where
    each takes the whole batch's router and GEMM paths).  Routing outputs, when
    asked for, stay on the GPU.  The work runs on the current stream of the
    weights' device.

    ``done`` None: the stream completes with the copy back, and the call
    synchronises it unless ``non_blocking``.  ``done`` an event: the copy
    back's completion is recorded on it and the stream goes on without it, so
    the next call's block overlaps this call's copy back (and this call's copy
    in overlaps the previous call's block); ``out`` is ready after
    ``done.synchronize()``.  Until then ``x`` and ``out`` must stay alive and
    untouched."""
    if x.is_cuda:
        raise ValueError("x must be a host tensor (moe_block takes device tensors)")
    dev = _cuda(router_w, "router_w").device
    x = _contig(x, torch.bfloat16)
    T, H = x.shape
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, pin_memory=True)
    elif out.is_cuda or out.dtype != torch.bfloat16 or tuple(out.shape) != (T, H) or not out.is_contiguous():
        raise ValueError("out must be a contiguous bf16 host tensor shaped like x")
    rsplit = None
    if router_w.shape[0] % 128 == 0:
        rsplit = router_w_split if router_w_split is not None else router_split(router_w)
    rw = _contig(router_w, torch.float32)
    b = _contig(_cuda(bias, "bias"), torch.float32) if bias is not None else None
    E, I = experts.num_experts, experts.inter
    idx = w = None
    if return_routing:
        idx = torch.empty(T, top_k, dtype=torch.int32, device=dev)
        w = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    nbytes = size_call("nkimoe_moe_block_host_workspace_bytes", T, H, I, E, top_k)
    with torch.cuda.device(dev):
        ws = _host_workspace(dev, nbytes)
        ev = None
        if done is not None:
            done.record(torch.cuda.current_stream(dev))  # creates the CUDA event on this device
            ev = ctypes.c_void_p(done.cuda_event)
        call("nkimoe_moe_block_host", _p(x), _p(rw), _p(b), _p(rsplit), _p(experts.w13), _p(experts.w2), _p(out),
             _p(idx), _p(w), T, H, I, E, top_k, int(chunk_tokens), _p(ws), ws.numel(), ev, _s(rw))
        if sync_check_enabled():
            read_status(ws)
            if done is not None:
                done.synchronize()
        elif not non_blocking and done is None:
            torch.cuda.current_stream(dev).synchronize()
    return (out, idx, w) if return_routing else out


def moe_block_rmsnorm(h: torch.Tensor, norm_weight: torch.Tensor, router_w: torch.Tensor, experts: PackedExperts,
                      top_k: int, eps: float = 1e-6, bias: torch.Tensor | None = None, return_x: bool = False,
                      return_routing: bool = False, router_w_split: torch.Tensor | None = None):
    """The block with the RMSNorm in front of it inside the call:
    ``moe_block(rmsnorm(h) * norm_weight)``, equal bit for bit to
    :func:`rmsnorm` + :func:`moe_block`.  For prefill batches (more than 512
    tokens, 128 experts) the norm and the router logits are one tensor-core
    kernel that writes the normalised rows once.  With
    ``return_x`` also returns the normalised rows (bf16)."""
    h = _contig(_cuda(h, "h"), torch.bfloat16)
    rsplit = None
    if router_w.shape[0] % 128 == 0:
        rsplit = router_w_split if router_w_split is not None else router_split(router_w)
    rw = _contig(_cuda(router_w, "router_w"), torch.float32)
    wdt = torch.float32 if norm_weight.dtype == torch.float32 else torch.bfloat16
    nw = _contig(_cuda(norm_weight, "norm_weight"), wdt)
    b = _contig(bias, torch.float32) if bias is not None else None
    T, H = h.shape
    E, I = experts.num_experts, experts.inter
    out = torch.empty(T, H, dtype=torch.bfloat16, device=h.device)
    x = torch.empty_like(h) if return_x else None
    idx = w = None
    if return_routing:
        idx = torch.empty(T, top_k, dtype=torch.int32, device=h.device)
        w = torch.empty(T, top_k, dtype=torch.float32, device=h.device)
    nbytes = size_call("nkimoe_moe_block_rmsnorm_workspace_bytes", T, H, I, E, top_k)
    ws = workspace(h.device, nbytes)
    call("nkimoe_moe_block_rmsnorm", _p(h), _p(nw), _DT[wdt], float(eps), _p(x), _p(rw), _p(b), _p(rsplit),
         _p(experts.w13), _p(experts.w2), _p(out), _p(idx), _p(w), T, H, I, E, top_k, _p(ws), ws.numel(), _s(h))
    if sync_check_enabled():
        read_status(ws)
    res = (out,)
    if return_x:
        res += (x,)
    if return_routing:
        res += (idx, w)
    return res if len(res) > 1 else out


def moe_block_add_rmsnorm(x: torch.Tensor, router_w: torch.Tensor, experts: PackedExperts, top_k: int,
                          residual: torch.Tensor, norm_weight: torch.Tensor, eps: float = 1e-6,
                          residual_out: torch.Tensor | None = None, router_w_split: torch.Tensor | None = None):
    """The MoE block on ``x`` followed by the decoder's residual add and the
    next RMSNorm: returns ``(rmsnorm(r) * norm_weight, r)`` with
    ``r = residual + moe(x)`` (bf16).  ``residual_out`` may be ``residual``
    (in place).  Equal bit for bit to :func:`moe_block` + :func:`add_rmsnorm`;
    up to 512 tokens the block's combine and the norm are one kernel."""
    x = _contig(_cuda(x, "x"), torch.bfloat16)
    residual = _contig(_cuda(residual, "residual"), torch.bfloat16)
    rsplit = None
    if router_w.shape[0] % 128 == 0:
        rsplit = router_w_split if router_w_split is not None else router_split(router_w)
    rw = _contig(_cuda(router_w, "router_w"), torch.float32)
    wdt = torch.float32 if norm_weight.dtype == torch.float32 else torch.bfloat16
    nw = _contig(_cuda(norm_weight, "norm_weight"), wdt)
    T, H = x.shape
    if residual.shape != x.shape:
        raise ValueError(f"residual {tuple(residual.shape)} does not match x {tuple(x.shape)}")
    if residual_out is None:
        residual_out = torch.empty_like(residual)
    out = torch.empty_like(x)
    E, I = experts.num_experts, experts.inter
    nbytes = size_call("nkimoe_moe_workspace_bytes", T, H, I, E, top_k)
    ws = workspace(x.device, nbytes)
    call("nkimoe_moe_block_add_rmsnorm", _p(x), _p(rw), None, _p(rsplit), _p(experts.w13), _p(experts.w2),
         _p(residual), _p(residual_out), _p(nw), _DT[wdt], float(eps), _p(out), None, None, T, H, I, E, top_k,
         _p(ws), ws.numel(), _s(x))
    if sync_check_enabled():
        read_status(ws)
    return out, residual_out


# ---------------------------------------------------------------- pieces
def grouped_gemm(a: torch.Tensor, w_packed: torch.Tensor, offsets: torch.Tensor,
                 out_row_map: torch.Tensor | None = None, out_rows: int | None = None) -> torch.Tensor:
    """``out[r] = a[r] @ w_packed[e]^T`` for rows r of expert segment e."""
    a = _contig(_cuda(a, "a"), torch.bfloat16)
    w = _contig(_cuda(w_packed, "w_packed"), torch.bfloat16)
    off = _contig(_cuda(offsets, "offsets"), torch.int32)
    M, Kd = a.shape
    E, N, Kw = w.shape
    if Kw != Kd:
        raise ValueError("inner dimensions differ")
    rows = M if out_rows is None else out_rows
    out = torch.empty(rows, N, dtype=torch.bfloat16, device=a.device)
    rm = _contig(out_row_map, torch.int32) if out_row_map is not None else None
    st = workspace(a.device, 256)
    call("nkimoe_grouped_gemm", _p(a), _p(w), _p(off), _p(rm), _p(out), M, N, Kd, E, _p(st), _s(a))
    return out


def swiglu(gate_up: torch.Tensor) -> torch.Tensor:
    g = _contig(_cuda(gate_up, "gate_up"), torch.bfloat16)
    M, N2 = g.shape
    out = torch.empty(M, N2 // 2, dtype=torch.bfloat16, device=g.device)
    call("nkimoe_swiglu", _p(g), _p(out), M, N2 // 2, _s(g))
    return out


def aggregate(expert_outputs: torch.Tensor) -> torch.Tensor:
    eo = _contig(_cuda(expert_outputs, "expert_outputs"), torch.bfloat16)
    K, T, H = eo.shape
    out = torch.empty(T, H, dtype=torch.bfloat16, device=eo.device)
    call("nkimoe_aggregate", _p(eo), _p(out), K, T, H, _s(eo))
    return out


# ---------------------------------------------------------------- expert-parallel pieces
def route(x: torch.Tensor, router_w: torch.Tensor, top_k: int, bias: torch.Tensor | None = None,
          tensor_router: bool = True):
    """Router + softmax/top-k/renormalise: ``(idx int32 [T,K], w fp32 [T,K])``."""
    x = _contig(_cuda(x, "x"), torch.bfloat16)
    rsplit = router_split(router_w) if tensor_router and router_w.shape[0] % 128 == 0 else None
    rw = _contig(_cuda(router_w, "router_w"), torch.float32)
    b = _contig(bias, torch.float32) if bias is not None else None
    T, H = x.shape
    E = rw.shape[0]
    idx = torch.empty(T, top_k, dtype=torch.int32, device=x.device)
    w = torch.empty(T, top_k, dtype=torch.float32, device=x.device)
    ws = workspace(x.device, size_call("nkimoe_route_workspace_bytes", T, H, E, top_k))
    call("nkimoe_route", _p(x), _p(rw), _p(b), _p(rsplit), _p(idx), _p(w), T, H, E, top_k, _p(ws), ws.numel(), _s(x))
    return idx, w


def dispatch(x: torch.Tensor, idx: torch.Tensor, weights: torch.Tensor, num_experts: int):
    """Group the (token, slot) rows by global expert: returns ``(x_perm [T*K, H],
    row_weight [T*K], slot_row [T*K], expert_counts [E])``."""
    x = _contig(_cuda(x, "x"), torch.bfloat16)
    idx = _contig(_cuda(idx, "idx"))
    if idx.dtype not in (torch.int32, torch.int64):
        idx = idx.to(torch.int64)
    w = _contig(_cuda(weights, "weights"), torch.float32)
    T, H = x.shape
    K = idx.shape[1]
    dev = x.device
    x_perm = torch.empty(T * K, H, dtype=torch.bfloat16, device=dev)
    row_weight = torch.empty(T * K, dtype=torch.float32, device=dev)
    slot_row = torch.empty(T * K, dtype=torch.int32, device=dev)
    counts = torch.empty(num_experts, dtype=torch.int32, device=dev)
    ws = workspace(dev, size_call("nkimoe_dispatch_workspace_bytes", T, K, num_experts))
    call("nkimoe_dispatch", _p(x), _p(idx), _DT[idx.dtype], _p(w), T, H, num_experts, K, _p(x_perm), _p(row_weight),
         _p(slot_row), _p(counts), _p(ws), ws.numel(), _s(x))
    if sync_check_enabled():
        read_status(ws)
    return x_perm, row_weight, slot_row, counts


def segment_experts(a: torch.Tensor, row_weight: torch.Tensor, segment_counts: torch.Tensor,
                    experts: PackedExperts) -> torch.Tensor:
    """``y[r] = row_weight[r] * FFN_{s % E_local}(a[r])`` for rows r of segment s."""
    a = _contig(_cuda(a, "a"), torch.bfloat16)
    rw = _contig(_cuda(row_weight, "row_weight"), torch.float32)
    sc = _contig(_cuda(segment_counts, "segment_counts").reshape(-1), torch.int32)
    R, H = a.shape
    S = sc.numel()
    y = torch.empty(R, H, dtype=torch.bfloat16, device=a.device)
    ws = workspace(a.device, size_call("nkimoe_segment_experts_workspace_bytes", R, experts.inter, S))
    call("nkimoe_segment_experts", _p(a), _p(rw), _p(sc), S, experts.num_experts, _p(experts.w13), _p(experts.w2),
         _p(y), R, H, experts.inter, _p(ws), ws.numel(), _s(a))
    if sync_check_enabled():
        read_status(ws)
    return y


def combine(y: torch.Tensor, slot_row: torch.Tensor, tokens: int, top_k: int,
            slot_weight: torch.Tensor | None = None) -> torch.Tensor:
    """``out[t] = sum_k (w[t,k]) * y[slot_row[t*K+k]]`` (fp32 sum, k ascending)."""
    y = _contig(_cuda(y, "y"), torch.bfloat16)
    sr = _contig(_cuda(slot_row, "slot_row"), torch.int32)
    sw = _contig(slot_weight, torch.float32) if slot_weight is not None else None
    H = y.shape[1]
    out = torch.empty(tokens, H, dtype=torch.bfloat16, device=y.device)
    call("nkimoe_combine", _p(y), _p(sr), _p(sw), _p(out), tokens, top_k, H, _s(y))
    return out


def ep_dispatch(x: torch.Tensor, idx: torch.Tensor, weights: torch.Tensor, num_ranks: int, experts_per_rank: int):
    """De-duplicated expert-parallel dispatch: one send row per (token, rank).

    Returns ``(x_send [R, H], slots [R, K] int32, wts [R, K] fp32, rank_counts [P]
    int32, slot_row [T, P] int32)``; the buffers hold ``T*min(P, K)`` rows, of
    which ``rank_counts.sum()`` are valid.
    """
    x = _contig(_cuda(x, "x"), torch.bfloat16)
    idx = _contig(_cuda(idx, "idx"), torch.int32)
    w = _contig(_cuda(weights, "weights"), torch.float32)
    T, H = x.shape
    K = idx.shape[1]
    P = num_ranks
    dev = x.device
    cap = T * min(P, K)
    x_send = torch.empty(cap, H, dtype=torch.bfloat16, device=dev)
    slots = torch.empty(cap, K, dtype=torch.int32, device=dev)
    wts = torch.empty(cap, K, dtype=torch.float32, device=dev)
    counts = torch.empty(P, dtype=torch.int32, device=dev)
    slot_row = torch.empty(T, P, dtype=torch.int32, device=dev)
    ws = workspace(dev, size_call("nkimoe_ep_dispatch_workspace_bytes", T, P))
    call("nkimoe_ep_dispatch", _p(x), _p(idx), _p(w), T, H, K, P, experts_per_rank, _p(x_send), _p(slots), _p(wts),
         _p(counts), _p(slot_row), _p(ws), ws.numel(), _s(x))
    if sync_check_enabled():
        read_status(ws)
    return x_send, slots, wts, counts, slot_row
