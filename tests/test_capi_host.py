"""CPU checks of the C ABI: the library loads, exports every symbol that
include/nkimoe.h declares, and rejects bad arguments before touching a GPU."""

import ctypes
import os
import re

import pytest

from nki_moe_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(REPO, "include", "nkimoe.h")).read()
    return sorted(set(re.findall(r"NKIMOE_API\s+[\w\s\*]+?\b(nkimoe_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "nkimoe_moe_block" in names and "nkimoe_rmsnorm" in names
    assert len(names) >= 19


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in nkimoe.h but not exported"
    # the Python binding covers exactly the declared ABI
    assert set(_lib.SIGNATURES) == set(declared_symbols())


def test_version_and_options():
    lib = _lib.load()
    assert lib.nkimoe_version() >= 1
    _lib.set_option("gemm_schedule", 2)
    _lib.set_option("gemm_schedule", 0)
    with pytest.raises(_lib.NKIMoEError) as ei:
        _lib.set_option("no_such_option", 1)
    assert ei.value.code == _lib.ERR_INVALID_ARG
    _lib.set_option("pdl", 0)
    _lib.set_option("pdl", 1)
    with pytest.raises(_lib.NKIMoEError):
        _lib.set_option("pdl", 2)
    _lib.set_option("router_permutes", 0)
    _lib.set_option("router_permutes", 1)
    _lib.set_option("router_halves", 0)
    _lib.set_option("router_halves", 1)
    _lib.set_option("weights_balance", 0)
    _lib.set_option("weights_balance", 1)
    with pytest.raises(_lib.NKIMoEError):
        _lib.set_option("weights_balance", 2)


def test_workspace_sizes_are_host_functions():
    small = _lib.size_call("nkimoe_moe_workspace_bytes", 64, 2048, 768, 128, 8)
    big = _lib.size_call("nkimoe_moe_workspace_bytes", 8192, 2048, 768, 128, 8)
    # dominated by the gathered rows (T*K*H bf16) and the SwiGLU output (T*K*I bf16)
    assert big > 8192 * 8 * (2048 + 768) * 2
    assert small < big
    assert _lib.size_call("nkimoe_permute_workspace_bytes", 8192, 8, 128) > 0


def test_argument_validation_without_gpu():
    null = ctypes.c_void_p(0)
    with pytest.raises(_lib.NKIMoEError) as ei:  # 600 experts > 512
        _lib.call("nkimoe_moe_experts", null, null, null, null, _lib.I32, null, null, 4, 2048, 768, 600, 8,
                  null, 0, null)
    assert ei.value.code == _lib.ERR_UNSUPPORTED
    with pytest.raises(_lib.NKIMoEError) as ei:  # hidden not a multiple of 8
        _lib.call("nkimoe_rmsnorm", null, _lib.BF16, null, _lib.F32, null, _lib.BF16, 4, 100, 1e-6, null)
    assert ei.value.code == _lib.ERR_UNSUPPORTED
    with pytest.raises(_lib.NKIMoEError) as ei:  # workspace too small
        _lib.call("nkimoe_moe_block", null, null, null, null, null, null, null, null, null, 64, 2048, 768, 128, 8,
                  null, 16, null)
    assert ei.value.code == _lib.ERR_WORKSPACE
    with pytest.raises(_lib.NKIMoEError) as ei:
        _lib.call("nkimoe_qk_norm_rope", null, null, null, null, _lib.F32, null, 4, 32, 4, 64, 1e6, 1e-6, null)
    assert ei.value.code == _lib.ERR_UNSUPPORTED
    # zero tokens is a valid no-op that touches nothing
    _lib.call("nkimoe_rmsnorm", null, _lib.BF16, null, _lib.F32, null, _lib.BF16, 0, 2048, 1e-6, null)


def test_host_block_validation_without_gpu():
    """The host-buffer block checks its shapes, workspace and host pointers
    before the first CUDA call."""
    null = ctypes.c_void_p(0)
    need = _lib.size_call("nkimoe_moe_block_host_workspace_bytes", 8192, 2048, 768, 128, 8)
    # the block workspace of any chunk plus two slots of staged input and output rows
    assert need >= _lib.size_call("nkimoe_moe_workspace_bytes", 8192, 2048, 768, 128, 8) + 4 * 8192 * 2048 * 2

    def host(T, E, ws, ws_bytes, x=null):
        _lib.call("nkimoe_moe_block_host", x, null, null, null, null, null, null, null, null, T, 2048, 768, E, 8, 0,
                  ws, ws_bytes, null, null)

    for args, code in (((64, 600, null, 0), _lib.ERR_UNSUPPORTED),             # 600 experts
                       ((8192, 128, null, need), _lib.ERR_WORKSPACE),          # no workspace
                       ((8192, 128, ctypes.c_void_p(256), need - 1), _lib.ERR_WORKSPACE),
                       ((8192, 128, ctypes.c_void_p(256), need), _lib.ERR_INVALID_ARG)):  # null host rows
        with pytest.raises(_lib.NKIMoEError) as ei:
            host(*args)
        assert ei.value.code == code


def test_decode_attention_validation_without_gpu():
    null = ctypes.c_void_p(0)

    def attn(B, nq, nkv, hd, S, ws_bytes, ws=null):
        _lib.call("nkimoe_decode_attention", null, null, null, _lib.BF16, null, 0, null, null, null, B, nq, nkv, hd, S,
                  1e6, 1e-6, 0.088, ws, ws_bytes, null)

    for args, code in (((8, 32, 4, 64, 640, 1 << 20), _lib.ERR_UNSUPPORTED),    # head_dim 64
                       ((8, 30, 4, 128, 640, 1 << 20), _lib.ERR_INVALID_ARG),   # 30 heads over 4 kv heads
                       ((8, 64, 2, 128, 640, 1 << 20), _lib.ERR_UNSUPPORTED),   # 32 q heads per kv head
                       ((8, 32, 4, 128, 640, 1 << 20), _lib.ERR_INVALID_ARG)):  # null pointers
        with pytest.raises(_lib.NKIMoEError) as ei:
            attn(*args)
        assert ei.value.code == code
    need = _lib.size_call("nkimoe_decode_attention_workspace_bytes", 8, 32, 4, 128, 640)
    # status + counters + partials: 8 sequences x 4 kv heads x 10 splits x 8 heads x (128 + 4) floats
    assert need >= 8 * 4 * 10 * 8 * 132 * 4
    assert _lib.size_call("nkimoe_decode_attention_workspace_bytes", 8, 32, 4, 64, 640) == 0
    attn(0, 32, 4, 128, 640, 0)  # an empty batch is a no-op


def test_reference_module_aliases():
    import sys
    import nki_moe_b200
    nki_moe_b200.install_reference_aliases()
    for name in nki_moe_b200.REFERENCE_MODULES:
        assert sys.modules[name].__name__ == f"nki_moe_b200.{name}"
    from nki_moe_integrated import NKIMoESimple, NKIMoEWrapper, enable_nki_moe, replace_with_nki_moe  # noqa
    from nki_custom_rmsnorm import NKIRMSNorm, get_nki_rmsnorm_cls, nki_rmsnorm_kernel  # noqa
    assert get_nki_rmsnorm_cls() is NKIRMSNorm
    n = NKIRMSNorm(16)
    with pytest.raises(ValueError):
        n(__import__("torch").ones(16))  # 1-D input: ValueError, as nki_custom_rmsnorm.py:115


def test_no_cpu_path_for_host_weights():
    """The block never computes on the CPU: a host batch is accepted only with
    the weights on a GPU (the block runs there); host weights raise."""
    import torch
    from nki_moe_b200 import ops
    from nki_moe_b200.nki_moe_integrated import NKIMoESimple
    moe = NKIMoESimple(128, 64, 4, 2)
    x = torch.randn(1, 3, 128)
    with pytest.raises(ValueError, match="CUDA"):
        moe(x)
    with pytest.raises(ValueError, match="CUDA"):
        ops.moe_block_host(x[0].bfloat16(), moe.router.weight, None, 2)
    with pytest.raises(ValueError, match="CUDA"):
        ops.moe_block(x[0].bfloat16(), moe.router.weight, None, 2)


def _plan(T, E=128, K=8, split=True, chunk=0):
    n, c = ctypes.c_int64(0), ctypes.c_int64(0)
    _lib.call("nkimoe_moe_block_host_plan", T, E, K, int(split), chunk, ctypes.byref(n), ctypes.byref(c))
    lens = [n.value] * (c.value - 1)
    return lens + [T - sum(lens)]


def test_host_batch_chunk_plan():
    """Chunks of a host-batch call: cut only where every chunk takes the whole
    batch's path (the tensor-core router at 256 tokens or more with the
    router planes given; more than 48 rows per expert under the auto GEMM
    schedule), so the output is the whole-batch block's bit for bit."""
    assert _plan(8192) == [4096, 4096]                         # default: halves
    assert _plan(2048) == [1024, 1024]
    assert _plan(2048, chunk=1000) == [1000, 1048]             # a short tail joins the chunk before
    assert _plan(3000, chunk=769) == [769, 769, 1462]
    assert _plan(3000, chunk=500) == [769, 769, 1462]          # at least 48 * 128 / 8 + 1 = 769 tokens
    assert _plan(8192, chunk=100) == [769] * 9 + [1271]        # at most 16 chunks, tail >= 769
    assert _plan(8192, chunk=1 << 30) == [8192]
    assert _plan(1400) == [1400]                               # halves would be shorter than 769
    assert _plan(300) == [300]                                 # weight-streaming GEMMs: one chunk
    assert _plan(8192, split=False) == [8192]                  # CUDA-core router: its split-K follows T
    assert _plan(0) == [0]
    try:
        _lib.set_option("router", 1)                           # CUDA-core router forced
        assert _plan(8192) == [8192]
        _lib.set_option("router", 0)
        _lib.set_option("gemm_schedule", 2)                    # weight-streaming GEMMs forced
        assert _plan(8192) == [8192]
        _lib.set_option("gemm_schedule", 1)                    # tile-rows GEMMs forced: 256-token minimum
        assert _plan(2048, chunk=300) == [300] * 5 + [548]
    finally:
        _lib.set_option("router", 0)
        _lib.set_option("gemm_schedule", 0)
    with pytest.raises(_lib.NKIMoEError):
        _lib.call("nkimoe_moe_block_host_plan", 10, 0, 8, 1, 0, None, None)


def test_replace_with_nki_moe_raises_when_weights_are_missing():
    """The reference leaves randomly initialised experts in place when it cannot
    find a layer's weights (nki_moe_integrated.py:545-563); this package
    raises and replaces no layer."""
    import types

    import torch.nn as nn
    from nki_moe_b200.nki_moe_integrated import replace_with_nki_moe

    class NoWeights(nn.Module):
        pass

    layers = [types.SimpleNamespace(mlp=NoWeights()) for _ in range(2)]
    model = types.SimpleNamespace(model=types.SimpleNamespace(layers=layers))
    cfg = types.SimpleNamespace(hidden_size=128, moe_intermediate_size=64, num_experts=4, num_experts_per_tok=2)
    with pytest.raises(AttributeError, match="layer 0"):
        replace_with_nki_moe(model, cfg)
    assert all(isinstance(layer.mlp, NoWeights) for layer in layers)


def test_peer_wait_budget_option():
    """The expert-parallel waits' budget is settable; values outside
    [1000, 1e12] cycles are rejected."""
    _lib.set_option("peer_wait_cycles", 2_000_000)
    _lib.set_option("peer_wait_cycles", 20_000_000_000)
    for bad in (0, 999, 10 ** 13):
        with pytest.raises(_lib.NKIMoEError):
            _lib.set_option("peer_wait_cycles", bad)
