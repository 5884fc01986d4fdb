"""The MoE block entry point that allocates nothing (nkimoe_moe_block_noalloc).

It serves callers that cannot allocate GPU memory or pass a workspace: a
server that reserved all device memory up front, a runtime whose allocator
cannot be entered where the layer is issued, or an embedding that forbids
allocation while it records CUDA graphs.  Its scratch is a fixed array inside
the library.  The test calls it through the C ABI twice in a row, on two
different token batches (the second call must not be affected by what the
first left in the shared array), and compares each result with the workspace
entry point's.  Both run the same kernels on the same inputs, only the scratch
address differs, so the outputs and the routing must be identical bit for bit.

This file is collected last on purpose, and it sets up everything it needs so
that it also passes alone in a fresh process.
"""

import ctypes

import pytest
import torch

from nki_moe_b200 import _lib, ops
from nki_moe_b200.workloads import WORKLOADS, make_moe_inputs

pytestmark = pytest.mark.gpu

# largest batch whose scratch fits the library's array at hidden 2048,
# intermediate 768, 128 experts, top-8 (the limit the header states)
MAX_TOKENS = 175


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _noalloc(x, router_w, rsplit, pe, top_k, tokens=None):
    T, H = x.shape
    out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
    idx = torch.empty(T, top_k, dtype=torch.int32, device=x.device)
    w = torch.empty(T, top_k, dtype=torch.float32, device=x.device)
    _lib.call("nkimoe_moe_block_noalloc", _p(x), _p(router_w), None, _p(rsplit), _p(pe.w13), _p(pe.w2), _p(out),
              _p(idx), _p(w), T if tokens is None else tokens, H, pe.inter, pe.num_experts, top_k, _stream())
    return out, idx, w


def _noalloc_status():
    st = ctypes.c_int(-1)
    _lib.call("nkimoe_noalloc_read_status", _stream(), ctypes.byref(st))
    return st.value


@pytest.fixture(scope="module")
def setup():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    _lib.load()
    wl = WORKLOADS["c2"]
    inp = make_moe_inputs(wl, device="cuda")
    pe = ops.packed_experts(inp["gate_up"].to(torch.bfloat16), inp["down"].to(torch.bfloat16), "nxd")
    rw = inp["router"].contiguous()
    return wl, rw, ops.router_split(rw), pe


def test_noalloc_matches_workspace_entry_point_on_two_calls(setup):
    wl, rw, rsplit, pe = setup
    for seed, T in ((11, 64), (12, 100)):
        g = torch.Generator(device="cuda").manual_seed(seed)
        x = torch.randn(T, wl.hidden, generator=g, device="cuda").to(torch.bfloat16)
        ref, ref_idx, ref_w = ops.moe_block(x, rw, pe, wl.top_k, return_routing=True, router_w_split=rsplit)
        out, idx, w = _noalloc(x, rw, rsplit, pe, wl.top_k)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"call with {T} tokens: max diff {(out.float() - ref.float()).abs().max()}"
        assert torch.equal(idx, ref_idx)
        assert torch.equal(w, ref_w)
        assert _noalloc_status() == 0


def test_noalloc_accepts_its_stated_maximum_and_rejects_one_more(setup):
    wl, rw, rsplit, pe = setup
    fits = _lib.size_call("nkimoe_moe_workspace_bytes", MAX_TOKENS, wl.hidden, wl.intermediate, wl.experts, wl.top_k)
    over = _lib.size_call("nkimoe_moe_workspace_bytes", MAX_TOKENS + 1, wl.hidden, wl.intermediate, wl.experts,
                          wl.top_k)
    assert fits <= (8 << 20) < over
    g = torch.Generator(device="cuda").manual_seed(13)
    x = torch.randn(MAX_TOKENS, wl.hidden, generator=g, device="cuda").to(torch.bfloat16)
    out, idx, _ = _noalloc(x, rw, rsplit, pe, wl.top_k)
    ref, ref_idx, _ = ops.moe_block(x, rw, pe, wl.top_k, return_routing=True, router_w_split=rsplit)
    torch.cuda.synchronize()
    assert torch.equal(out, ref) and torch.equal(idx, ref_idx)
    x1 = torch.zeros(MAX_TOKENS + 1, wl.hidden, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.NKIMoEError) as ei:
        _noalloc(x1, rw, rsplit, pe, wl.top_k)
    assert ei.value.code == _lib.ERR_WORKSPACE
    assert "scratch" in str(ei.value)


def test_noalloc_rejects_bad_shapes_before_the_size_check(setup):
    wl, rw, rsplit, pe = setup
    x = torch.zeros(4, wl.hidden, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.NKIMoEError) as ei:
        _noalloc(x, rw, rsplit, pe, wl.top_k, tokens=-1)
    assert ei.value.code == _lib.ERR_INVALID_ARG
