"""The MoE block entry point that allocates nothing (nkimoe_moe_block_noalloc).

It serves callers that cannot allocate GPU memory or pass a workspace: a
server that reserved all device memory up front, a runtime whose allocator
cannot be entered where the layer is issued, or an embedding that forbids
allocation while it records CUDA graphs.  Its scratch is a fixed array inside
the library.  The test calls it through the C ABI twice in a row, on two
different token batches (the second call must not be affected by what the
first left in the shared array), and compares each result with the workspace
entry point's, within the block-output tolerance of the other parity tests.

This file is collected last on purpose, and it sets up everything it needs so
that it also passes alone in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle
from nki_moe_b200 import _lib, ops
from nki_moe_b200.workloads import WORKLOADS, make_moe_inputs

pytestmark = pytest.mark.gpu

NORM_TOL = 2e-2
COS_TOL = 0.999


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _noalloc(x, router_w, rsplit, pe, top_k):
    T, H = x.shape
    out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
    idx = torch.empty(T, top_k, dtype=torch.int32, device=x.device)
    w = torch.empty(T, top_k, dtype=torch.float32, device=x.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.call("nkimoe_moe_block_noalloc", _p(x), _p(router_w), None, _p(rsplit), _p(pe.w13), _p(pe.w2), _p(out),
              _p(idx), _p(w), T, H, pe.inter, pe.num_experts, top_k, stream)
    return out, idx, w


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
        ref, ref_idx, ref_w = ops.moe_block(x, rw, pe, wl.top_k, return_routing=True)
        out, idx, w = _noalloc(x, rw, rsplit, pe, wl.top_k)
        torch.cuda.synchronize()
        y, y_ref = out.float().cpu().numpy(), ref.float().cpu().numpy()
        err, cos = oracle.normwise_rel_err(y, y_ref), oracle.cosine(y, y_ref)
        assert err <= NORM_TOL and cos >= COS_TOL, f"call with {T} tokens: normwise {err:.3e}, cosine {cos:.6f}"
        assert torch.equal(idx, ref_idx)
        np.testing.assert_allclose(w.cpu().numpy(), ref_w.cpu().numpy(), rtol=1e-6)


def test_noalloc_rejects_batches_beyond_its_scratch(setup):
    wl, rw, rsplit, pe = setup
    x = torch.zeros(4096, wl.hidden, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.NKIMoEError) as ei:
        _noalloc(x, rw, rsplit, pe, wl.top_k)
    assert ei.value.code == _lib.ERR_WORKSPACE
    assert "scratch" in str(ei.value)
