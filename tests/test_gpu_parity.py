"""Parity of the sm_100a kernels (called through the C ABI) with the oracle.

Bars (stated per test):
* integer/index work (top-k indices, permutation, offsets): bit-exact;
* routing weights: within 8 ulp of the oracle on identical fp32 logits;
* router logits: fp32, rtol 1e-5; full-router indices identical outside near
  ties (p_k - p_{k+1} <= 1e-5);
* bf16 block outputs: normwise max|y - y_ref| / max|y_ref| <= 2e-2 and
  cosine >= 0.999 against the fp32 oracle on the same bf16-rounded inputs.
"""

import os

import numpy as np
import pytest
import torch

import oracle
from nki_moe_b200 import _lib, ops
from nki_moe_b200.workloads import WORKLOADS, make_moe_inputs
from tests.golden import recipes

pytestmark = pytest.mark.gpu

NORM_TOL = 2e-2
COS_TOL = 0.999


@pytest.fixture(scope="module", autouse=True)
def _cuda_env():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    old = os.environ.get("NKIMOE_SYNC_CHECK")
    os.environ["NKIMOE_SYNC_CHECK"] = "1"
    _lib.load()
    yield
    _lib.set_option("gemm_schedule", 0)
    _lib.set_option("weights_rows", 0)
    if old is None:
        os.environ.pop("NKIMOE_SYNC_CHECK", None)
    else:
        os.environ["NKIMOE_SYNC_CHECK"] = old


def bf(t):
    """bf16-round a CPU tensor and return (cuda bf16 tensor, numpy fp32 copy)."""
    b = t.to(torch.bfloat16)
    return b.cuda(), b.float().numpy()


def assert_block_close(y, y_ref, tol=NORM_TOL):
    err = oracle.normwise_rel_err(y, y_ref)
    cos = oracle.cosine(y, y_ref)
    assert err <= tol and cos >= COS_TOL, f"normwise {err:.3e}, cosine {cos:.6f}"


def ulp_diff(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return np.abs(a.view(np.int32).astype(np.int64) - b.view(np.int32).astype(np.int64))


# ---------------------------------------------------------------- K1 / K6
def test_rmsnorm_fp32_matches_reference(golden_dir):
    g = np.load(os.path.join(golden_dir, "rmsnorm.npz"))
    r = recipes.rmsnorm_case()
    y = ops.rmsnorm(r["x"].cuda(), r["w"].cuda(), r["eps"]).cpu().numpy()
    np.testing.assert_allclose(y, g["y_ref"], rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("rows,hidden", [(1, 2048), (77, 2048), (4096, 2048), (33, 128), (5, 4096), (3, 8)])
def test_rmsnorm_bf16(rows, hidden):
    g = torch.Generator().manual_seed(rows * 7 + hidden)
    x = torch.randn(rows, hidden, generator=g) * 2
    w = 1 + 0.1 * torch.randn(hidden, generator=g)
    xb, xn = bf(x)
    y = ops.rmsnorm(xb, w.cuda(), 1e-6).float().cpu().numpy()
    ref = oracle.rmsnorm(xn, w.numpy(), 1e-6)
    assert np.max(np.abs(y - ref) / (np.abs(ref) + 1e-3)) < 8e-3  # one bf16 rounding of the output


@pytest.mark.parametrize("rows,hidden,in_place", [(100, 2048, False), (8, 2048, True), (1000, 2048, True),
                                                  (3, 8192, False), (5, 10240, True)])
def test_add_rmsnorm(rows, hidden, in_place):
    """Row-per-CTA path (few rows), warp-per-row path (many rows or long
    rows), and the decoder's in-place residual update."""
    g = torch.Generator().manual_seed(3 + rows)
    x, res = torch.randn(rows, hidden, generator=g), torch.randn(rows, hidden, generator=g)
    w = 1 + 0.1 * torch.randn(hidden, generator=g)
    xb, xn = bf(x)
    rb, rn = bf(res)
    out, r_out = ops.add_rmsnorm(xb, rb, w.cuda(), 1e-6, residual_out=rb if in_place else None)
    s = oracle.bf16_round(xn + rn)
    np.testing.assert_array_equal(r_out.float().cpu().numpy(), s)
    ref = oracle.rmsnorm(s, w.numpy(), 1e-6)
    assert_block_close(out.float().cpu().numpy(), ref, tol=8e-3)


def test_qk_norm_rope_matches_hf(golden_dir):
    g = np.load(os.path.join(golden_dir, "qk_rope.npz"))
    q = recipes.qk_rope_case()
    qkv_b, qkv_n = bf(q["qkv"])
    out = ops.qk_norm_rope(qkv_b, q["q_w"].cuda(), q["k_w"].cuda(), q["positions"].cuda(), q["n_heads"],
                           q["n_kv_heads"], q["head_dim"], q["theta"], q["eps"]).float().cpu().numpy()
    ref = oracle.qk_norm_rope(qkv_n, q["q_w"].numpy(), q["k_w"].numpy(), q["positions"].numpy(), q["n_heads"],
                              q["n_kv_heads"], q["head_dim"], q["theta"], q["eps"])
    assert_block_close(out, ref, tol=1e-2)
    assert_block_close(out, g["out"], tol=2e-2)  # HF on the unrounded fp32 input
    # in place
    inplace = qkv_b.clone()
    ops.qk_norm_rope(inplace, q["q_w"].cuda(), q["k_w"].cuda(), q["positions"].cuda(), q["n_heads"],
                     q["n_kv_heads"], q["head_dim"], q["theta"], q["eps"], out=inplace)
    np.testing.assert_array_equal(inplace.float().cpu().numpy(), out)


def test_qk_norm_rope_long_positions():
    g = torch.Generator().manual_seed(11)
    T, nh, nkv = 300, 32, 4
    qkv = torch.randn(T, (nh + 2 * nkv) * 128, generator=g)
    pos = torch.randint(0, 4096, (T,), generator=g)
    qw, kw = 1 + 0.1 * torch.randn(128, generator=g), 1 + 0.1 * torch.randn(128, generator=g)
    qb, qn = bf(qkv)
    out = ops.qk_norm_rope(qb, qw.cuda(), kw.cuda(), pos.cuda(), nh, nkv).float().cpu().numpy()
    ref = oracle.qk_norm_rope(qn, qw.numpy(), kw.numpy(), pos.numpy(), nh, nkv, 128, 1e6, 1e-6)
    assert_block_close(out, ref, tol=1e-2)
    # V passes through unchanged
    np.testing.assert_array_equal(out[:, (nh + nkv) * 128:], qn[:, (nh + nkv) * 128:])


# ---------------------------------------------------------------- K2
def test_topk_bit_exact_on_reference_logits(golden_dir):
    """Routing protocol (1)."""
    g = np.load(os.path.join(golden_dir, "moe_c1.npz"))
    idx, w = ops.topk_softmax(torch.from_numpy(g["logits"]).cuda(), 8)
    idx, w = idx.cpu().numpy(), w.cpu().numpy()
    assert np.array_equal(idx, g["idx"])
    _, w_or = oracle.topk_softmax(g["logits"], 8)
    assert ulp_diff(w, w_or).max() <= 8
    assert ulp_diff(w, g["w"]).max() <= 8


@pytest.mark.parametrize("T,E,K", [(1, 128, 8), (513, 128, 8), (64, 4, 2), (40, 64, 6), (10, 256, 8), (7, 32, 32)])
def test_topk_shapes(T, E, K):
    g = torch.Generator().manual_seed(T + E + K)
    lg = torch.randn(T, E, generator=g)
    lg[0, : min(E, 4)] = 0.5  # exact ties: lower id first
    idx, w = ops.topk_softmax(lg.cuda(), K)
    ri, rw = oracle.topk_softmax(lg.numpy(), K)
    assert np.array_equal(idx.cpu().numpy(), ri)
    assert ulp_diff(w.cpu().numpy(), rw).max() <= 8


@pytest.fixture(scope="module")
def c1_inputs():
    inp = make_moe_inputs(WORKLOADS["c1"])
    return inp


def test_router_logits_and_routing(c1_inputs, golden_dir):
    """Routing protocol (2): fp32 logits; identical idx outside near ties."""
    xb, xn = bf(c1_inputs["x"])
    rw = c1_inputs["router"]
    lg = ops.router_logits(xb, rw.cuda()).cpu().numpy()
    ref = oracle.router_logits(xn, rw.numpy())
    np.testing.assert_allclose(lg, ref, rtol=1e-5, atol=2e-5)
    idx, _ = ops.topk_softmax(torch.from_numpy(lg).cuda(), 8)
    ri, _ = oracle.topk_softmax(ref, 8)
    ties = oracle.near_tie_tokens(ref, 8)
    same = np.all(idx.cpu().numpy() == ri, axis=1)
    assert np.all(same | ties), f"{(~same & ~ties).sum()} non-tie tokens routed differently"


@pytest.mark.parametrize("router", [1, 2])
@pytest.mark.parametrize("T", [128, 1000])
def test_block_router_paths(c1_inputs, router, T):
    """Both router paths (CUDA-core split-K, tensor-core split-fp32) give fp32
    logits: identical routing to the oracle outside near ties."""
    _lib.set_option("router", router)
    try:
        x = torch.randn(T, 2048, generator=torch.Generator().manual_seed(T))
        xb, xn = bf(x)
        rw = c1_inputs["router"]
        pe = ops.packed_experts(*[bf(c1_inputs[k])[0] for k in ("gate_up", "down")], "nxd")
        _, idx, w = ops.moe_block(xb, rw.cuda(), pe, 8, return_routing=True)
        lg = oracle.router_logits(xn, rw.numpy())
        ri, rwt = oracle.topk_softmax(lg, 8)
        ties = oracle.near_tie_tokens(lg, 8)
        same = np.all(idx.cpu().numpy() == ri, axis=1)
        assert np.all(same | ties), f"{(~same & ~ties).sum()} non-tie tokens routed differently"
        ok = same & ~ties
        np.testing.assert_allclose(w.cpu().numpy()[ok], rwt[ok], rtol=2e-5, atol=1e-6)
    finally:
        _lib.set_option("router", 0)


@pytest.mark.parametrize("T,E,K,H", [(1, 128, 8, 2048), (7, 128, 8, 2048), (9, 128, 8, 2048), (64, 128, 8, 2048),
                                     (383, 128, 8, 2048), (384, 128, 8, 2048), (385, 128, 8, 2048),
                                     (40, 256, 8, 2048), (13, 64, 6, 128), (5, 32, 32, 256)])
def test_decode_router_token_groups(T, E, K, H):
    """The one-launch decode router (hidden slices, per-8-token-group last-CTA
    top-k) across token-group counts up to its limit of 48 groups (384
    tokens; 385 takes the split-K + top-k path), expert counts 32..256 and a
    router bias: identical routing to the oracle outside near ties, weights
    to fp32 rounding."""
    g = torch.Generator().manual_seed(T * 7 + E + K)
    x = torch.randn(T, H, generator=g)
    rw = torch.randn(E, H, generator=g) * 0.02
    bias = torch.randn(E, generator=g) * 0.1
    xb, xn = bf(x)
    idx, w = ops.route(xb, rw.cuda(), K, bias=bias.cuda(), tensor_router=False)
    lg = oracle.router_logits(xn, rw.numpy()) + bias.numpy()
    ri, rwt = oracle.topk_softmax(lg, K)
    ties = oracle.near_tie_tokens(lg, K)
    same = np.all(idx.cpu().numpy() == ri, axis=1)
    assert np.all(same | ties), f"{(~same & ~ties).sum()} non-tie tokens routed differently"
    ok = same & ~ties
    np.testing.assert_allclose(w.cpu().numpy()[ok], rwt[ok], rtol=2e-5, atol=1e-6)
    # the counters the router leaves behind are zero: a second call routes the same
    idx2, w2 = ops.route(xb, rw.cuda(), K, bias=bias.cuda(), tensor_router=False)
    assert torch.equal(idx2, idx) and torch.equal(w2, w)


# ---------------------------------------------------------------- K3
def _check_permute(idx_np, E, dtype=torch.int32):
    rt, rs, sr, off = ops.permute(torch.from_numpy(idx_np).to(dtype).cuda(), E)
    ert, ers, eoff, esr = oracle.permute(idx_np, E)
    assert np.array_equal(off.cpu().numpy(), eoff)
    assert np.array_equal(rs.cpu().numpy(), ers)
    assert np.array_equal(rt.cpu().numpy(), ert)
    assert np.array_equal(sr.cpu().numpy(), esr)


def test_permute_matches_reference_order(golden_dir):
    """Routing protocol (3): bit-identical grouping, (k, t) inside an expert."""
    g = np.load(os.path.join(golden_dir, "moe_c1.npz"))
    _check_permute(g["idx"], 128)
    _check_permute(g["idx"], 128, torch.int64)


@pytest.mark.parametrize("T,K,E", [(1, 8, 128), (8192, 8, 128), (1000, 2, 4), (333, 8, 512), (16384, 8, 128)])
def test_permute_shapes(T, K, E):
    rng = np.random.default_rng(T * K + E)
    idx = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    _check_permute(idx, E)


def test_permute_skewed_and_empty_experts():
    rng = np.random.default_rng(5)
    T, K, E = 4096, 8, 128
    idx = np.empty((T, K), np.int32)
    for t in range(T):
        idx[t] = rng.choice(np.arange(16), size=K, replace=False)  # only 16 experts used
    _check_permute(idx, E)


def test_bad_expert_id_is_reported():
    idx = torch.tensor([[0, 1], [2, 9]], dtype=torch.int32).cuda()
    with pytest.raises(_lib.NKIMoEError) as ei:
        ops.permute(idx, 4)
    assert ei.value.code == _lib.ERR_DEVICE


# ---------------------------------------------------------------- K4/K5
@pytest.mark.parametrize("counts", [(5, 0, 130, 64, 1), (300, 17, 0, 256, 513, 16)])
@pytest.mark.parametrize("schedule,rows", [(1, 0), (2, 16), (2, 32), (2, 64), (3, 0), (4, 0), (5, 0)])
def test_grouped_gemm(schedule, rows, counts):
    """Ragged segments: empty, one-row, exact multiples of the tile and
    partial last tiles (300 = 256 + 44 rows) for every schedule."""
    _lib.set_option("gemm_schedule", schedule)
    _lib.set_option("weights_rows", rows)
    try:
        g = torch.Generator().manual_seed(17)
        counts = list(counts)
        E, N, Kd = len(counts), 256, 192
        M = sum(counts)
        a = torch.randn(M, Kd, generator=g)
        w = torch.randn(E, N, Kd, generator=g) * 0.05
        ab, an = bf(a)
        wb, wn = bf(w)
        off = torch.tensor(np.concatenate([[0], np.cumsum(counts)]), dtype=torch.int32).cuda()
        out = ops.grouped_gemm(ab, wb, off).float().cpu().numpy()
        ref = np.zeros((M, N), np.float32)
        o = 0
        for e, c in enumerate(counts):
            ref[o:o + c] = an[o:o + c] @ wn[e].T
            o += c
        np.testing.assert_allclose(out, ref, rtol=1e-2, atol=2e-2)
    finally:
        _lib.set_option("gemm_schedule", 0)
        _lib.set_option("weights_rows", 0)


@pytest.mark.parametrize("schedule,rows", [(0, 0), (1, 0), (2, 16), (2, 32), (2, 64), (3, 0), (4, 0), (5, 0)])
def test_moe_experts_tiny(golden_dir, schedule, rows):
    """The reference test's module case (H=256, I=512, E=4, top-2) given routing."""
    _lib.set_option("gemm_schedule", schedule)
    _lib.set_option("weights_rows", rows)
    try:
        g = np.load(os.path.join(golden_dir, "moe_tiny.npz"))
        t = recipes.tiny_moe()
        xb, xn = bf(t["x"])
        gub, gun = bf(t["gate_up"])
        db, dn = bf(t["down"])
        pe = ops.packed_experts(gub, db, "nxd")
        idx = torch.from_numpy(g["idx"]).cuda()
        w = torch.from_numpy(g["w"]).cuda()
        out = ops.moe_experts(xb, pe, idx, w).float().cpu().numpy()
        ref = oracle.experts_forward(xn, gun, dn, g["idx"], g["w"])
        assert_block_close(out, ref)
        assert_block_close(out, g["out"])  # the reference's own fp32 output
    finally:
        _lib.set_option("gemm_schedule", 0)
        _lib.set_option("weights_rows", 0)


def _block_case(inp, T=None, bias=False):
    xb, xn = bf(inp["x"] if T is None else inp["x"][:T])
    gub, gun = bf(inp["gate_up"])
    db, dn = bf(inp["down"])
    rw = inp["router"]
    b = inp["router_bias"] if bias else None
    pe = ops.packed_experts(gub, db, "nxd")
    out, idx, w = ops.moe_block(xb, rw.cuda(), pe, 8, bias=b.cuda() if b is not None else None, return_routing=True)
    return out.float().cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), (xn, gun, dn, rw.numpy(),
                                                                              b.numpy() if b is not None else None)


def _oracle_block(xn, gun, dn, rwn, bias, idx_gpu, w_gpu):
    lg = oracle.router_logits(xn, rwn)
    if bias is not None:
        lg = lg + bias
    ri, rwt = oracle.topk_softmax(lg, 8)
    ties = oracle.near_tie_tokens(lg, 8)
    same = np.all(idx_gpu == ri, axis=1)
    assert np.all(same | ties)
    # compare the expert stage on the GPU's own routing (near-tie tokens may differ)
    return oracle.experts_forward(xn, gun, dn, idx_gpu, w_gpu)


@pytest.mark.parametrize("schedule", [0, 1, 2, 3, 4, 5])
def test_moe_block_c1(c1_inputs, golden_dir, schedule):
    _lib.set_option("gemm_schedule", schedule)
    try:
        out, idx, w, (xn, gun, dn, rwn, _) = _block_case(c1_inputs)
        ref = _oracle_block(xn, gun, dn, rwn, None, idx, w)
        assert_block_close(out, ref)
        # the reference's own fp32 run on the unrounded inputs, over the tokens
        # whose routing the bf16 rounding of x did not move (about 1 in 8 tokens
        # has a top-8 margin below the ~1e-3 logit change that rounding causes)
        g = np.load(os.path.join(golden_dir, "moe_c1.npz"))
        keep = np.all(idx == g["idx"], axis=1)
        assert keep.mean() > 0.75
        assert_block_close(out[keep], g["out"][keep])
    finally:
        _lib.set_option("gemm_schedule", 0)


def test_moe_block_c2_decode():
    inp = make_moe_inputs(WORKLOADS["c2"])
    out, idx, w, (xn, gun, dn, rwn, _) = _block_case(inp)
    ref = _oracle_block(xn, gun, dn, rwn, None, idx, w)
    assert_block_close(out, ref)
    assert len(np.unique(idx)) > 100  # natural routing touches ~all experts


@pytest.mark.parametrize("schedule", [0, 1, 4, 5])
def test_moe_block_c3_prefill_sampled_tokens(schedule):
    """Full prefill size (8192 tokens); each token's output depends only on
    that token, so 256 sampled tokens are checked against the oracle."""
    _lib.set_option("gemm_schedule", schedule)
    try:
        inp = make_moe_inputs(WORKLOADS["c3"])
        out, idx, w, (xn, gun, dn, rwn, _) = _block_case(inp)
    finally:
        _lib.set_option("gemm_schedule", 0)
    rng = np.random.default_rng(0)
    sel = np.sort(rng.choice(xn.shape[0], 256, replace=False))
    ref = oracle.experts_forward(xn[sel], gun, dn, idx[sel], w[sel])
    assert_block_close(out[sel], ref)
    lg = oracle.router_logits(xn[sel], rwn)
    ri, _ = oracle.topk_softmax(lg, 8)
    assert np.all(np.all(idx[sel] == ri, axis=1) | oracle.near_tie_tokens(lg, 8))
    # a checksum of the whole output: finite and the right scale
    assert np.isfinite(out).all()


@pytest.mark.parametrize("schedule", [0, 4, 5])
def test_moe_block_skewed_routing(schedule):
    wl = WORKLOADS["c4"]
    inp = make_moe_inputs(wl, tokens=2048)
    _lib.set_option("gemm_schedule", schedule)
    try:
        out, idx, w, (xn, gun, dn, rwn, bias) = _block_case(inp, bias=True)
    finally:
        _lib.set_option("gemm_schedule", 0)
    counts = np.bincount(idx.ravel(), minlength=128)
    assert counts.max() > 8 * counts.mean()  # heavily imbalanced
    ref = _oracle_block(xn, gun, dn, rwn, bias, idx, w)
    assert_block_close(out, ref)


def test_moe_block_odd_token_counts():
    inp = make_moe_inputs(WORKLOADS["c2"], tokens=3)
    out, idx, w, (xn, gun, dn, rwn, _) = _block_case(inp)
    ref = _oracle_block(xn, gun, dn, rwn, None, idx, w)
    assert_block_close(out, ref)


@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("schedule", [1, 2])
def test_moe_block_gather_fused(c1_inputs, schedule, mode):
    """GEMM-1 loading its gathered token rows itself (1: cp.async, 2: TMA
    gather4) instead of the separate gather kernel gives the same result."""
    _lib.set_option("gemm_schedule", schedule)
    try:
        _lib.set_option("gather_fused", 0)
        ref = _block_case(c1_inputs)[0]
        _lib.set_option("gather_fused", mode)
        out = _block_case(c1_inputs)[0]
        assert np.array_equal(out, ref)
    finally:
        _lib.set_option("gather_fused", 0)
        _lib.set_option("gemm_schedule", 0)


@pytest.mark.parametrize("schedule,rows", [(2, 16), (2, 32), (2, 64), (1, 0)])
def test_moe_block_gather4_skewed(schedule, rows):
    """TMA gather4 row loads on ragged, heavily skewed expert segments (rows
    past a segment's end inside a tile, one-row segments) equal the separate
    gather kernel bit for bit, for every decode tile width."""
    inp = make_moe_inputs(WORKLOADS["c4"], tokens=600)
    _lib.set_option("gemm_schedule", schedule)
    _lib.set_option("weights_rows", rows)
    try:
        _lib.set_option("gather_fused", 0)
        ref, idx, w, _ = _block_case(inp, bias=True)
        _lib.set_option("gather_fused", 2)
        out, idx2, _, _ = _block_case(inp, bias=True)
        assert np.array_equal(idx, idx2)
        assert np.array_equal(out, ref)
    finally:
        _lib.set_option("gather_fused", 0)
        _lib.set_option("weights_rows", 0)
        _lib.set_option("gemm_schedule", 0)


@pytest.mark.parametrize("staging", [0, 1, 2])
def test_epilogue_staging_is_bit_identical(staging):
    """Writing the GEMM outputs through the shared-memory staging tile changes
    only how the same bf16 values reach memory."""
    inp = make_moe_inputs(WORKLOADS["c3"], tokens=1500)
    try:
        _lib.set_option("epilogue_staging", 3)
        ref = _block_case(inp)[0]
        _lib.set_option("epilogue_staging", staging)
        out = _block_case(inp)[0]
        assert np.array_equal(out, ref)
    finally:
        _lib.set_option("epilogue_staging", 3)


@pytest.mark.parametrize("T,in_place,w_dtype", [(1, False, torch.bfloat16), (8, True, torch.bfloat16),
                                                (64, False, torch.float32), (512, True, torch.bfloat16),
                                                (513, True, torch.bfloat16), (1000, False, torch.float32)])
def test_moe_block_add_rmsnorm_equals_unfused(c1_inputs, T, in_place, w_dtype):
    """The block followed by the decoder's residual add + next RMSNorm
    (qwen_with_nki.py:447-454) in one call -- one fused combine + norm kernel
    up to 512 tokens, combine then add + norm above -- equals moe_block +
    add_rmsnorm bit for bit."""
    g = torch.Generator().manual_seed(T + 3)
    xb = torch.randn(T, 2048, generator=g).bfloat16().cuda()
    res = torch.randn(T, 2048, generator=g).bfloat16().cuda()
    nw = (1 + 0.1 * torch.randn(2048, generator=g)).to(w_dtype).cuda()
    rw = c1_inputs["router"].cuda()
    pe = ops.packed_experts(*[bf(c1_inputs[k])[0] for k in ("gate_up", "down")], "nxd")
    h = ops.moe_block(xb, rw, pe, 8)
    ref_xn, ref_res = ops.add_rmsnorm(h, res, nw, 1e-6)
    res_in = res.clone()
    xn, r = ops.moe_block_add_rmsnorm(xb, rw, pe, 8, res_in, nw, 1e-6, residual_out=res_in if in_place else None)
    assert torch.equal(r, ref_res)
    assert torch.equal(xn, ref_xn)


@pytest.mark.parametrize("T", [1, 5, 8, 9, 64, 255])
def test_router_permutation_equals_permute_kernel(c1_inputs, T):
    """Decode routers also write the expert permutation (no separate
    permutation launch): up to 8 tokens the split router's last CTA, from 9
    to 255 tokens the cluster router's last CTA.  The block's output equals,
    bit for bit, the experts stage run on the same routing with the
    permutation kernel."""
    g = torch.Generator().manual_seed(40 + T)
    xb = torch.randn(T, 2048, generator=g).bfloat16().cuda()
    rw = c1_inputs["router"].cuda()
    pe = ops.packed_experts(*[bf(c1_inputs[k])[0] for k in ("gate_up", "down")], "nxd")
    out, idx, w = ops.moe_block(xb, rw, pe, 8, return_routing=True)
    ref = ops.moe_experts(xb, pe, idx, w)
    assert torch.equal(out, ref)


def test_programmatic_dependent_launch_off_is_bit_identical(c1_inputs):
    """The decode-path kernels launched without programmatic dependent launch
    (option pdl=0) give the same bits as with it."""
    g = torch.Generator().manual_seed(77)
    rw = c1_inputs["router"].cuda()
    pe = ops.packed_experts(*[bf(c1_inputs[k])[0] for k in ("gate_up", "down")], "nxd")
    res = torch.randn(8, 2048, generator=g).bfloat16().cuda()
    nw = torch.ones(2048, dtype=torch.bfloat16, device="cuda")
    xs = [torch.randn(T, 2048, generator=g).bfloat16().cuda() for T in (8, 64)]
    outs = []
    for pdl in (1, 0):
        _lib.set_option("pdl", pdl)
        try:
            outs.append([ops.moe_block(x, rw, pe, 8) for x in xs] +
                        list(ops.moe_block_add_rmsnorm(xs[0], rw, pe, 8, res, nw)))
        finally:
            _lib.set_option("pdl", 1)
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_back_to_back_decode_blocks_read_their_own_offsets(c1_inputs):
    """Decode blocks launched back to back on one stream (no synchronisation
    between calls, the workspace and its expert offsets reused by every call,
    the routing different each time) equal the same blocks run one at a time
    without programmatic dependent launch, bit for bit.  The decode GEMMs read
    the offsets and start their weight loads before their dependency wait, so
    a GEMM that saw the previous call's offsets would show here."""
    g = torch.Generator().manual_seed(91)
    rw = c1_inputs["router"].cuda()
    pe = ops.packed_experts(*[bf(c1_inputs[k])[0] for k in ("gate_up", "down")], "nxd")
    xs = [torch.randn((8, 8, 64)[i % 3], 2048, generator=g).bfloat16().cuda() for i in range(24)]
    _lib.set_option("pdl", 0)
    try:
        ref = []
        for x in xs:
            ref.append(ops.moe_block(x, rw, pe, 8))
            torch.cuda.synchronize()
    finally:
        _lib.set_option("pdl", 1)
    outs = [ops.moe_block(x, rw, pe, 8) for x in xs]
    torch.cuda.synchronize()
    for a, b in zip(outs, ref):
        assert torch.equal(a, b)


@pytest.mark.parametrize("T,chunk,pinned", [(2048, 0, True), (2048, 1000, False), (3000, 769, True),
                                            (300, 0, True), (5, 0, True), (0, 0, True)])
def test_moe_block_host_equals_device_block(c1_inputs, T, chunk, pinned):
    """The block on host buffers (copies of token chunks overlapping the block
    on the chunk before) equals the device call on the whole batch bit for
    bit: output and routing, two calls in a row.  Chunks hold at least 769
    tokens here (more than 48 rows per expert at 128 experts, top-8): 2048
    tokens go as 1024 + 1024 (default: halves) or 1000 + 1048 (a short tail merged),
    3000 as 769 + 769 + 1462; 300 tokens (weight-streaming GEMMs) and 5
    tokens in one chunk; 0 tokens is a no-op."""
    g = torch.Generator().manual_seed(T + chunk)
    rw = c1_inputs["router"].cuda()
    pe = ops.packed_experts(*[bf(c1_inputs[k])[0] for k in ("gate_up", "down")], "nxd")
    for _ in range(2):
        xh = torch.randn(T, 2048, generator=g).bfloat16()
        if pinned:
            xh = xh.pin_memory()
        ref, ridx, rwt = ops.moe_block(xh.cuda(), rw, pe, 8, return_routing=True)
        out, idx, w = ops.moe_block_host(xh, rw, pe, 8, chunk_tokens=chunk, return_routing=True)
        assert not out.is_cuda and out.shape == (T, 2048)
        assert torch.equal(out.view(torch.int16), ref.cpu().view(torch.int16))
        assert torch.equal(idx, ridx) and torch.equal(w.view(torch.int32), rwt.view(torch.int32))


@pytest.mark.parametrize("chunk", [0, 1 << 30])
def test_moe_block_host_overlapped_calls(c1_inputs, chunk):
    """Successive host-buffer calls with completion events (each call's copy
    in overlapping the previous call's block, its copy back the next call's
    block; two output buffers in turn): every batch's output equals the device
    block's on that batch."""
    g = torch.Generator().manual_seed(90 + (chunk > 0))
    rw = c1_inputs["router"].cuda()
    pe = ops.packed_experts(*[bf(c1_inputs[k])[0] for k in ("gate_up", "down")], "nxd")
    xs = [torch.randn(2048, 2048, generator=g).bfloat16().pin_memory() for _ in range(4)]
    outs = [torch.empty(2048, 2048, dtype=torch.bfloat16).pin_memory() for _ in range(4)]
    dones = [torch.cuda.Event() for _ in range(4)]
    os.environ["NKIMOE_SYNC_CHECK"] = "0"  # no synchronisation inside the calls
    try:
        for x, o, d in zip(xs, outs, dones):
            ops.moe_block_host(x, rw, pe, 8, out=o, chunk_tokens=chunk, done=d)
    finally:
        os.environ["NKIMOE_SYNC_CHECK"] = "1"
    for x, o, d in zip(xs, outs, dones):
        d.synchronize()
        ref = ops.moe_block(x.cuda(), rw, pe, 8).cpu()
        assert torch.equal(o.view(torch.int16), ref.view(torch.int16))


def test_moe_block_host_overlapped_calls_of_changing_size(c1_inputs):
    """Successive host-buffer calls with completion events whose batch size
    changes from call to call (2048, 1000, 2048, 600, 2048 tokens) on one
    workspace: the staging rows' place follows the batch size, so a call
    after a change must not overwrite rows an earlier call's block or copy back
    still uses.  Every output equals the device block's bit for bit."""
    g = torch.Generator().manual_seed(97)
    rw = c1_inputs["router"].cuda()
    pe = ops.packed_experts(*[bf(c1_inputs[k])[0] for k in ("gate_up", "down")], "nxd")
    sizes = (2048, 1000, 2048, 600, 2048)
    xs = [torch.randn(T, 2048, generator=g).bfloat16().pin_memory() for T in sizes]
    outs = [torch.empty(T, 2048, dtype=torch.bfloat16).pin_memory() for T in sizes]
    dones = [torch.cuda.Event() for _ in sizes]
    os.environ["NKIMOE_SYNC_CHECK"] = "0"  # no synchronisation inside the calls
    try:
        for x, o, d in zip(xs, outs, dones):
            ops.moe_block_host(x, rw, pe, 8, out=o, done=d)
    finally:
        os.environ["NKIMOE_SYNC_CHECK"] = "1"
    for x, o, d in zip(xs, outs, dones):
        d.synchronize()
        ref = ops.moe_block(x.cuda(), rw, pe, 8).cpu()
        assert torch.equal(o.view(torch.int16), ref.view(torch.int16)), f"{x.shape[0]} tokens"


def test_workspace_captured_by_a_graph_survives_a_larger_call(c1_inputs):
    """A CUDA graph that captured the block keeps its workspace alive after a
    later, larger call on the same stream replaced it: replaying the graph
    still gives the eager result."""
    rw = c1_inputs["router"].cuda()
    pe = ops.packed_experts(*[bf(c1_inputs[k])[0] for k in ("gate_up", "down")], "nxd")
    g = torch.Generator().manual_seed(98)
    x = torch.randn(64, 2048, generator=g).bfloat16().cuda()
    big = torch.randn(4096, 2048, generator=g).bfloat16().cuda()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    os.environ["NKIMOE_SYNC_CHECK"] = "0"
    try:
        with torch.cuda.stream(s):
            ops.release_captured_workspaces()
            ops._ws.pop((x.device.index, s.cuda_stream), None)  # start this stream small
            ops.moe_block(x, rw, pe, 8)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                y = ops.moe_block(x, rw, pe, 8)
            ops.moe_block(big, rw, pe, 8)  # grows (replaces) this stream's workspace
            assert len(ops._ws_retired) >= 1
            torch.cuda.synchronize()
            y.zero_()
            graph.replay()
        torch.cuda.synchronize()
    finally:
        os.environ["NKIMOE_SYNC_CHECK"] = "1"
    ref = ops.moe_block(x, rw, pe, 8)
    assert torch.equal(y, ref)
    del graph
    ops.release_captured_workspaces()


def test_module_on_host_batch_equals_device_batch(c1_inputs):
    """NKIMoESimple called on a host tensor (as the reference's module test
    calls it) runs on the weights' GPU and returns the device call's result on
    the host."""
    from nki_moe_b200.nki_moe_integrated import NKIMoESimple
    moe = NKIMoESimple(2048, 768, 128, 8, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        moe.router.weight.copy_(c1_inputs["router"])
    xh = torch.randn(2, 1000, 2048, generator=torch.Generator().manual_seed(5)).bfloat16()  # 1000 + 1000
    with torch.no_grad():
        y_host = moe(xh)
        y_dev = moe(xh.cuda())
    assert not y_host.is_cuda
    assert torch.equal(y_host.view(torch.int16), y_dev.cpu().view(torch.int16))


def test_moe_block_deterministic(c1_inputs):
    a = _block_case(c1_inputs)[0]
    b = _block_case(c1_inputs)[0]
    assert np.array_equal(a, b)


# ---------------------------------------------------------------- pieces
def test_pieces(golden_dir):
    g = np.load(os.path.join(golden_dir, "pieces.npz"))
    from nki_moe_b200.nki_moe_integrated import nki_matmul_tiled, nki_moe_aggregate, nki_swiglu
    a, b = recipes.matmul_case()
    out = nki_matmul_tiled(a.cuda(), b.cuda()).float().cpu().numpy()
    # The reference test's bar is max|diff| < 0.1 between two bf16 results
    # (test_nki_moe.py:54-67).  Against the fp32 product the bf16 output can
    # differ by half a bf16 ulp (0.25 at |x| >= 64; these outputs reach ~90),
    # so the bar here is one bf16 ulp relative.
    ref = g["matmul"]
    assert np.all(np.abs(out - ref) <= 2.0 ** -8 * np.abs(ref) + 1e-3)
    assert_block_close(out, ref, tol=1e-2)
    s = nki_swiglu(recipes.swiglu_case().cuda()).float().cpu().numpy()
    assert np.max(np.abs(s - g["swiglu"])) < 1e-1  # test_nki_moe.py:108
    eo = torch.randn(8, 37, 256).to(torch.bfloat16)
    agg = nki_moe_aggregate(eo.cuda()).float().cpu().numpy()
    assert_block_close(agg, oracle.aggregate(eo.float().numpy()), tol=1e-2)


def test_grouped_expert_gemm_and_single_expert():
    from nki_moe_b200.nki_moe_expert import nki_grouped_expert_gemm
    from nki_moe_b200.nki_moe_kernel import nki_moe_single_expert_forward
    g = torch.Generator().manual_seed(23)
    M, H, N, E = 300, 256, 384, 5
    x = torch.randn(M, H, generator=g)
    w = torch.randn(E, H, N, generator=g) * 0.05
    ids = torch.randint(0, E, (M,), generator=g)
    xb, xn = bf(x)
    wb, wn = bf(w)
    out = nki_grouped_expert_gemm(xb, wb, ids.cuda(), E).float().cpu().numpy()
    ref = np.stack([xn[m] @ wn[ids[m]] for m in range(M)])
    assert_block_close(out, ref, tol=1e-2)
    # the weight re-layout is made once per weight tensor, then reused
    assert ops.kmajor_weights(wb, 64, 128) is ops.kmajor_weights(wb, 64, 128)
    out2 = nki_grouped_expert_gemm(xb, wb, ids.cuda(), E).float().cpu().numpy()
    assert np.array_equal(out, out2)
    # single expert: w[t] * FFN(x[t])
    I = 128
    gu = torch.randn(H, 2 * I, generator=g) * 0.05
    dw = torch.randn(I, H, generator=g) * 0.05
    tw = torch.rand(M, generator=g)
    gub, gun = bf(gu)
    dwb, dwn = bf(dw)
    y = nki_moe_single_expert_forward(xb, gub, dwb, tw.cuda()).float().cpu().numpy()
    ref = tw.numpy()[:, None] * oracle.expert_ffn(xn, gun, dwn)
    assert_block_close(y, ref)


def test_invalid_shapes_raise():
    x = torch.zeros(4, 100, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.NKIMoEError) as ei:
        ops.rmsnorm(x, torch.ones(100, device="cuda"))
    assert ei.value.code == _lib.ERR_UNSUPPORTED
    with pytest.raises(ValueError):
        ops.rmsnorm(torch.zeros(4, 128), torch.ones(128))  # CPU tensors: no CPU path


@pytest.mark.parametrize("T", [256, 300, 8192])
def test_fused_tensor_core_router_equals_two_kernels(T):
    """The one-kernel tensor-core router logits (the three weight planes
    summed in the epilogue) issue the same MMAs and sums as the router GEMM's
    partials added by the top-k kernel: routing indices and weights identical
    bit for bit, with and without a router bias, on full and ragged row tiles,
    with 64 experts per CTA (two CTAs per row block, the default) and 128."""
    g = torch.Generator().manual_seed(T)
    x = torch.randn(T, 2048, generator=g).bfloat16().cuda()
    rw = (torch.randn(128, 2048, generator=g) * 0.02).cuda()
    bias = (torch.randn(128, generator=g) * 0.1).cuda()
    for b in (None, bias):
        outs = []
        for fused, halves in ((1, 1), (1, 0), (0, 1)):
            _lib.set_option("router_fused", fused)
            _lib.set_option("router_halves", halves)
            try:
                outs.append(ops.route(x, rw, 8, bias=b))
            finally:
                _lib.set_option("router_fused", 1)
                _lib.set_option("router_halves", 1)
        i0, w0 = outs[-1]
        for i1, w1 in outs[:-1]:
            assert torch.equal(i1, i0)
            assert torch.equal(w1.view(torch.int32), w0.view(torch.int32))


@pytest.mark.parametrize("T", [300, 2048, 8192])
@pytest.mark.parametrize("wdt", [torch.float32, torch.bfloat16])
def test_moe_block_with_fused_rmsnorm_equals_separate_calls(c1_inputs, T, wdt):
    """The block with the post-attention RMSNorm inside the call equals
    rmsnorm + block bit for bit: the normalised rows, the routing and the
    output.  Above 512 tokens the norm and the router logits are one
    tensor-core kernel; at 300 tokens the norm kernel runs first."""
    g = torch.Generator().manual_seed(T + 7)
    h = (torch.randn(T, 2048, generator=g) * 3).bfloat16().cuda()
    nw = (torch.rand(2048, generator=g) + 0.5).to(wdt).cuda()
    rw = c1_inputs["router"].cuda()
    pe = ops.packed_experts(*[bf(c1_inputs[k])[0] for k in ("gate_up", "down")], "nxd")
    out, x, idx, w = ops.moe_block_rmsnorm(h, nw, rw, pe, 8, eps=1e-6, return_x=True, return_routing=True)
    x_ref = ops.rmsnorm(h, nw, 1e-6, out_dtype=torch.bfloat16)
    ref, ridx, rwt = ops.moe_block(x_ref, rw, pe, 8, return_routing=True)
    assert torch.equal(x, x_ref)
    assert torch.equal(idx, ridx) and torch.equal(w.view(torch.int32), rwt.view(torch.int32))
    assert torch.equal(out, ref)


def test_module_with_fused_post_attention_norm(c1_inputs):
    """NKIMoESimple.fuse_rmsnorm(norm): forward(h) = moe(norm(h)), as the
    reference's fused MoE module receives post_attention_layernorm."""
    from nki_moe_b200.nki_custom_rmsnorm import NKIRMSNorm
    from nki_moe_b200.nki_moe_integrated import NKIMoESimple
    moe = NKIMoESimple(2048, 768, 128, 8, device="cuda", dtype=torch.bfloat16)
    norm = NKIRMSNorm(2048).cuda()
    with torch.no_grad():
        moe.router.weight.copy_(c1_inputs["router"])
        norm.weight.copy_(torch.rand(2048, generator=torch.Generator().manual_seed(3)) + 0.5)
    h = torch.randn(2, 1024, 2048, generator=torch.Generator().manual_seed(8)).bfloat16().cuda()
    with torch.no_grad():
        ref = moe(norm(h).bfloat16())
        fused = moe.fuse_rmsnorm(norm)(h)
    assert torch.equal(fused, ref)


def test_pair_split_schedule_equals_one_sm_rows():
    """Schedule 5 (the SM pair over each expert's whole 256-row blocks, one SM
    past them) computes every output row with the same per-row arithmetic as
    the one-SM rows schedule: the prefill block's outputs are identical."""
    wl = WORKLOADS["c3"]
    inp = make_moe_inputs(wl, device="cuda", tokens=4096)
    x = inp["x"].to(torch.bfloat16)
    pe = ops.packed_experts(inp["gate_up"].to(torch.bfloat16), inp["down"].to(torch.bfloat16), "nxd")
    outs = []
    for sched in (1, 5):
        _lib.set_option("gemm_schedule", sched)
        try:
            outs.append(ops.moe_block(x, inp["router"], pe, wl.top_k))
        finally:
            _lib.set_option("gemm_schedule", 0)
    assert torch.equal(outs[0], outs[1]), f"max diff {(outs[0].float() - outs[1].float()).abs().max().item()}"
