"""Decode attention: q/k RMSNorm + RoPE of the step's token, KV-cache store and
split-KV attention in one kernel (``nkimoe_decode_attention``).

Checked against a plain PyTorch fp32 reference of the same step in the HF
Qwen3-MoE order (q_norm/k_norm per head, rotate-half RoPE, then
``softmax(q k^T * scale) v`` over positions ``0..p`` of the sequence's kv
head, ``nki_attention.py:252-373`` for the decode attention itself), with the
oracle's restatement of the norms and RoPE.  The new key is stored in bf16, so
the reference attends to the bf16-rounded key at ``p`` exactly as a cache
written by the prefill path would hold it.  Bars: normwise
``max|o - o_ref| / max|o_ref| <= 1e-2`` and cosine ``>= 0.9999`` on the bf16
output; the stored key bit-identical to ``nkimoe_qk_norm_rope``'s, the stored
value bit-identical to the input, every other cache row untouched.
"""

import numpy as np
import pytest
import torch

import oracle
from nki_moe_b200 import ops
from nki_moe_b200._lib import NKIMoEError

pytestmark = pytest.mark.gpu

HD = 128
NORM_BAR = 1e-2
COS_BAR = 0.9999


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def make_case(B, nq, nkv, max_seq, seed, w_dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(B, (nq + 2 * nkv) * HD, generator=g).bfloat16()
    qw = (1 + 0.1 * torch.randn(HD, generator=g)).to(w_dtype)
    kw = (1 + 0.1 * torch.randn(HD, generator=g)).to(w_dtype)
    kc = torch.randn(B, nkv, max_seq, HD, generator=g).bfloat16()
    vc = torch.randn(B, nkv, max_seq, HD, generator=g).bfloat16()
    return qkv, qw, kw, kc, vc


def reference(qkv, qw, kw, positions, kc, vc, nq, nkv, theta=1e6, eps=1e-6):
    """fp32 reference of one decode step; returns (out [B, nq*HD], k_new, v_new)."""
    B = qkv.shape[0]
    grp = nq // nkv
    pos = np.asarray(positions, dtype=np.int64)
    nr = oracle.qk_norm_rope(qkv.float().numpy(), qw.float().numpy(), kw.float().numpy(), pos, nq, nkv, HD,
                             theta, eps)
    nr = torch.from_numpy(nr)
    q = nr[:, : nq * HD].view(B, nq, HD)
    k_new = nr[:, nq * HD:(nq + nkv) * HD].view(B, nkv, HD).bfloat16()
    v_new = qkv[:, (nq + nkv) * HD:].view(B, nkv, HD)
    out = torch.empty(B, nq, HD)
    for b in range(B):
        p = int(pos[b])
        K = kc[b, :, : p + 1].float().clone()
        V = vc[b, :, : p + 1].float().clone()
        K[:, p] = k_new[b].float()
        V[:, p] = v_new[b].float()
        for h in range(nq):
            s = (K[h // grp] @ q[b, h]) * HD ** -0.5
            out[b, h] = torch.softmax(s.double(), 0).float() @ V[h // grp]
    return out.view(B, nq * HD), k_new, v_new


def run_and_check(B, nq, nkv, max_seq, positions, seed, broadcast=False, w_dtype=torch.bfloat16):
    qkv, qw, kw, kc, vc = make_case(B, nq, nkv, max_seq, seed, w_dtype)
    ref, k_new, v_new = reference(qkv, qw, kw, positions, kc, vc, nq, nkv)
    kc_d, vc_d = kc.cuda(), vc.cuda()
    pos_d = torch.tensor([positions[0]] if broadcast else positions, dtype=torch.int64, device="cuda")
    out = ops.decode_attention(qkv.cuda(), qw.cuda(), kw.cuda(), pos_d, kc_d, vc_d, nq, nkv)
    ws_status = ops._attention_workspace(out.device, 0)
    assert ops.read_status(ws_status) == 0
    o = out.float().cpu()
    err = oracle.normwise_rel_err(o.numpy(), ref.numpy())
    cos = oracle.cosine(o.numpy(), ref.numpy())
    assert err <= NORM_BAR and cos >= COS_BAR, f"normwise {err:.3e}, cosine {cos:.6f}"
    # cache: the new rows, bit for bit; nothing else changed
    kc_h, vc_h = kc_d.cpu(), vc_d.cpu()
    kcn, vcn = kc.clone(), vc.clone()
    nr = ops.qk_norm_rope(qkv.cuda(), qw.cuda(), kw.cuda(), torch.tensor(positions, device="cuda"), nq, nkv).cpu()
    k_lib = nr[:, nq * HD:(nq + nkv) * HD].view(B, nkv, HD)
    for b in range(B):
        kcn[b, :, positions[b]] = k_lib[b]
        vcn[b, :, positions[b]] = v_new[b]
    assert torch.equal(kc_h.view(torch.int16), kcn.view(torch.int16))
    assert torch.equal(vc_h.view(torch.int16), vcn.view(torch.int16))
    # the library's stored key is the oracle's within bf16 rounding
    assert (k_lib.float() - k_new.float()).abs().max() <= 2 ** -7 * k_new.float().abs().max()
    return out


def test_decode_attention_stack_shape():
    """Qwen3-30B-A3B attention (32 q / 4 kv heads), batch 8, one position for all."""
    run_and_check(8, 32, 4, 640, [512] * 8, seed=1, broadcast=True)


def test_decode_attention_ragged_positions():
    """Per-sequence positions across split boundaries: first position, the
    last of a chunk, the first of the next, mid-chunk, the cache's last."""
    run_and_check(5, 32, 4, 640, [0, 63, 64, 300, 639], seed=2)


def test_decode_attention_long_cache_and_wide_groups():
    """16 query heads per kv head (two heads per warp) and a cache long enough
    that each CTA stages several 64-position blocks."""
    run_and_check(2, 16, 1, 3000, [2999, 1500], seed=3)
    run_and_check(3, 8, 8, 200, [5, 199, 130], seed=4)


def test_decode_attention_single_sequence_fp32_norm_weights():
    """One sequence, fp32 q/k norm weights, a few positions into a long cache."""
    run_and_check(1, 32, 4, 4096, [3], seed=9, w_dtype=torch.float32)
    run_and_check(1, 32, 4, 4096, [4095], seed=10, w_dtype=torch.float32)


def test_decode_attention_consecutive_steps():
    """Two steps in a row on the same cache (the split counters reset), the
    second attending to the key the first stored."""
    B, nq, nkv, S = 4, 32, 4, 256
    qkv1, qw, kw, kc, vc = make_case(B, nq, nkv, S, seed=5)
    qkv2 = make_case(B, nq, nkv, S, seed=6)[0]
    kc_d, vc_d = kc.cuda(), vc.cuda()
    for step, qkv in ((200, qkv1), (201, qkv2)):
        pos = [step] * B
        ref, k_new, v_new = reference(qkv, qw, kw, pos, kc, vc, nq, nkv)
        out = ops.decode_attention(qkv.cuda(), qw.cuda(), kw.cuda(), torch.tensor(pos, device="cuda"), kc_d, vc_d,
                                   nq, nkv)
        o = out.float().cpu().numpy()
        assert oracle.normwise_rel_err(o, ref.numpy()) <= NORM_BAR
        assert oracle.cosine(o, ref.numpy()) >= COS_BAR
        kc[:, :, step] = k_new
        vc[:, :, step] = v_new


def test_decode_attention_in_graph():
    """Captured in a CUDA graph with the position in a device tensor (the
    decoder stack's decode step): replays at two positions."""
    B, nq, nkv, S = 8, 32, 4, 640
    qkv, qw, kw, kc, vc = make_case(B, nq, nkv, S, seed=7)
    qkv_d, qw_d, kw_d, kc_d, vc_d = qkv.cuda(), qw.cuda(), kw.cuda(), kc.cuda(), vc.cuda()
    pos_d = torch.zeros(1, dtype=torch.int64, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        out = ops.decode_attention(qkv_d, qw_d, kw_d, pos_d, kc_d.clone(), vc_d.clone(), nq, nkv)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            out = ops.decode_attention(qkv_d, qw_d, kw_d, pos_d, kc_d, vc_d, nq, nkv)
    torch.cuda.current_stream().wait_stream(s)
    for p in (100, 517):
        pos_d.fill_(p)
        graph.replay()
        torch.cuda.synchronize()
        ref, k_new, v_new = reference(qkv, qw, kw, [p] * B, kc, vc, nq, nkv)
        o = out.float().cpu().numpy()
        assert oracle.normwise_rel_err(o, ref.numpy()) <= NORM_BAR
        assert oracle.cosine(o, ref.numpy()) >= COS_BAR
        kc[:, :, p] = k_new
        vc[:, :, p] = v_new


def test_decode_attention_position_out_of_range_is_reported(monkeypatch):
    monkeypatch.setenv("NKIMOE_SYNC_CHECK", "0")  # read the status here, not inside the call
    B, nq, nkv, S = 2, 32, 4, 128
    qkv, qw, kw, kc, vc = make_case(B, nq, nkv, S, seed=8)
    kc_d, vc_d = kc.cuda(), vc.cuda()
    out = torch.zeros(B, nq * HD, dtype=torch.bfloat16, device="cuda")
    ops.decode_attention(qkv.cuda(), qw.cuda(), kw.cuda(), torch.tensor([5, S], device="cuda"), kc_d, vc_d, nq, nkv,
                         out=out)
    with pytest.raises(NKIMoEError):
        ops.read_status(ops._attention_workspace(out.device, 0))
    # the valid sequence was served, the other left alone, the caches intact outside position 5 of sequence 0
    assert torch.count_nonzero(out[1]) == 0
    assert torch.count_nonzero(out[0]) > 0
    assert torch.equal(kc_d[1].cpu().view(torch.int16), kc[1].view(torch.int16))
