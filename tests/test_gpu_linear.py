"""Skinny linear (``nkimoe_skinny_linear``): the decode step's projections,
y = x w^T for at most 16 rows of x, against a plain PyTorch fp32 reference.
Bars (one bf16 rounding of the output): normwise
``max|y - y_ref| / max|y_ref| <= 8e-3``, cosine ``>= 0.99999``; repeated calls
bit-identical (fixed reduction order)."""

import pytest
import torch

import oracle
from nki_moe_b200 import ops
from nki_moe_b200._lib import NKIMoEError

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.mark.parametrize("M,N,K", [(8, 2048, 4096), (8, 5120, 2048), (1, 2048, 4096), (13, 5120, 2048),
                                   (16, 1024, 2048), (3, 48, 96), (8, 151936, 2048)])
def test_skinny_linear_matches_fp32(M, N, K):
    g = torch.Generator().manual_seed(M * 131 + N + K)
    x = torch.randn(M, K, generator=g).bfloat16()
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16()
    y = ops.skinny_linear(x.cuda(), w.cuda())
    ref = (x.float() @ w.float().T).numpy()
    yh = y.float().cpu().numpy()
    err, cos = oracle.normwise_rel_err(yh, ref), oracle.cosine(yh, ref)
    assert err <= 8e-3 and cos >= 0.99999, f"normwise {err:.2e} cosine {cos:.7f}"
    assert torch.equal(ops.skinny_linear(x.cuda(), w.cuda()), y)


def test_skinny_linear_rejects_unsupported_shapes():
    x = torch.zeros(17, 64, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(32, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(NKIMoEError):
        ops.skinny_linear(x, w)  # 17 rows
    with pytest.raises(NKIMoEError):
        ops.skinny_linear(x[:4], torch.zeros(24, 64, dtype=torch.bfloat16, device="cuda"))  # N % 16
    assert ops.skinny_linear(x[:0], w).shape == (0, 32)
