"""Calibration-Hessian accumulation (tensor-core symmetric product) against the float64 CPU restatement."""
import numpy as np
import pytest
import torch

from oracle import hessian as OH


def _batches(seed, shapes, n, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    scale = torch.exp(torch.randn(n, generator=g))
    return [(torch.randn(*s, n, generator=g) * scale + 0.3).to(dtype) for s in shapes]


def test_oracle_quip_hook_is_the_covariance():
    x = np.random.default_rng(0).standard_normal((50, 6))
    H, mu, ct = OH.quip_hook([x[:20], x[20:]], 6)
    assert ct == 50
    np.testing.assert_allclose(H, np.cov(x.T, bias=True), rtol=1e-12, atol=1e-12)
    R = OH.regularize_H(H + np.outer(mu, mu), 6, 0.01)
    np.testing.assert_allclose(np.diag(R).mean(), 1.01, rtol=1e-12)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [300, 512])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_quip_hook_matches_oracle(cuda_dev, n, dtype):
    from mpq_b200.hessian import HessianAccumulator
    batches = _batches(1 + n, [(3, 97), (2, 64), (130,)], n, dtype)
    acc = HessianAccumulator(n, device=cuda_dev, mode="quip")
    for b in batches:
        acc.add_batch(b.to(cuda_dev))
    H, mu, ct = acc.finalize()
    Hw, muw, ctw = OH.quip_hook([b.float().numpy() for b in batches], n)
    assert ct == ctw
    np.testing.assert_allclose(mu.cpu().numpy(), muw, rtol=1e-5, atol=1e-5)
    # second moments are accumulated in FP32 (3xTF32 operands for f32, exact TF32 operands for bf16)
    second = Hw + np.outer(muw, muw)
    scale = np.abs(second).max()
    assert np.abs(H.cpu().double().numpy() - Hw).max() <= 2e-5 * scale


@pytest.mark.gpu
def test_gptq_add_batch_matches_oracle_and_is_symmetric(cuda_dev):
    from mpq_b200.hessian import HessianAccumulator
    n = 384
    batches = _batches(5, [(4, 33), (1, 50), (77,), (2, 129)], n)
    acc = HessianAccumulator(n, device=cuda_dev, mode="gptq")
    for b in batches:
        acc.add_batch(b.to(cuda_dev))
    H = acc.finalize()
    want = OH.gptq_add_batch([b.numpy() for b in batches], n)
    assert torch.equal(H, H.T)
    assert np.abs(H.cpu().double().numpy() - want).max() <= 2e-5 * np.abs(want).max()


@pytest.mark.gpu
def test_xtx_bf16_single_product_is_exact_products(cuda_dev):
    """bf16 activations are exact TF32 operands: X^T X in one TF32 product matches fp64 to FP32 accumulation."""
    from mpq_b200.hessian import accumulate_xtx
    n, T = 640, 4100
    X = _batches(9, [(T,)], n, torch.bfloat16)[0]
    H = torch.zeros(n, n, device=cuda_dev)
    accumulate_xtx(H, X.to(cuda_dev), alpha=1.0 / T, beta=0.0)
    want = X.double().T @ X.double() / T
    scale = (X.double().abs().T @ X.double().abs() / T).max().item()
    assert (H.cpu().double() - want).abs().max().item() <= 1e-5 * scale
    assert torch.equal(H, H.T)
