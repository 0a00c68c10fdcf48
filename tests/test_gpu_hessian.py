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


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,T,chunk", [(300, 5000, 1024), (256, 5000, 64), (520, 1100, 128)])
def test_xtx_chunked_running_sum(cuda_dev, dtype, n, T, chunk):
    """One launch over all tokens: chunks of `chunk` tokens accumulated on the tensor core and added, round to
    nearest, into the running sum kept in tensor memory (many chunks per tile, ragged token and row counts,
    beta != 0 reading the lower triangle); exactly symmetric and within FP32 accumulation of fp64."""
    import ctypes
    from mpq_b200._lib import call, ptr
    X = _batches(11 + n, [(T,)], n, dtype)[0].to(cuda_dev)
    g = torch.Generator().manual_seed(3)
    H0 = torch.randn(n, n, generator=g)
    H0 = (H0 + H0.T).to(cuda_dev)
    H = H0.clone()
    alpha, beta = 1.0 / T, 0.5
    st = torch.zeros(1, dtype=torch.int32, device=cuda_dev)  # the launch's own status word (0: no wait timed out)
    if dtype == torch.bfloat16:
        ld = (T + 7) // 8 * 8
        XT = torch.zeros(n, ld, device=cuda_dev, dtype=torch.bfloat16)
        XT[:, :T] = X.T
        call("mpq_syrk_bf16_acc", n, T, alpha, ptr(XT), ld, beta, ptr(H), H.stride(0), chunk, ptr(st))
    else:
        ld = (T + 3) // 4 * 4
        hi = torch.zeros(n, ld, device=cuda_dev)
        lo = torch.zeros(n, ld, device=cuda_dev)
        call("mpq_split_tf32_t", ptr(X), 0, X.stride(0), T, n, ptr(hi), ptr(lo), ld)
        arrA = (ctypes.c_void_p * 3)(hi.data_ptr(), hi.data_ptr(), lo.data_ptr())
        arrB = (ctypes.c_void_p * 3)(hi.data_ptr(), lo.data_ptr(), hi.data_ptr())
        call("mpq_syrk_tc_acc", 3, n, T, alpha, arrA, arrB, ld, beta, ptr(H), H.stride(0), chunk, ptr(st))
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    Xd = X.double().cpu()
    want = beta * H0.double().cpu() + alpha * (Xd.T @ Xd)
    scale = (Xd.abs().T @ Xd.abs() * alpha).max().item() + beta * H0.abs().max().item()
    assert torch.equal(H, H.T)
    assert (H.cpu().double() - want).abs().max().item() <= 1e-5 * scale


@pytest.mark.gpu
def test_xtx_chunked_rejects_bad_chunk(cuda_dev):
    from mpq_b200._lib import call, ptr
    n, T = 128, 256
    XT = torch.zeros(n, T, device=cuda_dev, dtype=torch.bfloat16)
    H = torch.zeros(n, n, device=cuda_dev)
    st = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    with pytest.raises(RuntimeError):
        call("mpq_syrk_bf16_acc", n, T, 1.0, ptr(XT), T, 0.0, ptr(H), n, 96, ptr(st))
