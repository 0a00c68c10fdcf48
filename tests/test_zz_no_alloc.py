"""The allocation-free 3xTF32 product (mpq_gemm_tf32x3_noalloc) against the allocating entry point.

mpq_gemm_tf32x3_noalloc keeps the TF32 operand split in a file-scope device array instead of caller buffers;
these tests call it through the C-ABI and compare it with mpq_split_tf32 + mpq_gemm_tc (ops.mm_nt) on two
calls in a row, so the second call runs on the array the first one left behind.  This file is named to be
collected last, after every other test has used the library on the same device.
"""
import pytest
import torch

MAX_OPERAND_FLOATS = 4194240  # (16 MiB - 256 B) / 4


def _noalloc(A, B, C, alpha, beta):
    from mpq_b200._lib import call, ptr
    M, K = A.shape
    N = B.shape[0]
    call("mpq_gemm_tf32x3_noalloc", M, N, K, float(alpha), ptr(A), A.stride(0), ptr(B), B.stride(0), float(beta),
         ptr(C), C.stride(0), None)
    return C


def test_noalloc_rejects_oversize_products():
    """Sizes beyond the array are refused before any device work (runs without a GPU)."""
    from mpq_b200 import _lib
    lib = _lib.load()
    fn = lib.mpq_gemm_tf32x3_noalloc
    M, N, K = 2048, 2048, 1024  # 2 * 4096 * 1024 = 8.4M floats > 4,194,240
    assert 2 * (M + N) * K > MAX_OPERAND_FLOATS
    dummy = 16  # never dereferenced: the size check comes first
    rc = fn(M, N, K, 1.0, dummy, K, dummy, K, 0.0, dummy, N, None, None)
    assert rc == 10001
    assert b"exceeds" in lib.mpq_last_error()


@pytest.mark.gpu
def test_noalloc_matches_allocating_entry_point(cuda_dev):
    from mpq_b200 import ops
    # tolerance of the tensor-core tests: 1e-5 of the |A| |B|^T scale (3xTF32 is FP32-class)
    tol = 1e-5
    cases = [((300, 200, 196), 1.0, 0.0, 11), ((512, 768, 1000), -0.5, 2.0, 12)]
    for (M, N, K), alpha, beta, seed in cases:
        g = torch.Generator(device="cpu").manual_seed(seed)
        A = torch.randn(M, K, generator=g).to(cuda_dev)
        Bt = torch.randn(N, K, generator=g).to(cuda_dev)
        C0 = torch.randn(M, N, generator=g).to(cuda_dev)
        assert 2 * (M + N) * ((K + 3) // 4 * 4) <= MAX_OPERAND_FLOATS
        want = ops.mm_nt(A, ops.Operand(Bt, "tf32x3"), out=C0.clone(), alpha=alpha, beta=beta, precision="tf32x3")
        got = _noalloc(A, Bt, C0.clone(), alpha, beta)
        torch.cuda.synchronize()
        ops.check_status(cuda_dev)
        scale = (A.double().abs() @ Bt.double().abs().T).max().item()
        err = (got.double() - want.double()).abs().max().item()
        assert err <= tol * scale, (M, N, K, err, scale)
        ref = beta * C0.double() + alpha * (A.double() @ Bt.double().T)
        assert (got.double() - ref).abs().max().item() <= tol * scale + 1e-5
