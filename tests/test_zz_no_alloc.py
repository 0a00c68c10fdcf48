"""The allocation-free 3xTF32 product (mpq_gemm_tf32x3_noalloc) against the allocating entry point.

mpq_gemm_tf32x3_noalloc keeps the TF32 operand split in a file-scope device array instead of caller buffers;
these tests call it through the C-ABI and compare it with mpq_split_tf32 + mpq_gemm_tc (ops.mm_nt) on two
calls in a row, so the second call runs on the array the first one left behind.  This file is named to be
collected last, after every other test has used the library on the same device.
"""
import pytest
import torch

MAX_OPERAND_FLOATS = 4194240  # (16 MiB - 256 B) / 4


def _noalloc(A, B, C, alpha, beta, status=None):
    from mpq_b200._lib import call, ptr
    M, K = A.shape
    N = B.shape[0]
    call("mpq_gemm_tf32x3_noalloc", M, N, K, float(alpha), ptr(A), A.stride(0), ptr(B), B.stride(0), float(beta),
         ptr(C), C.stride(0), None if status is None else ptr(status))
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
    # the third product is smaller than the second and has K % 4 != 0: it runs over the scratch the second call
    # left behind, with a TMA row width (K) narrower than the padded stride round_up(K, 4).  The first call uses the
    # status word inside the array (status=None); the others pass a caller-owned word, pre-set to a non-zero value
    # to show that the call clears it.
    cases = [((300, 200, 196), 1.0, 0.0, 11, False), ((512, 768, 1000), -0.5, 2.0, 12, True),
             ((130, 70, 97), 0.75, -1.0, 13, True)]
    for (M, N, K), alpha, beta, seed, own_status in cases:
        g = torch.Generator(device="cpu").manual_seed(seed)
        A = torch.randn(M, K, generator=g).to(cuda_dev)
        Bt = torch.randn(N, K, generator=g).to(cuda_dev)
        C0 = torch.randn(M, N, generator=g).to(cuda_dev)
        assert 2 * (M + N) * ((K + 3) // 4 * 4) <= MAX_OPERAND_FLOATS
        want = ops.mm_nt(A, ops.Operand(Bt, "tf32x3"), out=C0.clone(), alpha=alpha, beta=beta, precision="tf32x3")
        status = torch.full((1,), 7, dtype=torch.int32, device=cuda_dev) if own_status else None
        got = _noalloc(A, Bt, C0.clone(), alpha, beta, status)
        torch.cuda.synchronize()
        ops.check_status(cuda_dev)
        if status is not None:
            assert int(status.item()) == 0, "pipeline wait timed out inside mpq_gemm_tf32x3_noalloc"
        scale = (A.double().abs() @ Bt.double().abs().T).max().item()
        err = (got.double() - want.double()).abs().max().item()
        assert err <= tol * scale, (M, N, K, err, scale)
        ref = beta * C0.double() + alpha * (A.double() @ Bt.double().T)
        assert (got.double() - ref).abs().max().item() <= tol * scale + 1e-5


@pytest.mark.gpu
def test_second_device_in_one_process(cuda_dev):
    """Both GEMM entry points on cuda:1 after cuda:0 in one process: the shared-memory opt-in and the array's address
    are per device, so the second device needs its own set-up (skipped with one visible GPU)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two visible GPUs")
    from mpq_b200 import ops
    for dev in (torch.device("cuda:0"), torch.device("cuda:1")):
        with torch.cuda.device(dev):
            g = torch.Generator(device="cpu").manual_seed(21)
            A = torch.randn(200, 132, generator=g).to(dev)
            Bt = torch.randn(150, 132, generator=g).to(dev)
            want = A.double() @ Bt.double().T
            scale = (A.double().abs() @ Bt.double().abs().T).max().item()
            got_tc = ops.mm_nt(A, ops.Operand(Bt))
            status = torch.zeros(1, dtype=torch.int32, device=dev)
            got_na = _noalloc(A, Bt, torch.zeros(200, 150, device=dev), 1.0, 0.0, status)
            torch.cuda.synchronize(dev)
            ops.check_status(dev)
            assert int(status.item()) == 0
            assert (got_tc.double() - want).abs().max().item() <= 1e-5 * scale
            assert (got_na.double() - want).abs().max().item() <= 1e-5 * scale
