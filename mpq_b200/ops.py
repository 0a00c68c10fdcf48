"""Thin tensor-level wrappers over the C-ABI kernels (torch only allocates and passes pointers)."""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib, trace
from ._lib import call, ptr


def _check_cuda_f32(*ts):
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("mpq_b200 kernels require CUDA tensors (there is no CPU path)")


def group_layout(scale: torch.Tensor, n: int):
    """Return (ld_p, gshift) for scale/zero given either group-expanded (B, n) or per-group (B, G)."""
    cols = int(scale.shape[1])
    if cols == n:
        return int(scale.stride(0)), 0
    if cols <= 0 or n % cols != 0:
        raise ValueError(f"group params with {cols} columns do not tile n={n}")
    g = n // cols
    if g & (g - 1):
        raise ValueError(f"group size {g} must be a power of two")
    return int(scale.stride(0)), g.bit_length() - 1


def gemm_nt(A: torch.Tensor, Bt: torch.Tensor, out: Optional[torch.Tensor] = None, *, alpha: float = 1.0,
            beta: float = 0.0) -> torch.Tensor:
    """C = alpha * A @ Bt^T + beta * C  (A: M x K, Bt: N x K, both row-major float32)."""
    _check_cuda_f32(A, Bt, out)
    M, K = A.shape
    N = Bt.shape[0]
    if Bt.shape[1] != K:
        raise ValueError(f"gemm_nt shape mismatch {tuple(A.shape)} x {tuple(Bt.shape)}^T")
    if out is None:
        out = torch.empty(M, N, device=A.device, dtype=torch.float32)
    tok = trace.begin_timing("gemm")
    call("mpq_gemm_f32", 0, M, N, K, float(alpha), ptr(A), A.stride(0), ptr(Bt), Bt.stride(0), float(beta),
         ptr(out), out.stride(0))
    trace.end_timing("gemm", tok, 2.0 * M * N * K)
    return out


def gemm_nn(A: torch.Tensor, Bm: torch.Tensor, out: Optional[torch.Tensor] = None, *, alpha: float = 1.0,
            beta: float = 0.0) -> torch.Tensor:
    """C = alpha * A @ Bm + beta * C  (A: M x K, Bm: K x N, both row-major float32)."""
    _check_cuda_f32(A, Bm, out)
    M, K = A.shape
    N = Bm.shape[1]
    if Bm.shape[0] != K:
        raise ValueError(f"gemm_nn shape mismatch {tuple(A.shape)} x {tuple(Bm.shape)}")
    if out is None:
        out = torch.empty(M, N, device=A.device, dtype=torch.float32)
    tok = trace.begin_timing("gemm")
    call("mpq_gemm_f32", 1, M, N, K, float(alpha), ptr(A), A.stride(0), ptr(Bm), Bm.stride(0), float(beta),
         ptr(out), out.stride(0))
    trace.end_timing("gemm", tok, 2.0 * M * N * K)
    return out


def rankspace_error(Y_u: torch.Tensor, x: torch.Tensor, VsT: torch.Tensor, tmp: Optional[torch.Tensor] = None,
                    out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """rowsum((Y_u - x @ Vs)^2)  (mpq/linear.py:85-94); VsT is Vs transposed (R x n)."""
    B = x.shape[0]
    C = gemm_nt(x, VsT, tmp)
    if out is None:
        out = torch.empty(B, device=x.device, dtype=torch.float32)
    call("mpq_row_sqerr", ptr(Y_u), ptr(C), B, C.shape[1], Y_u.stride(0), C.stride(0), ptr(out))
    return out


def mean_rows(a: torch.Tensor, c: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(1, device=a.device, dtype=torch.float32)
    call("mpq_mean_rows", ptr(a), ptr(c), int(a.numel()), ptr(out))
    return out
