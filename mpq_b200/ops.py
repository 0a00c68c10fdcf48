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
    tok = trace.begin_timing("gemm_f32")
    call("mpq_gemm_f32", 0, M, N, K, float(alpha), ptr(A), A.stride(0), ptr(Bt), Bt.stride(0), float(beta),
         ptr(out), out.stride(0))
    trace.end_timing("gemm_f32", tok, 2.0 * M * N * K)
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
    tok = trace.begin_timing("gemm_f32")
    call("mpq_gemm_f32", 1, M, N, K, float(alpha), ptr(A), A.stride(0), ptr(Bm), Bm.stride(0), float(beta),
         ptr(out), out.stride(0))
    trace.end_timing("gemm_f32", tok, 2.0 * M * N * K)
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


# ------------------------------------------------------------------------------------------------
# tcgen05 tensor-core products (3xTF32 by default)
# ------------------------------------------------------------------------------------------------

import ctypes as _ct

_PRECISION = "f16x3"
_scratch = {}
_status = {}


def set_gemm_precision(mode: str) -> None:
    """'tf32x3' (FP32-faithful 3xTF32 split products), 'f16x3' (FP32-faithful row-scaled 3xFP16 split products on the
    fp16 tensor cores, twice the TF32 rate), 'tf32' (single TF32 product) or 'fp32' (CUDA-core FP32 kernel)."""
    global _PRECISION
    if mode not in ("tf32x3", "f16x3", "tf32", "fp32"):
        raise ValueError(f"unknown GEMM precision {mode!r}")
    _PRECISION = mode


def gemm_precision() -> str:
    return _PRECISION


def status_word(device: torch.device) -> torch.Tensor:
    key = (device.type, device.index)
    t = _status.get(key)
    if t is None:
        t = torch.zeros(1, device=device, dtype=torch.int32)
        _status[key] = t
    return t


def check_status(device: torch.device) -> None:
    """Raise if a tensor-core pipeline wait timed out since the last check (host sync)."""
    t = status_word(device)
    v = int(t.item())
    if v:
        t.zero_()
        raise RuntimeError(f"mpq_gemm_tc: pipeline wait timed out (code {v})")


def _tma_ok(t: torch.Tensor) -> bool:
    return t.stride(-1) == 1 and t.stride(0) % 4 == 0 and t.data_ptr() % 16 == 0


def split_tf32(x: torch.Tensor, hi: Optional[torch.Tensor] = None, lo: Optional[torch.Tensor] = None):
    """hi = round-to-nearest TF32 of x, lo = x - hi (exact)."""
    rows, cols = x.shape
    if hi is None:
        hi = torch.empty(rows, cols, device=x.device, dtype=torch.float32)
    if lo is None:
        lo = torch.empty_like(hi)
    call("mpq_split_tf32", ptr(x), x.stride(0), ptr(hi), ptr(lo), hi.stride(0), rows, cols)
    return hi, lo


def split_f16(x: torch.Tensor, bufs=None):
    """Row-scaled fp16 split: hi = fp16(x s), lo = fp16(x s - hi) with s = 2^(15 - E), max|x_row| < 2^E;
    returns (hi, lo, 1 / s) with hi / lo row-major, leading dimension a multiple of 8."""
    rows, cols = x.shape
    if bufs is None:
        ld = (cols + 7) // 8 * 8
        hi = torch.empty(rows, ld, device=x.device, dtype=torch.float16)
        bufs = (hi, torch.empty_like(hi), torch.empty(rows, device=x.device, dtype=torch.float32))
    hi, lo, inv = bufs
    call("mpq_split_f16", ptr(x), x.stride(0), rows, cols, ptr(hi), ptr(lo), hi.stride(0), ptr(inv))
    return hi, lo, inv


class Operand:
    """A row-major K-major matrix used as the B side of repeated products, with its split for the precision."""

    def __init__(self, t: torch.Tensor, precision: Optional[str] = None):
        self.full = t
        self.precision = precision or _PRECISION
        self.hi = self.lo = None
        self.f16 = None
        if self.precision == "tf32x3" and _tma_ok(t):
            self.hi, self.lo = split_tf32(t)
        elif self.precision == "f16x3" and t.dim() == 2 and t.dtype == torch.float32:
            self.f16 = split_f16(t)

    @classmethod
    def presplit(cls, full: torch.Tensor, f16) -> "Operand":
        """An f16x3 operand whose row-scaled split (hi, lo, inv) is already made (``full`` gives the shape only)."""
        op = cls.__new__(cls)
        op.full, op.precision, op.hi, op.lo, op.f16 = full, "f16x3", None, None, tuple(f16)
        return op

    def reload(self, t: torch.Tensor) -> None:
        """Copy new values (same shape) into this operand's buffers and re-split them in place: products captured in a
        CUDA graph against this operand see the new matrix."""
        self.full.copy_(t)
        if self.hi is not None:
            split_tf32(self.full, self.hi, self.lo)
        if self.f16 is not None:
            split_f16(self.full, self.f16)

    @property
    def shape(self):
        return self.full.shape


def _stream_key(dev: torch.device):
    """Scratch buffers are private to one (device, stream): work ordered on one stream never races on them, and work
    on concurrent streams (the chained solve's polish streams) never shares them.  Inside a CUDA-graph capture the
    scratch is private to the capture (graph-pool memory must not leak into eager calls)."""
    s = torch.cuda.current_stream(dev)
    if torch.cuda.is_current_stream_capturing():
        return ("capture", id(_capture_scratch()))
    return (dev.index, s.cuda_stream)


_capture_local = {}


def _capture_scratch():
    import threading
    d = _capture_local.get(threading.get_ident())
    if d is None:
        raise RuntimeError("tensor-core products inside a CUDA-graph capture need ops.graph_scratch()")
    return d


class graph_scratch:
    """Context for a CUDA-graph capture: the products captured inside use scratch buffers private to this capture
    (allocated from the graph's memory pool); keep the returned dict alive as long as the graph."""

    def __enter__(self):
        import threading
        self.key = threading.get_ident()
        self.prev = _capture_local.get(self.key)
        self.d = {}
        _capture_local[self.key] = self.d
        return self.d

    def __exit__(self, *exc):
        if self.prev is None:
            _capture_local.pop(self.key, None)
        else:
            _capture_local[self.key] = self.prev
        return False


def _scratch_dict(dev: torch.device):
    if torch.cuda.is_current_stream_capturing():
        return _capture_scratch()
    return _scratch


def _scratch_split(A: torch.Tensor):
    key = ("tf32", _stream_key(A.device), tuple(A.shape))
    sd = _scratch_dict(A.device)
    buf = sd.get(key)
    if buf is None:
        buf = (torch.empty(A.shape, device=A.device, dtype=torch.float32),
               torch.empty(A.shape, device=A.device, dtype=torch.float32))
        sd[key] = buf
    return split_tf32(A, buf[0], buf[1])


def _scratch_split16(A: torch.Tensor):
    key = ("f16", _stream_key(A.device), tuple(A.shape))
    sd = _scratch_dict(A.device)
    buf = sd.get(key)
    if buf is None:
        ld = (A.shape[1] + 7) // 8 * 8
        hi = torch.empty(A.shape[0], ld, device=A.device, dtype=torch.float16)
        buf = (hi, torch.empty_like(hi), torch.empty(A.shape[0], device=A.device, dtype=torch.float32))
        sd[key] = buf
    return split_f16(A, buf)


def _splitk_workspace(dev: torch.device, floats: int) -> torch.Tensor:
    key = ("splitk", _stream_key(dev))
    sd = _scratch_dict(dev)
    ws = sd.get(key)
    if ws is None or ws.numel() < floats:
        ws = torch.empty(max(int(floats), 1), device=dev, dtype=torch.float32)
        sd[key] = ws
    return ws


_NUM_SMS = {}


def num_sms(dev: torch.device) -> int:
    n = _NUM_SMS.get(dev.index)
    if n is None:
        n = torch.cuda.get_device_properties(dev).multi_processor_count
        _NUM_SMS[dev.index] = n
    return n


def splitk_for(M: int, N: int, K: int, sms: int) -> int:
    """K-splits for a 3-region fp16 product: 1 when the 128 x 256 tiles already fill half the SMs; otherwise enough
    splits to reach about one unit per SM, with at least 8 of the 3 * ceil(K / 64) k-blocks per unit."""
    tiles = ((M + 127) // 128) * ((N + 255) // 256)
    total_kb = 3 * ((K + 63) // 64)
    if tiles * 2 >= sms or total_kb < 16:
        return 1
    return max(1, min(sms // tiles, total_kb // 8))


def mm_nt(A: torch.Tensor, B, out: Optional[torch.Tensor] = None, *, alpha: float = 1.0, beta: float = 0.0,
          precision: Optional[str] = None) -> torch.Tensor:
    """C = alpha * A @ B^T + beta * C on the tensor cores.  B: Operand or (N x K) tensor; A: (M x K) tensor, or an
    Operand whose f16x3 split is already made (Operand.presplit)."""
    A_split = None
    if isinstance(A, Operand):
        A_split = A.f16
        A = A.full
    if not isinstance(B, Operand):
        B = Operand(B, precision)
    prec = precision or B.precision
    M, K = A.shape
    N = B.full.shape[0]
    if B.full.shape[1] != K:
        raise ValueError(f"mm_nt shape mismatch {tuple(A.shape)} x {tuple(B.full.shape)}^T")
    if out is None:
        out = torch.empty(M, N, device=A.device, dtype=torch.float32)
    if prec == "f16x3" and B.f16 is None:
        B = Operand(B.full, "f16x3")
    if prec == "f16x3" and A.dtype == torch.float32 and (A_split is not None or A.stride(-1) == 1):
        Ah, Al, Ai = A_split if A_split is not None else _scratch_split16(A)
        Bh, Bl, Bi = B.f16
        st = status_word(A.device)
        splits = splitk_for(M, N, K, num_sms(A.device)) if M and N else 1
        tok = trace.begin_timing("gemm_tc")
        if splits > 1:
            ws = _splitk_workspace(A.device, splits * M * N)
            call("mpq_gemm_f16x3_splitk", M, N, K, float(alpha), ptr(Ah), ptr(Al), Ah.stride(0), ptr(Ai), ptr(Bh),
                 ptr(Bl), Bh.stride(0), ptr(Bi), float(beta), ptr(out), out.stride(0), splits, ptr(ws), ws.numel(),
                 ptr(st))
        else:
            call("mpq_gemm_f16x3", M, N, K, float(alpha), ptr(Ah), ptr(Al), Ah.stride(0), ptr(Ai), ptr(Bh), ptr(Bl),
                 Bh.stride(0), ptr(Bi), float(beta), ptr(out), out.stride(0), ptr(st))
        trace.end_timing("gemm_tc", tok, 2.0 * M * N * K)
        return out
    if prec == "fp32" or not (_tma_ok(A) and _tma_ok(B.full) and (prec != "tf32x3" or B.hi is not None)):
        return gemm_nt(A, B.full, out, alpha=alpha, beta=beta)
    if prec == "tf32x3":
        Ah, Al = _scratch_split(A)
        As = [Ah, Ah, Al]
        Bs = [B.hi, B.lo, B.hi]
        lda = Ah.stride(0)
        ldb = B.hi.stride(0)
    else:
        As, Bs = [A], [B.full]
        lda, ldb = A.stride(0), B.full.stride(0)
    arrA = (_ct.c_void_p * 3)(*[t.data_ptr() for t in As])
    arrB = (_ct.c_void_p * 3)(*[t.data_ptr() for t in Bs])
    st = status_word(A.device)
    tok = trace.begin_timing("gemm_tc")
    call("mpq_gemm_tc", len(As), M, N, K, float(alpha), arrA, lda, arrB, ldb, float(beta), ptr(out), out.stride(0),
         ptr(st))
    trace.end_timing("gemm_tc", tok, 2.0 * M * N * K)
    return out
