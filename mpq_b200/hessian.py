"""Calibration-Hessian accumulation H = X^T X on the tensor cores (tcgen05 symmetric product).

The MPQ drivers consume Hessians collected by third-party forward hooks (not part of the reference tree):

* QUIP# ``utils.register_H_hook``: per batch H += x^T x, mu += sum_t x_t, ct += tokens; ``done()`` returns
  (H, mu, ct), which MPQ finalises as H / ct - (mu / ct)(mu / ct)^T (mpq/quip_generic.py:906-918) and
  re-centres with + mu mu^T before ``regularize_H`` (mpq/quip_generic.py:373-378);
* GPTQModel ``GPTQ.add_batch``: H <- H * ns / (ns + b) + (2 / (ns + b)) x^T x with b the leading (batch)
  dimension of the hooked input and ns += b; ``run_mpq_quantization`` takes this H (2/n convention,
  mpq/adapters/gptqmodel.py:650-679).

Both are restated here from their published sources; their parity is unpinned (the code is absent from
the reference tree).  Activations may be float32 (3xTF32: FP32-faithful) or bfloat16 (bf16 tensor-core products,
exact up to the FP32 accumulation).
"""
from __future__ import annotations

import ctypes as _ct
from typing import Optional, Tuple

import torch

from . import ops
from ._lib import call, ptr


def _as_tokens(x: torch.Tensor, n: int) -> Tuple[torch.Tensor, int]:
    x = x.reshape(-1, n)
    if x.dtype not in (torch.float32, torch.bfloat16):
        x = x.float()
    if x.stride(-1) != 1:
        x = x.contiguous()
    return x, (1 if x.dtype == torch.bfloat16 else 0)


class _Split:
    """Reusable K-major TF32 halves of X^T (n x round_up(T, 4))."""

    def __init__(self):
        self.hi = self.lo = None

    def get(self, n: int, tokens: int, device, need_lo: bool):
        ld = (tokens + 3) // 4 * 4
        if self.hi is None or self.hi.shape[0] != n or self.hi.shape[1] < ld or self.hi.device != device:
            self.hi = torch.empty(n, ld, device=device, dtype=torch.float32)
            self.lo = torch.empty(n, ld, device=device, dtype=torch.float32)
        return self.hi, (self.lo if need_lo else None), self.hi.stride(0)


_split_cache: dict = {}
_bf16_cache: dict = {}

# The tensor core's FP32 accumulator does not round to nearest (its error grows with the K extent of one
# accumulation: 1.7e-5 relative low after 4100 tokens).  The symmetric product accumulates at most CHUNK_TOKENS
# tokens at a time in tensor memory and adds the chunks, round to nearest, into a running sum kept there (one
# launch over all tokens, H read and written once per tile), which keeps H within a few 1e-6 of an FP32 FMA
# product.
CHUNK_TOKENS = 1024


def accumulate_xtx(H: torch.Tensor, x: torch.Tensor, *, alpha: float = 1.0, beta: float = 1.0) -> torch.Tensor:
    """H <- beta H + alpha X^T X for token-major activations x (..., n); H is n x n fp32, symmetric on entry
    when beta != 0, exactly symmetric on exit."""
    n = H.shape[0]
    if H.shape != (n, n) or H.dtype != torch.float32 or not H.is_cuda or H.stride(-1) != 1:
        raise ValueError("H must be an n x n float32 CUDA tensor with unit column stride")
    X, dtype = _as_tokens(x, n)
    if X.device != H.device:
        raise ValueError("x and H must be on the same device")
    T = X.shape[0]
    if T == 0:
        if beta != 1.0:
            H.mul_(beta)
        return H
    key = (H.device.type, H.device.index)
    st = ptr(ops.status_word(H.device))
    if dtype == 1:  # bf16 activations: exact bf16 operands on the kind::f16 tensor-core path
        ld = (T + 7) // 8 * 8
        XT = _bf16_cache.get(key)
        if XT is None or XT.shape[0] != n or XT.shape[1] < ld:
            XT = _bf16_cache[key] = torch.empty(n, ld, device=H.device, dtype=torch.bfloat16)
        ld = XT.stride(0)
        call("mpq_transpose_bf16", ptr(X), X.stride(0), T, n, ptr(XT), ld)
        call("mpq_syrk_bf16_acc", n, T, float(alpha), ptr(XT), ld, float(beta), ptr(H), H.stride(0), CHUNK_TOKENS, st)
        return H
    sp = _split_cache.setdefault(key, _Split())
    hi, lo, ld = sp.get(n, T, H.device, need_lo=(dtype == 0))
    call("mpq_split_tf32_t", ptr(X), dtype, X.stride(0), T, n, ptr(hi), ptr(lo), ld)
    if dtype == 0:
        As, Bs = [hi, hi, lo], [hi, lo, hi]
    else:
        As, Bs = [hi], [hi]
    arrA = (_ct.c_void_p * 3)(*[t.data_ptr() for t in As])
    arrB = (_ct.c_void_p * 3)(*[t.data_ptr() for t in Bs])
    call("mpq_syrk_tc_acc", len(As), n, T, float(alpha), arrA, arrB, ld, float(beta), ptr(H), H.stride(0),
         CHUNK_TOKENS, st)
    return H


class HessianAccumulator:
    """Running Hessian of one linear layer's inputs.  mode "quip" (sum, running mean, token count) or
    "gptq" (running average with the 2/n scale)."""

    def __init__(self, n: int, *, device, mode: str = "quip"):
        if mode not in ("quip", "gptq"):
            raise ValueError(f"unknown Hessian mode {mode!r}")
        self.n, self.mode = int(n), mode
        self.device = torch.device(device)
        self.H = torch.zeros(self.n, self.n, device=self.device, dtype=torch.float32)
        self.mu = torch.zeros(self.n, device=self.device, dtype=torch.float32) if mode == "quip" else None
        self.ct = 0        # tokens (quip)
        self.nsamples = 0  # leading-dimension samples (gptq)

    @torch.inference_mode()
    def add_batch(self, inp: torch.Tensor) -> None:
        if inp.shape[-1] != self.n:
            raise ValueError(f"expected inputs with last dimension {self.n}, got {tuple(inp.shape)}")
        if self.mode == "quip":
            X, dtype = _as_tokens(inp, self.n)
            accumulate_xtx(self.H, X, alpha=1.0, beta=1.0)
            call("mpq_col_sum", ptr(X), dtype, X.stride(0), X.shape[0], self.n, 1.0, 1.0, ptr(self.mu))
            self.ct += X.shape[0]
        else:
            b = int(inp.shape[0]) if inp.dim() == 3 else 1  # GPTQ: 2-D inputs count as one sample
            total = self.nsamples + b
            beta = self.nsamples / total
            self.nsamples = total
            accumulate_xtx(self.H, inp, alpha=2.0 / total, beta=beta)

    @torch.inference_mode()
    def finalize(self):
        """quip: (H / ct - mu mu^T, mu, ct) with mu = sum / ct (the hook's done() as MPQ finalises it);
        gptq: H."""
        ops.check_status(self.device)
        if self.mode == "gptq":
            return self.H
        if self.ct == 0:
            raise RuntimeError("no activations were accumulated")
        mu = self.mu / self.ct
        H = self.H / self.ct
        H.addr_(mu, mu, alpha=-1.0)
        return H, mu, self.ct


def regularize_H(H: torch.Tensor, n: int, sigma_reg: float) -> torch.Tensor:
    """QUIP# utils.regularize_H as called at mpq/quip_generic.py:378: H / mean(diag H) + sigma_reg I (in place)."""
    H.div_(torch.diagonal(H).mean())
    idx = torch.arange(int(n), device=H.device)
    H[idx, idx] += float(sigma_reg)
    return H


def covariance_to_second_moment(H: torch.Tensor, mu: torch.Tensor) -> torch.Tensor:
    """H + mu mu^T: the re-centring of a stored (H, mu) pair before the solve (mpq/quip_generic.py:373-375)."""
    return H.addr_(mu, mu)
