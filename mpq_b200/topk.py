"""Top-k candidate sets of the "topk_block_cd" polish.

Reference: mpq/priors/uniform.py:253-284 (uniform_map_topk) and mpq/priors/e8p12.py:453-538
(vamp_vector_map_topk_e8p12).  Both run in libmpq_b200.so (``mpq_uniform_topk``, ``mpq_e8p12_topk``).
"""
from __future__ import annotations

from typing import Dict, Optional

import torch

from . import ops
from ._lib import call, ptr
from .codebook import factor_tables

E8P12_TOPK_CANDIDATES = 1024  # 2 branches x 256 abs patterns x {best, second-best sign pattern}


@torch.inference_mode()
def uniform_map_topk(*, r1: torch.Tensor, gamma1: torch.Tensor, scale_full: torch.Tensor, zero_full: torch.Tensor,
                     maxq: int, prior_center: Optional[torch.Tensor], prior_tau: float, k: int,
                     atoms: Optional[torch.Tensor] = None) -> Dict[str, torch.Tensor]:
    """The k best grid levels per coordinate under score(q) = -g/2 (a_q - r1)^2 [- (a_q - W)^2 / (2 (tau s)^2)],
    a_q = s (q - z); descending, ties to the lower level.  ``atoms`` (the reference's optional precomputed
    s (q - z)) is accepted for call compatibility; the kernel forms the same atoms itself.

    Returns {"topk_q": int64 (B, n, k_eff), "topk_values": float32, "topk_scores": float32}, k_eff = min(k, maxq+1).
    """
    if not r1.is_cuda:
        raise ValueError("uniform_map_topk requires CUDA tensors (there is no CPU path)")
    dev = r1.device
    B, n = r1.shape
    maxq = int(maxq)
    k_eff = min(max(int(k), 1), maxq + 1)
    r = r1.to(torch.float32).contiguous()
    s = scale_full.to(device=dev, dtype=torch.float32)
    z = zero_full.to(device=dev, dtype=torch.float32)
    if s.stride(-1) != 1 or z.stride(-1) != 1 or s.stride(0) != z.stride(0):
        s, z = s.contiguous(), z.contiguous()
    ld_p, gshift = ops.group_layout(s, n)
    g = gamma1.reshape(B).to(device=dev, dtype=torch.float32).contiguous()
    tau = float(prior_tau)
    c = None
    if tau > 0.0:
        if prior_center is None:
            raise ValueError("prior_tau > 0 needs prior_center")
        c = prior_center.to(device=dev, dtype=torch.float32).contiguous()
    q = torch.empty(B, n, k_eff, device=dev, dtype=torch.int32)
    v = torch.empty(B, n, k_eff, device=dev, dtype=torch.float32)
    sc = torch.empty(B, n, k_eff, device=dev, dtype=torch.float32)
    call("mpq_uniform_topk", ptr(r), r.stride(0), ptr(c), c.stride(0) if c is not None else 0, ptr(s), ptr(z), ld_p,
         gshift, ptr(g), B, n, maxq, tau if c is not None else 0.0, k_eff, ptr(q), ptr(v), ptr(sc))
    return {"topk_q": q.to(torch.int64), "topk_values": v, "topk_scores": sc}


@torch.inference_mode()
def vamp_vector_map_topk_e8p12(*, r1_blocks: torch.Tensor, gamma1: torch.Tensor, cb, k: int,
                               blocks_per_chunk: int = 64, prior_center_blocks: Optional[torch.Tensor] = None,
                               prior_scale_blocks: Optional[torch.Tensor] = None, prior_tau: float = 0.0,
                               prior_tau_scale_mode: str = "absmax") -> Dict[str, torch.Tensor]:
    """Per block, the k highest-scoring of the 1024 candidates {best, second-best parity-valid sign pattern} x
    (branch, abs pattern) under the folded message.  ``blocks_per_chunk`` is accepted for call compatibility (one
    launch covers every block).

    Returns {"topk_idxs": int64 (B, nb, k_eff), "topk_scores": float32 (B, nb, k_eff), "topk_vals": float32
    (B, nb, k_eff, 8)}, k_eff = min(k, 1024).
    """
    from .e8p12 import _fold_args, _tab_ptrs
    B, nb, codesz = r1_blocks.shape
    if int(codesz) != 8:
        raise ValueError(f"E8P12 top-k expects codesz=8, got {codesz}.")
    k = int(k)
    if k <= 0:
        raise ValueError(f"expected k>0, got k={k}")
    if not r1_blocks.is_cuda:
        raise ValueError("vamp_vector_map_topk_e8p12 requires CUDA tensors (there is no CPU path)")
    k_eff = min(k, E8P12_TOPK_CANDIDATES)
    r1, center, pscale, tau = _fold_args(r1_blocks, prior_center_blocks, prior_scale_blocks, prior_tau,
                                         prior_tau_scale_mode)
    dev = r1.device
    t = factor_tables(cb, dev)
    g = gamma1.reshape(B).to(device=dev, dtype=torch.float32).contiguous()
    idx = torch.empty(B, nb, k_eff, device=dev, dtype=torch.int32)
    sc = torch.empty(B, nb, k_eff, device=dev, dtype=torch.float32)
    vals = torch.empty(B, nb, k_eff, 8, device=dev, dtype=torch.float32)
    call("mpq_e8p12_topk", ptr(r1), r1.stride(0), ptr(center), center.stride(0) if center is not None else 0,
         ptr(pscale), pscale.stride(0) if pscale is not None else 0, ptr(g), float(tau), B, nb, *_tab_ptrs(t), k_eff,
         ptr(idx), ptr(sc), ptr(vals))
    if idx.numel() and int(idx.min()) < 0:
        raise RuntimeError("failed to map factorized E8P12 top-k sign patterns back to full codebook indices.")
    return {"topk_idxs": idx.to(torch.int64), "topk_scores": sc, "topk_vals": vals}
