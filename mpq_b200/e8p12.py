"""E8P12 prior (factorized posterior / MAP / nearest codeword) and the gram-metric block CD engine.

Reference: mpq/priors/e8p12.py (prior_scale_from_center :47-63, vamp_vector_map_e8p12 :541-631,
vamp_vector_discrete_mmse_e8p12 :815-968) and mpq/polish/block_cd.py (block_coordinate_descent_rankspace
:332-625 with the E8P12 gram provider).  All numerical work runs in libmpq_b200.so.
"""
from __future__ import annotations

from typing import Any, Dict, Optional, Tuple

import torch

from . import ops
from ._lib import call, ptr
from .codebook import factor_tables


def prior_scale_from_center(prior_center_blocks: Optional[torch.Tensor], mode: str) -> Optional[torch.Tensor]:
    """mpq/priors/e8p12.py:47-63 (per-block prior scale; plumbing on B x nb values)."""
    if prior_center_blocks is None:
        return None
    mode = str(mode or "absmax").strip().lower()
    c = prior_center_blocks.to(torch.float32)
    if mode in ("none", "unit", "legacy"):
        return torch.ones(c.shape[:-1] + (1,), dtype=torch.float32, device=c.device)
    if mode in ("absmax", "exact_full", "exact_full_absmax"):
        s = c.abs().amax(dim=-1, keepdim=True)
    elif mode in ("rms", "std"):
        s = c.square().mean(dim=-1, keepdim=True).sqrt()
    elif mode in ("mean_abs", "l1"):
        s = c.abs().mean(dim=-1, keepdim=True)
    else:
        raise ValueError(f"unsupported prior_tau_scale_mode={mode!r}; supported: none|absmax|rms|mean_abs")
    return s.clamp_min_(1e-12)


def _tab_ptrs(t):
    return (ptr(t["base_abs"]), ptr(t["base_sqnorm"]), ptr(t["base_parity"]), ptr(t["idx_lut"]), ptr(t["grid"]))


def e8p12_map_rows(r1: torch.Tensor, cb, *, gamma: Optional[torch.Tensor] = None, fixed_gamma: float = 0.0,
                   center: Optional[torch.Tensor] = None, pscale: Optional[torch.Tensor] = None,
                   prior_tau: float = 0.0) -> Tuple[torch.Tensor, torch.Tensor]:
    """MAP codewords of a (B, n) message (n = 8 nb): returns (values (B, n), indices (B, nb) int32)."""
    if not r1.is_cuda:
        raise ValueError("E8P12 kernels require CUDA tensors (there is no CPU path)")
    B, n = r1.shape
    nb = n // 8
    t = factor_tables(cb, r1.device)
    idx = torch.empty(B, nb, device=r1.device, dtype=torch.int32)
    vals = torch.empty(B, n, device=r1.device, dtype=torch.float32)
    call("mpq_e8p12_map", ptr(r1), r1.stride(0), ptr(center), center.stride(0) if center is not None else 0,
         ptr(pscale), pscale.stride(0) if pscale is not None else 0, ptr(gamma), float(fixed_gamma), float(prior_tau),
         B, nb, *_tab_ptrs(t), ptr(idx), idx.stride(0), ptr(vals), vals.stride(0))
    return vals, idx


def e8p12_nearest(X: torch.Tensor, cb) -> Tuple[torch.Tensor, torch.Tensor]:
    """Nearest codeword of each 8-vector (N, 8): the MAP at unit precision without prior."""
    X = X.to(torch.float32).reshape(-1, 8)
    N = X.shape[0]
    per = 64
    rows = (N + per - 1) // per
    pad = rows * per - N
    Xp = torch.cat([X, X.new_zeros(pad, 8)]) if pad else X.contiguous()
    vals, idx = e8p12_map_rows(Xp.reshape(rows, per * 8), cb, fixed_gamma=1.0)
    return vals.reshape(-1, 8)[:N], idx.reshape(-1)[:N].to(torch.int64)


def _fold_args(r1_blocks, prior_center_blocks, prior_scale_blocks, prior_tau, prior_tau_scale_mode):
    B, nb, _ = r1_blocks.shape
    r1 = r1_blocks.reshape(B, nb * 8).to(torch.float32).contiguous()
    center = pscale = None
    tau = float(prior_tau)
    if tau > 0.0 and prior_center_blocks is not None:
        center = prior_center_blocks.reshape(B, nb * 8).to(torch.float32).contiguous()
        if prior_scale_blocks is None:
            prior_scale_blocks = prior_scale_from_center(prior_center_blocks, prior_tau_scale_mode)
        pscale = prior_scale_blocks.reshape(B, nb).to(torch.float32).contiguous()
    else:
        tau = 0.0
    return r1, center, pscale, tau


@torch.inference_mode()
def vamp_vector_map_e8p12(*, r1_blocks, gamma1, cb, blocks_per_chunk: int = 64, need_stats: bool = False,
                          prior_center_blocks=None, prior_scale_blocks=None, prior_tau: float = 0.0,
                          prior_tau_scale_mode: str = "absmax") -> Dict[str, Any]:
    """mpq/priors/e8p12.py:541-631."""
    B, nb, _ = r1_blocks.shape
    r1, center, pscale, tau = _fold_args(r1_blocks, prior_center_blocks, prior_scale_blocks, prior_tau,
                                         prior_tau_scale_mode)
    g = gamma1.reshape(B).to(device=r1.device, dtype=torch.float32).contiguous()
    vals, idx = e8p12_map_rows(r1, cb, gamma=g, center=center, pscale=pscale, prior_tau=tau)
    out: Dict[str, Any] = {"map_idxs": idx.to(torch.int64), "map_vals": vals.reshape(B, nb, 8)}
    if need_stats:
        out["margin"] = 0.0
    return out


@torch.inference_mode()
def vamp_vector_discrete_mmse_e8p12(*, r1_blocks, gamma1, cb, blocks_per_chunk: int = 64, need_stats: bool = False,
                                    prior_center_blocks=None, prior_scale_blocks=None, prior_tau: float = 0.0,
                                    prior_tau_scale_mode: str = "absmax", compile_prior: bool = True,
                                    return_logZ_blocks: bool = False, return_margin_blocks: bool = False,
                                    return_entropy_blocks: bool = False) -> Dict[str, Any]:
    """mpq/priors/e8p12.py:815-968.  need_stats / return_*_blocks add the diagnostics (per-block log-partition,
    entropy and top-2 margin, and the means "entropy" / "margin" over the reference's item chunks) from the
    unpruned diagnostics kernel."""
    want_stats = bool(need_stats) or bool(return_margin_blocks) or bool(return_entropy_blocks)
    B, nb, _ = r1_blocks.shape
    r1, center, pscale, tau = _fold_args(r1_blocks, prior_center_blocks, prior_scale_blocks, prior_tau,
                                         prior_tau_scale_mode)
    dev = r1.device
    t = factor_tables(cb, dev)
    g = gamma1.reshape(B).to(device=dev, dtype=torch.float32).contiguous()
    x1 = torch.empty(B, nb * 8, device=dev, dtype=torch.float32)
    var1 = torch.empty(B, nb, device=dev, dtype=torch.float32)
    idx = torch.empty(B, nb, device=dev, dtype=torch.int32)
    mvals = torch.empty(B, nb * 8, device=dev, dtype=torch.float32)
    vsum = torch.empty(B, device=dev, dtype=torch.float32)
    call("mpq_e8p12_mmse", ptr(r1), r1.stride(0), ptr(center), center.stride(0) if center is not None else 0,
         ptr(pscale), pscale.stride(0) if pscale is not None else 0, ptr(g), float(tau), B, nb, *_tab_ptrs(t),
         ptr(x1), x1.stride(0), ptr(var1), var1.stride(0), ptr(idx), idx.stride(0), ptr(mvals), mvals.stride(0),
         ptr(vsum))
    alpha1 = gamma1.to(device=dev, dtype=torch.float32).reshape(B, 1) * (vsum / float(nb)).reshape(B, 1)
    out = {"x1_blocks": x1.reshape(B, nb, 8), "var1": var1, "map_idxs": idx.to(torch.int64),
           "map_vals": mvals.reshape(B, nb, 8), "alpha1": alpha1, "entropy": 0.0, "margin": 0.0}
    if want_stats or return_logZ_blocks:
        ps = posterior_stats(r1, g, cb, center=center, pscale=pscale, prior_tau=tau,
                             blocks_per_chunk=int(blocks_per_chunk), means=want_stats)
        if return_logZ_blocks:
            out["logZ_blocks"] = ps["logZ_blocks"]
        if return_margin_blocks:
            out["margin_blocks"] = ps["margin_blocks"]
        if return_entropy_blocks:
            out["entropy_blocks"] = ps["entropy_blocks"]
        if want_stats:
            out["entropy"], out["margin"] = ps["entropy"], ps["margin"]
    return out


def posterior_stats(r1: torch.Tensor, gamma: torch.Tensor, cb, *, center=None, pscale=None, prior_tau: float = 0.0,
                    blocks_per_chunk: int = 64, means: bool = True) -> Dict[str, Any]:
    """Posterior diagnostics of a (B, n) message under the folded prior (mpq/priors/e8p12.py:292-306, :945-960):
    logZ_blocks, entropy_blocks, margin_blocks (B x nb) and, with means, the means "entropy" / "margin" as the
    reference forms them (per item chunk, then over the chunks)."""
    B, n = r1.shape
    nb = n // 8
    dev = r1.device
    t = factor_tables(cb, dev)
    r1 = r1.to(torch.float32).contiguous()
    g = gamma.reshape(B).to(device=dev, dtype=torch.float32).contiguous()
    tau = float(prior_tau) if center is not None else 0.0
    logz = torch.empty(B, nb, device=dev, dtype=torch.float32)
    ent = torch.empty_like(logz)
    mar = torch.empty_like(logz)
    call("mpq_e8p12_stats", ptr(r1), r1.stride(0), ptr(center), center.stride(0) if center is not None else 0,
         ptr(pscale), pscale.stride(0) if pscale is not None else 0, ptr(g), tau, B, nb, *_tab_ptrs(t),
         ptr(logz), ptr(ent), ptr(mar), nb)
    out: Dict[str, Any] = {"logZ_blocks": logz, "entropy_blocks": ent, "margin_blocks": mar}
    if means:
        bpc = _stats_chunk_blocks(B, nb, int(blocks_per_chunk), dev)
        ents = [ent[:, c:c + bpc].mean() for c in range(0, nb, bpc)]
        mars = [mar[:, c:c + bpc].mean() for c in range(0, nb, bpc)]
        vals = torch.stack(ents + mars).double().cpu().tolist()
        k = len(ents)
        out["entropy"] = float(sum(vals[:k]) / k)
        out["margin"] = float(sum(vals[k:]) / k)
    return out


def _stats_chunk_blocks(B: int, nb: int, requested: int, dev: torch.device) -> int:
    """Blocks per item chunk of the reference's posterior loop (mpq/priors/e8p12.py:67-80, CUDA branch)."""
    requested = max(int(requested or 1), 1)
    if nb <= requested:
        return nb
    total = int(torch.cuda.get_device_properties(dev).total_memory)
    budget = min(max(total // 8, 256 * 1024 ** 2), 4 * 1024 ** 3)
    auto = max(1, int(budget // max(B * 256 * 4 * 48, 1)))
    return int(min(nb, max(requested, auto)))


class GramLayer:
    """Per-layer operands of the gram-metric CD, shared by every row block of a layer: the 8x8 block metadata
    (grams, Cholesky factors, inverses; mpq_gram_meta) and the cross-block grams Vs Vs^T."""

    def __init__(self, Vs: torch.Tensor, opVs: Optional[ops.Operand] = None, opVsT: Optional[ops.Operand] = None):
        dev = Vs.device
        self.Vs = Vs.to(torch.float32).contiguous()
        n, R = self.Vs.shape
        nb = n // 8
        self.opVs = opVs or ops.Operand(self.Vs)
        self.opVsT = opVsT or ops.Operand(self.Vs.t().contiguous())
        self.meta = torch.empty(nb, 196, device=dev, dtype=torch.float32)
        self.fails = torch.zeros(1, device=dev, dtype=torch.int32)
        self.Hf = torch.empty(n, n, device=dev, dtype=torch.float32)
        self.refresh()

    def refresh(self) -> None:
        """Recompute the metadata in place from self.Vs (after its values changed)."""
        n, R = self.Vs.shape
        self.fails.zero_()
        call("mpq_gram_meta", ptr(self.Vs), self.Vs.stride(0), R, n // 8, ptr(self.meta), ptr(self.fails))
        ops.mm_nt(self.Vs, self.opVs, self.Hf)  # Vs Vs^T: cross-block grams


@torch.inference_mode()
def gram_block_cd(*, x: torch.Tensor, Y_u: torch.Tensor, Vs: torch.Tensor, cb, sweeps: int,
                  idxs_init: torch.Tensor, accept_tol: float = 0.0, opVs: Optional[ops.Operand] = None,
                  opVsT: Optional[ops.Operand] = None, on_sweep=None, topk_vals: Optional[torch.Tensor] = None,
                  topk_idx: Optional[torch.Tensor] = None, layer: Optional[GramLayer] = None,
                  deferred: bool = False) -> Tuple[torch.Tensor, torch.Tensor, Dict[str, Any]]:
    """Gram-metric greedy block CD over E8P12 8-blocks (mpq/polish/block_cd.py:332-625, E8P12Provider, metric
    'gram').  Returns (x, idxs int64 (B, nb), stats).  on_sweep(sweep, x, idx, res_norm, accepted_total) is
    called before the first sweep (sweep 0) and after each sweep.  With ``topk_vals`` (B, nb, k, 8) and
    ``topk_idx`` (B, nb, k) every block decision picks among the block's k candidates (E8P12TopKProvider,
    _topk_gram_step_impl :137-172) instead of searching the full grid.  ``layer`` carries the per-layer
    metadata when several row blocks of one layer are polished.  ``deferred``: no host synchronisation --
    the stats hold device tensors (``finish_gram_stats`` converts them once the work has completed)."""
    dev = x.device
    B, n = x.shape
    nb = n // 8
    R = int(Vs.shape[1])
    t = factor_tables(cb, dev)
    if layer is None:
        layer = GramLayer(Vs, opVs, opVsT)
    Vs, opVs, opVsT, meta, fails, Hf = layer.Vs, layer.opVs, layer.opVsT, layer.meta, layer.fails, layer.Hf
    x_work = x.to(torch.float32).clone()
    idx = idxs_init.to(device=dev, dtype=torch.int32).contiguous().clone()
    res_u = ops.mm_nt(x_work, opVsT)
    res_norm = torch.empty(B, device=dev, dtype=torch.float32)
    call("mpq_residual", ptr(Y_u), ptr(res_u), B, R, res_u.stride(0), ptr(res_norm))
    gain = torch.empty(nb, device=dev, dtype=torch.float32)
    order = torch.empty(nb, device=dev, dtype=torch.int32)
    VsJ = torch.empty(128, R, device=dev, dtype=torch.float32)
    VsJT = torch.empty(R, 128, device=dev, dtype=torch.float32)
    # the chunk's rows of Vs come pre-split from the layer's split of Vs (no split per chunk)
    vs16 = opVs.f16 if (opVs is not None and opVs.f16 is not None and ops.gemm_precision() == "f16x3") else None
    topk_vals_given = topk_vals is not None
    if vs16 is not None:
        hiJ = torch.empty(128, vs16[0].shape[1], device=dev, dtype=torch.float16)
        loJ = torch.empty_like(hiJ)
        invJ = torch.empty(128, device=dev, dtype=torch.float32)
        # Per chunk: the gather writes the split of VsJT and the chunk kernel the split of delta and sums the rhs
        # product's split-K planes, so the chunk's two products take their operands as they are (the same splits
        # and sums that mm_nt's split and reduction launches would produce, bit for bit).
        dhi = torch.empty(B, 128, device=dev, dtype=torch.float16)
        dlo = torch.empty_like(dhi)
        dinv = torch.empty(B, device=dev, dtype=torch.float32)
        ld16 = (R + 7) // 8 * 8
        rhi = torch.empty(B, ld16, device=dev, dtype=torch.float16)
        rlo = torch.empty_like(rhi)
        rinv = torch.empty(B, device=dev, dtype=torch.float32)
        rsplits = ops.splitk_for(B, 128, R, ops.num_sms(dev)) if B else 1
        planes = torch.empty(max(rsplits, 1) * B * 128, device=dev, dtype=torch.float32)
        st_word = ops.status_word(dev)
        if not topk_vals_given:
            # The block order is fixed for a whole sweep, so one launch per sweep gathers every chunk's operands
            # (chunk-major slices of these buffers: Vs rows' split, VsJT's split, Hsub) instead of one small
            # launch per chunk.
            nch = (nb + 15) // 16
            hiJa = torch.empty(nch, 128, hiJ.shape[1], device=dev, dtype=torch.float16)
            loJa = torch.empty_like(hiJa)
            invJa = torch.empty(nch, 128, device=dev, dtype=torch.float32)
            hiTa = torch.empty(nch, R, 128, device=dev, dtype=torch.float16)
            loTa = torch.empty_like(hiTa)
            invTa = torch.empty(nch, R, device=dev, dtype=torch.float32)
            Hsuba = torch.empty(nch, 128, 128, device=dev, dtype=torch.float32)
    Hsub = torch.empty(128, 128, device=dev, dtype=torch.float32)
    rhsJ = torch.empty(B, 128, device=dev, dtype=torch.float32)
    delta = torch.empty(B, 128, device=dev, dtype=torch.float32)
    accepted = torch.zeros(1, device=dev, dtype=torch.int32)
    evals = torch.zeros(1, device=dev, dtype=torch.int64)
    n_cand = 0
    if topk_vals is not None:
        topk_vals = topk_vals.to(device=dev, dtype=torch.float32).contiguous()
        topk_idx = topk_idx.to(device=dev, dtype=torch.int32).contiguous()
        n_cand = int(topk_idx.shape[2])
        if tuple(topk_vals.shape) != (B, nb, n_cand, 8) or tuple(topk_idx.shape) != (B, nb, n_cand):
            raise ValueError(f"top-k candidates must be (B, nb, k, 8) / (B, nb, k); got {tuple(topk_vals.shape)}, "
                             f"{tuple(topk_idx.shape)}")
    trace_dev = torch.empty(max(int(sweeps), 0) + 1, device=dev, dtype=torch.float64)
    trace_dev[0:1].copy_(res_norm.double().mean().reshape(1))
    if on_sweep is not None:
        on_sweep(0, x_work, idx, res_norm, 0)
    for sweep in range(1, max(int(sweeps), 0) + 1):
        rhs_all = ops.mm_nt(res_u, opVs)
        call("mpq_gram_gain", ptr(rhs_all), rhs_all.stride(0), B, nb, ptr(meta), ptr(gain))
        del rhs_all
        call("mpq_argsort_desc", ptr(gain), nb, ptr(order))
        fused = vs16 is not None and not n_cand
        if fused:
            call("mpq_gram_gather_sweep", ptr(Vs), Vs.stride(0), R, ptr(Hf), Hf.stride(0), ptr(order), nb,
                 ptr(vs16[0]), ptr(vs16[1]), vs16[0].stride(0), ptr(vs16[2]), ptr(hiJa), ptr(loJa), hiJa.stride(1),
                 ptr(invJa), ptr(Hsuba), ptr(hiTa), ptr(loTa), hiTa.stride(1), ptr(invTa))
        for c0 in range(0, nb, 16):
            Kb = min(16, nb - c0)
            kc = 8 * Kb
            if fused:
                ci = c0 // 16
                hJ, lJ, iJ, hT, lT, iT = hiJa[ci], loJa[ci], invJa[ci], hiTa[ci], loTa[ci], invTa[ci]
                ops.split_f16(res_u, (rhi, rlo, rinv))
                spl = min(ops.splitk_for(B, kc, R, ops.num_sms(dev)), rsplits) if B else 1
                call("mpq_gemm_f16x3_parts", B, kc, R, ptr(rhi), ptr(rlo), rhi.stride(0), ptr(rinv), ptr(hJ),
                     ptr(lJ), hJ.stride(0), ptr(iJ), spl, ptr(planes), planes.numel(), ptr(st_word))
                call("mpq_gram_chunk_planes", ptr(x_work), x_work.stride(0), ptr(planes), kc, spl, B * kc,
                     ptr(Hsuba[ci]), ptr(meta), ptr(order), c0, Kb, ptr(t["base_abs"]), ptr(t["base_parity"]),
                     ptr(t["grid"]), ptr(t["sign_id"]), ptr(res_norm), ptr(idx), idx.stride(0), ptr(delta), ptr(dhi),
                     ptr(dlo), dhi.stride(0), ptr(dinv), ptr(accepted), ptr(evals), B, float(accept_tol))
                ops.mm_nt(ops.Operand.presplit(delta[:, :kc], (dhi[:, :kc], dlo[:, :kc], dinv)),
                          ops.Operand.presplit(VsJT[:, :kc], (hT[:, :kc], lT[:, :kc], iT)),
                          out=res_u, alpha=-1.0, beta=1.0)
                continue
            if vs16 is not None:
                call("mpq_gram_gather_split", ptr(Vs), Vs.stride(0), R, ptr(Hf), Hf.stride(0), ptr(order), c0, Kb,
                     ptr(vs16[0]), ptr(vs16[1]), vs16[0].stride(0), ptr(vs16[2]), ptr(hiJ), ptr(loJ), hiJ.stride(0),
                     ptr(invJ), ptr(VsJT), ptr(Hsub), None, None, 0, None)
                ops.mm_nt(res_u, ops.Operand.presplit(VsJ[:kc], (hiJ[:kc], loJ[:kc], invJ[:kc])), out=rhsJ[:, :kc])
            else:
                call("mpq_gram_gather", ptr(Vs), Vs.stride(0), R, ptr(Hf), Hf.stride(0), ptr(order), c0, Kb, ptr(VsJ),
                     ptr(VsJT), ptr(Hsub))
                ops.mm_nt(res_u, VsJ[:kc], out=rhsJ[:, :kc])
            if n_cand:
                call("mpq_gram_chunk_topk", ptr(x_work), x_work.stride(0), ptr(rhsJ), rhsJ.stride(0), ptr(Hsub),
                     ptr(meta), ptr(order), c0, Kb, ptr(topk_vals), ptr(topk_idx), n_cand, nb, ptr(res_norm), ptr(idx),
                     idx.stride(0), ptr(delta), ptr(accepted), ptr(evals), B, float(accept_tol))
            else:
                call("mpq_gram_chunk", ptr(x_work), x_work.stride(0), ptr(rhsJ), rhsJ.stride(0), ptr(Hsub), ptr(meta),
                     ptr(order), c0, Kb, ptr(t["base_abs"]), ptr(t["base_parity"]), ptr(t["grid"]), ptr(t["sign_id"]),
                     ptr(res_norm), ptr(idx), idx.stride(0), ptr(delta), ptr(accepted), ptr(evals), B,
                     float(accept_tol))
            ops.mm_nt(delta[:, :kc], VsJT[:, :kc], out=res_u, alpha=-1.0, beta=1.0)
        trace_dev[sweep:sweep + 1].copy_(res_norm.double().mean().reshape(1))
        if on_sweep is not None:
            on_sweep(sweep, x_work, idx, res_norm, int(accepted.item()))
    st = {"accepted_updates": accepted, "exact_score_evals": evals, "stabilized_objective_trace": trace_dev,
          "_fails": fails}
    if deferred:
        return x_work, idx.to(torch.int64), st
    return x_work, idx.to(torch.int64), finish_gram_stats(st)


def finish_gram_stats(st: Dict[str, Any]) -> Dict[str, Any]:
    """Host values of a deferred gram_block_cd's stats (synchronises with the work that produced them)."""
    if int(st["_fails"].item()):
        raise RuntimeError("stabilize_cholesky failed for an E8P12 block gram")
    trace = [float(v) for v in st["stabilized_objective_trace"].cpu().tolist()]
    nonincreasing = all(b <= a + max(1e-8, abs(a) * 1e-7) for a, b in zip(trace, trace[1:]))
    return {"accepted_updates": float(st["accepted_updates"].item()), "exact_score_evals": int(st["exact_score_evals"].item()),
            "stabilized_objective_trace": trace, "stabilized_objective_nonincreasing": bool(nonincreasing)}


@torch.inference_mode()
def gram_search(targets: torch.Tensor, chol: torch.Tensor, cb, lam_bounds: Optional[Tuple[float, float]] = None
                ) -> torch.Tensor:
    """Exact first-minimum gram-metric search of N targets (N, 8) under one lower Cholesky factor (8, 8)."""
    dev = targets.device
    t = factor_tables(cb, dev)
    L = chol.to(device=dev, dtype=torch.float32).contiguous()
    if lam_bounds is None:
        S = (L.double() @ L.double().T)
        ev = torch.linalg.eigvalsh(S.cpu())
        lam_bounds = (max(float(ev.min()) * (1 - 1e-6), 0.0), float(ev.max()) * (1 + 1e-6))
    tg = targets.to(torch.float32).contiguous()
    out = torch.empty(tg.shape[0], device=dev, dtype=torch.int32)
    call("mpq_gram_search", ptr(tg), tg.shape[0], ptr(L), float(lam_bounds[0]), float(lam_bounds[1]),
         ptr(t["base_abs"]), ptr(t["base_parity"]), ptr(t["grid"]), ptr(t["sign_id"]), ptr(out))
    return out.to(torch.int64)
