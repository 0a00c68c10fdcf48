"""Per-linear E8P12 driver (the QUIP# hook point).

Reference: mpq/adapters/quip_sharp.py:396-878 (mpq_refine_codebook), :33-67 (_vamp_hessian_eigen, fp64),
:97-122 (exact surrogate audits), :190-262 (initializations), :370-393 (_build_vamp_cfg).

The default recipe (solver 'vamp', polish 'block_cd' with the gram metric) runs on the CUDA path; the
comparison solvers (ldlq/cdquant/quantease/ojbkq) and top-k polish raise ``ValueError``.
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional, Tuple

import torch

from .. import ops
from .._lib import call, ptr
from ..e8p12 import e8p12_nearest
from ..rotation import stable_seed
from ..chain import chain_supported, e8p12_layer_chain
from ..solver import E8P12VampConfig, solve_e8p12_rankspace_vamp
from .gptqmodel import vamp_hessian_eigen


@dataclass(frozen=True)
class QuipAdapterConfig:
    block_rows: int = 128
    jitter_base: float = 1e-6
    eigen_floor_scale: float = 1e-6


def _build_vamp_cfg(args: Any, *, polish_mode: str) -> E8P12VampConfig:
    """mpq/adapters/quip_sharp.py:370-393."""
    g = lambda k, d: getattr(args, k, d)
    return E8P12VampConfig(
        iters=int(g("mpq_iters", 16)), damping=float(g("mpq_damping", 0.5)),
        gamma_start=float(g("mpq_gamma_start", 1.0)), gamma_retry_factor=float(g("mpq_gamma_retry_factor", 4.0)),
        gamma_retry_steps=int(g("mpq_gamma_retry_steps", 3)), prior_tau=float(g("mpq_prior_tau", 0.25)),
        prior_tau_scale_mode=str(g("mpq_prior_tau_scale_mode", "absmax")),
        compile_prior=bool(g("mpq_compile_prior", True)), obs_precision=float(g("mpq_obs_precision", 0.0)),
        em_obs_precision=bool(g("mpq_em_obs_precision", True)),
        em_obs_precision_damping=float(g("mpq_em_obs_precision_damping", 0.3)),
        em_obs_precision_min=float(g("mpq_em_obs_precision_min", 1e-4)),
        em_obs_precision_max=float(g("mpq_em_obs_precision_max", 1e8)),
        blocks_per_chunk=int(g("mpq_blocks_per_chunk", 16)), polish_sweeps=int(g("mpq_polish_sweeps", 3)),
        polish_mode=str(polish_mode), polish_metric=str(g("mpq_polish_metric", "gram")),
        polish_metric_rows_per_chunk=int(g("mpq_metric_rows_per_chunk", 0)),
        polish_max_blocks=int(g("mpq_polish_max_blocks", 0)),
        topk_k=int(g("mpq_topk_k", g("quant_topk_k", 16)) or 16), best_iterate=bool(g("mpq_best_iterate", False)))


def _resolve_solver(args: Any) -> Tuple[str, str]:
    """Solver and polish mode of the recipe (mpq/adapters/quip_sharp.py:339-367)."""
    solver = getattr(args, "quant_solver", None) or getattr(args, "mpq_solver", None)
    if solver is not None:
        polish = str(getattr(args, "quant_polish_mode", getattr(args, "mpq_polish_mode", "none")) or "none")
        return str(solver).strip().lower(), polish.strip().lower()
    legacy = str(getattr(args, "mpq_method", "vamp") or "vamp").strip().lower()
    polish = "topk_block_cd" if legacy == "vamp-topk-polish" else "block_cd"
    if int(getattr(args, "mpq_polish_sweeps", 3) or 0) <= 0:
        polish = "none"
    return "vamp", polish


class _Surrogate:
    """Row-chunked exact surrogate (W - hat) H (W - hat)^T (mpq/adapters/quip_sharp.py:70-117)."""

    def __init__(self, H: torch.Tensor):
        self.op = ops.Operand(H.t().contiguous())

    def rows(self, W: torch.Tensor, hat: torch.Tensor) -> torch.Tensor:
        d = torch.empty_like(W)
        call("mpq_sub", ptr(W), ptr(hat), ptr(d), W.shape[0], W.shape[1], d.stride(0))
        dH = ops.mm_nt(d, self.op)
        out = torch.empty(W.shape[0], device=W.device, dtype=torch.float32)
        call("mpq_row_dot", ptr(dH), dH.stride(0), ptr(d), d.stride(0), W.shape[0], W.shape[1], ptr(out))
        return out

    def chunk_means_dev(self, W, hat, block_rows) -> torch.Tensor:
        """chunk_means without the read-back: float64 device tensor [chunk means..., overall mean]."""
        m = W.shape[0]
        if m == 0:
            return torch.zeros(1, device=W.device, dtype=torch.float64)
        s = self.rows(W, hat).double()
        nfull = m // block_rows
        parts = [s[:nfull * block_rows].reshape(nfull, block_rows).mean(1)] if nfull else []
        if m % block_rows:
            parts.append(s[nfull * block_rows:].mean().reshape(1))
        return torch.cat(parts + [s.mean().reshape(1)])

    def chunk_means(self, W, hat, block_rows) -> Tuple[float, List[float]]:
        """Per-row surrogates of all rows in one product (rows are independent), then the means of the block_rows
        chunks and of all rows, read back together."""
        m = W.shape[0]
        if m == 0:
            return 0.0, []
        s = self.rows(W, hat).double()
        nfull = m // block_rows
        parts = [s[:nfull * block_rows].reshape(nfull, block_rows).mean(1)] if nfull else []
        if m % block_rows:
            parts.append(s[nfull * block_rows:].mean().reshape(1))
        means = torch.cat(parts + [s.mean().reshape(1)]).cpu().tolist()
        return float(means[-1]), [float(v) for v in means[:-1]]


@torch.inference_mode()
def mpq_refine_codebook(
    Wr: torch.Tensor,
    Hr: torch.Tensor,
    hatWr0: torch.Tensor,
    Qidxs0: torch.Tensor,
    cb: Any,
    args: Any,
    *,
    module_name: str = "",
    adapter_cfg: QuipAdapterConfig = QuipAdapterConfig(),
    eigen: Optional[Tuple[torch.Tensor, torch.Tensor, float]] = None,
    after_enqueue: Optional[Callable[[], None]] = None,
) -> Tuple[torch.Tensor, torch.Tensor, Dict[str, Any]]:
    """QUIP# adapter: refine codebook decisions with VAMP + greedy gram-metric polish.

    eigen: (lam, V, floor) of vamp_hessian_eigen(Hr, fp64=True) with this adapter_cfg's jitter and floor, computed
    ahead (by mpq_b200.pipeline while the previous layer was solved, or on another rank); None computes it here, as
    the reference does.  after_enqueue: called once the solve's device work is enqueued (the chained path) or
    before it starts (the block-by-block path).

    Returns (hatWr (m, n), Qidxs int64 (m, n/8), stats)."""
    start = time.time()
    if not Wr.is_cuda:
        raise ValueError("mpq_refine_codebook requires CUDA tensors (there is no CPU path)")
    device = Wr.device
    Wr = Wr.to(torch.float32).contiguous()
    Hr = Hr.to(device=device, dtype=torch.float32).contiguous()
    m, n = Wr.shape
    if int(getattr(cb, "codesz", 8)) != 8 or n % 8 != 0:
        raise ValueError(f"mpq QUIP adapter expects E8P12 codesz=8; got n={n}.")
    nb = n // 8
    solver, polish_mode = _resolve_solver(args)
    if solver != "vamp":
        raise ValueError(f"QUIP adapter solver {solver!r} is not on the CUDA path (only 'vamp').")
    if polish_mode in ("topk_cd", "topk", "vamp_topk"):
        polish_mode = "topk_block_cd"
    if polish_mode not in ("block_cd", "topk_block_cd", "none"):
        raise ValueError(f"QUIP adapter polish {polish_mode!r} is not on the CUDA path.")
    init_mode = str(getattr(args, "mpq_init", "rtn") or "rtn").strip().lower()
    seed = int(getattr(args, "seed", getattr(args, "mpq_seed", 0)) or 0)
    if init_mode == "rtn":
        v, i = e8p12_nearest(Wr.reshape(-1, 8), cb)
        hat_init, idx_init = v.reshape(m, n), i.reshape(m, nb)
    elif init_mode in ("float", "paper", "unquantized"):
        _, i = e8p12_nearest(Wr.reshape(-1, 8), cb)
        hat_init, idx_init = Wr.clone(), i.reshape(m, nb)
    elif init_mode == "zero":
        _, i = e8p12_nearest(torch.zeros(m * nb, 8, device=device), cb)
        hat_init, idx_init = torch.zeros_like(Wr), i.reshape(m, nb)
    elif init_mode == "ldlq":
        hat_init = hatWr0.to(device=device, dtype=torch.float32).clone()
        idx_init = Qidxs0.to(device=device, dtype=torch.int64).clone()
    elif init_mode == "random":
        gen = torch.Generator(device="cpu")
        gen.manual_seed(stable_seed(f"{module_name}:mpq_init", base_seed=seed))
        idx_init = torch.randint(0, int(cb.grid.shape[0]), (m, nb), generator=gen, dtype=torch.int64).to(device)
        hat_init = cb.grid.to(device=device, dtype=torch.float32).index_select(0, idx_init.reshape(-1)).reshape(m, n)
    else:
        raise ValueError(f"unknown mpq_init={init_mode!r} (expected 'float', 'random', 'rtn', 'zero', or 'ldlq').")

    if eigen is None:
        eigen = vamp_hessian_eigen(Hr, jitter_base=adapter_cfg.jitter_base, floor_scale=adapter_cfg.eigen_floor_scale,
                                   fp64=True)
    lam, V, eigen_floor = eigen
    if lam.shape != (n,) or V.shape != (n, n) or lam.device != device or V.device != device:
        raise ValueError(f"eigen: expected lam ({n},) and V ({n}, {n}) on {device}; got {tuple(lam.shape)} and "
                         f"{tuple(V.shape)}")
    V = V.contiguous()
    Vh = V.T.contiguous()
    S = torch.sqrt(lam).contiguous()
    Vs = (V * S.unsqueeze(0)).contiguous()
    R = int(S.numel())
    block_rows = min(m, max(int(getattr(args, "mpq_block_rows", adapter_cfg.block_rows) or adapter_cfg.block_rows), 1))
    opVsT = ops.Operand(Vs.T.contiguous())
    requested_obs = float(getattr(args, "mpq_obs_precision", 0.0) or 0.0)
    if requested_obs > 0.0:
        obs_precision = requested_obs
    else:
        # (:520-535) the mean squared rank-space RTN error over all rows; rows are independent, so one product
        d = torch.empty_like(Wr)
        call("mpq_sub", ptr(Wr), ptr(hat_init), ptr(d), m, n, d.stride(0))
        du = ops.mm_nt(d, opVsT)
        zeros = torch.zeros_like(du)
        e = torch.empty(m, device=device, dtype=torch.float32)
        call("mpq_row_sqerr", ptr(du), ptr(zeros), m, R, du.stride(0), zeros.stride(0), ptr(e))
        # kept on the device (float64, the reference's Python float arithmetic): read back with the statistics
        obs_precision = 1.0 / torch.clamp(e.double().sum() / float(max(m * R, 1)), min=1e-12)
    vamp_cfg = _build_vamp_cfg(args, polish_mode=polish_mode)
    sur = _Surrogate(Hr)
    # the surrogate audits (:97-122) stay on the device until the end: one read-back per layer
    ldlq_t = sur.chunk_means_dev(Wr, hatWr0.to(device=device, dtype=torch.float32).contiguous(), block_rows)
    final_hat = hat_init.clone()
    final_idx = idx_init.clone()
    before_t = sur.chunk_means_dev(Wr, hat_init, block_rows)
    obs_block = obs_precision
    gamma_sum, gamma_count, changed, changed_total = 0.0, 0, 0, 0
    stats_chunk: Dict[str, Any] = {}
    if chain_supported(vamp_cfg):
        # the serial chain of row blocks on the device (VAMP chain on one stream, polish overlapped on others)
        final_hat, final_idx, per_block = e8p12_layer_chain(
            Wr=Wr, hat_init=hat_init, cb=cb, V=V, Vh=Vh, S=S, Vs=Vs, cfg=vamp_cfg, block_rows=block_rows,
            obs_init=obs_precision, after_enqueue=after_enqueue)
        for bst in per_block:
            gamma_sum += bst.pop("_gamma1_sum")
            gamma_count += bst.pop("_gamma1_count")
            bst.pop("_gamma1_min")
            bst.pop("_gamma1_max")
            changed += bst.pop("_changed_count")
            changed_total += bst.pop("_changed_total")
            bst["module"] = str(module_name)
        stats_chunk = per_block[-1] if per_block else {}
        if bool(vamp_cfg.em_obs_precision) and float(vamp_cfg.obs_precision) <= 0.0 and per_block:
            obs_block = float(per_block[-1]["obs_precision_final"])
    else:
        if after_enqueue is not None:
            after_enqueue()
        for r0 in range(0, m, block_rows):
            rb = slice(r0, min(r0 + block_rows, m))
            dbg: Dict[str, Any] = {"summary_only": True}
            hat_c, idx_c, _err, stats_chunk = solve_e8p12_rankspace_vamp(
                Wr=Wr[rb], hatWr_init=final_hat[rb], cb=cb, V=V, Vh=Vh, S=S, Vs=Vs, cfg=vamp_cfg,
                module_name=module_name, obs_precision_init=float(obs_block), log_stats=False, debug_out=dbg)
            final_hat[rb] = hat_c
            final_idx[rb] = idx_c
            if bool(vamp_cfg.em_obs_precision) and float(vamp_cfg.obs_precision) <= 0.0:
                obs_block = float(stats_chunk.get("obs_precision_final", obs_block))
            gamma_sum += float(dbg.get("gamma1_sum", 0.0))
            gamma_count += int(dbg.get("gamma1_count", 0))
            changed += int(dbg.get("changed_count", 0))
            changed_total += int(dbg.get("changed_total", 0))
    after_t = sur.chunk_means_dev(Wr, final_hat, block_rows)
    k = int(ldlq_t.numel())
    host = torch.cat([ldlq_t, before_t, after_t, torch.as_tensor(obs_precision, device=device,
                                                                 dtype=torch.float64).reshape(1)]).cpu().tolist()
    split = lambda v: (float(v[-1]), [float(x) for x in v[:-1]])
    exact_ldlq, exact_ldlq_chunks = split(host[:k])
    exact_before, exact_before_chunks = split(host[k:2 * k])
    exact_after, exact_after_chunks = split(host[2 * k:3 * k])
    obs_precision = float(host[-1])
    if not torch.is_tensor(obs_block):
        obs_block = float(obs_block)
    else:
        obs_block = obs_precision
    violations, max_delta, max_ratio = 0, 0.0, 0.0
    for ld, mp in zip(exact_ldlq_chunks, exact_after_chunks):
        if mp > ld + 1e-8:
            violations += 1
            max_delta = max(max_delta, mp - ld)
            if ld > 0:
                max_ratio = max(max_ratio, mp / ld)
    stats: Dict[str, Any] = {
        "method": "mpq", "backend": "quip", "solver": solver, "polish_mode": polish_mode,
        "module": str(module_name), "init_mode": init_mode, "seed": seed, "m": m, "n": n, "rank": R,
        "eigen_floor": float(eigen_floor), "obs_precision_initial": float(obs_precision),
        "obs_precision_final": float(obs_block), "block_rows": int(block_rows),
        "exact_surrogate_ldlq_mean": float(exact_ldlq), "exact_surrogate_ldlq_chunk_means": exact_ldlq_chunks,
        "exact_surrogate_before_mean": float(exact_before), "exact_surrogate_before_chunk_means": exact_before_chunks,
        "exact_surrogate_after_mean": float(exact_after), "exact_surrogate_after_chunk_means": exact_after_chunks,
        "exact_surrogate_gain_mean": float(exact_before - exact_after),
        "surrogate_chunk_violation_count": int(violations), "surrogate_chunk_violation_max_delta": float(max_delta),
        "surrogate_chunk_violation_max_ratio": float(max_ratio), "solver_time_s": float(time.time() - start),
        "solver_stats": stats_chunk,
        "mechanism": {"regime": "2bit_e8p12", "cleanup_unit": "e8p12_block", "module": str(module_name),
                      "rows": m, "cols": n, "nblocks": nb,
                      "stage1_gamma1_mean": float(gamma_sum / max(gamma_count, 1)),
                      "cleanup_changed_count": int(changed), "cleanup_total_count": int(changed_total or m * nb),
                      "cleanup_changed_fraction": float(changed / max(changed_total or m * nb, 1))},
    }
    return final_hat.to(dtype=hatWr0.dtype if hatWr0 is not None else torch.float32), final_idx, stats
