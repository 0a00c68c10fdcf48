"""numpy restatement of the grouped-scalar (uniform grid) VAMP solve + scalar greedy CD.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

All arithmetic is float32 and follows the operation order of the reference's eager
torch code so that discrete decisions (codes, argmax) agree bit-for-bit on the
standalone rounding steps.  Host scalars (observation precision, EM, best-iterate
means) are Python floats (float64), as in the reference.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Dict, Optional, Tuple

import numpy as np

f32 = np.float32
ALPHA_EPS = 1e-7


# ---------------------------------------------------------------------------
# small helpers (mpq/utils.py)
# ---------------------------------------------------------------------------

def log_damp_positive(prev: np.ndarray, new: np.ndarray, damping: float) -> np.ndarray:
    """mpq/utils.py:24-33 (tensor version, float32)."""
    damping = float(damping)
    if damping >= 1.0:
        return new
    if damping <= 0.0:
        return prev
    prev = np.maximum(prev, f32(1e-12))
    new = np.maximum(new, f32(1e-12))
    lp = np.log(prev.astype(np.float64)).astype(f32)  # correctly rounded float32 log/exp, as torch's CPU kernels
    ln = np.log(new.astype(np.float64)).astype(f32)
    return np.exp((f32(1.0 - damping) * lp + f32(damping) * ln).astype(np.float64)).astype(f32)


def log_damp_positive_scalar(prev: float, new: float, damping: float) -> float:
    """mpq/utils.py:36-45 (host float64)."""
    damping = float(damping)
    if damping >= 1.0:
        return float(new)
    if damping <= 0.0:
        return float(prev)
    prev = max(float(prev), 1e-12)
    new = max(float(new), 1e-12)
    return float(math.exp((1.0 - damping) * math.log(prev) + damping * math.log(new)))


def alpha_valid_mask(alpha: np.ndarray, eps: float = ALPHA_EPS) -> np.ndarray:
    """mpq/utils.py:52-53."""
    return np.isfinite(alpha) & (alpha > f32(eps)) & (alpha < f32(1.0 - eps))


def precision_valid_mask(gamma: np.ndarray, eps: float = 1e-12) -> np.ndarray:
    """mpq/utils.py:56-57."""
    return np.isfinite(gamma) & (gamma > f32(eps))


def nan_to_num(x: np.ndarray, nan: float, posinf: float, neginf: float) -> np.ndarray:
    return np.nan_to_num(x, nan=f32(nan), posinf=f32(posinf), neginf=f32(neginf)).astype(f32)


# ---------------------------------------------------------------------------
# priors (mpq/priors/uniform.py)
# ---------------------------------------------------------------------------

def make_atoms(scale_full: np.ndarray, zero_full: np.ndarray, maxq: int) -> np.ndarray:
    """mpq/solver.py:468-470 / mpq/priors/uniform.py:140-144: atoms = s * (q - z)."""
    cand = np.arange(maxq + 1, dtype=f32).reshape(1, 1, -1)
    return (scale_full[..., None] * (cand - zero_full[..., None])).astype(f32)


def uniform_scores(r1, gamma1, scale_full, prior_center, prior_tau, atoms) -> np.ndarray:
    """Per-atom log-scores, mpq/priors/uniform.py:177-180 operation order."""
    d = atoms - r1[..., None]
    scores = (f32(-0.5) * gamma1[..., None]) * (d * d)
    if float(prior_tau) > 0.0:
        st = f32(prior_tau) * np.maximum(scale_full, f32(1e-12))
        scaled_tau2 = (st * st)[..., None]
        e = atoms - prior_center[..., None]
        scores = scores - (f32(0.5) * (e * e)) / scaled_tau2
    return scores.astype(f32)


def discrete_uniform_mmse(*, r1, gamma1, scale_full, zero_full, maxq, prior_center, prior_tau,
                          atoms: Optional[np.ndarray] = None) -> Dict[str, Any]:
    """Exact discrete posterior per entry, mpq/priors/uniform.py:99-213 (eager path)."""
    if atoms is None:
        atoms = make_atoms(scale_full, zero_full, maxq)
    gamma1 = gamma1.astype(f32)
    scores = uniform_scores(r1, gamma1, scale_full, prior_center, prior_tau, atoms)
    m = scores.max(axis=-1, keepdims=True)
    # float64 evaluation rounded once: the correctly rounded float32 exp/log of torch's CPU kernels
    lse = m + np.log(np.exp((scores - m).astype(np.float64)).sum(axis=-1, keepdims=True).astype(f32).astype(np.float64)).astype(f32)
    probs = np.exp((scores - lse).astype(np.float64)).astype(f32)
    mean = (probs * atoms).sum(axis=-1)
    second = (probs * (atoms * atoms)).sum(axis=-1)
    var = np.maximum(second - mean * mean, f32(0.0))
    map_idx = scores.argmax(axis=-1)  # first max = lowest index on ties
    map_value = np.take_along_axis(atoms, map_idx[..., None], axis=-1)[..., 0]
    alpha1 = gamma1 * var.mean(axis=1, keepdims=True, dtype=f32)
    return {"mean": mean.astype(f32), "var": var.astype(f32), "map_value": map_value.astype(f32),
            "map_idx": map_idx.astype(np.int64), "alpha1": alpha1.astype(f32)}


def nearest_atom_idx(*, x, scale_full, zero_full, maxq) -> np.ndarray:
    """mpq/priors/uniform.py:287-299: q = clamp(round(x / max(s,1e-12) + z), 0, maxq)."""
    scale = np.maximum(scale_full.astype(f32), f32(1e-12))
    q = np.round(x.astype(f32) / scale + zero_full.astype(f32))
    return np.clip(q, 0, int(maxq)).astype(np.int32)


def dequant_from_q(*, q_int, scale_full, zero_full) -> np.ndarray:
    """mpq/priors/uniform.py:302-309."""
    return (scale_full.astype(f32) * (q_int.astype(f32) - zero_full.astype(f32))).astype(f32)


def uniform_hard_decision(*, x_mean, x_map, scale_full, zero_full, maxq, final_decision="map"):
    """mpq/solver.py:833-850."""
    src = x_map if final_decision == "map" else x_mean
    q = nearest_atom_idx(x=src, scale_full=scale_full, zero_full=zero_full, maxq=maxq)
    return q, dequant_from_q(q_int=q, scale_full=scale_full, zero_full=zero_full)


# ---------------------------------------------------------------------------
# linear module (mpq/linear.py)
# ---------------------------------------------------------------------------

def linear_mmse_exact(r2, gamma2, *, Y_u, V, Vh, S, obs_precision):
    """mpq/linear.py:10-56."""
    n = r2.shape[1]
    rank = S.size
    s = S[None, :].astype(f32)
    obs = f32(obs_precision)
    denom = obs * (s * s) + gamma2
    r2_v = r2 @ V
    residual_before = Y_u - r2_v * s
    coeff = (obs * s) / denom
    delta = (residual_before * coeff) @ Vh
    x2 = r2 + delta
    alpha2 = f32(1.0 - (float(rank) / float(n))) + (gamma2 / f32(n)) * (f32(1.0) / denom).sum(axis=1, keepdims=True, dtype=f32)
    residual_after = residual_before * (gamma2 / denom)
    return x2.astype(f32), alpha2.astype(f32), residual_after.astype(f32)


def em_update_obs_precision_rankspace(*, residual_u, gamma2, S, obs_precision, num_obs,
                                      damping=0.3, min_value=1e-4, max_value=1e8) -> float:
    """mpq/linear.py:59-82."""
    if S.size == 0 or num_obs <= 0:
        return float(obs_precision)
    s2 = (S * S)[None, :].astype(f32)
    trace_term = (s2 / (f32(obs_precision) * s2 + gamma2)).sum(axis=1, keepdims=True, dtype=f32)
    resid_term = (residual_u * residual_u).sum(axis=1, keepdims=True, dtype=f32)
    denom = max(float((resid_term + trace_term).mean(dtype=f32)), 1e-12)
    beta_new = float(num_obs / denom)
    beta_old = max(float(obs_precision), 1e-12)
    beta = log_damp_positive_scalar(beta_old, beta_new, damping)
    return float(min(max(beta, float(min_value)), float(max_value)))


def vamp_rankspace_error(*, Y_u, x, Vs) -> np.ndarray:
    """mpq/linear.py:85-94."""
    d = Y_u - x @ Vs
    return (d * d).sum(axis=1, dtype=f32).astype(f32)


def hessian_objective_mean(*, target, x, gram) -> float:
    """mpq/linear.py:97-118."""
    delta = (target - x).astype(f32)
    return float(((delta @ gram) * delta).sum(axis=1, dtype=f32).mean(dtype=f32))


# ---------------------------------------------------------------------------
# scalar greedy CD (mpq/polish/triton_scalar_cd.py torch twin, :164-307)
# ---------------------------------------------------------------------------

def uniform_scalar_diag_greedy_cd(*, x, Y_u, Vs, gram_full, scale, zero, maxq, sweeps, accept_tol=0.0):
    """Column-sequential greedy CD with raw-H rank-1 rhs updates.

    Follows the torch twin mpq/polish/triton_scalar_cd.py:188-307 (the arithmetic of the
    Triton kernel :28-110, with the twin's reciprocal-multiply target).
    Returns (x_polished, stats).
    """
    x_work = x.astype(f32).copy()
    Vs = Vs.astype(f32)
    gram = gram_full.astype(f32)
    scale = scale.astype(f32)
    zero = zero.astype(f32)
    residual_u = Y_u.astype(f32) - x_work @ Vs
    rhs_all = (residual_u @ np.ascontiguousarray(Vs.T)).astype(f32)
    residual_norm = (residual_u * residual_u).sum(axis=1, dtype=f32)
    diag = np.maximum((Vs * Vs).sum(axis=1, dtype=f32), f32(1e-12))
    diag_inv = (f32(1.0) / diag).astype(f32)
    accepted = 0
    B = x_work.shape[0]
    for _ in range(max(int(sweeps), 0)):
        gain = (rhs_all * rhs_all * diag_inv[None, :]).sum(axis=0, dtype=f32) / f32(max(B, 1))
        order = np.argsort(-gain, kind="stable")
        for col in order:
            rhs = rhs_all[:, col]
            x_col = x_work[:, col]
            scale_col = np.maximum(scale[:, col], f32(1e-12))
            zero_col = zero[:, col]
            diag_col = diag[col]
            target = x_col + rhs * diag_inv[col]
            q = np.clip(np.round(target / scale_col + zero_col), 0, int(maxq))
            xq = scale_col * (q.astype(f32) - zero_col)
            delta = xq - x_col
            cand_err = np.maximum(residual_norm + (delta * delta) * diag_col - (f32(2.0) * rhs) * delta, f32(0.0))
            accept = (cand_err + f32(1e-12)) < residual_norm * f32(1.0 + accept_tol)
            if not accept.any():
                continue
            x_work[:, col] = np.where(accept, xq, x_col)
            residual_norm = np.where(accept, cand_err, residual_norm).astype(f32)
            delta_m = np.where(accept, delta, f32(0.0)).astype(f32)
            accepted += int(accept.sum())
            rhs_all -= delta_m[:, None] * gram[col][None, :]
    return x_work, {"accepted_updates": float(accepted)}


def polish_uniform_gpu_semantics(*, x_init, Y_u, Vs, scale_full, zero_full, maxq, sweeps, gram_full):
    """mpq/solver.py:299-333: the CUDA dispatch of the uniform polish (raw-H greedy CD)."""
    x_pol, st = uniform_scalar_diag_greedy_cd(x=x_init, Y_u=Y_u, Vs=Vs, gram_full=gram_full,
                                              scale=scale_full, zero=zero_full, maxq=maxq, sweeps=sweeps)
    q = nearest_atom_idx(x=x_pol, scale_full=scale_full, zero_full=zero_full, maxq=maxq)
    x_out = dequant_from_q(q_int=q, scale_full=scale_full, zero_full=zero_full)
    err = vamp_rankspace_error(Y_u=Y_u, x=x_out, Vs=Vs)
    return q, x_out, err, st


# ---------------------------------------------------------------------------
# the scalar VAMP loop (mpq/solver.py:426-830)
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class UniformVampConfig:
    """mpq/solver.py:35-55 (fields used by the solve)."""
    iters: int = 10
    damping: float = 0.5
    final_decision: str = "map"
    init_from: str = "rtn"
    gamma_start: float = 1.0
    gamma_retry_factor: float = 4.0
    gamma_retry_steps: int = 3
    prior_tau: float = 0.2
    obs_precision: float = 0.0
    em_obs_precision: bool = True
    em_obs_precision_damping: float = 0.3
    em_obs_precision_min: float = 1e-4
    em_obs_precision_max: float = 1e8
    polish_sweeps: int = 3
    polish_mode: str = "block_cd"  # "block_cd" | "topk_block_cd"
    topk_k: int = 16


def solve_uniform_rankspace_vamp(*, W, x_rtn, scale_full, zero_full, maxq, V, Vh, S, Vs, cfg,
                                 gram_full=None, obs_precision_init=None, debug=None):
    """mpq/solver.py:426-830 with the CUDA polish dispatch (:299-333) when gram_full is given."""
    W = W.astype(f32)
    x_rtn = x_rtn.astype(f32)
    scale_full = scale_full.astype(f32)
    zero_full = zero_full.astype(f32)
    iters = max(int(cfg.iters), 0)
    damping = float(cfg.damping)
    prior_tau = float(cfg.prior_tau)
    B, n = W.shape
    rank = int(S.size)
    atoms = make_atoms(scale_full, zero_full, maxq)
    if cfg.init_from == "zero":
        r1 = np.zeros_like(W)
    elif cfg.init_from == "float":
        r1 = W.copy()
    else:
        r1 = x_rtn.copy()
    d0 = W - x_rtn
    mse = np.maximum((d0 * d0).mean(axis=1, keepdims=True, dtype=f32), f32(1e-12))
    gamma1 = (f32(cfg.gamma_start) * (f32(0.25) / mse)).astype(f32)
    Y_u = (W @ Vs).astype(f32)
    if obs_precision_init is not None and float(obs_precision_init) > 0.0:
        obs0 = float(obs_precision_init)
    elif float(cfg.obs_precision) > 0.0:
        obs0 = float(cfg.obs_precision)
    else:
        dd = Y_u - x_rtn @ Vs
        obs0 = 1.0 / max(float((dd * dd).mean(dtype=f32)), 1e-12)
    obs = float(obs0)
    em_active = bool(cfg.em_obs_precision) and float(cfg.obs_precision) <= 0.0
    factor = max(float(cfg.gamma_retry_factor), 1.000001)
    retry_steps = max(int(cfg.gamma_retry_steps), 0)

    def hard_state(r1_s, g1_s):
        post = discrete_uniform_mmse(r1=r1_s, gamma1=g1_s, scale_full=scale_full, zero_full=zero_full,
                                     maxq=maxq, prior_center=W, prior_tau=prior_tau, atoms=atoms)
        q, x = uniform_hard_decision(x_mean=post["mean"], x_map=post["map_value"], scale_full=scale_full,
                                     zero_full=zero_full, maxq=maxq, final_decision=cfg.final_decision)
        return q, x, vamp_rankspace_error(Y_u=Y_u, x=x, Vs=Vs)

    best_q, best_x, best_err = hard_state(r1, gamma1)
    best_err_mean = float(best_err.mean(dtype=f32))
    best = dict(r1=r1.copy(), g1=gamma1.copy(), r2p=None, g2p=None, obs=obs)
    best_iter = -1
    stop_iter = -1
    r2_prev = None
    g2_prev = None
    retries = 0
    g2_invalid = 0
    iters_run = 0
    for it in range(iters):
        iters_run += 1
        g1w = gamma1
        for retry_idx in range(retry_steps + 1):
            post = discrete_uniform_mmse(r1=r1, gamma1=g1w, scale_full=scale_full, zero_full=zero_full,
                                         maxq=maxq, prior_center=W, prior_tau=prior_tau, atoms=atoms)
            a1 = post["alpha1"]
            valid = alpha_valid_mask(a1)
            if valid.all():
                alpha1 = a1
                x1 = post["mean"]
                break
            if retry_idx >= retry_steps:
                if not np.isfinite(a1).all():
                    raise RuntimeError("alpha1 invalid")
                alpha1 = np.clip(nan_to_num(a1, 0.5, 1.0 - ALPHA_EPS, ALPHA_EPS), f32(ALPHA_EPS), f32(1.0 - ALPHA_EPS))
                x1 = post["mean"]
                break
            retries += int((~valid).sum())
            g1w = np.where(a1 <= f32(ALPHA_EPS), g1w / f32(factor), g1w)
            g1w = np.where(a1 >= f32(1.0 - ALPHA_EPS), g1w * f32(factor), g1w)
            g1w = np.maximum(g1w, f32(1e-12)).astype(f32)
        eta1 = g1w / alpha1
        g2_new = np.maximum(nan_to_num(eta1 - g1w, 1e-12, 1e12, 1e-12), f32(1e-12))
        if not precision_valid_mask(g2_new).all():
            g2_invalid += 1
            continue
        r2_new = (eta1 * x1 - g1w * r1) / g2_new
        if r2_prev is None or g2_prev is None or damping >= 1.0:
            gamma2, r2 = g2_new, r2_new
        else:
            gamma2 = log_damp_positive(g2_prev, g2_new, damping)
            r2 = f32(1.0 - damping) * r2_prev + f32(damping) * r2_new
        if not precision_valid_mask(gamma2).all():
            g2_invalid += 1
            continue
        x2, alpha2_raw, residual_u = linear_mmse_exact(r2, gamma2, Y_u=Y_u, V=V, Vh=Vh, S=S, obs_precision=obs)
        alpha2 = np.clip(nan_to_num(alpha2_raw, 0.5, 1.0 - ALPHA_EPS, ALPHA_EPS), f32(ALPHA_EPS), f32(1.0 - ALPHA_EPS))
        if em_active and rank > 0:
            obs = em_update_obs_precision_rankspace(
                residual_u=residual_u, gamma2=gamma2, S=S, obs_precision=obs, num_obs=rank,
                damping=cfg.em_obs_precision_damping, min_value=cfg.em_obs_precision_min,
                max_value=cfg.em_obs_precision_max)
        eta2 = gamma2 / alpha2
        g1_new = np.maximum(nan_to_num(eta2 - gamma2, 1e-12, 1e12, 1e-12), f32(1e-12))
        r1_new = (eta2 * x2 - gamma2 * r2) / g1_new
        if damping >= 1.0:
            gamma1, r1 = g1_new, r1_new
        else:
            gamma1 = log_damp_positive(gamma1, g1_new, damping)
            r1 = (f32(1.0 - damping) * r1 + f32(damping) * r1_new).astype(f32)
        r2_prev, g2_prev = r2, gamma2
        cq, cx, ce = hard_state(r1, gamma1)
        ce_mean = float(ce.mean(dtype=f32))
        tol = max(1e-10, abs(best_err_mean) * 1e-8)
        if ce_mean + tol < best_err_mean:
            best_q, best_x, best_err, best_err_mean = cq, cx, ce, ce_mean
            best = dict(r1=r1.copy(), g1=gamma1.copy(), r2p=r2_prev.copy(), g2p=g2_prev.copy(), obs=obs)
            best_iter = it
        else:
            r1 = best["r1"].copy()
            gamma1 = best["g1"].copy()
            obs = float(best["obs"])
            stop_iter = it
            break

    q_final, x_final, err_final = best_q, best_x, best_err
    polish_updates = 0.0
    topk = str(getattr(cfg, "polish_mode", "block_cd")) == "topk_block_cd"
    if int(cfg.polish_sweeps) > 0 and Vs.size and (gram_full is not None or topk):
        err_before = vamp_rankspace_error(Y_u=Y_u, x=x_final, Vs=Vs)
        if topk:  # mpq/solver.py:704-745 with polish_uniform_rankspace :292-366 (generic engine, top-k provider)
            from . import block_cd as OB
            from . import topk as OT
            tk = OT.uniform_map_topk(r1=r1, gamma1=gamma1, scale_full=scale_full, zero_full=zero_full, maxq=maxq,
                                     prior_center=W, prior_tau=float(cfg.prior_tau), k=max(int(cfg.topk_k), 1))
            q0 = nearest_atom_idx(x=x_final, scale_full=scale_full, zero_full=zero_full, maxq=maxq)
            _, q_p, pst = OB.block_coordinate_descent_rankspace(
                x=x_final, Y_u=Y_u, Vs=Vs, block_size=1, propose=OT.uniform_topk_provider(tk["topk_values"], tk["topk_q"]),
                sweeps=int(cfg.polish_sweeps), metric="diag", order_mode="greedy_gain", idxs_init=q0)
            q_p = q_p.astype(np.int32)
            x_p = dequant_from_q(q_int=q_p, scale_full=scale_full, zero_full=zero_full)
            err_after = vamp_rankspace_error(Y_u=Y_u, x=x_p, Vs=Vs)
        else:
            q_p, x_p, err_after, pst = polish_uniform_gpu_semantics(
                x_init=x_final, Y_u=Y_u, Vs=Vs, scale_full=scale_full, zero_full=zero_full, maxq=maxq,
                sweeps=int(cfg.polish_sweeps), gram_full=gram_full)
        improve = (err_after + f32(1e-12)) < err_before
        if improve.any():
            q_final = np.where(improve[:, None], q_p, q_final)
            x_final = np.where(improve[:, None], x_p, x_final)
            err_final = np.where(improve, err_after, err_final)
        polish_updates = pst["accepted_updates"]
    rtn_err = vamp_rankspace_error(Y_u=Y_u, x=x_rtn, Vs=Vs)
    if debug is not None:  # mpq/solver.py:757-777 (capture_r1)
        debug["r1"] = r1.copy()
        debug["gamma1"] = gamma1.copy()
    stats = {"obs_precision_initial": obs0, "obs_precision_final": obs, "best_iter": best_iter,
             "stop_iter": stop_iter, "alpha1_retry_count": retries, "gamma2_invalid_count": g2_invalid,
             "best_rankspace_error_mean": best_err_mean, "polish_updates": polish_updates,
             "rankspace_error_mean": float(err_final.mean(dtype=f32)), "iters_run": iters_run}
    return q_final.astype(np.int32), x_final.astype(f32), err_final.astype(f32), rtn_err, stats
