"""Rank-space VAMP solvers: the public plugin interface of the reference, on sm_100a kernels.

Reference: mpq/solver.py (UniformVampConfig :35-55, E8P12VampConfig :58-82,
polish_uniform_rankspace :260-366, solve_uniform_rankspace_vamp :426-830,
_uniform_hard_decision :833-850).

Signatures, argument meaning, return values and error behaviour follow the reference:
keyword-only, pure (fresh outputs), ``ValueError`` for bad configuration or shapes,
``RuntimeError`` for numerical invalidity.  All tensors must live on one CUDA device; the
computation runs on the current torch stream through ``libmpq_b200.so``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Dict, Optional, Tuple

import torch

from . import ops, trace
from ._lib import call, ptr

ALPHA_EPS = 1e-7


@dataclass(frozen=True)
class UniformVampConfig:
    iters: int = 10
    damping: float = 0.5
    final_decision: str = "map"  # "map" | "round_mean"
    init_from: str = "rtn"  # "rtn" | "float" | "zero"
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
    polish_mode: str = "block_cd"  # "none" | "block_cd" | "topk_block_cd"
    topk_k: int = 16
    vamp_backend: str = "auto"  # accepted for interface compatibility; always the CUDA kernels
    compile_block_cd: bool = True
    block_cd_backend: str = "eager"


@dataclass(frozen=True)
class E8P12VampConfig:
    """Scalar-precision VAMP config for QUIP E8P12 (mpq/solver.py:58-82)."""

    iters: int = 16
    damping: float = 0.5
    gamma_start: float = 1.0
    gamma_retry_factor: float = 4.0
    gamma_retry_steps: int = 3
    prior_tau: float = 0.25
    prior_tau_scale_mode: str = "absmax"
    compile_prior: bool = True
    obs_precision: float = 0.0
    em_obs_precision: bool = True
    em_obs_precision_damping: float = 0.3
    em_obs_precision_min: float = 1e-4
    em_obs_precision_max: float = 1e8
    blocks_per_chunk: int = 16
    polish_sweeps: int = 3
    polish_mode: str = "block_cd"
    polish_metric: str = "gram"
    polish_metric_rows_per_chunk: int = 0
    polish_max_blocks: int = 0
    topk_k: int = 16
    best_iterate: bool = False


def _resolve_polish_mode(*, sweeps: int, mode: str) -> str:
    """mpq/solver.py:164-175."""
    if int(sweeps) <= 0:
        return "none"
    mode_norm = str(mode or "block_cd").strip().lower()
    if mode_norm in {"none", "off"}:
        return "none"
    if mode_norm in {"block_cd", "cd", "full_cd"}:
        return "block_cd"
    if mode_norm in {"topk_block_cd", "topk_cd", "topk", "vamp_topk"}:
        return "topk_block_cd"
    raise ValueError(f"unsupported polish_mode={mode!r}; expected none|block_cd|topk_block_cd.")


def _resolve_block_cd_backend(*, block_cd_backend: Optional[str], compile_block_cd: bool) -> str:
    """mpq/solver.py:189-197: "triton"/"auto" select the raw-Hessian greedy scalar CD (here a CUDA kernel),
    "eager"/"compile" the generic rank-space block CD engine with the scalar provider."""
    backend = str(block_cd_backend or "").strip().lower()
    if not backend:
        return "compile" if bool(compile_block_cd) else "eager"
    if backend not in {"eager", "compile", "triton", "auto"}:
        raise ValueError(f"unsupported block_cd_backend={block_cd_backend!r}; expected eager|compile|triton|auto.")
    return backend


def _expand_groups(p: torch.Tensor, n: int) -> torch.Tensor:
    """(B, n/group) -> (B, n) group-expanded; (B, n) unchanged."""
    if p.shape[1] == n:
        return p.contiguous()
    return p.repeat_interleave(n // p.shape[1], dim=1).contiguous()


def _generic_uniform_polish(*, x_init, Y_u, Vs, scale, zero, maxq, sweeps, order_mode, backend, raw_target, raw_gram,
                            q_init):
    """The generic engine with the scalar provider (mpq/solver.py:337-366)."""
    from .block_cd import BlockCDConfig, UniformScalarProvider, block_coordinate_descent_rankspace
    n = x_init.shape[1]
    sf, zf = _expand_groups(scale, n), _expand_groups(zero, n)
    x_pol, q_cd, st = block_coordinate_descent_rankspace(
        x=x_init, Y_u=Y_u, Vs=Vs, block_size=1, provider=UniformScalarProvider(scale=sf, zero=zf, maxq=int(maxq)),
        cfg=BlockCDConfig(sweeps=int(sweeps), metric="diag", accept_tol=0.0, order_mode=str(order_mode or "greedy_gain"),
                          compile_steps=backend in {"compile", "auto"}),
        idxs_init=q_init, raw_target=raw_target, raw_gram=raw_gram)
    st = dict(st)
    st["block_cd_backend"] = "cuda_generic"
    return x_pol, q_cd, st


def _uniform_topk_polish(*, x_init, Y_u, Vs, topk_values, topk_q, sweeps, order_mode, backend, raw_target, raw_gram,
                         q_init):
    """The generic engine with the top-k provider (mpq/solver.py:292-295, 341-366)."""
    from .block_cd import BlockCDConfig, UniformTopKProvider, block_coordinate_descent_rankspace
    x_pol, q_cd, st = block_coordinate_descent_rankspace(
        x=x_init, Y_u=Y_u, Vs=Vs, block_size=1, provider=UniformTopKProvider(topk_values=topk_values, topk_q=topk_q),
        cfg=BlockCDConfig(sweeps=int(sweeps), metric="diag", accept_tol=0.0, order_mode=str(order_mode or "greedy_gain"),
                          compile_steps=backend in {"compile", "auto"}),
        idxs_init=q_init, raw_target=raw_target, raw_gram=raw_gram)
    st = dict(st)
    st["block_cd_backend"] = "cuda_generic"
    return x_pol, q_cd, st


def _dequant(q: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor) -> torch.Tensor:
    """s (q - z) in float32 with group-compressed or expanded scale / zero."""
    n = q.shape[1]
    return _expand_groups(scale, n) * (q.to(torch.float32) - _expand_groups(zero, n))


@torch.inference_mode()
def build_uniform_vamp_topk_candidates(*, r1: torch.Tensor, gamma1: torch.Tensor, W: torch.Tensor,
                                       scale_full: torch.Tensor, zero_full: torch.Tensor, maxq: int, prior_tau: float,
                                       k: int, atoms: Optional[torch.Tensor] = None) -> Dict[str, torch.Tensor]:
    """mpq/solver.py:201-224: the k best grid levels per coordinate under the final VAMP message."""
    from .topk import uniform_map_topk
    return uniform_map_topk(r1=r1, gamma1=gamma1, scale_full=scale_full, zero_full=zero_full, maxq=maxq,
                            prior_center=W, prior_tau=float(prior_tau), k=max(int(k), 1), atoms=atoms)


@torch.inference_mode()
def build_e8p12_vamp_topk_candidates(*, r1: torch.Tensor, gamma1: torch.Tensor, Wr: torch.Tensor, cb: object,
                                     blocks_per_chunk: int, prior_tau: float, prior_tau_scale_mode: str,
                                     k: int) -> Dict[str, torch.Tensor]:
    """mpq/solver.py:227-260: the k best of the 1024 {best, second-best} sign-pattern candidates per block."""
    from .e8p12 import prior_scale_from_center
    from .topk import vamp_vector_map_topk_e8p12
    B, n = Wr.shape
    codesz = int(getattr(cb, "codesz", 8))
    if codesz != 8 or (n % codesz) != 0:
        raise ValueError(f"E8P12 top-k expects n divisible by 8; got n={n}, codesz={codesz}.")
    nb = n // codesz
    W_blocks = Wr.reshape(B, nb, codesz)
    prior_scale_blocks = prior_scale_from_center(W_blocks, prior_tau_scale_mode) if float(prior_tau) > 0.0 else None
    return vamp_vector_map_topk_e8p12(
        r1_blocks=r1.reshape(B, nb, codesz), gamma1=gamma1, cb=cb, k=max(int(k), 1),
        blocks_per_chunk=max(int(blocks_per_chunk), 1),
        prior_center_blocks=W_blocks if float(prior_tau) > 0.0 else None, prior_scale_blocks=prior_scale_blocks,
        prior_tau=float(prior_tau), prior_tau_scale_mode=str(prior_tau_scale_mode))


def _log_damp_scalar(prev: float, new: float, damping: float) -> float:
    """mpq/utils.py:36-45."""
    if damping >= 1.0:
        return float(new)
    if damping <= 0.0:
        return float(prev)
    prev = max(float(prev), 1e-12)
    new = max(float(new), 1e-12)
    return float(math.exp((1.0 - damping) * math.log(prev) + damping * math.log(new)))


class _UniformCtx:
    """Device-side operands of one grouped-scalar solve (shared by VAMP and polish)."""

    def __init__(self, W, scale_full, zero_full, maxq, V, Vh, S, Vs):
        self.dev = W.device
        self.W = W
        self.B, self.n = W.shape
        self.R = int(S.numel())
        self.scale = scale_full
        self.zero = zero_full
        self.ld_p, self.gshift = ops.group_layout(scale_full, self.n)
        if zero_full.shape != scale_full.shape or zero_full.stride(0) != self.ld_p:
            raise ValueError("scale_full and zero_full must have the same shape and layout")
        self.maxq = int(maxq)
        self.V = V
        self.Vh = Vh
        self.S = S
        self.Vs = Vs
        self.VsT = Vs.t().contiguous()
        # B-side operands of the rank-space products, split once for the 3xTF32 tensor-core GEMM
        self.opV = ops.Operand(V)        # (resid * coeff) @ Vh  ==  u @ V^T
        self.opVh = ops.Operand(Vh)      # r2 @ V                ==  r2 @ Vh^T
        self.opVsT = ops.Operand(self.VsT)  # x @ Vs
        self.opVs = ops.Operand(Vs)      # residual_u @ Vs^T
        # Y_u anchors every residual of the solve: one FP32-faithful split product (the solve's parity tests at
        # 4096 columns hold with it; a single-pass TF32 product would not be faithful enough)
        self.Y_u = ops.mm_nt(W, self.opVsT)

    def err(self, x, out=None, tmp=None):
        C = ops.mm_nt(x, self.opVsT, tmp)
        if out is None:
            out = torch.empty(x.shape[0], device=x.device, dtype=torch.float32)
        call("mpq_row_sqerr", ptr(self.Y_u), ptr(C), x.shape[0], C.shape[1], self.Y_u.stride(0), C.stride(0), ptr(out))
        return out

    def nearest(self, x, q_out, x_out):
        call("mpq_uniform_nearest", ptr(x), x.stride(0), ptr(self.scale), ptr(self.zero), self.ld_p, self.gshift,
             self.B, self.n, self.maxq, ptr(q_out), ptr(x_out), x_out.stride(0))


def _f32c(t: torch.Tensor, device) -> torch.Tensor:
    return t.to(device=device, dtype=torch.float32).contiguous()


@torch.inference_mode()
def scalar_greedy_cd(ctx: _UniformCtx, x_init: torch.Tensor, gram_full: torch.Tensor, *, sweeps: int,
                     accept_tol: float = 0.0) -> Tuple[torch.Tensor, Dict[str, Any]]:
    """Raw-Hessian scalar greedy CD (mpq/polish/triton_scalar_cd.py:164-307) in 128-column blocks.

    Returns (x_polished, stats).  Each sweep orders columns by the greedy gain, then for every
    block of 128 columns runs the per-row sequential decisions (mpq_cd_block) and applies the
    block's accepted steps to the right-hand side with one GEMM.
    """
    dev, B, n, R = ctx.dev, ctx.B, ctx.n, ctx.R
    x_work = x_init.clone()
    res_u = ops.mm_nt(x_work, ctx.opVsT)
    res_norm = torch.empty(B, device=dev, dtype=torch.float32)
    call("mpq_residual", ptr(ctx.Y_u), ptr(res_u), B, R, res_u.stride(0), ptr(res_norm))
    rhs = ops.mm_nt(res_u, ctx.opVs)  # residual_u @ Vs^T  (B x n)
    del res_u
    diag = torch.empty(n, device=dev, dtype=torch.float32)
    diag_inv = torch.empty(n, device=dev, dtype=torch.float32)
    call("mpq_cd_diag", ptr(ctx.Vs), n, R, ctx.Vs.stride(0), ptr(diag), ptr(diag_inv))
    gain = torch.empty(n, device=dev, dtype=torch.float32)
    order = torch.empty(n, device=dev, dtype=torch.int32)
    HJT = torch.empty(n, 128, device=dev, dtype=torch.float32)
    Hsub = torch.empty(128, 128, device=dev, dtype=torch.float32)
    delta = torch.empty(B, 128, device=dev, dtype=torch.float32)
    accepted = torch.zeros(1, device=dev, dtype=torch.int32)
    H = gram_full
    for _ in range(max(int(sweeps), 0)):
        call("mpq_cd_gain", ptr(rhs), B, n, rhs.stride(0), ptr(diag_inv), ptr(gain))
        call("mpq_argsort_desc", ptr(gain), n, ptr(order))
        for c0 in range(0, n, 128):
            K = min(128, n - c0)
            call("mpq_cd_gather", ptr(H), H.stride(0), n, ptr(order), c0, K, ptr(HJT), ptr(Hsub))
            call("mpq_cd_block", ptr(x_work), x_work.stride(0), ptr(rhs), rhs.stride(0), ptr(ctx.scale),
                 ptr(ctx.zero), ctx.ld_p, ctx.gshift, ptr(diag), ptr(diag_inv), ptr(order), c0, K, ptr(Hsub),
                 ptr(res_norm), ptr(delta), ptr(accepted), B, ctx.maxq, float(accept_tol))
            ops.mm_nt(delta[:, :K], HJT[:, :K], out=rhs, alpha=-1.0, beta=1.0)
    return x_work, {"accepted_updates": float(accepted.item())}


@torch.inference_mode()
def polish_uniform_rankspace(
    *,
    x_init: torch.Tensor,
    Y_u: torch.Tensor,
    Vs: torch.Tensor,
    scale_full: torch.Tensor,
    zero_full: torch.Tensor,
    maxq: int,
    sweeps: int,
    polish_mode: str,
    topk_values: Optional[torch.Tensor] = None,
    topk_q: Optional[torch.Tensor] = None,
    compile_block_cd: bool = True,
    block_cd_backend: Optional[str] = None,
    gram_full: Optional[torch.Tensor] = None,
    order_mode: str = "greedy_gain",
    raw_target: Optional[torch.Tensor] = None,
    raw_gram: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, Dict[str, Any]]:
    """mpq/solver.py:260-366 on CUDA: backends "triton"/"auto" (greedy order, raw Hessian given) run the raw-Hessian
    greedy scalar CD kernel; the others run the generic block CD engine with the scalar provider."""
    mode = _resolve_polish_mode(sweeps=int(sweeps), mode=str(polish_mode))
    dev = x_init.device
    x_work = _f32c(x_init, dev)
    B, n = x_work.shape
    R = int(Vs.shape[1])
    scale_full = _f32c(scale_full, dev)
    zero_full = _f32c(zero_full, dev)
    Vs = _f32c(Vs, dev)
    VsT = Vs.t().contiguous()
    Y_u = _f32c(Y_u, dev)
    ld_p, gshift = ops.group_layout(scale_full, n)
    q_out = torch.empty(B, n, device=dev, dtype=torch.uint8)
    x_out = torch.empty(B, n, device=dev, dtype=torch.float32)

    def finish(x, stats):
        call("mpq_uniform_nearest", ptr(x), x.stride(0), ptr(scale_full), ptr(zero_full), ld_p, gshift, B, n,
             int(maxq), ptr(q_out), ptr(x_out), x_out.stride(0))
        C = ops.mm_nt(x_out, ops.Operand(VsT))
        err = torch.empty(B, device=dev, dtype=torch.float32)
        call("mpq_row_sqerr", ptr(Y_u), ptr(C), B, C.shape[1], Y_u.stride(0), C.stride(0), ptr(err))
        return q_out.to(torch.int32), x_out, err, stats

    if mode == "none" or Vs.numel() == 0:
        return finish(x_work, {"accepted_updates": 0.0})
    backend = _resolve_block_cd_backend(block_cd_backend=block_cd_backend, compile_block_cd=bool(compile_block_cd))
    if mode == "topk_block_cd":
        if topk_values is None:
            raise ValueError("topk_block_cd requires topk_values for uniform polish.")
        q0 = torch.empty(B, n, device=dev, dtype=torch.uint8)
        x0 = torch.empty(B, n, device=dev, dtype=torch.float32)
        call("mpq_uniform_nearest", ptr(x_work), x_work.stride(0), ptr(scale_full), ptr(zero_full), ld_p, gshift, B, n,
             int(maxq), ptr(q0), ptr(x0), x0.stride(0))
        x_pol, q_cd, st = _uniform_topk_polish(
            x_init=x_work, Y_u=Y_u, Vs=Vs, topk_values=topk_values, topk_q=topk_q, sweeps=int(sweeps),
            order_mode=order_mode, backend=backend, raw_target=raw_target,
            raw_gram=_f32c(raw_gram, dev) if raw_gram is not None else None, q_init=q0.to(torch.int32))
        if q_cd is None:
            return finish(x_pol, st)
        q_pol = q_cd.to(torch.int32)
        x_q = _dequant(q_pol, scale_full, zero_full).contiguous()
        C = ops.mm_nt(x_q, ops.Operand(VsT))
        err = torch.empty(B, device=dev, dtype=torch.float32)
        call("mpq_row_sqerr", ptr(Y_u), ptr(C), B, C.shape[1], Y_u.stride(0), C.stride(0), ptr(err))
        return q_pol, x_q, err, st
    use_raw = (str(order_mode or "greedy_gain").strip().lower() == "greedy_gain" and backend in {"triton", "auto"}
               and gram_full is not None)
    if not use_raw:
        q0 = torch.empty(B, n, device=dev, dtype=torch.uint8)
        x0 = torch.empty(B, n, device=dev, dtype=torch.float32)
        call("mpq_uniform_nearest", ptr(x_work), x_work.stride(0), ptr(scale_full), ptr(zero_full), ld_p, gshift, B, n,
             int(maxq), ptr(q0), ptr(x0), x0.stride(0))
        x_pol, _, st = _generic_uniform_polish(
            x_init=x_work, Y_u=Y_u, Vs=Vs, scale=scale_full, zero=zero_full, maxq=maxq, sweeps=int(sweeps),
            order_mode=order_mode, backend=backend, raw_target=raw_target,
            raw_gram=_f32c(raw_gram, dev) if raw_gram is not None else None, q_init=q0.to(torch.int32))
        return finish(x_pol, st)
    ctx = _UniformCtx.__new__(_UniformCtx)
    ctx.dev, ctx.B, ctx.n, ctx.R = dev, B, n, R
    ctx.scale, ctx.zero, ctx.ld_p, ctx.gshift, ctx.maxq = scale_full, zero_full, ld_p, gshift, int(maxq)
    ctx.Vs, ctx.VsT, ctx.Y_u = Vs, VsT, Y_u
    ctx.opVs, ctx.opVsT = ops.Operand(Vs), ops.Operand(VsT)
    x_pol, st = scalar_greedy_cd(ctx, x_work, _f32c(gram_full, dev), sweeps=int(sweeps))
    st = dict(st)
    st["block_cd_backend"] = "cuda"
    return finish(x_pol, st)


@torch.inference_mode()
def solve_uniform_rankspace_vamp(
    *,
    W: torch.Tensor,
    x_rtn: torch.Tensor,
    scale_full: torch.Tensor,
    zero_full: torch.Tensor,
    maxq: int,
    V: torch.Tensor,
    Vh: torch.Tensor,
    S: torch.Tensor,
    Vs: torch.Tensor,
    cfg: UniformVampConfig,
    gram_full: Optional[torch.Tensor] = None,
    obs_precision_init: Optional[float] = None,
    log_stats: bool = True,
    debug_out: Optional[Dict[str, Any]] = None,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, Dict[str, Any]]:
    """Scalar uniform exact-full VAMP in rank space (MMSE x1) with the greedy CD polish.

    mpq/solver.py:426-830.  Returns (q_int int32 (B, n), x_final (B, n), final_err (B,),
    rtn_err (B,), stats).
    """
    if not W.is_cuda:
        raise ValueError("solve_uniform_rankspace_vamp requires CUDA tensors (there is no CPU path)")
    dev = W.device
    W = _f32c(W, dev)
    x_rtn = _f32c(x_rtn, dev)
    scale_full = _f32c(scale_full, dev)
    zero_full = _f32c(zero_full, dev)
    V, Vh, S, Vs = (_f32c(t, dev) for t in (V, Vh, S, Vs))
    maxq = int(maxq)
    iters = max(int(cfg.iters), 0)
    damping = float(cfg.damping)
    prior_tau = float(cfg.prior_tau)
    final_decision = str(cfg.final_decision or "map").strip().lower()
    init_from = str(cfg.init_from or "rtn").strip().lower()
    if final_decision not in {"map", "round_mean"}:
        raise ValueError(f"unsupported final_decision={cfg.final_decision!r}")
    B, n = W.shape
    R = int(S.numel())
    if R == 0:
        raise ValueError("rank-0 spectra are not supported by the CUDA solver")
    ctx = _UniformCtx(W, scale_full, zero_full, maxq, V, Vh, S, Vs)
    f32 = dict(device=dev, dtype=torch.float32)

    if init_from == "zero":
        r1 = torch.zeros(B, n, **f32)
    elif init_from == "float":
        r1 = W.clone()
    elif init_from == "rtn":
        r1 = x_rtn.clone()
    else:
        raise ValueError(f"unknown init_from={init_from!r} (expected 'rtn', 'float', or 'zero').")

    gamma1 = torch.empty(B, **f32)
    call("mpq_gamma_init", ptr(W), ptr(x_rtn), B, n, W.stride(0), float(cfg.gamma_start), ptr(gamma1))
    tmpBR = torch.empty(B, R, **f32)
    if obs_precision_init is not None and float(obs_precision_init) > 0.0:
        obs_initial = float(obs_precision_init)
    elif float(cfg.obs_precision) > 0.0:
        obs_initial = float(cfg.obs_precision)
    else:
        e = ctx.err(x_rtn, tmp=tmpBR)
        obs_initial = 1.0 / max(float(ops.mean_rows(e).item()) / R, 1e-12)
    obs = float(obs_initial)
    em_active = bool(cfg.em_obs_precision) and float(cfg.obs_precision) <= 0.0

    def args_uniform(r, g):
        return (ptr(r), r.stride(0), ptr(W), W.stride(0), ptr(scale_full), ptr(zero_full), ctx.ld_p, ctx.gshift,
                ptr(g), B, n, maxq, prior_tau)

    mean_tmp = torch.empty(B, n, **f32) if final_decision == "round_mean" else None
    vsum_tmp = torch.empty(B, **f32) if final_decision == "round_mean" else None

    def hard_state(r, g, q_out, x_out, err_out):
        """mpq/solver.py:513-541 + _uniform_hard_decision :833-850: 'map' rounds the posterior's MAP atom,
        'round_mean' rounds the posterior mean to the nearest grid level."""
        if final_decision == "map":
            call("mpq_uniform_map_decision", *args_uniform(r, g), ptr(q_out), ptr(x_out), x_out.stride(0))
        else:
            call("mpq_uniform_mmse", *args_uniform(r, g), ptr(mean_tmp), mean_tmp.stride(0), None, None, None,
                 ptr(vsum_tmp))
            ctx.nearest(mean_tmp, q_out, x_out)
        ctx.err(x_out, out=err_out, tmp=tmpBR)

    best_q = torch.empty(B, n, device=dev, dtype=torch.uint8)
    best_x = torch.empty(B, n, **f32)
    best_err = torch.empty(B, **f32)
    cur_q = torch.empty_like(best_q)
    cur_x = torch.empty_like(best_x)
    cur_err = torch.empty_like(best_err)
    hard_state(r1, gamma1, best_q, best_x, best_err)
    best_err_mean = float(ops.mean_rows(best_err).item())
    best_r1 = r1.clone()
    best_g1 = gamma1.clone()
    best_obs = obs

    x1 = torch.empty(B, n, **f32)  # posterior mean, later reused for the linear-module delta
    r2 = torch.empty(B, n, **f32)
    r2_prev = torch.empty(B, n, **f32)
    have_prev = False
    u = torch.empty(B, R, **f32)
    rows = {k: torch.empty(B, **f32) for k in ("var", "g1w", "a1", "eta1", "g2n", "g2", "g2p", "a2", "eta2", "g1n",
                                               "g1next", "trace", "resid")}
    flags = torch.zeros(8, device=dev, dtype=torch.int32)
    means = torch.zeros(2, **f32)
    factor = max(float(cfg.gamma_retry_factor), 1.000001)
    retry_steps = max(int(cfg.gamma_retry_steps), 0)
    alpha1_retry_count = 0
    alpha2_clip_count = 0
    gamma2_invalid_count = 0
    obs_values = []
    best_iter_idx = -1
    stop_iter_idx = -1

    for it in range(iters):
        rows["g1w"].copy_(gamma1)
        for retry_idx in range(retry_steps + 1):
            final = retry_idx >= retry_steps
            call("mpq_uniform_mmse", *args_uniform(r1, rows["g1w"]), ptr(x1), x1.stride(0), None, None, None,
                 ptr(rows["var"]))
            flags.zero_()
            call("mpq_vamp_rows", ptr(rows["var"]), ptr(gamma1), ptr(rows["g1w"]), ptr(rows["a1"]), ptr(rows["eta1"]),
                 ptr(rows["g2n"]), ptr(rows["g2"]), ptr(rows["g2p"]) if (have_prev and damping < 1.0) else None,
                 ptr(rows["a2"]), ptr(rows["eta2"]), ptr(rows["g1n"]), ptr(rows["g1next"]), ptr(rows["trace"]),
                 ptr(flags), ptr(S), B, n, n, R, obs, damping, int(final))
            fl = flags.tolist()
            if fl[0] == 0:
                break
            if final:
                if fl[1] > 0:
                    raise RuntimeError(f"alpha1 invalid: expected all in ({ALPHA_EPS}, 1-{ALPHA_EPS}).")
                break
            alpha1_retry_count += int(fl[0])
            call("mpq_gamma_retry", ptr(rows["g1w"]), ptr(rows["var"]), B, n, factor)
        if fl[2] > 0 or fl[3] > 0:
            gamma2_invalid_count += 1
            continue
        alpha2_clip_count += int(fl[4])
        call("mpq_vamp_r2", ptr(x1), ptr(r1), ptr(r2_prev) if (have_prev and damping < 1.0) else None, ptr(r2),
             ptr(rows["eta1"]), ptr(rows["g1w"]), ptr(rows["g2n"]), B, n, r2.stride(0), damping)
        P = ops.mm_nt(r2, ctx.opVh, tmpBR)  # r2 @ V
        call("mpq_linear_epilogue", ptr(P), ptr(ctx.Y_u), ptr(S), ptr(rows["g2"]), obs, B, R, P.stride(0), ptr(u),
             ptr(rows["resid"]))
        D = ops.mm_nt(u, ctx.opV, x1)  # (resid * coeff) @ Vh
        call("mpq_vamp_r1", ptr(D), ptr(r2), ptr(r1), ptr(rows["eta2"]), ptr(rows["g2"]), ptr(rows["g1n"]), B, n,
             r1.stride(0), damping)
        gamma1.copy_(rows["g1next"])
        r2, r2_prev = r2_prev, r2
        rows["g2p"].copy_(rows["g2"])
        have_prev = True
        if em_active:
            ops.mean_rows(rows["resid"], rows["trace"], out=means[0:1])
        hard_state(r1, gamma1, cur_q, cur_x, cur_err)
        ops.mean_rows(cur_err, out=means[1:2])
        em_mean, cur_err_mean = means.tolist()
        if em_active:
            beta_new = float(R / max(em_mean, 1e-12))
            beta = _log_damp_scalar(max(obs, 1e-12), beta_new, float(cfg.em_obs_precision_damping))
            obs = float(min(max(beta, float(cfg.em_obs_precision_min)), float(cfg.em_obs_precision_max)))
        obs_values.append(obs)
        tol = max(1e-10, abs(best_err_mean) * 1e-8)
        if cur_err_mean + tol < best_err_mean:
            best_q, cur_q = cur_q, best_q
            best_x, cur_x = cur_x, best_x
            best_err, cur_err = cur_err, best_err
            best_err_mean = cur_err_mean
            best_r1.copy_(r1)
            best_g1.copy_(gamma1)
            best_obs = obs
            best_iter_idx = it
        else:
            r1.copy_(best_r1)
            gamma1.copy_(best_g1)
            obs = float(best_obs)
            stop_iter_idx = it
            break

    q_final, x_final, err_final = best_q, best_x, best_err
    polish_sweeps = max(int(cfg.polish_sweeps), 0)
    polish_mode = _resolve_polish_mode(sweeps=polish_sweeps, mode=str(getattr(cfg, "polish_mode", "block_cd")))
    polish_stats: Dict[str, Any] = {}
    polish_updates = 0.0
    polish_gain = 0.0
    if polish_mode != "none":
        backend = _resolve_block_cd_backend(block_cd_backend=str(getattr(cfg, "block_cd_backend", "") or ""),
                                            compile_block_cd=bool(getattr(cfg, "compile_block_cd", True)))
        q_pol = torch.empty_like(q_final)
        x_out = torch.empty_like(x_final)
        if polish_mode == "topk_block_cd":
            topk = build_uniform_vamp_topk_candidates(
                r1=r1, gamma1=gamma1, W=W, scale_full=ctx.scale, zero_full=ctx.zero, maxq=ctx.maxq,
                prior_tau=prior_tau, k=max(int(getattr(cfg, "topk_k", 16) or 16), 1))
            x_pol, q_cd, polish_stats = _uniform_topk_polish(
                x_init=x_final, Y_u=ctx.Y_u, Vs=ctx.Vs, topk_values=topk["topk_values"], topk_q=topk["topk_q"],
                sweeps=polish_sweeps, order_mode="greedy_gain", backend=backend,
                raw_target=W if gram_full is not None else None,
                raw_gram=_f32c(gram_full, dev) if gram_full is not None else None, q_init=q_final.to(torch.int32))
            q_pol.copy_(q_cd.to(torch.uint8))
            x_out.copy_(_dequant(q_pol, ctx.scale, ctx.zero))
            del topk
        elif backend in {"triton", "auto"} and gram_full is not None:
            x_pol, polish_stats = scalar_greedy_cd(ctx, x_final, _f32c(gram_full, dev), sweeps=polish_sweeps)
            polish_stats = dict(polish_stats, block_cd_backend="cuda")
            ctx.nearest(x_pol, q_pol, x_out)
        else:
            x_pol, q_cd, polish_stats = _generic_uniform_polish(
                x_init=x_final, Y_u=ctx.Y_u, Vs=ctx.Vs, scale=ctx.scale, zero=ctx.zero, maxq=ctx.maxq,
                sweeps=polish_sweeps, order_mode="greedy_gain", backend=backend,
                raw_target=W if gram_full is not None else None,
                raw_gram=_f32c(gram_full, dev) if gram_full is not None else None, q_init=q_final.to(torch.int32))
            q_pol.copy_(q_cd.to(torch.uint8))
            call("mpq_uniform_nearest", ptr(x_pol), x_pol.stride(0), ptr(ctx.scale), ptr(ctx.zero), ctx.ld_p,
                 ctx.gshift, B, n, ctx.maxq, ptr(q_pol), ptr(x_out), x_out.stride(0))
        err_after = ctx.err(x_out, tmp=tmpBR)
        err_before = err_final.clone()
        improved = torch.zeros(1, device=dev, dtype=torch.int32)
        call("mpq_polish_merge", ptr(err_after), ptr(err_final), ptr(err_before), ptr(x_out), ptr(x_final),
             ptr(q_pol), ptr(q_final), B, n, x_final.stride(0), ptr(improved))
        polish_updates = float(polish_stats.get("accepted_updates", 0.0))
        polish_stats = dict(polish_stats)
        polish_stats["rows_improved"] = int(improved.item())

    rtn_err = ctx.err(x_rtn, tmp=tmpBR)
    ops.check_status(dev)
    if debug_out is not None:
        debug_out["solver"] = "uniform_exact_vamp"
        g64 = gamma1.double()
        debug_out["gamma1_sum"] = float(g64.sum())
        debug_out["gamma1_count"] = int(g64.numel())
        debug_out["gamma1_min"] = float(g64.min()) if B else 0.0
        debug_out["gamma1_max"] = float(g64.max()) if B else 0.0
        if bool(debug_out.get("capture_r1", False)):
            debug_out["r1"] = r1.detach().cpu()
        debug_out["gamma1"] = gamma1.detach().cpu()
    stats: Dict[str, Any] = {
        "solver": "uniform_exact_vamp",
        "iters": int(iters),
        "rank": int(R),
        "init_from": init_from,
        "damping": damping,
        "prior_tau": prior_tau,
        "vamp_backend": "cuda",
        "vamp_backend_used": "cuda",
        "gamma_start": float(cfg.gamma_start),
        "gamma_retry_factor": float(factor),
        "gamma_retry_steps": int(retry_steps),
        "obs_precision_initial": float(obs_initial),
        "obs_precision_final": float(obs),
        "obs_precision_mean": float(sum(obs_values) / len(obs_values)) if obs_values else float(obs),
        "alpha1_retry_count": int(alpha1_retry_count),
        "alpha2_clip_count": int(alpha2_clip_count),
        "gamma2_invalid_count": int(gamma2_invalid_count),
        "final_decision": final_decision,
        "best_iterate_enabled": True,
        "best_iter": int(best_iter_idx),
        "stop_iter": int(stop_iter_idx),
        "best_rankspace_error_mean": float(best_err_mean),
        "polish_sweeps": int(polish_sweeps),
        "polish_mode": polish_mode,
        "polish_gain": float(polish_gain),
        "polish_updates": float(polish_updates),
        "polish_trace": polish_stats,
        "block_cd_backend": "cuda",
        "rankspace_error_mean": float(ops.mean_rows(err_final).item()),
        "rtn_rankspace_error_mean": float(ops.mean_rows(rtn_err).item()),
    }
    return q_final.to(torch.int32), x_final, err_final, rtn_err, stats


# ------------------------------------------------------------------------------------------------
# E8P12 (QUIP# 2-bit lattice codebook)
# ------------------------------------------------------------------------------------------------

def _resolve_e8p12_polish_metric(metric: str) -> str:
    """mpq/solver.py:178-185."""
    m = str(metric or "gram").strip().lower()
    if m in ("isotropic", "diag"):
        return "diag"
    if m == "gram":
        return "gram"
    raise ValueError(f"unsupported polish_metric={metric!r}; expected 'gram'|'diag'.")


@torch.inference_mode()
def polish_e8p12_rankspace(
    *,
    x_init: torch.Tensor,
    idxs_init: torch.Tensor,
    Y_u: torch.Tensor,
    Vs: torch.Tensor,
    cb: object,
    sweeps: int,
    polish_mode: str,
    polish_metric: str,
    metric_rows_per_chunk: int = 0,
    polish_max_blocks: int = 0,
    topk_idxs: Optional[torch.Tensor] = None,
    order_mode: str = "greedy_gain",
    snapshot_budgets=None,
    snapshots_out=None,
    _ops: Optional[Tuple[Any, Any]] = None,
    topk_vals: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, Dict[str, Any]]:
    """mpq/solver.py:369-423: gram-metric greedy block CD over the full E8P12 grid ("block_cd") or over each block's
    precomputed top-k codewords ("topk_block_cd"; ``topk_vals`` optionally carries their values)."""
    from .e8p12 import gram_block_cd
    mode = _resolve_polish_mode(sweeps=int(sweeps), mode=str(polish_mode))
    metric = _resolve_e8p12_polish_metric(polish_metric)
    dev = x_init.device
    x_work = _f32c(x_init, dev)
    Vs = _f32c(Vs, dev)
    Y_u = _f32c(Y_u, dev)
    opVs, opVsT = _ops if _ops is not None else (ops.Operand(Vs), ops.Operand(Vs.t().contiguous()))

    def err_of(x):
        C = ops.mm_nt(x, opVsT)
        e = torch.empty(x.shape[0], device=dev, dtype=torch.float32)
        call("mpq_row_sqerr", ptr(Y_u), ptr(C), x.shape[0], C.shape[1], Y_u.stride(0), C.stride(0), ptr(e))
        return e

    if mode == "none" or Vs.numel() == 0:
        return x_work, idxs_init, err_of(x_work), {"accepted_updates": 0.0}
    from .block_cd import BlockCDConfig, E8P12Provider, E8P12TopKProvider, block_coordinate_descent_rankspace
    if mode == "topk_block_cd":
        if topk_idxs is None:
            raise ValueError("topk_block_cd requires topk_idxs for E8P12 polish.")
        provider = E8P12TopKProvider(cb=cb, topk_idxs=topk_idxs, topk_vals=topk_vals)
    else:
        provider = E8P12Provider(cb=cb, metric_rows_per_chunk=int(metric_rows_per_chunk))
    x_out, idx_out, st = block_coordinate_descent_rankspace(
        x=x_work, Y_u=Y_u, Vs=Vs, block_size=int(getattr(cb, "codesz", 8)), provider=provider,
        cfg=BlockCDConfig(sweeps=int(sweeps), metric="gram" if metric == "gram" else "diag", accept_tol=0.0,
                          metric_rows_per_chunk=int(metric_rows_per_chunk), max_blocks_per_sweep=int(polish_max_blocks),
                          order_mode=str(order_mode or "greedy_gain")),
        idxs_init=idxs_init, snapshot_budgets=snapshot_budgets, snapshots_out=snapshots_out)
    if idx_out is None:
        raise RuntimeError("E8P12 polish must return block indices.")
    return x_out, idx_out, err_of(x_out), st


# ------------------------------------------------------------------------------------------------
# device-resident E8P12 VAMP loop (no host round trip inside a row block or between chained blocks)
# ------------------------------------------------------------------------------------------------

# int32 view of the 64-byte control block (csrc/common.cuh VampCtl): obs is the float64 at ints 0-1
_CTL_ACTIVE, _CTL_SKIP, _CTL_HAVE_PREV, _CTL_STOPPED, _CTL_FAIL = 2, 3, 4, 5, 6
_CTL_RETRY, _CTL_CLIP, _CTL_INVALID, _CTL_COMMITTED, _CTL_BEST, _CTL_STOP = 7, 8, 9, 10, 11, 12


def vamp_ctl_new(device, obs: Optional[float] = None) -> torch.Tensor:
    """A zeroed control block (16 int32 = 64 bytes) with best/stop iteration -1 and, optionally, obs set."""
    ctl = torch.zeros(16, device=device, dtype=torch.int32)
    vamp_ctl_reset(ctl)
    if obs is not None:
        ctl.view(torch.float64)[0:1].fill_(float(obs))
    return ctl


def vamp_ctl_reset(ctl: torch.Tensor) -> None:
    """Clear every field but obs (the chain's warm start for the next row block); asynchronous."""
    ctl[2:].zero_()
    ctl[_CTL_BEST:_CTL_STOP + 1].fill_(-1)


def _posterior_chunks(B: int, nb: int, slots: int = 148 * 4) -> int:
    """Item chunks per row of the posterior launch (CTA slots: 148 SMs x 4 resident CTAs of k_e8p12<1>).  Rows alone
    fill the GPU from about two waves up; below that, the chunk count whose last wave is fullest (>= 32 items per
    chunk)."""
    if B <= 0 or B >= 2 * slots:
        return 1
    best, best_eff = 1, 0.0
    for c in range(1, max(1, nb // 32) + 1):
        ctas = B * c
        waves = -(-ctas // slots)
        eff = ctas / (waves * slots) * min(1.0, ctas / (2.0 * slots))
        if eff > best_eff + 1e-9:
            best, best_eff = c, eff
    return best


class E8Layer:
    """Operands of one E8P12 layer solve shared by all its row blocks: the factor tables, the rank-space basis with
    its pre-split tensor-core operands, and (for the gram-metric polish) the per-layer block metadata."""

    def __init__(self, *, V, Vh, S, Vs, cb, device):
        from .codebook import factor_tables
        self.dev = device
        self.cb = cb
        self.V, self.Vh, self.S, self.Vs = V, Vh, S, Vs
        self.R = int(S.numel())
        self.tab = factor_tables(cb, device)
        # the device-resident loop's products take the row-scaled fp16 split of V and Vh
        self.opV, self.opVh = ops.Operand(V, "f16x3"), ops.Operand(Vh, "f16x3")
        self.V, self.Vh = self.opV.full, self.opVh.full
        self.VsT = Vs.t().contiguous()
        self.opVs, self.opVsT = ops.Operand(Vs), ops.Operand(self.VsT)
        self.Vs, self.VsT = self.opVs.full, self.opVsT.full
        self._gram = None

    def gram(self):
        from .e8p12 import GramLayer
        if self._gram is None:
            self._gram = GramLayer(self.Vs, self.opVs, self.opVsT)
        return self._gram

    @classmethod
    def static(cls, *, n: int, R: int, cb, device) -> "E8Layer":
        """A layer whose operand buffers are reused for every layer of this shape (load() fills them): products and
        CUDA graphs captured against them stay valid from layer to layer."""
        z = lambda r, c: torch.zeros(r, c, device=device, dtype=torch.float32)
        return cls(V=z(n, R), Vh=z(R, n), S=torch.ones(R, device=device), Vs=z(n, R), cb=cb, device=device)

    def load(self, *, V, Vh, S, Vs) -> None:
        """Copy a layer's basis into this layer's buffers and refresh every derived operand in place."""
        self.opV.reload(V)
        self.opVh.reload(Vh)
        self.S.copy_(S)
        self.opVs.reload(Vs)
        self.opVsT.reload(Vs.t())
        if self._gram is not None:
            self._gram.refresh()

    def tab_ptrs(self):
        t = self.tab
        return ptr(t["base_abs"]), ptr(t["base_sqnorm"]), ptr(t["base_parity"]), ptr(t["idx_lut"]), ptr(t["grid"])


class E8VampState:
    """Device buffers of the VAMP loop for row blocks of B rows (reused from block to block)."""

    def __init__(self, B: int, n: int, R: int, iters: int, device):
        f32 = dict(device=device, dtype=torch.float32)
        self.B, self.n, self.R = B, n, R
        nb = n // 8
        self.r1 = torch.empty(B, n, **f32)
        self.x1 = torch.empty(B, n, **f32)
        self.r2 = torch.empty(B, n, **f32)
        self.r2_prev = torch.empty(B, n, **f32)
        self.u = torch.empty(B, R, **f32)
        self.P = torch.empty(B, R, **f32)
        self.gamma1 = torch.empty(B, **f32)
        self.rows = {k: torch.empty(B, **f32) for k in ("var", "g1w", "a1", "eta1", "g2n", "g2", "g2p", "a2", "eta2",
                                                          "g1n", "g1next", "trace", "resid")}
        self.flags = torch.zeros(8, device=device, dtype=torch.int32)
        self.round_counter = torch.zeros(1, device=device, dtype=torch.int32)  # the fused row stage's arrivals
        # per iteration: obs, mean alpha1, mean alpha2 (NaN for skipped iterations)
        self.hist = torch.empty(3, max(iters, 1), device=device, dtype=torch.float64)
        self.obs_hist, self.a1_hist, self.a2_hist = self.hist[0], self.hist[1], self.hist[2]
        self.chunks = _posterior_chunks(B, nb)
        self.work = torch.zeros(B * (self.chunks + 1), device=device, dtype=torch.int32)
        # row-scaled fp16 splits of the products' A operands (r2, u), written by their producers, and the split-K
        # partial planes of the two products (added by their consumers)
        h16 = dict(device=device, dtype=torch.float16)
        ldn, ldr = (n + 7) // 8 * 8, (R + 7) // 8 * 8
        self.r2_hi, self.r2_lo, self.r2_inv = torch.empty(B, ldn, **h16), torch.empty(B, ldn, **h16), torch.empty(B, **f32)
        self.u_hi, self.u_lo, self.u_inv = torch.empty(B, ldr, **h16), torch.empty(B, ldr, **h16), torch.empty(B, **f32)
        sms = ops.num_sms(torch.device(device))
        self.splits_p = ops.splitk_for(B, R, n, sms)
        self.splits_d = ops.splitk_for(B, n, R, sms)
        self.ws = torch.empty(max(self.splits_p * B * R, self.splits_d * B * n, 1), **f32)


def e8_vamp_device(st: E8VampState, ctl: torch.Tensor, L: E8Layer, *, Wr, hat0, center, pscale, tau: float, Y_u,
                   cfg: "E8P12VampConfig", em_active: bool) -> None:
    """Enqueue the VAMP iterations of one row block (mpq/solver.py:961-1122 with best_iterate off) on the current
    stream.  ctl holds the starting observation precision and receives the final one; nothing is read back."""
    B, n, R = st.B, st.n, st.R
    nb = n // 8
    rows, flags = st.rows, st.flags
    damping = float(cfg.damping)
    factor = max(float(cfg.gamma_retry_factor), 1.000001)
    retry_steps = max(int(cfg.gamma_retry_steps), 0)
    c = ptr(ctl)
    st.r1.copy_(hat0)
    call("mpq_gamma_init", ptr(Wr), ptr(hat0), B, n, Wr.stride(0), float(cfg.gamma_start), ptr(st.gamma1))
    tabs = L.tab_ptrs()
    iters = max(int(cfg.iters), 0)
    for it in range(iters):
        if it == 0:  # later iterations are opened by the previous commit
            call("mpq_vamp_ctl_begin", c, ptr(st.gamma1), ptr(rows["g1w"]), B, ptr(flags))
        for rnd in range(retry_steps + 1):
            final = int(rnd >= retry_steps)
            # retry rounds usually do nothing (the device skips them): only the first round's launch is timed
            # the posterior with the round's row stage fused behind it (the CTA completing a row's variance sum runs
            # that row's stage; the last row takes the round's decision)
            tok = trace.begin_timing("e8p12_mmse" if rnd == 0 else "e8p12_mmse_retry")
            call("mpq_e8p12_mmse_rows_round_ctl", ptr(st.r1), st.r1.stride(0), ptr(center),
                 center.stride(0) if center is not None else 0, ptr(pscale),
                 pscale.stride(0) if pscale is not None else 0, ptr(rows["g1w"]), tau, B, nb, *tabs, ptr(st.x1),
                 st.x1.stride(0), ptr(rows["var"]), st.chunks, ptr(st.work), c + 8, ptr(st.gamma1), ptr(rows["a1"]),
                 ptr(rows["eta1"]), ptr(rows["g2n"]), ptr(rows["g2"]), ptr(rows["g2p"]), ptr(rows["a2"]),
                 ptr(rows["eta2"]), ptr(rows["g1n"]), ptr(rows["g1next"]), ptr(rows["trace"]), ptr(flags), ptr(L.S), n,
                 R, damping, final, c, factor, ptr(st.round_counter))
            trace.end_timing("e8p12_mmse" if rnd == 0 else "e8p12_mmse_retry", tok,
                             4.0 * B * n * (3 if center is not None else 2) + 8.0 * B
                             + (4.0 * B * nb if pscale is not None else 0.0))
        # r2 and its fp16 split -> P = r2 V (partial planes) -> linear epilogue (adds the planes, writes u split)
        # -> D = u V^T (partial planes) -> r1 update (adds the planes)
        call("mpq_vamp_r2_split_ctl", ptr(st.x1), ptr(st.r1), ptr(st.r2_prev), ptr(st.r2), ptr(rows["eta1"]),
             ptr(rows["g1w"]), ptr(rows["g2n"]), B, n, st.r2.stride(0), damping, ptr(st.r2_hi), ptr(st.r2_lo),
             st.r2_hi.stride(0), ptr(st.r2_inv), c)
        Bh, Bl, Bi = L.opVh.f16
        status = ops.status_word(L.dev)
        tok = trace.begin_timing("gemm_tc")
        call("mpq_gemm_f16x3_parts", B, R, n, ptr(st.r2_hi), ptr(st.r2_lo), st.r2_hi.stride(0), ptr(st.r2_inv), ptr(Bh),
             ptr(Bl), Bh.stride(0), ptr(Bi), st.splits_p, ptr(st.ws), st.ws.numel(), ptr(status))
        trace.end_timing("gemm_tc", tok, 2.0 * B * R * n)
        call("mpq_linear_epilogue_parts_ctl", ptr(st.ws), st.splits_p, ptr(Y_u), Y_u.stride(0), ptr(L.S), ptr(rows["g2"]),
             B, R, ptr(st.u), ptr(st.u_hi), ptr(st.u_lo), st.u_hi.stride(0), ptr(st.u_inv), ptr(rows["resid"]), c)
        Bh, Bl, Bi = L.opV.f16
        tok = trace.begin_timing("gemm_tc")
        call("mpq_gemm_f16x3_parts", B, n, R, ptr(st.u_hi), ptr(st.u_lo), st.u_hi.stride(0), ptr(st.u_inv), ptr(Bh),
             ptr(Bl), Bh.stride(0), ptr(Bi), st.splits_d, ptr(st.ws), st.ws.numel(), ptr(status))
        trace.end_timing("gemm_tc", tok, 2.0 * B * R * n)
        call("mpq_vamp_r1_parts_ctl", ptr(st.ws), st.splits_d, ptr(st.r2), ptr(st.r1), ptr(rows["eta2"]), ptr(rows["g2"]),
             ptr(rows["g1n"]), B, n, st.r1.stride(0), damping, ptr(st.r2_prev) if damping < 1.0 else None, c)
        call("mpq_vamp_ctl_commit", c, ptr(st.gamma1), ptr(rows["g1next"]), ptr(rows["g2p"]), ptr(rows["g2"]),
             ptr(rows["resid"]), ptr(rows["trace"]), B, R, int(em_active), float(cfg.em_obs_precision_damping),
             float(cfg.em_obs_precision_min), float(cfg.em_obs_precision_max), ptr(st.obs_hist), ptr(rows["a1"]),
             ptr(rows["a2"]), ptr(st.a1_hist), ptr(st.a2_hist), it,
             ptr(rows["g1w"]) if it + 1 < iters else None, ptr(flags) if it + 1 < iters else None)


def vamp_ctl_stats(ctl_host, obs_hist_host, iters: int, a1_hist_host=None, a2_hist_host=None) -> Dict[str, Any]:
    """Host view of a finished loop's control block (int32 numpy array of 16) and per-iteration histories."""
    import numpy as np
    c = np.asarray(ctl_host, dtype=np.int32)
    obs = float(c[:2].view(np.float64)[0])
    live = lambda h: [float(v) for v in list(h)[:iters] if v == v] if h is not None else []
    hist = live(obs_hist_host)
    a1, a2 = live(a1_hist_host), live(a2_hist_host)
    return {"obs": obs, "obs_values": hist, "fail": int(c[_CTL_FAIL]), "alpha1_retry_count": int(c[_CTL_RETRY]),
            "alpha2_clip_count": int(c[_CTL_CLIP]), "gamma2_invalid_count": int(c[_CTL_INVALID]),
            "best_iter": int(c[_CTL_BEST]), "stop_iter": int(c[_CTL_STOP]),
            "alpha1_mean": float(sum(a1) / len(a1)) if a1 else 0.0,
            "alpha2_mean": float(sum(a2) / len(a2)) if a2 else 0.0}


def _e8_host_loop(*, Wr, hat0, B, n, nb, R, iters, cfg, obs, em_active, mmse, map_state, err_of, opV, opVh, S, Y_u,
                  tmpBR, dev, best_iterate=True, post_stats=None):
    """The E8P12 VAMP loop with the host deciding between launches (needed for the best-iterate test,
    mpq/solver.py:1089-1122, which restores the best iterate and stops, and for the per-iteration posterior
    diagnostics of log_stats: post_stats(r1, gamma1_work) -> (entropy, margin) of the accepted posterior)."""
    damping = float(cfg.damping)
    f32 = dict(device=dev, dtype=torch.float32)
    r1 = hat0.clone()
    gamma1 = torch.empty(B, **f32)
    call("mpq_gamma_init", ptr(Wr), ptr(hat0), B, n, Wr.stride(0), float(cfg.gamma_start), ptr(gamma1))

    best_err_mean = float("inf")
    best_iter_idx = -1
    stop_iter_idx = -1
    reported_iters = iters
    best_r1 = best_g1 = None
    best_obs = obs
    if best_iterate:
        hx, _ = map_state(r1, gamma1)
        best_err_mean = float(ops.mean_rows(err_of(hx)).item())
        best_r1, best_g1 = r1.clone(), gamma1.clone()

    x1 = torch.empty(B, n, **f32)
    r2 = torch.empty(B, n, **f32)
    r2_prev = torch.empty(B, n, **f32)
    have_prev = False
    u = torch.empty(B, R, **f32)
    rows = {k: torch.empty(B, **f32) for k in ("var", "g1w", "a1", "eta1", "g2n", "g2", "g2p", "a2", "eta2", "g1n",
                                               "g1next", "trace", "resid")}
    flags = torch.zeros(8, device=dev, dtype=torch.int32)
    em_mean_t = torch.zeros(1, **f32)
    factor = max(float(cfg.gamma_retry_factor), 1.000001)
    retry_steps = max(int(cfg.gamma_retry_steps), 0)
    alpha1_retry_count = alpha2_clip_count = gamma2_invalid_count = 0
    obs_values = []
    a1_values, a2_values, ent_values, mar_values = [], [], [], []
    for it in range(iters):
        rows["g1w"].copy_(gamma1)
        for retry_idx in range(retry_steps + 1):
            final = retry_idx >= retry_steps
            mmse(r1, rows["g1w"], x1, rows["var"])
            flags.zero_()
            call("mpq_vamp_rows", ptr(rows["var"]), ptr(gamma1), ptr(rows["g1w"]), ptr(rows["a1"]), ptr(rows["eta1"]),
                 ptr(rows["g2n"]), ptr(rows["g2"]), ptr(rows["g2p"]) if (have_prev and damping < 1.0) else None,
                 ptr(rows["a2"]), ptr(rows["eta2"]), ptr(rows["g1n"]), ptr(rows["g1next"]), ptr(rows["trace"]),
                 ptr(flags), ptr(S), B, n, nb, R, obs, damping, int(final))
            fl = flags.tolist()
            if fl[0] == 0:
                break
            if final:
                if fl[1] > 0:
                    raise RuntimeError(f"alpha1 invalid: expected all in ({ALPHA_EPS}, 1-{ALPHA_EPS}).")
                break
            alpha1_retry_count += int(fl[0])
            call("mpq_gamma_retry", ptr(rows["g1w"]), ptr(rows["var"]), B, nb, factor)
        if fl[2] > 0 or fl[3] > 0:
            gamma2_invalid_count += 1
            continue
        it_stats = post_stats(r1, rows["g1w"]) if post_stats is not None else None
        alpha2_clip_count += int(fl[4])
        call("mpq_vamp_r2", ptr(x1), ptr(r1), ptr(r2_prev) if (have_prev and damping < 1.0) else None, ptr(r2),
             ptr(rows["eta1"]), ptr(rows["g1w"]), ptr(rows["g2n"]), B, n, r2.stride(0), damping)
        P = ops.mm_nt(r2, opVh, tmpBR)
        call("mpq_linear_epilogue", ptr(P), ptr(Y_u), ptr(S), ptr(rows["g2"]), obs, B, R, P.stride(0), ptr(u),
             ptr(rows["resid"]))
        D = ops.mm_nt(u, opV, x1)
        call("mpq_vamp_r1", ptr(D), ptr(r2), ptr(r1), ptr(rows["eta2"]), ptr(rows["g2"]), ptr(rows["g1n"]), B, n,
             r1.stride(0), damping)
        gamma1.copy_(rows["g1next"])
        r2, r2_prev = r2_prev, r2
        rows["g2p"].copy_(rows["g2"])
        have_prev = True
        if em_active:
            ops.mean_rows(rows["resid"], rows["trace"], out=em_mean_t)
            em_mean = float(em_mean_t.item())
            beta_new = float(R / max(em_mean, 1e-12))
            beta = _log_damp_scalar(max(obs, 1e-12), beta_new, float(cfg.em_obs_precision_damping))
            obs = float(min(max(beta, float(cfg.em_obs_precision_min)), float(cfg.em_obs_precision_max)))
        obs_values.append(obs)
        a1_values.append(float(rows["a1"].mean()))
        a2_values.append(float(rows["a2"].mean()))
        if it_stats is not None:
            ent_values.append(it_stats[0])
            mar_values.append(it_stats[1])
        if best_iterate:
            hx, _ = map_state(r1, gamma1)
            cur = float(ops.mean_rows(err_of(hx)).item())
            if cur + max(1e-10, abs(best_err_mean) * 1e-8) < best_err_mean:
                best_err_mean = cur
                best_r1.copy_(r1)
                best_g1.copy_(gamma1)
                best_obs = obs
                best_iter_idx = it
            else:
                r1.copy_(best_r1)
                gamma1.copy_(best_g1)
                obs = float(best_obs)
                stop_iter_idx = it
                reported_iters = it + 1
                break

    mean = lambda v: float(sum(v) / len(v)) if v else 0.0
    extra = {"alpha1_mean": mean(a1_values), "alpha2_mean": mean(a2_values), "mean_entropy": mean(ent_values),
             "mean_margin": mean(mar_values)}
    return (r1, gamma1, obs, obs_values, (alpha1_retry_count, alpha2_clip_count, gamma2_invalid_count), best_err_mean,
            best_iter_idx, stop_iter_idx, reported_iters, extra)


@torch.inference_mode()
def solve_e8p12_rankspace_vamp(
    *,
    Wr: torch.Tensor,
    hatWr_init: torch.Tensor,
    cb: object,
    V: torch.Tensor,
    Vh: torch.Tensor,
    S: torch.Tensor,
    Vs: torch.Tensor,
    cfg: E8P12VampConfig,
    module_name: str = "",
    obs_precision_init: Optional[float] = None,
    log_stats: bool = True,
    debug_out: Optional[Dict[str, Any]] = None,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, Dict[str, Any]]:
    """Scalar-precision VAMP for QUIP E8P12 in rank space with the gram-metric polish (mpq/solver.py:853-1276).

    Returns (hatWr (B, n), Qidxs int64 (B, n/8), final_err (B,), stats)."""
    from .e8p12 import prior_scale_from_center, e8p12_map_rows
    from .codebook import factor_tables
    if not Wr.is_cuda:
        raise ValueError("solve_e8p12_rankspace_vamp requires CUDA tensors (there is no CPU path)")
    dev = Wr.device
    Wr = _f32c(Wr, dev)
    hat0 = _f32c(hatWr_init, dev)
    B, n = Wr.shape
    codesz = int(getattr(cb, "codesz", 8))
    if codesz != 8 or n % 8 != 0:
        raise ValueError(f"E8P12 solver expects n divisible by 8; got n={n}, codesz={codesz}.")
    nb = n // 8
    V, Vh, S, Vs = (_f32c(t, dev) for t in (V, Vh, S, Vs))
    R = int(S.numel())
    if R == 0:
        raise ValueError("rank-0 spectra are not supported by the CUDA solver")
    iters = max(int(cfg.iters), 0)
    reported_iters = iters
    damping = float(cfg.damping)
    tau = float(cfg.prior_tau)
    mode_scale = str(cfg.prior_tau_scale_mode or "absmax").strip().lower()
    tab = factor_tables(cb, dev)
    f32 = dict(device=dev, dtype=torch.float32)
    W_blocks = Wr.reshape(B, nb, 8)
    pscale = prior_scale_from_center(W_blocks, mode_scale).reshape(B, nb).contiguous() if tau > 0.0 else None
    center = Wr if tau > 0.0 else None
    opV, opVh = ops.Operand(V), ops.Operand(Vh)
    VsT = Vs.t().contiguous()
    opVs, opVsT = ops.Operand(Vs), ops.Operand(VsT)
    Y_u = ops.mm_nt(Wr, opVsT)  # FP32-faithful split product, once per solve
    tmpBR = torch.empty(B, R, **f32)

    def err_of(x, out=None):
        C = ops.mm_nt(x, opVsT, tmpBR)
        out = torch.empty(B, **f32) if out is None else out
        call("mpq_row_sqerr", ptr(Y_u), ptr(C), B, R, Y_u.stride(0), C.stride(0), ptr(out))
        return out

    if float(cfg.obs_precision) > 0.0:
        obs_start = float(cfg.obs_precision)
    elif obs_precision_init is not None and float(obs_precision_init) > 0.0:
        obs_start = float(obs_precision_init)
    else:
        obs_start = 1.0 / max(float(ops.mean_rows(err_of(hat0)).item()) / R, 1e-12)
    # algorithmic bytes of one posterior launch: r1 and x1 (and the prior centre), gamma and the row sums
    mmse_bytes = 4.0 * B * n * (3 if center is not None else 2) + 8.0 * B + (4.0 * B * nb if pscale is not None else 0.0)

    def mmse(r, g, x_out, vsum):
        tok = trace.begin_timing("e8p12_mmse")
        call("mpq_e8p12_mmse", ptr(r), r.stride(0), ptr(center), center.stride(0) if center is not None else 0,
             ptr(pscale), pscale.stride(0) if pscale is not None else 0, ptr(g), tau, B, nb, ptr(tab["base_abs"]),
             ptr(tab["base_sqnorm"]), ptr(tab["base_parity"]), ptr(tab["idx_lut"]), ptr(tab["grid"]), ptr(x_out),
             x_out.stride(0), None, 0, None, 0, None, 0, ptr(vsum))
        trace.end_timing("e8p12_mmse", tok, mmse_bytes)

    def map_state(r, g):
        return e8p12_map_rows(r, cb, gamma=g, center=center, pscale=pscale, prior_tau=tau)

    obs = float(obs_start)
    em_active = bool(cfg.em_obs_precision) and float(cfg.obs_precision) <= 0.0
    best_iterate = bool(getattr(cfg, "best_iterate", False))
    best_err_mean = float("inf")
    best_iter_idx = -1
    stop_iter_idx = -1

    extra: Dict[str, float] = {"mean_entropy": 0.0, "mean_margin": 0.0}
    if not best_iterate and not log_stats:
        # device-resident loop: one host synchronisation after the iterations instead of one per iteration
        L = E8Layer.__new__(E8Layer)
        L.dev, L.cb, L.R, L.tab, L._gram = dev, cb, R, tab, None
        L.V, L.Vh, L.S, L.Vs, L.VsT = V, Vh, S, Vs, VsT
        L.opV = opV if opV.f16 is not None else ops.Operand(V, "f16x3")
        L.opVh = opVh if opVh.f16 is not None else ops.Operand(Vh, "f16x3")
        L.opVs, L.opVsT = opVs, opVsT
        st_dev = E8VampState(B, n, R, iters, dev)
        ctl = vamp_ctl_new(dev, obs)
        e8_vamp_device(st_dev, ctl, L, Wr=Wr, hat0=hat0, center=center, pscale=pscale, tau=tau, Y_u=Y_u, cfg=cfg,
                       em_active=em_active)
        r1, gamma1 = st_dev.r1, st_dev.gamma1
        hist_h = st_dev.hist.cpu().tolist()
        cst = vamp_ctl_stats(ctl.cpu().numpy(), hist_h[0], iters, hist_h[1], hist_h[2])
        if cst["fail"]:
            raise RuntimeError(f"alpha1 invalid: expected all in ({ALPHA_EPS}, 1-{ALPHA_EPS}).")
        obs = cst["obs"]
        obs_values = cst["obs_values"]
        extra.update(alpha1_mean=cst["alpha1_mean"], alpha2_mean=cst["alpha2_mean"])
        alpha1_retry_count = cst["alpha1_retry_count"]
        alpha2_clip_count = cst["alpha2_clip_count"]
        gamma2_invalid_count = cst["gamma2_invalid_count"]
        factor = max(float(cfg.gamma_retry_factor), 1.000001)
        retry_steps = max(int(cfg.gamma_retry_steps), 0)
    else:
        from .e8p12 import posterior_stats

        def post_stats(r, g):
            ps = posterior_stats(r, g, cb, center=center, pscale=pscale, prior_tau=tau,
                                 blocks_per_chunk=int(cfg.blocks_per_chunk))
            return ps["entropy"], ps["margin"]

        r1, gamma1, obs, obs_values, counts, best_err_mean, best_iter_idx, stop_iter_idx, reported_iters, extra = \
            _e8_host_loop(Wr=Wr, hat0=hat0, B=B, n=n, nb=nb, R=R, iters=iters, cfg=cfg, obs=obs, em_active=em_active,
                          mmse=mmse, map_state=map_state, err_of=err_of, opV=opV, opVh=opVh, S=S, Y_u=Y_u, tmpBR=tmpBR,
                          dev=dev, best_iterate=best_iterate, post_stats=post_stats if log_stats else None)
        alpha1_retry_count, alpha2_clip_count, gamma2_invalid_count = counts
        factor = max(float(cfg.gamma_retry_factor), 1.000001)
        retry_steps = max(int(cfg.gamma_retry_steps), 0)

    final_hat, final_idx32 = map_state(r1, gamma1)
    final_idx = final_idx32.to(torch.int64)
    idxs_stage1 = final_idx
    final_err = err_of(final_hat)
    polish_sweeps = max(int(cfg.polish_sweeps), 0)
    polish_mode = _resolve_polish_mode(sweeps=polish_sweeps, mode=str(getattr(cfg, "polish_mode", "block_cd")))
    polish_metric = _resolve_e8p12_polish_metric(str(cfg.polish_metric or "gram"))
    polish_stats: Dict[str, Any] = {}
    polish_gain = polish_updates = 0.0
    if polish_mode != "none":
        err_before = final_err
        topk = None
        if polish_mode == "topk_block_cd":
            topk = build_e8p12_vamp_topk_candidates(
                r1=r1, gamma1=gamma1, Wr=Wr, cb=cb, blocks_per_chunk=int(getattr(cfg, "blocks_per_chunk", 64) or 64),
                prior_tau=tau, prior_tau_scale_mode=mode_scale, k=max(int(getattr(cfg, "topk_k", 16) or 16), 1))
        final_hat, final_idx, err_after, polish_stats = polish_e8p12_rankspace(
            x_init=final_hat, idxs_init=final_idx, Y_u=Y_u, Vs=Vs, cb=cb, sweeps=polish_sweeps,
            polish_mode=polish_mode, polish_metric=polish_metric,
            metric_rows_per_chunk=int(cfg.polish_metric_rows_per_chunk),
            polish_max_blocks=int(getattr(cfg, "polish_max_blocks", 0) or 0), _ops=(opVs, opVsT),
            topk_idxs=None if topk is None else topk["topk_idxs"], topk_vals=None if topk is None else topk["topk_vals"])
        if debug_out is not None and topk is not None and not bool(debug_out.get("summary_only", False)):
            debug_out["topk_idxs"] = topk["topk_idxs"].detach().to(device="cpu")
        del topk
        polish_gain = float((err_before.double() - err_after.double()).mean().item())
        polish_updates = float(polish_stats.get("accepted_updates", 0.0))
        final_err = err_after
    ops.check_status(dev)
    if debug_out is not None:
        g64 = gamma1.double()
        debug_out["solver"] = "e8p12_exact_vamp"
        debug_out["gamma1_sum"] = float(g64.sum())
        debug_out["gamma1_count"] = int(g64.numel())
        debug_out["gamma1_min"] = float(g64.min()) if B else 0.0
        debug_out["gamma1_max"] = float(g64.max()) if B else 0.0
        if bool(debug_out.get("summary_only", False)):
            debug_out["changed_count"] = int((idxs_stage1 != final_idx).sum().item())
            debug_out["changed_total"] = int(final_idx.numel())
        if bool(debug_out.get("capture_r1", False)):
            debug_out["r1"] = r1.detach().cpu()
        if not bool(debug_out.get("summary_only", False)):
            debug_out["gamma1"] = gamma1.detach().cpu()
        if bool(debug_out.get("capture_block_stats", False)):
            # per-block diagnostics at the VAMP fixed point (mpq/solver.py:96-145)
            from .e8p12 import posterior_stats, vamp_vector_discrete_mmse_e8p12
            post = vamp_vector_discrete_mmse_e8p12(r1_blocks=r1.reshape(B, nb, 8), gamma1=gamma1.reshape(B, 1), cb=cb,
                                                   blocks_per_chunk=int(cfg.blocks_per_chunk),
                                                   prior_center_blocks=W_blocks if tau > 0.0 else None,
                                                   prior_scale_blocks=pscale.reshape(B, nb, 1) if pscale is not None
                                                   else None, prior_tau=tau, prior_tau_scale_mode=mode_scale,
                                                   return_margin_blocks=True, return_entropy_blocks=True)
            debug_out["block_stats"] = {"top2_gap": post["margin_blocks"].float().cpu(),
                                        "entropy": post["entropy_blocks"].float().cpu(),
                                        "cov_trace": (8.0 * post["var1"].float()).cpu()}
    stats: Dict[str, Any] = {
        "solver": "e8p12_exact_vamp",
        "module": str(module_name),
        "iters": int(reported_iters),
        "rank": R,
        "nblocks": nb,
        "damping": damping,
        "prior_tau": tau,
        "prior_tau_scale_mode": mode_scale,
        "gamma_start": float(cfg.gamma_start),
        "gamma_retry_factor": float(factor),
        "gamma_retry_steps": int(retry_steps),
        "obs_precision_initial": float(obs_start),
        "obs_precision_final": float(obs),
        "obs_precision_mean": float(sum(obs_values) / len(obs_values)) if obs_values else float(obs),
        "alpha1_retry_count": int(alpha1_retry_count),
        "alpha2_clip_count": int(alpha2_clip_count),
        "gamma2_invalid_count": int(gamma2_invalid_count),
        "polish_sweeps": polish_sweeps,
        "polish_mode": polish_mode,
        "polish_metric": polish_metric,
        "polish_gain": polish_gain,
        "polish_updates": polish_updates,
        "polish_trace": polish_stats,
        "best_iterate_enabled": best_iterate,
        "best_iter": int(best_iter_idx),
        "stop_iter": int(stop_iter_idx),
        "best_rankspace_error_mean": float(best_err_mean) if best_iterate else 0.0,
        "rankspace_error_mean": float(ops.mean_rows(final_err).item()),
        "alpha1_mean": float(extra.get("alpha1_mean", 0.0)),
        "alpha2_mean": float(extra.get("alpha2_mean", 0.0)),
        "mean_entropy": float(extra.get("mean_entropy", 0.0)),
        "mean_margin": float(extra.get("mean_margin", 0.0)),
        "compile_prior": bool(getattr(cfg, "compile_prior", True)),
        "blocks_per_chunk": int(getattr(cfg, "blocks_per_chunk", 16)),
        "topk_k": int(getattr(cfg, "topk_k", 16)),
    }
    return final_hat, final_idx, final_err, stats
