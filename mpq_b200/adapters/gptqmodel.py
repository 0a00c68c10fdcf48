"""Per-linear grouped-scalar driver (the GPTQModel hook point).

Reference: mpq/adapters/gptqmodel.py:650-1163 (run_mpq_quantization), :276-310
(_vamp_hessian_eigen), :313-327 (_resolve_block_rows), :46-118 (_resolve_internal_rotation), :330-358
(_uniform_vamp_cfg_from_qcfg), :1250-1470 (postprocess_gptq_quantization: the MPQ polish of a GPTQ solution).

Only the default ``vamp`` solver is on this path; the research baselines (cdquant, quantease,
ojbkq) raise ``ValueError``.  ``desc_act`` (activation order) permutes the solver-basis columns by
descending Hessian diagonal as the reference does (:700-738) and un-permutes the outputs (:819-822).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

import torch

from .. import ops
from .._lib import call, ptr
from ..rotation import (apply_right_block_hadamard, apply_right_block_hadamard_inverse, resolve_block_hadamard_plan,
                        sample_rademacher_signs)
from ..solver import UniformVampConfig, solve_uniform_rankspace_vamp


@dataclass(frozen=True)
class GPTQAdapterConfig:
    hessian_scale: float = 0.5  # GPTQModel stores H = 2/m X^T X; 0.5 gives X^T X / m
    block_rows: int = 128
    jitter_base: float = 1e-6
    eigen_floor_scale: float = 1e-6
    rotation_seed: int = 0
    # True: grow block_rows to the memory budget as the reference does on CUDA
    # (mpq/adapters/gptqmodel.py:313-327).  False: use block_rows as given (parity pinning).
    grow_block_rows: bool = True
    # Optional dict shared by the linears of one layer: modules fed by the same input (q/k/v, gate/up) get the
    # same Hessian tensor, and its floored eigendecomposition (taken before the per-module rotation) is reused.
    eigen_cache: Optional[dict] = field(default=None, compare=False, hash=False)


@torch.inference_mode()
def vamp_hessian_eigen(H: torch.Tensor, *, jitter_base: float = 1e-6, floor_scale: float = 1e-6,
                       fp64: bool = False) -> Tuple[torch.Tensor, torch.Tensor, float]:
    """Floored, descending eigendecomposition (cuSOLVER through torch.linalg.eigh).

    mpq/adapters/gptqmodel.py:276-310 (fp32) and mpq/adapters/quip_sharp.py:33-67 (fp64).
    """
    Hd = H.to(torch.float64 if fp64 else torch.float32)
    Hd = 0.5 * (Hd + Hd.T)
    if not torch.isfinite(Hd).all():
        Hd = torch.nan_to_num(Hd, nan=0.0, posinf=0.0, neginf=0.0)
    lam, V = torch.linalg.eigh(Hd)
    lam = lam.to(torch.float32)
    V = V.to(torch.float32)
    max_lam = float(lam.max().item()) if lam.numel() else 0.0
    diag_mean = float(torch.diagonal(Hd).mean().abs().item()) if Hd.numel() else 0.0
    floor = max(float(jitter_base), float(floor_scale) * max(diag_mean, max_lam, 1e-12))
    lam = lam.clamp_min_(floor).flip(0).contiguous()
    V = V.flip(1).contiguous()
    return lam, V, float(floor)


def resolve_block_rows(rows: int, cols: int, maxq: int, requested: int, device: torch.device, grow: bool = True) -> int:
    """mpq/adapters/gptqmodel.py:313-327."""
    block_rows = min(int(rows), max(int(requested), 1))
    if not grow or device.type != "cuda":
        return block_rows
    with torch.cuda.device(device):
        free_bytes, _ = torch.cuda.mem_get_info()
    bytes_per_row = 4 * (8 * int(cols) + 4 * int(cols) * (int(maxq) + 1))
    budget = min(4 * 1024**3, int(free_bytes) // 2)
    auto = max(8, min(int(rows), int(budget // max(bytes_per_row, 1))))
    return min(int(rows), max(block_rows, int(auto)))


def group_params(W: torch.Tensor, group_size: int, maxq: int, quantizer: Any = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-(row, group) scale/zero.  With ``quantizer`` (a GPTQModel ``Quantizer``) its
    ``find_params`` is called per group as the reference does (:899-909); otherwise the CUDA
    min-max kernel (the restated asymmetric GPTQ grid) computes them."""
    rows, cols = W.shape
    ng = (cols + group_size - 1) // group_size
    if quantizer is not None and hasattr(quantizer, "find_params"):
        sc, zc = [], []
        for g in range(ng):
            quantizer.find_params(W[:, g * group_size:(g + 1) * group_size].contiguous(), weight=True)
            sc.append(quantizer.scale.to(torch.float32).reshape(rows, 1).clone())
            zc.append(quantizer.zero.to(torch.float32).reshape(rows, 1).clone())
        return torch.cat(sc, 1).contiguous(), torch.cat(zc, 1).contiguous()
    scale = torch.empty(rows, ng, device=W.device, dtype=torch.float32)
    zero = torch.empty(rows, ng, device=W.device, dtype=torch.float32)
    call("mpq_group_minmax", ptr(W), W.stride(0), rows, cols, int(group_size), int(maxq), ptr(scale), ptr(zero),
         scale.stride(0))
    return scale, zero


def _expand(g: torch.Tensor, group_size: int, cols: int) -> torch.Tensor:
    return torch.repeat_interleave(g, group_size, dim=1)[:, :cols].contiguous()


@torch.inference_mode()
def run_mpq_quantization(
    *,
    W: torch.Tensor,
    H: torch.Tensor,
    quantizer: Any,
    qcfg: Any,
    module_name: str,
    vamp_cfg: UniformVampConfig,
    adapter_cfg: GPTQAdapterConfig = GPTQAdapterConfig(),
) -> Tuple[torch.Tensor, Optional[torch.Tensor], Optional[torch.Tensor], Optional[torch.Tensor],
           Optional[torch.Tensor], float, Dict[str, Any]]:
    """Run MPQ on one linear layer given its weights and accumulated Hessian.

    Returns (Q dense float32 in the original basis, q_int uint8 in the solver basis,
    scale_groups, zero_groups, g_idx int32, quant_time_s, stats).
    """
    start = time.time()
    if not W.is_cuda:
        raise ValueError("run_mpq_quantization requires CUDA tensors (there is no CPU path)")
    device = W.device
    W = W.to(torch.float32).contiguous()
    H = H.to(device=device, dtype=torch.float32).contiguous()
    rows, cols = W.shape
    bits = int(getattr(qcfg, "bits"))
    maxq = int(2**bits - 1)
    group_size = int(getattr(qcfg, "group_size", cols))
    if group_size == -1:
        group_size = cols
    mpq_cfg = getattr(qcfg, "mpq", None)
    solver_name = str(getattr(mpq_cfg, "dispatch_solver", getattr(mpq_cfg, "solver", "vamp")) or "vamp").lower()
    if solver_name != "vamp":
        raise ValueError(f"unsupported GPTQModel MPQ solver={solver_name!r} (only 'vamp' is on the CUDA path).")
    use_activation_order = bool(getattr(qcfg, "desc_act", False))
    rotation = str(getattr(mpq_cfg, "rotation_mode", getattr(qcfg, "rotation", None) or "none") or "none").lower()
    if rotation not in {"none", "internal_hadamard", "model_hadamard", "model_random"}:
        raise ValueError("mpq only supports rotation in {none, model_hadamard, model_random, internal_hadamard}; "
                         f"got rotation={rotation!r}.")

    H_work = float(adapter_cfg.hessian_scale) * H
    cache = adapter_cfg.eigen_cache
    key = (H.data_ptr(), tuple(H.shape), float(adapter_cfg.hessian_scale), float(adapter_cfg.jitter_base),
           float(adapter_cfg.eigen_floor_scale))
    lam = V = None
    eigen_floor = 0.0
    if use_activation_order:
        pass  # (:716-721, :885-892) decomposed below in the permuted solver basis
    elif cache is not None and key in cache:
        lam, V, eigen_floor = cache[key]
    else:
        lam, V, eigen_floor = vamp_hessian_eigen(H_work, jitter_base=adapter_cfg.jitter_base,
                                                 floor_scale=adapter_cfg.eigen_floor_scale)
        if cache is not None:
            cache[key] = (lam, V, eigen_floor)
    signs = None
    had_dim = 1
    effective = rotation
    if rotation == "internal_hadamard":
        mode, had_dim = resolve_block_hadamard_plan(cols)
        if mode == "block":
            signs = sample_rademacher_signs(width=cols, key=f"{module_name}:full", seed=int(adapter_cfg.rotation_seed),
                                            device=device)
            effective = "internal_block_hadamard"
        else:
            effective = "none"
    if signs is not None:
        W_work = apply_right_block_hadamard(W, signs=signs, had_dim=had_dim)
        H_metric = apply_right_block_hadamard(H_work.T.contiguous(), signs=signs, had_dim=had_dim).T.contiguous()
        H_metric = apply_right_block_hadamard(H_metric, signs=signs, had_dim=had_dim)
        if V is not None:
            V = apply_right_block_hadamard(V.T.contiguous(), signs=signs, had_dim=had_dim).T.contiguous()
    else:
        W_work, H_metric = W, H_work.contiguous()
    activation_invperm = None
    if use_activation_order:
        # (:731-736) columns by descending Hessian diagonal in the solver basis; a stable sort keeps equal
        # diagonals in column order
        activation_perm = torch.argsort(torch.diagonal(H_metric), descending=True, stable=True)
        activation_invperm = torch.argsort(activation_perm)
        W_work = W_work.index_select(1, activation_perm).contiguous()
        H_metric = H_metric.index_select(0, activation_perm).index_select(1, activation_perm).contiguous()
    dead = torch.diagonal(H_metric) == 0
    has_dead = bool(dead.any().item())
    if has_dead:
        # mpq/adapters/gptqmodel.py:743-749
        H_metric = H_metric.clone()
        W_work = W_work.clone()
        H_metric[dead, dead] = 1
        W_work[:, dead] = 0
    if has_dead or V is None:
        # re-decomposition of the exact solver-basis Hessian (:885-892)
        lam, V, eigen_floor = vamp_hessian_eigen(H_metric, jitter_base=adapter_cfg.jitter_base,
                                                 floor_scale=adapter_cfg.eigen_floor_scale)
    V = V.contiguous()
    Vh = V.T.contiguous()
    S = torch.sqrt(lam).contiguous()
    Vs = (V * S.unsqueeze(0)).contiguous()
    R = int(S.numel())

    scale_groups, zero_groups = group_params(W_work, group_size, maxq, quantizer)
    block_rows = resolve_block_rows(rows, cols, maxq, int(adapter_cfg.block_rows), device,
                                    grow=bool(adapter_cfg.grow_block_rows))

    def block_params(rb):
        sg, zg = scale_groups[rb], zero_groups[rb]
        if cols % group_size == 0 and (group_size & (group_size - 1)) == 0:
            return sg.contiguous(), zg.contiguous()
        return _expand(sg, group_size, cols), _expand(zg, group_size, cols)

    def rtn(rb, sb, zb):
        Wb = W_work[rb]
        ld_p, gshift = ops.group_layout(sb, cols)
        x = torch.empty_like(Wb)
        call("mpq_uniform_rtn", ptr(Wb), Wb.stride(0), ptr(sb), ptr(zb), ld_p, gshift, Wb.shape[0], cols, maxq, None,
             ptr(x), x.stride(0))
        return x

    opVsT = ops.Operand(Vs.T.contiguous())
    if float(getattr(vamp_cfg, "obs_precision", 0.0)) > 0.0:
        obs_precision = float(vamp_cfg.obs_precision)
    else:
        sum_sq = 0.0
        count = 0
        for r0 in range(0, rows, block_rows):
            rb = slice(r0, min(r0 + block_rows, rows))
            sb, zb = block_params(rb)
            x_rtn = rtn(rb, sb, zb)
            delta = torch.empty_like(x_rtn)
            call("mpq_sub", ptr(W_work[rb]), ptr(x_rtn), ptr(delta), delta.shape[0], cols, delta.stride(0))
            diff_u = ops.mm_nt(delta, opVsT)
            zeros = torch.zeros_like(diff_u)
            e = torch.empty(diff_u.shape[0], device=device, dtype=torch.float32)
            call("mpq_row_sqerr", ptr(diff_u), ptr(zeros), diff_u.shape[0], R, diff_u.stride(0), zeros.stride(0), ptr(e))
            sum_sq += float(e.double().sum().item())
            count += int(diff_u.numel())
        obs_precision = 1.0 / float(max(sum_sq / max(count, 1), 1e-12))

    opHT = ops.Operand(H_metric.T.contiguous())  # (W - Q) @ H for the raw audit
    Q_work = torch.empty_like(W_work)
    q_int_work = torch.empty((rows, cols), dtype=torch.uint8, device=device)
    obs_block = float(obs_precision)
    layer_err_sum = 0.0
    raw_err_sum = 0.0
    rtn_err_sum = 0.0
    block_stats: List[Dict[str, Any]] = []
    gamma_sum, gamma_count = 0.0, 0
    for r0 in range(0, rows, block_rows):
        rb = slice(r0, min(r0 + block_rows, rows))
        sb, zb = block_params(rb)
        x_rtn = rtn(rb, sb, zb)
        dbg: Dict[str, Any] = {"summary_only": True}
        q_int, x_final, final_err, rtn_err, st = solve_uniform_rankspace_vamp(
            W=W_work[rb], x_rtn=x_rtn, scale_full=sb, zero_full=zb, maxq=maxq, V=V, Vh=Vh, S=S, Vs=Vs, cfg=vamp_cfg,
            gram_full=H_metric, obs_precision_init=obs_block, log_stats=False, debug_out=dbg)
        Q_work[rb] = x_final
        q_int_work[rb] = q_int.to(torch.uint8)
        layer_err_sum += float(final_err.double().sum().item())
        # raw Hessian audit (:1048-1056): (W - Q) H (W - Q)^T per row
        delta = torch.empty_like(x_final)
        call("mpq_sub", ptr(W_work[rb]), ptr(x_final), ptr(delta), delta.shape[0], cols, delta.stride(0))
        dH = ops.mm_nt(delta, opHT)
        raw = torch.empty(delta.shape[0], device=device, dtype=torch.float32)
        call("mpq_row_dot", ptr(dH), dH.stride(0), ptr(delta), delta.stride(0), delta.shape[0], cols, ptr(raw))
        raw_err_sum += float(raw.double().sum().item())
        rtn_err_sum += float(rtn_err.double().sum().item())
        if bool(getattr(vamp_cfg, "em_obs_precision", True)):
            obs_block = float(st.get("obs_precision_final", obs_block))
        gamma_sum += float(dbg.get("gamma1_sum", 0.0))
        gamma_count += int(dbg.get("gamma1_count", 0))
        block_stats.append(st)

    g_idx = torch.arange(cols, device=device, dtype=torch.int32) // int(group_size)
    if activation_invperm is not None:  # (:819-822)
        Q_work = Q_work.index_select(1, activation_invperm).contiguous()
        q_int_work = q_int_work.index_select(1, activation_invperm).contiguous()
        g_idx = g_idx.index_select(0, activation_invperm).contiguous()
    Q = apply_right_block_hadamard_inverse(Q_work, signs=signs, had_dim=had_dim) if signs is not None else Q_work
    stats: Dict[str, Any] = {
        "method": "mpq",
        "solver": solver_name,
        "module": str(module_name),
        "bits": bits,
        "group_size": group_size,
        "rotation_requested": rotation,
        "rotation_effective": effective,
        "rotation_internal": signs is not None,
        "rotation_block_dim": int(had_dim),
        "desc_act": bool(use_activation_order),
        "rows": int(rows),
        "cols": int(cols),
        "rank": R,
        "eigen_floor": float(eigen_floor),
        "block_rows": int(block_rows),
        "block_cd_backend": "cuda",
        "obs_precision_initial": float(obs_precision),
        "obs_precision_final": float(obs_block),
        "layer_error_sum": float(layer_err_sum),
        "stabilized_objective_mean_final": float(layer_err_sum / max(rows, 1)),
        "raw_objective_mean_final": float(raw_err_sum / max(rows, 1)),
        "rtn_error_sum": float(rtn_err_sum),
        "block_stats": block_stats,
        "quant_time_s": float(time.time() - start),
        "stage1_gamma1_mean": float(gamma_sum / max(gamma_count, 1)),
    }
    return Q, q_int_work, scale_groups, zero_groups, g_idx, float(time.time() - start), stats


def uniform_vamp_cfg_from_qcfg(qcfg: Any) -> UniformVampConfig:
    """mpq/adapters/gptqmodel.py:330-358: the scalar VAMP knobs from GPTQModel's ``qcfg.mpq``."""
    mpq_cfg = getattr(qcfg, "mpq", None)
    g = lambda k, d: getattr(mpq_cfg, k, d)
    backend = str(g("block_cd_backend", "") or "").strip().lower()
    if not backend:
        backend = "compile" if bool(g("compile_block_cd", False)) else "eager"
    return UniformVampConfig(
        iters=int(g("iters", 10)), damping=float(g("damping", 0.5)), final_decision=str(g("final_decision", "map") or "map"),
        init_from="rtn", gamma_start=float(g("gamma_start", 1.0)), gamma_retry_factor=float(g("gamma_retry_factor", 4.0)),
        gamma_retry_steps=int(g("gamma_retry_steps", 3)), prior_tau=float(g("prior_tau", 0.2)),
        obs_precision=float(g("obs_precision", 0.0)), em_obs_precision=bool(g("em_obs_precision", True)),
        em_obs_precision_damping=float(g("em_obs_precision_damping", 0.3)),
        em_obs_precision_min=float(g("em_obs_precision_min", 1e-4)),
        em_obs_precision_max=float(g("em_obs_precision_max", 1e8)), polish_sweeps=int(g("polish_sweeps", 3)),
        polish_mode=str(g("polish_mode", "block_cd") or "block_cd"), topk_k=int(g("topk_k", 16) or 16),
        vamp_backend=str(g("vamp_backend", "auto") or "auto"), compile_block_cd=bool(g("compile_block_cd", False)),
        block_cd_backend=backend)


def _tensor_sha256(t: torch.Tensor) -> str:
    """mpq/data.py:14-20: sha256 over dtype, shape and the C-order bytes."""
    import hashlib
    import json
    v = t.detach().to("cpu").contiguous()
    h = hashlib.sha256()
    h.update(str(v.dtype).encode("ascii"))
    h.update(json.dumps(list(v.shape), separators=(",", ":")).encode("ascii"))
    h.update(v.numpy().tobytes(order="C"))
    return h.hexdigest()


def _input_fingerprint(W: torch.Tensor, H: torch.Tensor, basis: str) -> Dict[str, Any]:
    """The paired (W, H) record of mpq/adapters/gptqmodel.py:121-144 with the on-disk cache disabled."""
    return {"protocol": "paired_w_h_sha256_v1", "w_sha256": _tensor_sha256(W), "h_sha256": _tensor_sha256(H),
            "w_shape": [int(d) for d in W.shape], "h_shape": [int(d) for d in H.shape], "basis": str(basis),
            "cache": "disabled"}


def _raw_objective(W: torch.Tensor, Q: torch.Tensor, opHT) -> torch.Tensor:
    """(W - Q) H (W - Q)^T per row."""
    d = torch.empty_like(W)
    call("mpq_sub", ptr(W), ptr(Q), ptr(d), d.shape[0], d.shape[1], d.stride(0))
    dH = ops.mm_nt(d, opHT)
    out = torch.empty(d.shape[0], device=W.device, dtype=torch.float32)
    call("mpq_row_dot", ptr(dH), dH.stride(0), ptr(d), d.stride(0), d.shape[0], d.shape[1], ptr(out))
    return out


@torch.inference_mode()
def postprocess_gptq_quantization(
    *,
    W: torch.Tensor,
    H: torch.Tensor,
    Q_init: torch.Tensor,
    scale_groups: torch.Tensor,
    zero_groups: torch.Tensor,
    g_idx: torch.Tensor,
    qcfg: Any,
    module_name: str,
    adapter_cfg: GPTQAdapterConfig = GPTQAdapterConfig(),
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, float, Dict[str, Any]]:
    """Polish a finished GPTQ solution in the rank space of H (mpq/adapters/gptqmodel.py:1250-1470).

    GPTQModel's own solve produced ``Q_init`` on the grid ``scale_groups``/``zero_groups`` (columns mapped to
    groups by ``g_idx``).  Its codes are the starting point of the rank-space block CD (``qcfg.mpq.polish_mode``
    "block_cd", or "topk_block_cd" with candidates from an auxiliary VAMP solve of the whole module); rows whose
    rank-space error does not drop keep the GPTQ codes, and the module keeps the GPTQ solution outright when the
    result is not finite or its mean error rose (fail closed).

    Returns (Q dense float32, q_int int32, scale_groups, zero_groups, g_idx int32, seconds, stats).
    """
    start = time.time()
    if not W.is_cuda:
        raise ValueError("postprocess_gptq_quantization requires CUDA tensors (there is no CPU path)")
    dev = W.device
    W = W.to(torch.float32).contiguous()
    H = H.to(device=dev, dtype=torch.float32).contiguous()
    Q_init = Q_init.to(device=dev, dtype=torch.float32).contiguous()
    scale_groups = scale_groups.to(device=dev, dtype=torch.float32)
    zero_groups = zero_groups.to(device=dev, dtype=torch.float32)
    g_idx = g_idx.to(device=dev, dtype=torch.int32)
    bits = int(getattr(qcfg, "bits"))
    maxq = int(2**bits - 1)
    rows, cols = W.shape
    block_rows = resolve_block_rows(rows, cols, maxq, int(adapter_cfg.block_rows), dev,
                                    grow=bool(adapter_cfg.grow_block_rows))
    gl = g_idx.to(torch.long)
    scale_full = scale_groups.index_select(1, gl).contiguous()
    zero_full = zero_groups.index_select(1, gl).contiguous()
    q_init8 = torch.empty(rows, cols, device=dev, dtype=torch.uint8)
    x_snap = torch.empty_like(Q_init)
    call("mpq_uniform_nearest", ptr(Q_init), Q_init.stride(0), ptr(scale_full), ptr(zero_full), scale_full.stride(0), 0,
         rows, cols, maxq, ptr(q_init8), ptr(x_snap), x_snap.stride(0))
    q_init = q_init8.to(torch.int32)

    mpq_cfg = getattr(qcfg, "mpq", None)
    H_work = float(adapter_cfg.hessian_scale) * H
    fingerprint = _input_fingerprint(W, H_work, str(getattr(mpq_cfg, "rotation_effective", "internal_block_hadamard")))
    lam, V, eigen_floor = vamp_hessian_eigen(H_work, jitter_base=adapter_cfg.jitter_base,
                                             floor_scale=adapter_cfg.eigen_floor_scale)
    V = V.contiguous()
    Vh = V.T.contiguous()
    S = torch.sqrt(lam).contiguous()
    Vs = (V * S.unsqueeze(0)).contiguous()
    VsT = Vs.T.contiguous()
    Y_u = ops.gemm_nt(W, VsT)  # W Vs in FP32
    opHT = ops.Operand(H_work.T.contiguous())

    polish_mode = str(getattr(mpq_cfg, "polish_mode", "none") or "none").strip().lower()
    polish_sweeps = int(getattr(mpq_cfg, "polish_sweeps", 0))
    vamp_cfg = uniform_vamp_cfg_from_qcfg(qcfg)
    err_before = ops.rankspace_error(Y_u, Q_init, VsT)
    raw_before = _raw_objective(W, Q_init, opHT)

    topk = None
    aux_stats: Dict[str, Any] = {}
    if polish_mode in {"topk_block_cd", "topk_cd", "topk", "vamp_topk"}:
        from dataclasses import replace
        aux_debug: Dict[str, Any] = {"capture_r1": True}
        aux_cfg = replace(vamp_cfg, init_from="rtn", polish_sweeps=0, polish_mode="none")
        _, _, _, _, aux_stats = solve_uniform_rankspace_vamp(
            W=W, x_rtn=Q_init, scale_full=scale_full, zero_full=zero_full, maxq=maxq, V=V, Vh=Vh, S=S, Vs=Vs,
            cfg=aux_cfg, gram_full=H_work, log_stats=False, debug_out=aux_debug)
        from ..solver import build_uniform_vamp_topk_candidates
        topk = build_uniform_vamp_topk_candidates(
            r1=aux_debug["r1"].to(dev), gamma1=aux_debug["gamma1"].to(dev), W=W, scale_full=scale_full,
            zero_full=zero_full, maxq=maxq, prior_tau=float(vamp_cfg.prior_tau), k=int(vamp_cfg.topk_k))

    from ..solver import polish_uniform_rankspace
    q_pol, x_pol, err_after, polish_stats = polish_uniform_rankspace(
        x_init=Q_init, Y_u=Y_u, Vs=Vs, scale_full=scale_full, zero_full=zero_full, maxq=maxq, sweeps=polish_sweeps,
        polish_mode=polish_mode, topk_values=None if topk is None else topk["topk_values"],
        topk_q=None if topk is None else topk["topk_q"], compile_block_cd=bool(vamp_cfg.compile_block_cd),
        block_cd_backend=str(vamp_cfg.block_cd_backend or ""), gram_full=H_work, raw_target=W, raw_gram=H_work)
    improve = (err_after + 1e-12 < err_before).unsqueeze(-1)
    Q_final = torch.where(improve, x_pol, Q_init)
    q_final = torch.where(improve, q_pol.to(torch.int32), q_init)
    err_final = ops.rankspace_error(Y_u, Q_final, VsT)
    before_mean = float(err_before.double().mean().item()) if err_before.numel() else 0.0
    final_mean = float(err_final.double().mean().item()) if err_final.numel() else 0.0
    fail_closed = (not bool(torch.isfinite(err_final).all().item())) or (final_mean > before_mean + 1e-9)
    if fail_closed:
        Q_final, q_final, err_final, final_mean = Q_init, q_init, err_before, before_mean
    raw_final = _raw_objective(W, Q_final, opHT)
    stats: Dict[str, Any] = {
        "method": "mpq",
        "solver": "gptq",
        "polish_mode": polish_mode,
        "module": str(module_name),
        "bits": bits,
        "group_size": int(getattr(qcfg, "group_size", cols)),
        "rows": int(rows),
        "cols": int(cols),
        "rank": int(S.numel()),
        "eigen_floor": float(eigen_floor),
        "block_rows": int(block_rows),
        "polish_sweeps": polish_sweeps,
        "topk_k": int(getattr(mpq_cfg, "topk_k", 16) or 16),
        "rankspace_error_mean_before": before_mean,
        "rankspace_error_mean_after": float(err_after.double().mean().item()) if err_after.numel() else 0.0,
        "rankspace_error_mean_final": final_mean,
        "raw_objective_mean_before": float(raw_before.double().mean().item()) if raw_before.numel() else 0.0,
        "raw_objective_mean_final": float(raw_final.double().mean().item()) if raw_final.numel() else 0.0,
        "polish_gain": float((err_before.double() - err_after.double()).mean().item()) if err_after.numel() else 0.0,
        "polish_updates": float(polish_stats.get("accepted_updates", 0.0)),
        "cd_trace": list(polish_stats.get("cd_trace") or polish_stats.get("sweep_trace") or []),
        "polish_assignment_changes": int((q_final != q_init).sum().item()),
        "polish_assignments_total": int(q_init.numel()),
        "block_cd_backend": str(polish_stats.get("block_cd_backend", vamp_cfg.block_cd_backend)),
        "module_fail_closed": bool(fail_closed),
        "aux_vamp": aux_stats if topk is not None else {},
        "quant_time_s": float(time.time() - start),
        "input_fingerprint": fingerprint,
    }
    bucket = getattr(mpq_cfg, "_layer_stats", None)
    if mpq_cfg is not None:
        if not isinstance(bucket, list):
            bucket = []
            setattr(mpq_cfg, "_layer_stats", bucket)
        bucket.append(stats)
    return Q_final, q_final, scale_groups, zero_groups, g_idx, float(time.time() - start), stats


@torch.inference_mode()
def resolve_internal_rotation(*, requested: str, cols: int, module_name: str, seed: int,
                              device: torch.device) -> Dict[str, Any]:
    """The rotation plan of one linear (mpq/adapters/gptqmodel.py:46-118): requested / effective basis, block
    Hadamard width and the module's Rademacher signs (None unless the internal block Hadamard applies)."""
    req = str(requested or "none").strip().lower()
    plan = {"requested": req or "none", "effective": req or "none", "mode": "none", "signs": None, "block_dim": 1,
            "fallback_reason": "", "internal": False}
    if req in {"", "none", "model_random", "model_hadamard"}:
        plan["requested"] = plan["effective"] = req or "none"
        return plan
    if req != "internal_hadamard":
        raise ValueError("mpq only supports rotation in {none, model_hadamard, model_random, internal_hadamard}; "
                         f"got rotation={requested!r}.")
    mode, block_dim = resolve_block_hadamard_plan(int(cols))
    if mode == "none":
        plan.update(effective="none", fallback_reason=f"unsupported_block_hadamard_width:{int(cols)}")
        return plan
    plan.update(effective="internal_block_hadamard", mode="block", block_dim=int(block_dim), internal=True,
                signs=sample_rademacher_signs(width=int(cols), key=f"{module_name}:full", seed=int(seed),
                                              device=device))
    return plan


@torch.inference_mode()
def prepare_gptq_internal_hadamard(*, W: torch.Tensor, H: torch.Tensor, qcfg: Any, module_name: str,
                                   adapter_cfg: GPTQAdapterConfig = GPTQAdapterConfig(),
                                   ) -> Tuple[torch.Tensor, torch.Tensor, Dict[str, Any]]:
    """W and H in the solver basis for GPTQModel's own solve (mpq/adapters/gptqmodel.py:593-633):
    W diag(s) Had and Had^T diag(s) H diag(s) Had, with the plan that undoes it."""
    mpq_cfg = getattr(qcfg, "mpq", None)
    plan = resolve_internal_rotation(
        requested=str(getattr(mpq_cfg, "rotation_mode", getattr(qcfg, "rotation", None) or "none")),
        cols=int(W.shape[1]), module_name=str(module_name), seed=int(adapter_cfg.rotation_seed), device=W.device)
    if float(adapter_cfg.hessian_scale) <= 0.0:
        raise ValueError(f"hessian_scale must be positive, got {float(adapter_cfg.hessian_scale)}")
    W32 = W.to(torch.float32).contiguous()
    H32 = H.to(device=W.device, dtype=torch.float32).contiguous()
    if not plan["internal"]:
        return W32, H32, plan
    s, had = plan["signs"], int(plan["block_dim"])
    W_work = apply_right_block_hadamard(W32, signs=s, had_dim=had)
    H_work = apply_right_block_hadamard(H32.T.contiguous(), signs=s, had_dim=had).T.contiguous()
    H_work = apply_right_block_hadamard(H_work, signs=s, had_dim=had).contiguous()
    return W_work, H_work, plan


@torch.inference_mode()
def finalize_gptq_internal_hadamard(*, Q_work: torch.Tensor, rotation_plan: Dict[str, Any]) -> torch.Tensor:
    """Back to the original basis (mpq/adapters/gptqmodel.py:636-648)."""
    if not bool(rotation_plan.get("internal", False)):
        return Q_work.to(torch.float32).contiguous()
    return apply_right_block_hadamard_inverse(Q_work.to(torch.float32), signs=rotation_plan["signs"],
                                              had_dim=int(rotation_plan["block_dim"])).contiguous()


@torch.inference_mode()
def install_internal_hadamard_input_hooks(model: torch.nn.Module, *, rotation_seed: int = 0) -> int:
    """Rotate the inputs of packed internal-Hadamard linears at load time (mpq/adapters/gptqmodel.py:1166-1247).

    The packed qweight/qzeros/scales of such a module hold the codes in the solver basis; the pre-hook applies
    the module's signed block Hadamard (same key "<module>:full" and seed as the solve) to its input, so the
    packed weights reproduce the dense inverse-rotated weights.  Returns the number of hooks installed."""
    installed = 0
    for name, module in model.named_modules():
        if not name or getattr(module, "_mpq_internal_hadamard_hook", None) is not None:
            continue
        if not all(hasattr(module, a) for a in ("qweight", "qzeros", "scales")):
            continue
        width = int(getattr(module, "in_features", 0) or getattr(module, "infeatures", 0) or 0)
        if width <= 0:
            qweight = getattr(module, "qweight", None)
            bits = int(getattr(module, "bits", 0) or 0)
            pdt = getattr(qweight, "dtype", torch.int32)
            pack_bits = torch.iinfo(pdt).bits if isinstance(pdt, torch.dtype) and not pdt.is_floating_point else 32
            if isinstance(qweight, torch.Tensor) and bits > 0:
                width = int(qweight.shape[0]) * int(pack_bits // bits)
        if width <= 0:
            raise RuntimeError(f"Cannot determine MPQ input width for quantized module {name!r}")
        mode, block_dim = resolve_block_hadamard_plan(width)
        if mode == "none":
            continue
        cache: Dict[torch.device, torch.Tensor] = {}

        def _rotate(_module, args, *, _name=name, _width=width, _block=block_dim, _cache=cache):
            if not args or not isinstance(args[0], torch.Tensor):
                return args
            v = args[0]
            if int(v.shape[-1]) != int(_width):
                raise RuntimeError(f"MPQ input width mismatch for {_name!r}: expected {_width}, got {int(v.shape[-1])}")
            s = _cache.get(v.device)
            if s is None:
                s = sample_rademacher_signs(width=int(_width), key=f"{_name}:full", seed=int(rotation_seed),
                                            device=v.device)
                _cache[v.device] = s
            return (apply_right_block_hadamard(v, signs=s, had_dim=int(_block)).to(v.dtype), *args[1:])

        module._mpq_internal_hadamard_hook = module.register_forward_pre_hook(_rotate)
        installed += 1
    return installed
