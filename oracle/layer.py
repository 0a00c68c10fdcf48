"""numpy restatement of the per-linear scalar driver and its helpers.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

- block-Hadamard input rotation  (mpq/rotation.py:135-160, 325-340, 404-441)
- eigen decomposition + floor    (mpq/adapters/gptqmodel.py:276-310)
- GPTQ-style asymmetric min-max group parameters (GPTQModel ``Quantizer.find_params`` @ ed96f2e,
  un-vendored; restated from the published GPTQ quantizer, parity vs GPTQModel unpinned)
- serial row-block chain          (mpq/adapters/gptqmodel.py:911-1088)
- calibration Hessian             (H = X^T X / T, then + 0.01 * mean(diag) * I)
- GPTQ postprocess polish         (mpq/adapters/gptqmodel.py:1250-1470)
"""
from __future__ import annotations

import hashlib
import math
from typing import Any, Dict, Optional, Tuple

import numpy as np

from .uniform_vamp import UniformVampConfig, solve_uniform_rankspace_vamp, vamp_rankspace_error

f32 = np.float32


def stable_seed(key: str, base_seed: int = 0) -> int:
    """mpq/utils.py:10-21: sha256(key) little-endian 4 bytes + base_seed, mod 2^31-1."""
    digest = hashlib.sha256(str(key).encode("utf-8")).digest()
    extra = int.from_bytes(digest[:4], byteorder="little", signed=False)
    return int((int(base_seed) + extra) % (2**31 - 1))


def largest_pow2_factor(n: int) -> int:
    """mpq/rotation.py:17-21."""
    return int(n & -n)


def hadamard_last_dim(x: np.ndarray, had_dim: int) -> np.ndarray:
    """Normalized Sylvester Hadamard over blocks of ``had_dim`` of the last axis.

    Same butterfly order as mpq/rotation.py:135-157: the stage that runs while ``m`` rows
    remain combines row pairs (2i, 2i+1) of a (m, c) view into (a+b, a-b) and appends them
    to the column axis; then divides by sqrt(had_dim) in float32.
    """
    shape = x.shape
    N = int(np.prod(shape)) // had_dim
    y = x.astype(f32).reshape(N, had_dim, 1).copy()
    while y.shape[1] > 1:
        m, c = y.shape[1], y.shape[2]
        v = y.reshape(N, m // 2, 2, c)
        out = np.empty_like(v)
        out[:, :, 0, :] = v[:, :, 0, :] + v[:, :, 1, :]
        out[:, :, 1, :] = v[:, :, 0, :] - v[:, :, 1, :]
        y = out.reshape(N, m // 2, 2 * c)
    return (y.reshape(N, had_dim) / np.sqrt(f32(had_dim))).reshape(shape).astype(f32)


def right_block_hadamard(m: np.ndarray, signs: np.ndarray, had_dim: int) -> np.ndarray:
    """mpq/rotation.py:432-434: (M * signs) then block Hadamard of the last dim."""
    return hadamard_last_dim(m.astype(f32) * signs[None, :].astype(f32), had_dim)


def right_block_hadamard_inverse(m: np.ndarray, signs: np.ndarray, had_dim: int) -> np.ndarray:
    """mpq/rotation.py:437-439."""
    return (hadamard_last_dim(m.astype(f32), had_dim) * signs[None, :].astype(f32)).astype(f32)


def vamp_hessian_eigen(H: np.ndarray, *, jitter_base=1e-6, floor_scale=1e-6, fp64=False):
    """mpq/adapters/gptqmodel.py:276-310 (fp32) / mpq/adapters/quip_sharp.py:33-67 (fp64)."""
    Hd = H.astype(np.float64 if fp64 else f32)
    Hd = (0.5 * (Hd + Hd.T)).astype(Hd.dtype)
    lam, V = np.linalg.eigh(Hd)
    lam = lam.astype(f32)
    V = V.astype(f32)
    max_lam = float(lam.max()) if lam.size else 0.0
    diag_mean = abs(float(np.diagonal(Hd).mean())) if Hd.size else 0.0
    floor = max(float(jitter_base), float(floor_scale) * max(diag_mean, max_lam, 1e-12))
    lam = np.maximum(lam, f32(floor))[::-1].copy()
    V = V[:, ::-1].copy()
    return lam, V, floor


def find_params_minmax(Wg: np.ndarray, maxq: int) -> Tuple[np.ndarray, np.ndarray]:
    """Asymmetric per-row min-max grid (published GPTQ quantizer; GPTQModel find_params @ ed96f2e
    is un-vendored, so this restatement is shared by oracle and product — parity vs GPTQModel unpinned).

    xmin = min(row_min, 0), xmax = max(row_max, 0); all-zero rows get [-1, 1];
    scale = (xmax - xmin) / maxq; zero = round(-xmin / scale).
    """
    xmin = np.minimum(Wg.min(axis=1), f32(0.0))
    xmax = np.maximum(Wg.max(axis=1), f32(0.0))
    tmp = (xmin == 0) & (xmax == 0)
    xmin = np.where(tmp, f32(-1.0), xmin)
    xmax = np.where(tmp, f32(1.0), xmax)
    scale = ((xmax - xmin) / f32(maxq)).astype(f32)
    zero = np.round(-xmin / scale).astype(f32)
    return scale[:, None], zero[:, None]


def hessian_from_calibration(X: np.ndarray, *, reg: float = 0.01) -> np.ndarray:
    """H = X^T X / T + reg * mean(diag) * I (the synthetic-config convention)."""
    T = X.shape[0]
    H = (X.T.astype(f32) @ X.astype(f32)) / f32(T)
    H = H + f32(reg) * np.diagonal(H).mean(dtype=f32) * np.eye(H.shape[0], dtype=f32)
    return H.astype(f32)


def rademacher_signs_torch(width: int, key: str, seed: int = 0) -> np.ndarray:
    """mpq/rotation.py:325-340.  Uses torch's CPU generator (the only torch use in the oracle)
    because the sign stream is defined by torch.randint with a seeded generator."""
    import torch
    g = torch.Generator(device="cpu")
    g.manual_seed(stable_seed(str(key), base_seed=int(seed)))
    s = torch.randint(0, 2, (int(width),), generator=g, dtype=torch.int64)
    return (s.to(torch.float32) * 2.0 - 1.0).numpy().astype(f32)


def run_scalar_layer(*, W, H, bits, group_size, vamp_cfg: UniformVampConfig, block_rows: int,
                     module_name: str = "layer", rotation: str = "internal_hadamard",
                     hessian_scale: float = 0.5, rotation_seed: int = 0,
                     jitter_base=1e-6, eigen_floor_scale=1e-6, desc_act: bool = False) -> Dict[str, Any]:
    """mpq/adapters/gptqmodel.py:650-1163 (vamp solver, no dead columns, no paired-matrix cache), with the CUDA
    polish semantics of mpq/solver.py:299-333.  desc_act (:700-738, :819-822): the solver-basis columns are
    ordered by descending Hessian diagonal, the Hessian is decomposed in that basis, and the outputs (Q, q_int,
    g_idx) are put back in column order."""
    W = W.astype(f32)
    rows, cols = W.shape
    maxq = 2 ** int(bits) - 1
    H_work = (f32(hessian_scale) * H.astype(f32)).astype(f32)
    lam = V = None
    if not desc_act:
        lam, V, floor = vamp_hessian_eigen(H_work, jitter_base=jitter_base, floor_scale=eigen_floor_scale)
    if rotation == "internal_hadamard":
        had = largest_pow2_factor(cols)
        signs = rademacher_signs_torch(cols, f"{module_name}:full", rotation_seed)
        W_work = right_block_hadamard(W, signs, had)
        Hm = right_block_hadamard(np.ascontiguousarray(H_work.T), signs, had).T.copy()
        Hm = right_block_hadamard(Hm, signs, had)
        if V is not None:
            V = right_block_hadamard(np.ascontiguousarray(V.T), signs, had).T.copy()
    else:
        had, signs = 1, None
        W_work, Hm = W, H_work
    invperm = None
    if desc_act:
        perm = np.argsort(-np.diagonal(Hm), kind="stable")
        invperm = np.argsort(perm, kind="stable")
        W_work = np.ascontiguousarray(W_work[:, perm])
        Hm = np.ascontiguousarray(Hm[perm][:, perm])
        lam, V, floor = vamp_hessian_eigen(Hm, jitter_base=jitter_base, floor_scale=eigen_floor_scale)
    Vh = np.ascontiguousarray(V.T)
    S = np.sqrt(lam).astype(f32)
    Vs = (V * S[None, :]).astype(f32)
    ng = (cols + group_size - 1) // group_size
    scale_g = np.empty((rows, ng), f32)
    zero_g = np.empty((rows, ng), f32)
    for gi in range(ng):
        sg, zg = find_params_minmax(W_work[:, gi * group_size:(gi + 1) * group_size], maxq)
        scale_g[:, gi] = sg[:, 0]
        zero_g[:, gi] = zg[:, 0]
    widths = [min(group_size, cols - gi * group_size) for gi in range(ng)]

    def expand(g):
        return np.repeat(g, widths, axis=1).astype(f32)

    block_rows = min(rows, max(int(block_rows), 1))
    if float(vamp_cfg.obs_precision) > 0.0:
        obs = float(vamp_cfg.obs_precision)
    else:
        ssq = 0.0
        cnt = 0
        for r0 in range(0, rows, block_rows):
            rb = slice(r0, min(r0 + block_rows, rows))
            sf, zf = expand(scale_g[rb]), expand(zero_g[rb])
            q = np.clip(np.round(W_work[rb] / sf) + zf, 0, maxq).astype(f32)
            xr = sf * (q - zf)
            du = (W_work[rb] - xr) @ Vs
            ssq += float((du * du).sum(dtype=f32))
            cnt += du.size
        obs = 1.0 / max(ssq / max(cnt, 1), 1e-12)
    obs_init = obs
    Q = np.empty_like(W_work)
    q_int = np.empty((rows, cols), np.uint8)
    blocks = []
    for r0 in range(0, rows, block_rows):
        rb = slice(r0, min(r0 + block_rows, rows))
        sf, zf = expand(scale_g[rb]), expand(zero_g[rb])
        q = np.clip(np.round(W_work[rb] / sf) + zf, 0, maxq).astype(f32)
        xr = (sf * (q - zf)).astype(f32)
        qi, xf, err, rerr, st = solve_uniform_rankspace_vamp(
            W=W_work[rb], x_rtn=xr, scale_full=sf, zero_full=zf, maxq=maxq, V=V, Vh=Vh, S=S, Vs=Vs,
            cfg=vamp_cfg, gram_full=Hm, obs_precision_init=obs)
        Q[rb] = xf
        q_int[rb] = qi.astype(np.uint8)
        if vamp_cfg.em_obs_precision:
            obs = float(st["obs_precision_final"])
        blocks.append(st)
    g_idx = (np.arange(cols) // int(group_size)).astype(np.int32)
    Q_solver, q_solver = Q, q_int
    if invperm is not None:
        Q = np.ascontiguousarray(Q[:, invperm])
        q_int = np.ascontiguousarray(q_int[:, invperm])
        g_idx = np.ascontiguousarray(g_idx[invperm])
    Q_out = right_block_hadamard_inverse(Q, signs, had) if signs is not None else Q
    return {"Q": Q_out, "Q_work": Q_solver, "q_int": q_int, "q_solver": q_solver, "scale": scale_g, "zero": zero_g,
            "g_idx": g_idx, "W_work": W_work, "H_metric": Hm, "V": V, "S": S, "Vs": Vs, "signs": signs, "had_dim": had,
            "invperm": invperm, "obs_precision_initial": obs_init, "obs_precision_final": obs, "block_stats": blocks}


def proxy_loss(W_work: np.ndarray, Q_work: np.ndarray, H: np.ndarray) -> float:
    """tr((W - Q) H (W - Q)^T) — the proxy loss of the acceptance bar."""
    d = (W_work - Q_work).astype(np.float64)
    return float(((d @ H.astype(np.float64)) * d).sum())


def postprocess_gptq(*, W, H, Q_init, scale_groups, zero_groups, g_idx, bits, polish_mode, polish_sweeps, topk_k=16,
                     vamp_cfg: Optional[UniformVampConfig] = None, hessian_scale=0.5, jitter_base=1e-6,
                     eigen_floor_scale=1e-6) -> Dict[str, Any]:
    """mpq/adapters/gptqmodel.py:1250-1470 with the generic block CD (the eager/compile backends): the GPTQ codes
    start a rank-space block CD (scalar provider, or the top-k provider with candidates from an auxiliary VAMP
    solve); per-row improve merge; fail closed on a non-finite or worse module mean."""
    from . import block_cd as OB
    from . import topk as OT
    from .uniform_vamp import dequant_from_q, nearest_atom_idx
    W = W.astype(f32)
    Q_init = Q_init.astype(f32)
    maxq = 2 ** int(bits) - 1
    H_work = (f32(hessian_scale) * H.astype(f32)).astype(f32)
    lam, V, _ = vamp_hessian_eigen(H_work, jitter_base=jitter_base, floor_scale=eigen_floor_scale)
    S = np.sqrt(lam).astype(f32)
    Vs = (V * S[None, :]).astype(f32)
    sf = scale_groups.astype(f32)[:, g_idx]
    zf = zero_groups.astype(f32)[:, g_idx]
    q_init = nearest_atom_idx(x=Q_init, scale_full=sf, zero_full=zf, maxq=maxq).astype(np.int32)
    Y_u = (W @ Vs).astype(f32)
    err_before = vamp_rankspace_error(Y_u=Y_u, x=Q_init, Vs=Vs)
    if polish_mode == "topk_block_cd":
        cfg = vamp_cfg or UniformVampConfig()
        from dataclasses import replace
        dbg: Dict[str, Any] = {}
        solve_uniform_rankspace_vamp(W=W, x_rtn=Q_init, scale_full=sf, zero_full=zf, maxq=maxq, V=V,
                                     Vh=np.ascontiguousarray(V.T), S=S, Vs=Vs, cfg=replace(cfg, polish_sweeps=0),
                                     gram_full=None, debug=dbg)
        tk = OT.uniform_map_topk(r1=dbg["r1"], gamma1=dbg["gamma1"], scale_full=sf, zero_full=zf, maxq=maxq,
                                 prior_center=W, prior_tau=float(cfg.prior_tau), k=int(topk_k))
        propose = OT.uniform_topk_provider(tk["topk_values"], tk["topk_q"])
    else:
        propose = OB.scalar_provider(sf, zf, maxq)
    _, q_p, st = OB.block_coordinate_descent_rankspace(x=Q_init, Y_u=Y_u, Vs=Vs, block_size=1, propose=propose,
                                                       sweeps=int(polish_sweeps), metric="diag",
                                                       order_mode="greedy_gain", idxs_init=q_init)
    q_p = q_p.astype(np.int32)
    x_p = dequant_from_q(q_int=q_p, scale_full=sf, zero_full=zf)
    err_after = vamp_rankspace_error(Y_u=Y_u, x=x_p, Vs=Vs)
    improve = (err_after + f32(1e-12)) < err_before
    Q_final = np.where(improve[:, None], x_p, Q_init).astype(f32)
    q_final = np.where(improve[:, None], q_p, q_init).astype(np.int32)
    err_final = vamp_rankspace_error(Y_u=Y_u, x=Q_final, Vs=Vs)
    fail = (not np.isfinite(err_final).all()) or float(err_final.mean()) > float(err_before.mean()) + 1e-9
    if fail:
        Q_final, q_final, err_final = Q_init, q_init, err_before
    return {"Q": Q_final, "q": q_final, "err_before": err_before, "err_final": err_final, "fail_closed": bool(fail),
            "accepted_updates": st["accepted_updates"]}
