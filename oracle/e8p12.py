"""numpy restatement of the E8P12 codebook, its factorized posterior / MAP, and the gram-metric
block coordinate descent.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Codebook.  The QUIP# ``E8P12_codebook`` (lib/codebook/latticee8_padded12.py @ 1d8f873) is not
vendored with the reference.  Its construction is restated from the QUIP# paper (E8P, "E8 padded"):
256 absolute-value patterns from the half-integer coset of E8 — the 227 patterns of norm^2 <= 10 plus
29 of norm^2 12 — each combined with an even number of sign flips of its signed base pattern and a
+-1/4 shift, giving 2^16 points of E8 + 1/4.  Index layout (chosen so the reference's structural
asserts in mpq/priors/e8p12.py:83-151 hold): idx = (abs << 8) | s; parity p = popcount(s) & 1 selects
the shift (+1/4 even, -1/4 odd); the flip mask is s ^ p.  Which 29 norm-12 patterns pad the set and
the abs order are this restatement's choice (lexicographic), so indices are NOT pinned against real
QUIP# artifacts; the reference solver is pinned on this same codebook (tests/golden/e8p12_*.npz).
"""
from __future__ import annotations

import math
from typing import Any, Dict, Optional, Tuple

import numpy as np

f32 = np.float32
LOG2 = math.log(2.0)


def _cr(fn, x):
    """float32 result of a transcendental, correctly rounded (float64 evaluation, one rounding).

    torch's CPU float32 tanh/exp/log (what the reference runs) are correctly rounded for all but ~0.1-2% of
    inputs; numpy's float32 SIMD versions differ from correct rounding for 30-50%, which the reference's
    clamped-tanh algebra amplifies.  The float64 evaluation runs on torch's multi-threaded CPU kernels."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float64))
    return _TORCH_FN[fn](t).to(torch.float32).numpy()


def _torch_fns():
    import torch
    return {np.tanh: torch.tanh, np.exp: torch.exp, np.log: torch.log, np.log1p: torch.log1p, np.expm1: torch.expm1}


class _LazyFns(dict):
    def __missing__(self, key):
        self.update(_torch_fns())
        return dict.__getitem__(self, key)


_TORCH_FN = _LazyFns()


def _abs_patterns() -> np.ndarray:
    """256 x 8 abs patterns: the sorted abs patterns of half-integer E8 points with norm^2 <= 10 (227;
    every half-integer abs pattern has a signed version with even coordinate sum) followed by the first
    29, in lexicographic order, of the norm^2 = 12 patterns made of five 3/2 and three 1/2."""
    vals = np.array([0.5, 1.5, 2.5, 3.5])
    combos = np.stack(np.meshgrid(*([vals] * 8), indexing="ij"), axis=-1).reshape(-1, 8)
    small = combos[(combos ** 2).sum(axis=1) <= 10]
    small = np.asarray(sorted(map(tuple, small)))
    assert len(small) == 227
    two = np.array([0.5, 1.5])
    c12 = np.stack(np.meshgrid(*([two] * 8), indexing="ij"), axis=-1).reshape(-1, 8)
    pad = np.asarray(sorted(map(tuple, c12[(c12 ** 2).sum(axis=1) == 12])))
    assert len(pad) == 56
    return np.concatenate([small, pad[:29]]).astype(np.float32)


def _popcount8(s):
    s = np.asarray(s, dtype=np.int64)
    c = np.zeros_like(s)
    for k in range(8):
        c += (s >> k) & 1
    return c


class E8P12_codebook:
    """Stand-in with the attribute surface the reference reads: grid, grid_packed_abs, codesz,
    idx_dtype, quantize()."""

    codesz = 8

    def __init__(self):
        absp = _abs_patterns()  # (256, 8)
        base = absp.copy()
        odd = (np.rint(base.sum(axis=1)).astype(np.int64) % 2) == 1
        base[odd, 7] *= -1.0  # even coordinate sum -> point of the half-integer E8 coset
        self.base_signed = base
        s = np.arange(256, dtype=np.int64)
        p = _popcount8(s) & 1
        f = s ^ p
        flips = 1.0 - 2.0 * ((f[:, None] >> np.arange(8)[None, :]) & 1)  # (256, 8) +-1
        off = np.where(p == 1, -0.25, 0.25)
        grid = base[:, None, :] * flips[None, :, :] + off[None, :, None]
        self.grid = grid.reshape(65536, 8).astype(np.float32)
        self.grid_packed_abs = np.arange(256, dtype=np.int64)
        self.idx_dtype = np.int64

    def quantize(self, X, return_idx=True, **kw):
        """Nearest codeword: the factorized MAP with unit precision and no prior."""
        X = np.asarray(X, dtype=np.float32).reshape(-1, 8)
        idx = map_search(X, np.ones((X.shape[0], 1), np.float32), factor_cache(self))[0]
        vals = self.grid[idx]
        return (vals, idx) if return_idx else vals


_CACHE: Dict[int, Dict[str, np.ndarray]] = {}


def factor_cache(cb) -> Dict[str, np.ndarray]:
    """Same tables as mpq/priors/e8p12.py:83-151 (with its structural assertions)."""
    key = id(cb)
    if key in _CACHE:
        return _CACHE[key]
    grid = np.asarray(cb.grid, dtype=np.float32)
    base_template = grid[np.arange(256) << 8] - f32(0.25)
    base_sign_mask = (base_template < 0).astype(np.int64)
    base_parity = base_sign_mask.sum(axis=1) & 1
    base_abs = np.abs(base_template).astype(np.float32)
    base_sqnorm = (base_abs * base_abs).sum(axis=1, dtype=np.float32)
    full = np.arange(65536, dtype=np.int64)
    abs_idx = full >> 8
    branch = _popcount8(full & 255) & 1
    offset = np.where(branch == 1, f32(-0.25), f32(0.25)).astype(np.float32)
    residual = grid - offset[:, None]
    bits = (residual < 0).astype(np.int64)
    sign_id = (bits << np.arange(8)[None, :]).sum(axis=1)
    lut = np.full((2, 256, 256), -1, dtype=np.int64)
    lut[branch, abs_idx, sign_id] = full
    assert np.allclose(np.abs(residual), base_abs[abs_idx], atol=1e-6, rtol=1e-6)
    valid = (_popcount8(np.arange(256))[None, None, :] & 1) == base_parity[None, :, None]
    assert np.all(lut[np.broadcast_to(valid, lut.shape)] >= 0)
    assert np.all(lut[~np.broadcast_to(valid, lut.shape)] < 0)
    c = {"base_abs": base_abs, "base_parity": base_parity, "base_sqnorm": base_sqnorm, "idx_lut": lut}
    _CACHE[key] = c
    return c


def _branch_map(y, gamma, cache, branch):
    """mpq/priors/e8p12.py:367-449 (MAP part): per (item, abs) best parity-valid sign and its score.

    Float32 operation order: a = (gamma*y)*|b|; y_norm = sum_k y_k^2 (sequential k = 0..7);
    const = (-0.5*gamma) * (y_norm + |b|^2); linear = sum_k |a_k| (sequential) - 2*mismatch*min|a|.
    (torch CPU tensors with separate float32 multiplies and adds: the same roundings as numpy.)
    """
    import torch
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    base_abs = T(cache["base_abs"])  # (256, 8)
    yt, gt = T(y), T(gamma)
    gy = gt * yt  # (N, 8)
    a = gy[:, None, :] * base_abs[None, :, :]  # (N, 256, 8)
    y_norm = torch.zeros(yt.shape[0], dtype=torch.float32)
    for k in range(8):
        y_norm = y_norm + yt[:, k] * yt[:, k]
    const = (np.float32(-0.5) * gt[:, 0])[:, None] * (y_norm[:, None] + T(cache["base_sqnorm"])[None, :])
    abs_a = a.abs()
    sum_abs = torch.zeros(abs_a.shape[:2], dtype=torch.float32)
    for k in range(8):
        sum_abs = sum_abs + abs_a[:, :, k]
    neg = (a < 0)
    best_parity = neg.sum(dim=2) & 1
    min_abs, min_pos = abs_a.min(dim=2)  # first minimum
    mismatch = best_parity != T(cache["base_parity"])[None, :]
    bits = (1 << torch.arange(8, dtype=torch.int64))
    sid = (neg.to(torch.int64) * bits).sum(dim=2)
    sid = torch.where(mismatch, sid ^ bits[min_pos], sid)
    best_linear = sum_abs - np.float32(2.0) * mismatch.to(torch.float32) * min_abs
    best_logscore = const + best_linear
    idx = T(cache["idx_lut"][branch])[torch.arange(256)[None, :], sid]
    return best_logscore.numpy(), idx.numpy()


def _fold_prior(r1_blocks, gamma1, prior_center_blocks, prior_scale_blocks, prior_tau):
    """mpq/priors/e8p12.py:841-857: combine the channel message with the isotropic prior."""
    B, nb, _ = r1_blocks.shape
    g = np.broadcast_to(gamma1.astype(np.float32)[:, None, :], (B, nb, 1))
    if float(prior_tau) > 0.0 and prior_center_blocks is not None:
        sc = np.maximum(prior_scale_blocks.astype(np.float32), f32(1e-12))
        t = f32(max(float(prior_tau), 1e-12)) * sc
        pp = f32(1.0) / (t * t)
        gw = g + pp
        rw = (g * r1_blocks + pp * prior_center_blocks) / gw
        return rw.astype(np.float32), gw.astype(np.float32)
    return r1_blocks.astype(np.float32), np.ascontiguousarray(g, dtype=np.float32)


def prior_scale_from_center(center_blocks, mode="absmax"):
    """mpq/priors/e8p12.py:47-63."""
    mode = str(mode or "absmax").lower()
    if mode in ("none", "unit", "legacy"):
        return np.ones(center_blocks.shape[:-1] + (1,), np.float32)
    if mode in ("absmax", "exact_full", "exact_full_absmax"):
        s = np.abs(center_blocks).max(axis=-1, keepdims=True)
    elif mode in ("rms", "std"):
        s = np.sqrt((center_blocks * center_blocks).mean(axis=-1, keepdims=True))
    elif mode in ("mean_abs", "l1"):
        s = np.abs(center_blocks).mean(axis=-1, keepdims=True)
    else:
        raise ValueError(mode)
    return np.maximum(s.astype(np.float32), f32(1e-12))


def map_search(y, gamma, cache):
    """argmax over (branch, abs) of the factorized MAP score (mpq/priors/e8p12.py:603-611).
    y: (N, 8) folded message, gamma: (N, 1) folded precision.  Returns (idx, best_score)."""
    scores, idxs = [], []
    for b, off in enumerate((0.25, -0.25)):
        s, i = _branch_map((y - f32(off)).astype(np.float32), gamma, cache, b)
        scores.append(s)
        idxs.append(i)
    S = np.concatenate(scores, axis=1)  # (N, 512) in (branch, abs) order
    I = np.concatenate(idxs, axis=1)
    pos = S.argmax(axis=1)
    return I[np.arange(len(pos)), pos], S[np.arange(len(pos)), pos]


def vamp_vector_map_e8p12(*, r1_blocks, gamma1, cb, prior_center_blocks=None, prior_scale_blocks=None, prior_tau=0.0):
    """mpq/priors/e8p12.py:541-631."""
    B, nb, _ = r1_blocks.shape
    rw, gw = _fold_prior(r1_blocks, gamma1, prior_center_blocks, prior_scale_blocks, prior_tau)
    idx, _ = map_search(rw.reshape(-1, 8), gw.reshape(-1, 1), factor_cache(cb))
    return {"map_idxs": idx.reshape(B, nb), "map_vals": cb.grid[idx].reshape(B, nb, 8)}


def _log1mexp(x):
    return np.where(x < f32(-LOG2), _cr(np.log1p, -_cr(np.exp, x)), _cr(np.log, -_cr(np.expm1, x))).astype(np.float32)


def _branch_stats(y, gamma, offset, branch, cache):
    """mpq/priors/e8p12.py:169-308 (need_stats=False).

    Array work runs on torch CPU tensors (multi-threaded) in float32 with torch's own float32 CPU
    transcendentals, i.e. the reference's arithmetic when it runs on the CPU."""
    import torch
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    cr = lambda fn, x: fn(x)
    base_abs = T(cache["base_abs"])
    parity_even = T(cache["base_parity"] == 0)[None, :]
    yt, gt = T(y), T(gamma)
    a = (gt[:, :, None] * yt[:, None, :]) * base_abs[None, :, :]
    y_norm = (yt * yt).sum(dim=1, keepdim=True)
    const = np.float32(-0.5) * gt * (y_norm + T(cache["base_sqnorm"])[None, :])
    aa = a.abs()
    logC = (aa + cr(torch.log1p, cr(torch.exp, -2.0 * aa))).sum(dim=-1)  # logaddexp(a, -a)
    t = cr(torch.tanh, a).clamp(-0.99999988079071044921875, 0.99999988079071044921875)
    lpt = cr(torch.log, t.abs().clamp_min(1e-7)).sum(dim=-1)
    neg = ((t < 0).sum(dim=-1) & 1).bool()
    pabs = cr(torch.exp, lpt)
    prod = torch.where(neg, -pabs, pabs)
    lae = cr(torch.log1p, cr(torch.exp, lpt))  # logaddexp(0, lpt), lpt <= 0
    l1me = torch.where(lpt < -LOG2, cr(torch.log1p, -cr(torch.exp, lpt)), cr(torch.log, -cr(torch.expm1, lpt)))
    lop = torch.where(neg, l1me, lae)
    lom = torch.where(neg, lae, l1me)
    logZ = torch.where(parity_even, logC + lop - np.float32(LOG2), logC + lom - np.float32(LOG2))
    prefix = torch.ones_like(t)
    acc = torch.ones(t.shape[:2], dtype=torch.float32)
    for k in range(8):
        prefix[:, :, k] = acc
        acc = acc * t[:, :, k]
    de = 1.0 + prod
    do = 1.0 - prod
    de = torch.where(de.abs() > 1e-12, de, torch.ones_like(de))
    do = torch.where(do.abs() > 1e-12, do, torch.ones_like(do))
    sm = torch.empty_like(t)
    suffix = torch.ones(t.shape[:2], dtype=torch.float32)
    for k in reversed(range(8)):
        tk = t[:, :, k]
        ex = prefix[:, :, k] * suffix
        sm[:, :, k] = torch.where(parity_even, (tk + ex) / de, (tk - ex) / do)
        suffix = suffix * tk
    sm = torch.nan_to_num(sm, nan=0.0, posinf=0.0, neginf=0.0)
    off = np.float32(offset)
    mu_core = sm * base_abs[None, :, :]
    mu = mu_core + off
    second = T(cache["base_sqnorm"])[None, :] + np.float32(8 * offset * offset) + np.float32(2.0) * off * mu_core.sum(dim=-1)
    return {"log_component": (const + logZ).numpy(), "mu_component": mu.numpy(), "second_component": second.numpy()}


def vamp_vector_discrete_mmse_e8p12(*, r1_blocks, gamma1, cb, prior_center_blocks=None, prior_scale_blocks=None,
                                    prior_tau=0.0, chunk_items=4096):
    """mpq/priors/e8p12.py:815-968 (need_stats=False): posterior mean, per-block variance, MAP."""
    import torch
    B, nb, _ = r1_blocks.shape
    rw, gw = _fold_prior(r1_blocks, gamma1, prior_center_blocks, prior_scale_blocks, prior_tau)
    cache = factor_cache(cb)
    Y = rw.reshape(-1, 8)
    G = gw.reshape(-1, 1)
    N = Y.shape[0]
    x1 = np.empty((N, 8), np.float32)
    var1 = np.empty(N, np.float32)
    map_idx = np.empty(N, np.int64)
    for s0 in range(0, N, chunk_items):
        y = Y[s0:s0 + chunk_items]
        g = G[s0:s0 + chunk_items]
        outs = [_branch_stats((y - f32(o)).astype(np.float32), g, o, b, cache) for b, o in enumerate((0.25, -0.25))]
        lc = torch.from_numpy(np.concatenate([o["log_component"] for o in outs], axis=1))  # (n, 512)
        m = lc.max(dim=1, keepdim=True).values
        lz = m + torch.log(torch.exp(lc - m).sum(dim=1, keepdim=True))
        w = torch.exp(lc - lz)
        mu = torch.zeros((y.shape[0], 8), dtype=torch.float32)
        sec = torch.zeros(y.shape[0], dtype=torch.float32)
        for b in range(2):
            wb = w[:, b * 256:(b + 1) * 256]
            mu += (wb[:, :, None] * torch.from_numpy(outs[b]["mu_component"])).sum(dim=1)
            sec += (wb * torch.from_numpy(outs[b]["second_component"])).sum(dim=1)
        var = torch.clamp((sec - (mu * mu).sum(dim=1)) / np.float32(8.0), min=0.0).numpy()
        mu = mu.numpy()
        idx, _ = map_search(y, g, cache)
        hi = g[:, 0] >= f32(1e3)
        mu[hi] = cb.grid[idx[hi]]
        var[hi] = 0.0
        x1[s0:s0 + chunk_items] = mu
        var1[s0:s0 + chunk_items] = var
        map_idx[s0:s0 + chunk_items] = idx
    var1 = var1.reshape(B, nb)
    alpha1 = (gamma1.astype(np.float32) * var1.mean(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return {"x1_blocks": x1.reshape(B, nb, 8), "var1": var1, "map_idxs": map_idx.reshape(B, nb),
            "map_vals": cb.grid[map_idx].reshape(B, nb, 8), "alpha1": alpha1}


# ---------------------------------------------------------------------------------------------
# gram-metric block coordinate descent (mpq/polish/block_cd.py:332-625 with _cd_gram_step_impl :212-246)
# ---------------------------------------------------------------------------------------------

def stabilize_cholesky(gram, jitter=1e-6, max_tries=6):
    """mpq/linear.py:121-141 (float32)."""
    floor = float(np.abs(np.diagonal(gram)).max()) * jitter + jitter
    out = gram.astype(np.float32)
    for k in range(max_tries):
        try:
            return np.linalg.cholesky(out).astype(np.float32)
        except np.linalg.LinAlgError:
            out = (out + f32((2.0 ** k) * floor) * np.eye(out.shape[0], dtype=np.float32)).astype(np.float32)
    return np.linalg.cholesky(out).astype(np.float32)


def metric_grid(chol, grid):
    """gl = grid L (products and sums in index order k = 0..7, float32) and gn = |gl|^2 (order j = 0..7)."""
    gT = np.ascontiguousarray(grid.T, dtype=np.float32)
    cols = []
    for j in range(8):
        acc = np.zeros(grid.shape[0], np.float32)
        for k in range(8):
            if chol[k, j] != 0:  # exact zeros leave the float32 sum unchanged
                acc += gT[k] * chol[k, j]
        cols.append(acc)
    gn = np.zeros(grid.shape[0], np.float32)
    for j in range(8):
        gn += cols[j] * cols[j]
    return np.stack(cols, axis=1), gn


def gram_search(target, chol, grid, metric=None):
    """argmin_c of  |t L|^2 + |g L|^2 - 2 (t L).(g L)  over the full grid (first minimum).

    Float32 with the products and sums in index order k = 0..7 (the fixed order of the CUDA kernel):
    tl_j = sum_k t_k L[k, j]; gl_j likewise; score = (tn + gn) - 2 * sum_j tl_j gl_j.  `metric` is an
    optional precomputed metric_grid(chol, grid)."""
    tl = np.zeros((target.shape[0], 8), np.float32)
    for j in range(8):
        for k in range(8):
            tl[:, j] = tl[:, j] + target[:, k] * chol[k, j]
    gl, gn = metric if metric is not None else metric_grid(chol, grid)
    tn = np.zeros(target.shape[0], np.float32)
    for j in range(8):
        tn = tn + tl[:, j] * tl[:, j]
    glT = np.ascontiguousarray(gl.T)
    R, G, CH = target.shape[0], grid.shape[0], 4096
    best_s = np.full(R, np.inf, np.float32)
    best_i = np.zeros(R, np.int64)
    cross = np.empty((R, CH), np.float32)
    tmp = np.empty((R, CH), np.float32)
    rows = np.arange(R)
    for c0 in range(0, G, CH):  # grid tiles that stay in cache; strict < keeps the first minimum
        c1 = min(G, c0 + CH)
        cr, tp = cross[:, :c1 - c0], tmp[:, :c1 - c0]
        np.multiply(tl[:, 0:1], glT[0, None, c0:c1], out=cr)
        for j in range(1, 8):
            np.multiply(tl[:, j:j + 1], glT[j, None, c0:c1], out=tp)
            np.add(cr, tp, out=cr)
        np.add(tn[:, None], gn[None, c0:c1], out=tp)
        np.multiply(cr, np.float32(2.0), out=cr)
        np.subtract(tp, cr, out=tp)
        i = tp.argmin(axis=1)
        v = tp[rows, i]
        upd = v < best_s
        best_s = np.where(upd, v, best_s)
        best_i = np.where(upd, i + c0, best_i)
    return best_i


def block_metric_cache(Vs, cb):
    """Every 8-block's metric grid (the per-layer part of block_cd_gram), keyed like its metric_cache."""
    Vs = Vs.astype(np.float32)
    grid = np.asarray(cb.grid, np.float32)
    out = {}
    for bi in range(Vs.shape[0] // 8):
        vb = Vs[bi * 8:(bi + 1) * 8]
        out[bi] = metric_grid(stabilize_cholesky((vb @ vb.T).astype(np.float32)), grid)
    return out


def block_cd_gram(*, x, Y_u, Vs, cb, sweeps, idxs_init, accept_tol=0.0, metric_cache=None):
    """Gram-metric greedy block CD over 8-blocks (mpq/polish/block_cd.py:332-625, compiled-step path).
    `metric_cache` (dict, optional) keeps each block's metric grid across sweeps and calls."""
    B, n = x.shape
    x_work = x.astype(np.float32).copy()
    Vs = Vs.astype(np.float32)
    grid = np.asarray(cb.grid, np.float32)
    residual_u = (Y_u - x_work @ Vs).astype(np.float32)
    residual_norm = (residual_u * residual_u).sum(axis=1, dtype=np.float32)
    nb = n // 8
    meta = []
    for bi in range(nb):
        vb = Vs[bi * 8:(bi + 1) * 8]
        g = (vb @ vb.T).astype(np.float32)
        L = stabilize_cholesky(g)
        Linv = np.linalg.inv(L.astype(np.float64))
        ginv = (Linv.T @ Linv).astype(np.float32)
        meta.append((vb, g, L, ginv))
    ginv_stack = np.stack([m[3] for m in meta])
    idxs = idxs_init.copy()
    accepted = 0
    for _ in range(max(int(sweeps), 0)):
        rhs_all = (residual_u @ Vs.T).reshape(B, nb, 8)
        ds = np.einsum("bnk,nkl->bnl", rhs_all, ginv_stack)
        gain = (rhs_all * ds).sum(axis=2).mean(axis=0)
        order = np.argsort(-gain, kind="stable")
        for bi in order:
            vb, g, L, ginv = meta[bi]
            xb = x_work[:, bi * 8:(bi + 1) * 8]
            rhs = residual_u @ vb.T
            target = xb + rhs @ ginv
            mg = None
            if metric_cache is not None:
                mg = metric_cache.get(int(bi))
                if mg is None:
                    mg = metric_cache[int(bi)] = metric_grid(L, grid)
            best = gram_search(target.astype(np.float32), L, grid, metric=mg)
            out = grid[best]
            delta = out - xb
            cross_r = (rhs * delta).sum(axis=1)
            dn = np.maximum(((delta @ g) * delta).sum(axis=1), f32(0.0))
            cand = np.maximum(residual_norm + dn - f32(2.0) * cross_r, f32(0.0))
            acc = (cand + f32(1e-12)) < residual_norm * f32(1.0 + accept_tol)
            x_work[:, bi * 8:(bi + 1) * 8] = np.where(acc[:, None], out, xb)
            residual_u = residual_u - (delta * acc[:, None]) @ vb
            residual_norm = np.where(acc, cand, residual_norm).astype(np.float32)
            idxs[:, bi] = np.where(acc, best, idxs[:, bi])
            accepted += int(acc.sum())
    return x_work, idxs, {"accepted_updates": float(accepted)}


# ---------------------------------------------------------------------------------------------
# E8P12 VAMP loop (mpq/solver.py:853-1276) and the QUIP# per-linear driver (mpq/adapters/quip_sharp.py:396-878)
# ---------------------------------------------------------------------------------------------
from dataclasses import dataclass

from . import uniform_vamp as U


@dataclass(frozen=True)
class E8P12VampConfig:
    """mpq/solver.py:58-82 (fields used by the solve)."""
    iters: int = 16
    damping: float = 0.5
    gamma_start: float = 1.0
    gamma_retry_factor: float = 4.0
    gamma_retry_steps: int = 3
    prior_tau: float = 0.25
    prior_tau_scale_mode: str = "absmax"
    obs_precision: float = 0.0
    em_obs_precision: bool = True
    em_obs_precision_damping: float = 0.3
    em_obs_precision_min: float = 1e-4
    em_obs_precision_max: float = 1e8
    polish_sweeps: int = 3
    best_iterate: bool = False
    polish_mode: str = "block_cd"  # "block_cd" | "topk_block_cd"
    topk_k: int = 16


def solve_e8p12_rankspace_vamp(*, Wr, hatWr_init, cb, V, Vh, S, Vs, cfg, obs_precision_init=None, metric_cache=None):
    """mpq/solver.py:853-1276 (block_cd polish with the gram metric)."""
    Wr = Wr.astype(f32)
    hat0 = hatWr_init.astype(f32)
    B, n = Wr.shape
    nb = n // 8
    rank = int(S.size)
    damping = float(cfg.damping)
    tau = float(cfg.prior_tau)
    Wb = Wr.reshape(B, nb, 8)
    pscale = prior_scale_from_center(Wb, cfg.prior_tau_scale_mode) if tau > 0 else None
    pc = Wb if tau > 0 else None
    Y_u = (Wr @ Vs).astype(f32)
    if float(cfg.obs_precision) > 0:
        obs0 = float(cfg.obs_precision)
    elif obs_precision_init is not None and float(obs_precision_init) > 0:
        obs0 = float(obs_precision_init)
    else:
        dd = Y_u - hat0 @ Vs
        obs0 = 1.0 / max(float((dd * dd).mean(dtype=f32)), 1e-12)
    obs = obs0
    em_active = bool(cfg.em_obs_precision) and float(cfg.obs_precision) <= 0.0
    r1 = hat0.copy()
    d0 = Wr - hat0
    mse = np.maximum((d0 * d0).mean(axis=1, keepdims=True, dtype=f32), f32(1e-12))
    gamma1 = (f32(cfg.gamma_start) * (f32(0.25) / mse)).astype(f32)
    factor = max(float(cfg.gamma_retry_factor), 1.000001)
    retry_steps = max(int(cfg.gamma_retry_steps), 0)
    r2_prev = g2_prev = None
    retries = 0
    g2_invalid = 0

    def post(r, g):
        return vamp_vector_discrete_mmse_e8p12(r1_blocks=r.reshape(B, nb, 8), gamma1=g, cb=cb, prior_center_blocks=pc,
                                               prior_scale_blocks=pscale, prior_tau=tau)

    best = None
    best_err_mean = float("inf")
    best_iter = -1
    stop_iter = -1
    if cfg.best_iterate:
        p0 = post(r1, gamma1)
        bx = p0["map_vals"].reshape(B, n)
        be = U.vamp_rankspace_error(Y_u=Y_u, x=bx, Vs=Vs)
        best = dict(r1=r1.copy(), g1=gamma1.copy(), obs=obs)
        best_err_mean = float(be.mean(dtype=f32))
    for it in range(max(int(cfg.iters), 0)):
        g1w = gamma1
        for retry_idx in range(retry_steps + 1):
            p = post(r1, g1w)
            a1 = p["alpha1"]
            valid = U.alpha_valid_mask(a1)
            if valid.all():
                alpha1, x1 = a1, p["x1_blocks"].reshape(B, n)
                break
            if retry_idx >= retry_steps:
                if not np.isfinite(a1).all():
                    raise RuntimeError("alpha1 invalid")
                alpha1 = np.clip(U.nan_to_num(a1, 0.5, 1.0 - U.ALPHA_EPS, U.ALPHA_EPS), f32(U.ALPHA_EPS),
                                 f32(1.0 - U.ALPHA_EPS))
                x1 = p["x1_blocks"].reshape(B, n)
                break
            retries += int((~valid).sum())
            g1w = np.where(a1 <= f32(U.ALPHA_EPS), g1w / f32(factor), g1w)
            g1w = np.where(a1 >= f32(1.0 - U.ALPHA_EPS), g1w * f32(factor), g1w)
            g1w = np.maximum(g1w, f32(1e-12)).astype(f32)
        eta1 = g1w / alpha1
        g2n = np.maximum(U.nan_to_num(eta1 - g1w, 1e-12, 1e12, 1e-12), f32(1e-12))
        if not U.precision_valid_mask(g2n).all():
            g2_invalid += 1
            continue
        r2n = (eta1 * x1 - g1w * r1) / g2n
        if r2_prev is None or g2_prev is None or damping >= 1.0:
            g2, r2 = g2n, r2n
        else:
            g2 = U.log_damp_positive(g2_prev, g2n, damping)
            r2 = f32(1.0 - damping) * r2_prev + f32(damping) * r2n
        if not U.precision_valid_mask(g2).all():
            g2_invalid += 1
            continue
        x2, a2raw, res_u = U.linear_mmse_exact(r2, g2, Y_u=Y_u, V=V, Vh=Vh, S=S, obs_precision=obs)
        a2 = np.clip(U.nan_to_num(a2raw, 0.5, 1.0 - U.ALPHA_EPS, U.ALPHA_EPS), f32(U.ALPHA_EPS), f32(1.0 - U.ALPHA_EPS))
        if em_active and rank > 0:
            obs = U.em_update_obs_precision_rankspace(residual_u=res_u, gamma2=g2, S=S, obs_precision=obs,
                                                      num_obs=rank, damping=cfg.em_obs_precision_damping,
                                                      min_value=cfg.em_obs_precision_min,
                                                      max_value=cfg.em_obs_precision_max)
        eta2 = g2 / a2
        g1n = np.maximum(U.nan_to_num(eta2 - g2, 1e-12, 1e12, 1e-12), f32(1e-12))
        r1n = (eta2 * x2 - g2 * r2) / g1n
        if damping >= 1.0:
            gamma1, r1 = g1n, r1n
        else:
            gamma1 = U.log_damp_positive(gamma1, g1n, damping)
            r1 = (f32(1.0 - damping) * r1 + f32(damping) * r1n).astype(f32)
        r2_prev, g2_prev = r2, g2
        if cfg.best_iterate:
            ps = post(r1, gamma1)
            sx = ps["map_vals"].reshape(B, n)
            se = U.vamp_rankspace_error(Y_u=Y_u, x=sx, Vs=Vs)
            sm = float(se.mean(dtype=f32))
            if sm + max(1e-10, abs(best_err_mean) * 1e-8) < best_err_mean:
                best_err_mean = sm
                best = dict(r1=r1.copy(), g1=gamma1.copy(), obs=obs)
                best_iter = it
            else:
                r1, gamma1, obs = best["r1"].copy(), best["g1"].copy(), best["obs"]
                stop_iter = it
                break
    fin = vamp_vector_map_e8p12(r1_blocks=r1.reshape(B, nb, 8), gamma1=gamma1, cb=cb, prior_center_blocks=pc,
                                prior_scale_blocks=pscale, prior_tau=tau)
    hat = fin["map_vals"].reshape(B, n)
    idx = fin["map_idxs"]
    idx_stage1 = idx.copy()
    updates = 0.0
    if int(cfg.polish_sweeps) > 0 and str(getattr(cfg, "polish_mode", "block_cd")) == "topk_block_cd":
        # mpq/solver.py:1177-1215: top-k candidates from the final message, generic engine with the top-k provider
        from . import block_cd as OB
        from . import topk as OT
        tk = OT.vamp_vector_map_topk_e8p12(r1_blocks=r1.reshape(B, nb, 8), gamma1=gamma1, cb=cb,
                                           k=max(int(cfg.topk_k), 1), prior_center_blocks=pc,
                                           prior_scale_blocks=pscale, prior_tau=tau)
        hat, idx, st = OB.block_coordinate_descent_rankspace(
            x=hat, Y_u=Y_u, Vs=Vs, block_size=8, propose=OT.e8p12_topk_provider(tk["topk_idxs"], cb.grid),
            sweeps=int(cfg.polish_sweeps), metric="gram", order_mode="greedy_gain", idxs_init=idx)
        updates = st["accepted_updates"]
    elif int(cfg.polish_sweeps) > 0:
        hat, idx, st = block_cd_gram(x=hat, Y_u=Y_u, Vs=Vs, cb=cb, sweeps=int(cfg.polish_sweeps), idxs_init=idx,
                                     metric_cache=metric_cache)
        updates = st["accepted_updates"]
    err = U.vamp_rankspace_error(Y_u=Y_u, x=hat, Vs=Vs)
    stats = {"obs_precision_initial": obs0, "obs_precision_final": obs, "alpha1_retry_count": retries,
             "gamma2_invalid_count": g2_invalid, "polish_updates": updates, "best_iter": best_iter,
             "stop_iter": stop_iter, "changed_count": int((idx_stage1 != idx).sum())}
    return hat.astype(f32), idx, err, stats


def rtn_init(Wr, cb):
    """mpq/adapters/quip_sharp.py:212-241 with cb.quantize = nearest codeword."""
    m, n = Wr.shape
    vals, idx = cb.quantize(Wr.reshape(-1, 8))
    return vals.reshape(m, n).astype(f32), idx.reshape(m, n // 8)


def refine_codebook(*, Wr, Hr, cb, cfg: E8P12VampConfig, block_rows=128, jitter_base=1e-6, eigen_floor_scale=1e-6,
                    max_blocks=None):
    """mpq/adapters/quip_sharp.py:396-878 for the default recipe (mpq_init=rtn, solver=vamp, block_cd).
    max_blocks: solve only the first row blocks of the chain (the obs-precision warm start is still the layer's);
    the other rows keep their RTN codes."""
    from .layer import vamp_hessian_eigen
    m, n = Wr.shape
    hat0, idx0 = rtn_init(Wr, cb)
    lam, V, floor = vamp_hessian_eigen(Hr, jitter_base=jitter_base, floor_scale=eigen_floor_scale, fp64=True)
    Vh = np.ascontiguousarray(V.T)
    S = np.sqrt(lam).astype(f32)
    Vs = (V * S[None, :]).astype(f32)
    block_rows = min(m, max(int(block_rows), 1))
    ssq = 0.0
    cnt = 0
    for r0 in range(0, m, block_rows):
        du = (Wr[r0:r0 + block_rows] - hat0[r0:r0 + block_rows]) @ Vs
        ssq += float((du * du).sum(dtype=f32))
        cnt += du.size
    obs = 1.0 / max(ssq / max(cnt, 1), 1e-12)
    hat = hat0.copy()
    idx = idx0.copy()
    blocks = []
    mcache = {}
    for bi, r0 in enumerate(range(0, m, block_rows)):
        if max_blocks is not None and bi >= int(max_blocks):
            break
        rb = slice(r0, min(r0 + block_rows, m))
        h, i, e, st = solve_e8p12_rankspace_vamp(Wr=Wr[rb], hatWr_init=hat0[rb], cb=cb, V=V, Vh=Vh, S=S, Vs=Vs,
                                                 cfg=cfg, obs_precision_init=obs, metric_cache=mcache)
        hat[rb] = h
        idx[rb] = i
        if cfg.em_obs_precision and float(cfg.obs_precision) <= 0.0:
            obs = float(st["obs_precision_final"])
        blocks.append(st)
    return {"hatWr": hat, "Qidxs": idx, "rtn_hat": hat0, "rtn_idx": idx0, "V": V, "S": S, "Vs": Vs,
            "obs_precision_final": obs, "block_stats": blocks}


def posterior_stats_e8p12(*, r1_blocks, gamma1, cb, prior_center_blocks=None, prior_scale_blocks=None, prior_tau=0.0,
                          correctly_rounded=False):
    """Posterior diagnostics of mpq/priors/e8p12.py:815-968 with need_stats (per-block log-partition, entropy and
    top-2 log-score margin; the components' sign entropies and second-best sign patterns of :292-306).

    Float32 torch CPU arithmetic in the reference's formula order.  correctly_rounded evaluates tanh and the log
    of |tanh| in float64 and rounds once (the CUDA kernels' choice; on the fixtures' inputs it changes nothing).
    Returns logZ_blocks, entropy_blocks, margin_blocks (B x nb) and the means entropy, margin."""
    import torch
    if correctly_rounded:
        tanh = lambda x: torch.from_numpy(_cr(np.tanh, x.numpy()))
        log = lambda x: torch.from_numpy(_cr(np.log, x.numpy()))
    else:
        tanh, log = torch.tanh, torch.log
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    B, nb, _ = r1_blocks.shape
    rw, gw = _fold_prior(r1_blocks, gamma1, prior_center_blocks, prior_scale_blocks, prior_tau)
    cache = factor_cache(cb)
    Y = T(rw.reshape(-1, 8))
    G = T(gw.reshape(-1, 1))
    N = Y.shape[0]
    base_abs = T(cache["base_abs"])
    sqn = T(cache["base_sqnorm"])
    par = T(cache["base_parity"])
    even = (par == 0)[None, :]
    comps, entr, scores = [], [], []
    for offset in (0.25, -0.25):
        y = Y - np.float32(offset)
        a = (G[:, :, None] * y[:, None, :]) * base_abs[None, :, :]
        const = np.float32(-0.5) * G * ((y * y).sum(dim=1, keepdim=True) + sqn[None, :])
        logC = torch.logaddexp(a, -a).sum(dim=-1)
        t = tanh(a).clamp(-1.0 + 1e-7, 1.0 - 1e-7)
        lpt = log(t.abs().clamp_min(1e-7)).sum(dim=-1)
        neg = ((t < 0).sum(dim=-1) & 1).bool()
        pabs = torch.exp(lpt)
        prod = torch.where(neg, -pabs, pabs)
        l1me = torch.where(lpt < -LOG2, torch.log1p(-torch.exp(lpt)), torch.log(-torch.expm1(lpt)))
        lae = torch.logaddexp(torch.zeros_like(lpt), lpt)
        lzs = torch.where(even, logC + torch.where(neg, l1me, lae) - np.float32(LOG2),
                          logC + torch.where(neg, lae, l1me) - np.float32(LOG2))
        pre, acc = [], torch.ones_like(prod)
        for k in range(8):
            pre.append(acc)
            acc = acc * t[:, :, k]
        de = 1.0 + prod
        do = 1.0 - prod
        de = torch.where(de.abs() > 1e-12, de, torch.ones_like(de))
        do = torch.where(do.abs() > 1e-12, do, torch.ones_like(do))
        sm = torch.empty_like(t)
        suf = torch.ones_like(prod)
        for k in reversed(range(8)):
            ex = pre[k] * suf
            sm[:, :, k] = torch.where(even, (t[:, :, k] + ex) / de, (t[:, :, k] - ex) / do)
            suf = suf * t[:, :, k]
        sm = torch.nan_to_num(sm, nan=0.0, posinf=0.0, neginf=0.0)
        sign_ent = torch.where(torch.isfinite(lzs), (lzs - (a * sm).sum(dim=-1)).clamp_min(0.0), torch.zeros_like(lzs))
        aa = a.abs()
        sum_abs = aa.sum(dim=-1)
        min_abs, min_pos = aa.min(dim=-1)
        second = aa.clone()
        second.scatter_(-1, min_pos.unsqueeze(-1), float("inf"))
        min2 = second.min(dim=-1).values
        mismatch = ((a < 0).sum(dim=-1) & 1) != par[None, :]
        best_lin = sum_abs - 2.0 * mismatch.to(torch.float32) * min_abs
        second_lin = torch.where(mismatch, sum_abs - 2.0 * min2, sum_abs - 2.0 * (min_abs + min2))
        comps.append(const + lzs)
        entr.append(sign_ent)
        scores.append(torch.stack([const + best_lin, const + second_lin], dim=-1))
    lc = torch.stack(comps, dim=1).reshape(N, -1)
    lz = torch.logsumexp(lc, dim=-1)
    lw = lc - lz[:, None]
    w = torch.exp(lw)
    wlw = torch.where(torch.isfinite(lw), w * lw, torch.zeros_like(lw))
    ent = -wlw.sum(dim=1) + (w * torch.stack(entr, dim=1).reshape(N, -1)).sum(dim=1)
    top2 = torch.topk(torch.stack(scores, dim=1).reshape(N, -1), k=2, dim=-1).values
    margin = top2[:, 0] - top2[:, 1]
    return {"logZ_blocks": lz.view(B, nb).numpy(), "entropy_blocks": ent.view(B, nb).numpy(),
            "margin_blocks": margin.view(B, nb).numpy(), "entropy": float(ent.mean()), "margin": float(margin.mean())}
