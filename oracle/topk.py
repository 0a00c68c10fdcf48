"""CPU restatement of the top-k polish candidate sets and providers (TEST INFRASTRUCTURE ONLY).

mpq/priors/uniform.py:253-284 (uniform_map_topk), mpq/priors/e8p12.py:367-449 (_branch_factorized_map with
need_stats) and :453-538 (vamp_vector_map_topk_e8p12), mpq/polish/block_cd.py:657-685 (UniformTopKProvider) and
:93-101, :768-860 (_topk_metric_select_impl, E8P12TopKProvider).  float32 numpy.

Ordering: torch.topk leaves the order of equal scores unspecified; this restatement (and the CUDA kernels) break
ties by the candidate's position (lower grid level; lower flat index 2 (256 branch + abs) + s).
"""
import numpy as np

from . import e8p12 as OE
from .uniform_vamp import make_atoms, uniform_scores

f32 = np.float32


def _topk_desc(scores, k):
    """First k positions by (score descending, position ascending)."""
    order = np.argsort(-scores, axis=-1, kind="stable")[..., :k]
    return order, np.take_along_axis(scores, order, axis=-1)


def uniform_map_topk(*, r1, gamma1, scale_full, zero_full, maxq, prior_center, prior_tau, k):
    """mpq/priors/uniform.py:253-284."""
    atoms = make_atoms(scale_full.astype(f32), zero_full.astype(f32), maxq)
    scores = uniform_scores(r1.astype(f32), gamma1.astype(f32).reshape(-1, 1), scale_full.astype(f32),
                            None if prior_center is None else prior_center.astype(f32), prior_tau, atoms)
    k_eff = min(max(int(k), 1), maxq + 1)
    q, sc = _topk_desc(scores, k_eff)
    return {"topk_q": q.astype(np.int64), "topk_values": np.take_along_axis(atoms, q, axis=-1).astype(f32),
            "topk_scores": sc.astype(f32)}


def _branch_topk_stats(y, gamma, cache, branch):
    """mpq/priors/e8p12.py:367-449 with need_stats: per (item, abs) the best and second-best parity-valid sign
    patterns and their log-scores.  Sums over the 8 coordinates run sequentially (k = 0..7)."""
    base_abs = cache["base_abs"]
    N = y.shape[0]
    a = (gamma * y)[:, None, :] * base_abs[None, :, :]  # (N, 256, 8)
    y_norm = np.zeros(N, f32)
    for kk in range(8):
        y_norm = (y_norm + y[:, kk] * y[:, kk]).astype(f32)
    const = ((f32(-0.5) * gamma[:, 0])[:, None] * (y_norm[:, None] + cache["base_sqnorm"][None, :])).astype(f32)
    abs_a = np.abs(a)
    sum_abs = np.zeros(abs_a.shape[:2], f32)
    for kk in range(8):
        sum_abs = (sum_abs + abs_a[:, :, kk]).astype(f32)
    neg = a < 0
    parity = neg.sum(axis=2) & 1
    min_pos = abs_a.argmin(axis=2)  # first minimum
    min_abs = np.take_along_axis(abs_a, min_pos[..., None], axis=2)[..., 0]
    second = abs_a.copy()
    np.put_along_axis(second, min_pos[..., None], np.inf, axis=2)
    sec_pos = second.argmin(axis=2)
    sec_abs = np.take_along_axis(second, sec_pos[..., None], axis=2)[..., 0]
    mismatch = parity != cache["base_parity"][None, :]
    bits = (1 << np.arange(8, dtype=np.int64))
    sid = (neg.astype(np.int64) * bits).sum(axis=2)
    mb, sb = bits[min_pos], bits[sec_pos]
    best_sid = np.where(mismatch, sid ^ mb, sid)
    sec_sid = np.where(mismatch, sid ^ sb, sid ^ mb ^ sb)
    two = f32(2.0)
    best_lin = np.where(mismatch, (sum_abs - two * min_abs).astype(f32), sum_abs)
    sec_lin = np.where(mismatch, (sum_abs - two * sec_abs).astype(f32), (sum_abs - two * (min_abs + sec_abs)).astype(f32))
    lut = cache["idx_lut"][branch]
    ar = np.arange(256)[None, :]
    return ((const + best_lin).astype(f32), (const + sec_lin).astype(f32), lut[ar, best_sid], lut[ar, sec_sid])


def vamp_vector_map_topk_e8p12(*, r1_blocks, gamma1, cb, k, prior_center_blocks=None, prior_scale_blocks=None,
                               prior_tau=0.0):
    """mpq/priors/e8p12.py:453-538: candidates flattened as (branch, abs, {best, second})."""
    B, nb, _ = r1_blocks.shape
    rw, gw = OE._fold_prior(r1_blocks.astype(f32), gamma1.astype(f32).reshape(B, 1), prior_center_blocks,
                            prior_scale_blocks, prior_tau)
    y = rw.reshape(-1, 8)
    g = gw.reshape(-1, 1)
    cache = OE.factor_cache(cb)
    scores, idxs = [], []
    for br, off in enumerate((0.25, -0.25)):
        s1, s2, i1, i2 = _branch_topk_stats((y - f32(off)).astype(f32), g, cache, br)
        scores.append(np.stack([s1, s2], axis=-1))
        idxs.append(np.stack([i1, i2], axis=-1))
    S = np.stack(scores, axis=1).reshape(y.shape[0], -1)  # (N, 1024)
    I = np.stack(idxs, axis=1).reshape(y.shape[0], -1)
    k_eff = min(int(k), S.shape[1])
    pos, sc = _topk_desc(S, k_eff)
    ti = np.take_along_axis(I, pos, axis=1)
    if np.any(ti < 0):
        raise RuntimeError("failed to map factorized E8P12 top-k sign patterns back to full codebook indices.")
    return {"topk_idxs": ti.reshape(B, nb, k_eff), "topk_scores": sc.reshape(B, nb, k_eff).astype(f32)}


def uniform_topk_provider(topk_values, topk_q=None):
    """UniformTopKProvider.propose: the candidate nearest to the target (squared distance, first minimum)."""
    def propose(*, start, end, target, **_):
        cand = topk_values[:, start, :].astype(f32)  # (B, k)
        d = (cand - target.astype(f32)).astype(f32)
        best = np.argmin(d * d, axis=1)
        rows = np.arange(cand.shape[0])
        vals = cand[rows, best][:, None]
        return vals, None if topk_q is None else topk_q[:, start, :][rows, best].astype(np.int32)
    return propose


def e8p12_topk_provider(topk_idxs, grid):
    """E8P12TopKProvider.propose: gram metric |tL|^2 + |cL|^2 - 2 (tL).(cL) (clamped at 0, sums in coordinate order),
    otherwise the squared distance; first minimum."""
    grid = np.asarray(grid, f32)

    def propose(*, block_idx, target, metric, gram_chol, **_):
        ci = topk_idxs[:, block_idx, :]  # (B, k)
        cand = grid[ci]  # (B, k, 8)
        t = target.astype(f32)
        if metric == "gram":
            L = gram_chol.astype(f32)
            tm = np.zeros_like(t)
            cm = np.zeros_like(cand)
            for i in range(8):
                tm = (tm + t[:, i:i + 1] * L[i][None, :]).astype(f32)
                cm = (cm + cand[:, :, i:i + 1] * L[i][None, None, :]).astype(f32)
            tn = np.zeros(t.shape[0], f32)
            cn = np.zeros(cand.shape[:2], f32)
            cross = np.zeros(cand.shape[:2], f32)
            for j in range(8):
                tn = (tn + tm[:, j] * tm[:, j]).astype(f32)
                cn = (cn + cm[:, :, j] * cm[:, :, j]).astype(f32)
                cross = (cross + cm[:, :, j] * tm[:, None, j]).astype(f32)
            dist = np.maximum((tn[:, None] + cn) - f32(2.0) * cross, f32(0.0)).astype(f32)
        else:
            d = (cand - t[:, None, :]).astype(f32)
            dist = np.zeros(cand.shape[:2], f32)
            for j in range(8):
                dist = (dist + d[:, :, j] * d[:, :, j]).astype(f32)
        best = np.argmin(dist, axis=1)
        rows = np.arange(ci.shape[0])
        return cand[rows, best], ci[rows, best].astype(np.int64)
    return propose
