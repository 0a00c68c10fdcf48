"""Generic rank-space block coordinate descent with pluggable candidate providers.

Reference: mpq/polish/block_cd.py — CandidateProvider :12-25, BlockCDConfig :309-317,
block_coordinate_descent_rankspace :332-625, UniformScalarProvider :629-654, UniformTopKProvider :657-685,
E8P12Provider :688-764, E8P12TopKProvider :768-860.

Objective: minimise ||Y_u - x Vs||^2 over discrete block assignments proposed by a provider.  Two engines sit
behind one entry point:

* the E8P12 gram-metric recipe (E8P12Provider, metric "gram", greedy order over all blocks) runs the fused
  chunked CUDA kernels of ``mpq_b200.e8p12.gram_block_cd``;
* every other provider / metric / order runs the reference's per-block loop with device kernels for the
  target, the accept test and the residual products (``mpq_cd_target``, ``mpq_cd_accept``, GEMMs), calling
  ``provider.propose`` for each block, so user-defined providers plug in unchanged.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, Optional, Protocol, Tuple

import torch

from . import ops
from ._lib import call, ptr


class CandidateProvider(Protocol):
    def propose(self, *, block_idx: int, start: int, end: int, x_block: torch.Tensor, target: torch.Tensor,
                metric: str, gram_chol: Optional[torch.Tensor]) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        """Return (cand_vals (B, bs), cand_idxs (B,) or None) for this block."""


@dataclass(frozen=True)
class BlockCDConfig:
    sweeps: int = 3
    metric: str = "diag"  # "diag" | "gram"
    accept_tol: float = 0.0
    metric_rows_per_chunk: int = 0
    max_blocks_per_sweep: int = 0
    order_mode: str = "greedy_gain"  # "static" | "cyclic" | "greedy_gain"
    compile_steps: bool = True


@dataclass(frozen=True)
class UniformScalarProvider:
    """Nearest grid atom of the block's target (block_size 1)."""
    scale: torch.Tensor  # (B, n), group-expanded
    zero: torch.Tensor  # (B, n)
    maxq: int

    @torch.inference_mode()
    def propose(self, *, block_idx, start, end, x_block, target, metric, gram_chol):
        if end != start + 1:
            raise ValueError("UniformScalarProvider expects block_size=1.")
        B = target.shape[0]
        scale = self.scale.to(device=target.device, dtype=torch.float32)
        zero = self.zero.to(device=target.device, dtype=torch.float32)
        if scale.stride(-1) != 1 or zero.stride(-1) != 1 or scale.stride(0) != zero.stride(0):
            scale, zero = scale.contiguous(), zero.contiguous()
        q = torch.empty(B, 1, device=target.device, dtype=torch.uint8)
        x = torch.empty(B, 1, device=target.device, dtype=torch.float32)
        tg = target.to(torch.float32).contiguous()
        call("mpq_uniform_nearest", ptr(tg), tg.stride(0), ptr(scale[:, start:]), ptr(zero[:, start:]),
             scale.stride(0), 0, B, 1, int(self.maxq), ptr(q), ptr(x), 1)
        return x, q[:, 0].to(torch.int32)


@dataclass
class E8P12Provider:
    """Full-grid E8P12 proposal: exact gram-metric argmin (metric "gram") or the nearest codeword."""
    cb: object
    metric_rows_per_chunk: int = 0

    @torch.inference_mode()
    def propose(self, *, block_idx, start, end, x_block, target, metric, gram_chol):
        from .codebook import factor_tables
        from .e8p12 import e8p12_nearest, gram_search
        if (end - start) != int(getattr(self.cb, "codesz", 8)):
            raise ValueError("E8P12Provider expects block_size=codesz.")
        if metric == "gram":
            if gram_chol is None:
                raise ValueError("metric='gram' requires gram_chol.")
            idx = gram_search(target.contiguous(), gram_chol, self.cb)
            grid = factor_tables(self.cb, target.device)["grid"]
            return grid.index_select(0, idx.to(torch.int64)), idx.to(torch.int64)
        vals, idx = e8p12_nearest(target.contiguous(), self.cb)
        return vals, idx.to(torch.int64)


@dataclass
class UniformTopKProvider:
    """Nearest of the coordinate's precomputed top-k atoms (block_size 1, squared distance, first minimum)."""
    topk_values: torch.Tensor  # (B, n, k)
    topk_q: Optional[torch.Tensor] = None  # (B, n, k)
    _vals: Optional[torch.Tensor] = field(default=None, init=False, repr=False)
    _q: Optional[torch.Tensor] = field(default=None, init=False, repr=False)

    def _on_q(self, dev):
        if self._vals is None or self._vals.device != dev:
            self._vals = self.topk_values.to(device=dev, dtype=torch.float32).contiguous()
            self._q = None if self.topk_q is None else self.topk_q.to(device=dev, dtype=torch.int32).contiguous()
        return self._vals, self._q

    @torch.inference_mode()
    def propose(self, *, block_idx, start, end, x_block, target, metric, gram_chol):
        if end != start + 1:
            raise ValueError("UniformTopKProvider expects block_size=1.")
        dev = target.device
        self._on_q(dev)
        B, n, k = self._vals.shape
        tg = target.to(torch.float32).contiguous()
        out_v = torch.empty(B, 1, device=dev, dtype=torch.float32)
        out_q = None if self._q is None else torch.empty(B, device=dev, dtype=torch.int32)
        call("mpq_topk_pick", ptr(tg), tg.stride(0), ptr(self._vals[:, start]), n * k,
             ptr(None if self._q is None else self._q[:, start]), n * k, B, k, 1, None, ptr(out_v), 1, ptr(out_q))
        return out_v, out_q


@dataclass
class E8P12TopKProvider:
    """Best of the block's precomputed top-k E8P12 codewords: metric "gram" measures |(t - c) L|^2 through the
    block's Cholesky factor (|tL|^2 + |cL|^2 - 2 (tL).(cL), clamped at 0), otherwise |t - c|^2; first minimum."""
    cb: object
    topk_idxs: torch.Tensor  # (rows, nblocks, k)
    topk_vals: Optional[torch.Tensor] = None  # (rows, nblocks, k, 8); gathered from the grid when absent
    _idx: Optional[torch.Tensor] = field(default=None, init=False, repr=False)
    _vals: Optional[torch.Tensor] = field(default=None, init=False, repr=False)

    def _on(self, dev):
        if self._idx is None or self._idx.device != dev:
            self._idx = self.topk_idxs.to(device=dev, dtype=torch.int32).contiguous()
            if self.topk_vals is not None:
                self._vals = self.topk_vals.to(device=dev, dtype=torch.float32).contiguous()
            else:
                from .codebook import factor_tables
                grid = factor_tables(self.cb, dev)["grid"]
                self._vals = grid.index_select(0, self._idx.reshape(-1).to(torch.int64)).view(*self._idx.shape, 8)
        return self._idx, self._vals

    @torch.inference_mode()
    def propose(self, *, block_idx, start, end, x_block, target, metric, gram_chol):
        codesz = int(getattr(self.cb, "codesz", 8))
        if (end - start) != codesz:
            raise ValueError(f"E8P12TopKProvider expects block_size={codesz}, got {end - start}.")
        dev = target.device
        idx, vals = self._on(dev)
        B, nb, k = idx.shape
        chol = None
        if metric == "gram":
            if gram_chol is None:
                raise ValueError("metric='gram' requires gram_chol.")
            chol = gram_chol.to(device=dev, dtype=torch.float32).contiguous()
        tg = target.to(torch.float32).contiguous()
        out_v = torch.empty(B, 8, device=dev, dtype=torch.float32)
        out_i = torch.empty(B, device=dev, dtype=torch.int32)
        bi = int(block_idx)
        call("mpq_topk_pick", ptr(tg), tg.stride(0), ptr(vals[:, bi]), nb * k * 8, ptr(idx[:, bi]), nb * k, B, k, 8,
             ptr(chol), ptr(out_v), 8, ptr(out_i))
        return out_v, out_i.to(torch.int64)


def _resolve_blocks(n: int, block_size: int):
    if block_size <= 0:
        raise ValueError(f"block_size must be > 0, got {block_size}.")
    if n % block_size != 0:
        raise ValueError(f"n must be divisible by block_size; got n={n}, block_size={block_size}.")
    return [(s, s + block_size) for s in range(0, n, block_size)]


def hessian_objective_mean(*, target: torch.Tensor, x: torch.Tensor, gram: torch.Tensor) -> float:
    """mean_b (target - x)_b H (target - x)_b^T (mpq/linear.py:98-118)."""
    if target.shape != x.shape:
        raise ValueError(f"target/x shape mismatch: {tuple(target.shape)} != {tuple(x.shape)}")
    if x.numel() == 0:
        return 0.0
    D = torch.empty_like(x, dtype=torch.float32)
    B, n = x.shape
    t = target.to(torch.float32).contiguous()
    xx = x.to(torch.float32).contiguous()
    call("mpq_sub", ptr(t), ptr(xx), ptr(D), B, n, n)
    DG = ops.mm_nt(D, ops.Operand(gram.to(torch.float32).contiguous()))
    out = torch.empty(B, device=x.device, dtype=torch.float32)
    call("mpq_row_dot", ptr(DG), DG.stride(0), ptr(D), D.stride(0), B, n, ptr(out))
    return float(ops.mean_rows(out).item())


@torch.inference_mode()
def block_coordinate_descent_rankspace(*, x: torch.Tensor, Y_u: torch.Tensor, Vs: torch.Tensor, block_size: int,
                                       provider: CandidateProvider, cfg: BlockCDConfig,
                                       idxs_init: Optional[torch.Tensor] = None, snapshot_budgets=None,
                                       snapshots_out: Optional[Dict[int, torch.Tensor]] = None,
                                       raw_target: Optional[torch.Tensor] = None,
                                       raw_gram: Optional[torch.Tensor] = None):
    """Returns (x_new (B, n), idxs (provider-defined) or None, stats) as mpq/polish/block_cd.py:332-625."""
    sweeps = max(int(cfg.sweeps), 0)
    if sweeps <= 0 or x.numel() == 0 or Vs.numel() == 0:
        return x, idxs_init, {"accepted_updates": 0.0, "sweep_trace": [], "stabilized_objective_nonincreasing": True}
    metric = str(cfg.metric or "diag").strip().lower()
    if metric not in ("diag", "gram", "isotropic"):
        raise ValueError(f"unsupported metric={metric!r}; expected 'diag'|'gram'.")
    if metric == "isotropic":
        metric = "diag"
    order_mode = str(getattr(cfg, "order_mode", "greedy_gain") or "greedy_gain").strip().lower()
    if order_mode not in ("static", "cyclic", "greedy_gain"):
        raise ValueError(f"unsupported order_mode={order_mode!r}; expected 'static'|'cyclic'|'greedy_gain'.")
    if (raw_target is None) != (raw_gram is None):
        raise ValueError("raw_target and raw_gram must be provided together.")
    if not x.is_cuda:
        raise ValueError("block_coordinate_descent_rankspace requires CUDA tensors (there is no CPU path)")
    dev = x.device
    B, n = x.shape
    bs = int(block_size)
    blocks = _resolve_blocks(n, bs)
    if bs not in (1, 8):
        raise ValueError("block sizes 1 (scalar grids) and 8 (E8P12) are built")
    if metric == "gram" and bs != 8:
        raise ValueError("metric 'gram' needs 8-blocks")
    max_blocks = int(getattr(cfg, "max_blocks_per_sweep", 0) or 0)
    requested = {int(b) for b in (snapshot_budgets or set()) if 0 <= int(b) <= sweeps}

    fused_order = order_mode == "greedy_gain" and max_blocks == 0
    if (isinstance(provider, (E8P12Provider, E8P12TopKProvider)) and metric == "gram" and fused_order
            and idxs_init is not None):
        return _e8p12_gram_engine(x=x, Y_u=Y_u, Vs=Vs, cb=provider.cb, sweeps=sweeps, accept_tol=float(cfg.accept_tol),
                                  idxs_init=idxs_init, requested=requested, snapshots_out=snapshots_out,
                                  raw_target=raw_target, raw_gram=raw_gram,
                                  topk=provider if isinstance(provider, E8P12TopKProvider) else None)
    if (isinstance(provider, UniformTopKProvider) and provider.topk_q is not None and metric == "diag" and fused_order
            and idxs_init is not None and int(provider.topk_values.shape[-1]) <= 32):
        return _uniform_topk_engine(x=x, Y_u=Y_u, Vs=Vs, provider=provider, sweeps=sweeps,
                                    accept_tol=max(float(cfg.accept_tol), 0.0), idxs_init=idxs_init,
                                    requested=requested, snapshots_out=snapshots_out, raw_target=raw_target,
                                    raw_gram=raw_gram)
    return _generic_engine(x=x, Y_u=Y_u, Vs=Vs, bs=bs, blocks=blocks, provider=provider, metric=metric,
                           order_mode=order_mode, max_blocks=max_blocks, sweeps=sweeps,
                           accept_tol=max(float(cfg.accept_tol), 0.0), idxs_init=idxs_init, requested=requested,
                           snapshots_out=snapshots_out, raw_target=raw_target, raw_gram=raw_gram)


class _Trace:
    def __init__(self, raw_target, raw_gram, idxs0):
        self.items, self.raw_target, self.raw_gram, self.idxs0 = [], raw_target, raw_gram, idxs0

    def add(self, budget, res_norm, x, idxs, acc_sweep, acc_cum):
        it = {"budget": int(budget), "stabilized_objective_mean": float(ops.mean_rows(res_norm).item()),
              "accepted_updates_sweep": int(acc_sweep), "accepted_updates_cumulative": int(acc_cum),
              "assignment_changes_from_cd0": int((idxs != self.idxs0).sum().item())
              if idxs is not None and self.idxs0 is not None else 0,
              "assignments_total": int(idxs.numel()) if idxs is not None else 0}
        if self.raw_target is not None:
            it["raw_objective_mean"] = hessian_objective_mean(target=self.raw_target, x=x, gram=self.raw_gram)
        self.items.append(it)

    def stats(self, accepted, extra=None):
        vals = [it["stabilized_objective_mean"] for it in self.items]
        nonincreasing = all(b <= a + max(1e-8, abs(a) * 1e-7) for a, b in zip(vals, vals[1:]))
        out = {"accepted_updates": float(accepted), "sweep_trace": self.items,
               "stabilized_objective_nonincreasing": bool(nonincreasing)}
        out.update(extra or {})
        return out


def _e8p12_gram_engine(*, x, Y_u, Vs, cb, sweeps, accept_tol, idxs_init, requested, snapshots_out, raw_target,
                       raw_gram, topk=None):
    from .e8p12 import gram_block_cd
    dev = x.device
    idx0 = idxs_init.to(device=dev, dtype=torch.int64)
    tr = _Trace(raw_target, raw_gram, idx0)
    if snapshots_out is not None and 0 in requested:
        snapshots_out[0] = idx0.detach().cpu().clone()
    state = {"acc": 0}

    def on_sweep(sweep, x_work, idx, res_norm, accepted_total):
        idx64 = idx.to(torch.int64)
        tr.add(sweep, res_norm, x_work, idx64, accepted_total - state["acc"], accepted_total)
        state["acc"] = accepted_total
        if snapshots_out is not None and sweep in requested and sweep > 0:
            snapshots_out[sweep] = idx64.detach().cpu().clone()

    tv = ti = None
    if topk is not None:
        ti, tv = topk._on(dev)
    x_out, idx_out, st = gram_block_cd(x=x, Y_u=Y_u.to(torch.float32).contiguous(), Vs=Vs, cb=cb, sweeps=sweeps,
                                       idxs_init=idx0, accept_tol=accept_tol, on_sweep=on_sweep, topk_vals=tv,
                                       topk_idx=ti)
    return x_out.to(dtype=x.dtype), idx_out.to(getattr(cb, "idx_dtype", torch.int64)), tr.stats(
        st["accepted_updates"], {"exact_score_evals": st.get("exact_score_evals", 0)})


def _uniform_topk_engine(*, x, Y_u, Vs, provider, sweeps, accept_tol, idxs_init, requested, snapshots_out, raw_target,
                         raw_gram):
    """Scalar blocks, diag metric, greedy order with the top-k provider, in 128-column lazy blocks: per row one warp
    runs a block's sequential decisions against the block's rank-space grams G[J, J] (G = Vs Vs^T) in shared
    memory, and one GEMM applies the accepted steps to the right-hand side of every column."""
    dev = x.device
    B, n = x.shape
    R = int(Vs.shape[1])
    vals, qc = provider._on_q(dev)
    kc = int(vals.shape[2])
    if tuple(vals.shape) != (B, n, kc):
        raise ValueError(f"topk_values must be (B, n, k) = ({B}, {n}, k); got {tuple(vals.shape)}")
    x_work = x.to(torch.float32).contiguous().clone()
    Vs = Vs.to(device=dev, dtype=torch.float32).contiguous()
    opVs, opVsT = ops.Operand(Vs), ops.Operand(Vs.t().contiguous())
    res_u = ops.mm_nt(x_work, opVsT)
    res_norm = torch.empty(B, device=dev, dtype=torch.float32)
    Yc = Y_u.to(torch.float32).contiguous()
    call("mpq_residual", ptr(Yc), ptr(res_u), B, R, res_u.stride(0), ptr(res_norm))
    rhs = ops.mm_nt(res_u, opVs)  # residual_u Vs^T (B, n)
    del res_u
    G = ops.mm_nt(Vs, opVs)  # Vs Vs^T: the rank-space grams of every column pair
    diag = torch.empty(n, device=dev, dtype=torch.float32)
    diag_inv = torch.empty(n, device=dev, dtype=torch.float32)
    call("mpq_cd_diag", ptr(Vs), n, R, Vs.stride(0), ptr(diag), ptr(diag_inv))
    q = idxs_init.to(device=dev, dtype=torch.int32).reshape(B, n).contiguous().clone()
    tr = _Trace(raw_target, raw_gram, q.clone())
    if snapshots_out is not None and 0 in requested:
        snapshots_out[0] = q.detach().cpu().to(idxs_init.dtype).clone()
    tr.add(0, res_norm, x_work, q, 0, 0)
    gain = torch.empty(n, device=dev, dtype=torch.float32)
    order = torch.empty(n, device=dev, dtype=torch.int32)
    HJT = torch.empty(n, 128, device=dev, dtype=torch.float32)
    Hsub = torch.empty(128, 128, device=dev, dtype=torch.float32)
    delta = torch.empty(B, 128, device=dev, dtype=torch.float32)
    accepted = torch.zeros(1, device=dev, dtype=torch.int32)
    acc_prev = 0
    for sweep in range(1, sweeps + 1):
        call("mpq_cd_gain", ptr(rhs), B, n, rhs.stride(0), ptr(diag_inv), ptr(gain))
        call("mpq_argsort_desc", ptr(gain), n, ptr(order))
        for c0 in range(0, n, 128):
            K = min(128, n - c0)
            call("mpq_cd_gather", ptr(G), G.stride(0), n, ptr(order), c0, K, ptr(HJT), ptr(Hsub))
            call("mpq_cd_block_topk", ptr(x_work), x_work.stride(0), ptr(rhs), rhs.stride(0), ptr(vals), ptr(qc),
                 n * kc, kc, ptr(q), q.stride(0), ptr(diag), ptr(diag_inv), ptr(order), c0, K, ptr(Hsub),
                 ptr(res_norm), ptr(delta), ptr(accepted), B, float(accept_tol))
            ops.mm_nt(delta[:, :K], HJT[:, :K], out=rhs, alpha=-1.0, beta=1.0)
        acc_now = int(accepted.item())
        tr.add(sweep, res_norm, x_work, q, acc_now - acc_prev, acc_now)
        acc_prev = acc_now
        if snapshots_out is not None and sweep in requested:
            snapshots_out[sweep] = q.detach().cpu().clone()
    return x_work.to(dtype=x.dtype), q, tr.stats(acc_prev)


def _generic_engine(*, x, Y_u, Vs, bs, blocks, provider, metric, order_mode, max_blocks, sweeps, accept_tol, idxs_init,
                    requested, snapshots_out, raw_target, raw_gram):
    dev = x.device
    B, n = x.shape
    nb = len(blocks)
    x_work = x.to(torch.float32).contiguous().clone()
    Vs = Vs.to(device=dev, dtype=torch.float32).contiguous()
    R = int(Vs.shape[1])
    opVsT = ops.Operand(Vs.t().contiguous())
    residual = ops.mm_nt(x_work, opVsT)  # x Vs
    res_norm = torch.empty(B, device=dev, dtype=torch.float32)
    Yc = Y_u.to(torch.float32).contiguous()
    call("mpq_residual", ptr(Yc), ptr(residual), B, R, residual.stride(0), ptr(res_norm))
    diag = torch.empty(n, device=dev, dtype=torch.float32)
    diag_inv = torch.empty(n, device=dev, dtype=torch.float32)
    call("mpq_cd_diag", ptr(Vs), n, R, Vs.stride(0), ptr(diag), ptr(diag_inv))
    meta = None
    if bs == 8:
        meta = torch.empty(nb, 196, device=dev, dtype=torch.float32)
        fails = torch.zeros(1, device=dev, dtype=torch.int32)
        call("mpq_gram_meta", ptr(Vs), Vs.stride(0), R, nb, ptr(meta), ptr(fails))
        if int(fails.item()):
            raise RuntimeError("stabilize_cholesky failed for a block gram")
        grams = meta[:, :64].reshape(nb, 8, 8)
        chols = meta[:, 64:128].reshape(nb, 8, 8)
        ginvs = meta[:, 128:192].reshape(nb, 8, 8)
        importance = torch.diagonal(grams, dim1=1, dim2=2).sum(dim=1)
    else:
        grams = diag.reshape(nb, 1, 1)
        importance = diag
    static_order = torch.argsort(importance, descending=True, stable=True).tolist()
    opVs = ops.Operand(Vs)

    idxs = None
    if idxs_init is not None:
        idxs = idxs_init.to(device=dev, dtype=torch.int32).reshape(B, nb).contiguous().clone()
    idxs0 = None if idxs is None else idxs.clone()
    tr = _Trace(raw_target, raw_gram, idxs0)
    if snapshots_out is not None and idxs is not None and 0 in requested:
        snapshots_out[0] = idxs.detach().cpu().to(idxs_init.dtype).clone()
    tr.add(0, res_norm, x_work, idxs, 0, 0)

    accepted = torch.zeros(1, device=dev, dtype=torch.int32)
    rhs = torch.empty(B, bs, device=dev, dtype=torch.float32)
    target = torch.empty(B, bs, device=dev, dtype=torch.float32)
    delta = torch.empty(B, bs, device=dev, dtype=torch.float32)
    gain = torch.empty(nb, device=dev, dtype=torch.float32)
    order_t = torch.empty(nb, device=dev, dtype=torch.int32)
    idx_dtype = None
    acc_prev = 0
    for sweep in range(1, sweeps + 1):
        if order_mode == "greedy_gain":
            rhs_all = ops.mm_nt(residual, opVs)  # residual Vs^T (B, n)
            if metric == "gram":
                call("mpq_gram_gain", ptr(rhs_all), rhs_all.stride(0), B, nb, ptr(meta), ptr(gain))
            else:
                col_gain = torch.empty(n, device=dev, dtype=torch.float32)
                call("mpq_cd_gain", ptr(rhs_all), B, n, rhs_all.stride(0), ptr(diag_inv), ptr(col_gain))
                gain.copy_(col_gain.reshape(nb, bs).sum(dim=1) if bs > 1 else col_gain)
            del rhs_all
            call("mpq_argsort_desc", ptr(gain), nb, ptr(order_t))
            order = order_t.tolist()
        elif order_mode == "cyclic":
            order = list(range(nb))
        else:
            order = list(static_order)
        if max_blocks > 0:
            order = order[:max_blocks]
        for bi in order:
            s0, s1 = blocks[bi]
            Vb = Vs[s0:s1]
            ops.gemm_nt(residual, Vb, out=rhs)
            xb = x_work[:, s0:s1]
            call("mpq_cd_target", ptr(xb), x_work.stride(0), ptr(rhs), bs, B, bs,
                 ptr(ginvs[bi]) if metric == "gram" else None, None if metric == "gram" else ptr(diag_inv[s0:]),
                 ptr(target), bs)
            cand, cidx = provider.propose(block_idx=bi, start=s0, end=s1, x_block=xb, target=target, metric=metric,
                                          gram_chol=chols[bi] if metric == "gram" else None)
            cand = cand.to(device=dev, dtype=torch.float32).contiguous()
            ci = None
            if cidx is not None:
                if idx_dtype is None:
                    idx_dtype = cidx.dtype
                ci = cidx.to(device=dev, dtype=torch.int32).contiguous()
                if idxs is None:
                    idxs = torch.zeros(B, nb, device=dev, dtype=torch.int32)
            call("mpq_cd_accept", ptr(xb), x_work.stride(0), ptr(cand), cand.stride(0), ptr(rhs), bs, ptr(grams[bi]),
                 ptr(res_norm), B, bs, float(accept_tol), ptr(delta), bs, ptr(ci),
                 ptr(idxs[:, bi:]) if (ci is not None and idxs is not None) else None, nb, ptr(accepted))
            ops.gemm_nn(delta, Vb, out=residual, alpha=-1.0, beta=1.0)
        acc_now = int(accepted.item())
        tr.add(sweep, res_norm, x_work, idxs, acc_now - acc_prev, acc_now)
        acc_prev = acc_now
        if snapshots_out is not None and idxs is not None and sweep in requested:
            snapshots_out[sweep] = idxs.detach().cpu().clone()
    out_idx = None
    if idxs is not None:
        out_idx = idxs.to(idx_dtype or (idxs_init.dtype if idxs_init is not None else torch.int32))
    return x_work.to(dtype=x.dtype), out_idx, tr.stats(acc_prev)
