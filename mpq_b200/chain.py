"""Chained row-block E8P12 layer solve on one GPU.

The QUIP# adapter solves a layer in row blocks (128 rows by default, mpq/adapters/quip_sharp.py:28) whose only
coupling is the observation precision: each block starts from the previous block's final EM value
(:555-586).  Here the chain stays on the device:

* the VAMP iterations of a block are one CUDA graph over static buffers (control decisions taken by kernels,
  mpq_b200.solver.e8_vamp_device), replayed block after block on one stream -- the control block carrying the
  observation precision from one replay to the next;
* the gram-metric polish of block b depends only on block b's VAMP result, so it runs on one of a few polish
  streams (one CUDA graph per stream) while the VAMP iterations of block b+1 proceed;
* statistics are collected into device tensors and read back once per layer.

The first block runs without graphs (it initialises every kernel's launch state), then the graphs are captured.
"""
from __future__ import annotations

import time
from typing import Any, Callable, Dict, List, Optional, Tuple

import torch

from . import ops, trace
from ._lib import call, ptr
from .solver import (E8Layer, E8P12VampConfig, E8VampState, _resolve_e8p12_polish_metric, _resolve_polish_mode,
                     e8_vamp_device, vamp_ctl_new, vamp_ctl_reset, vamp_ctl_stats, ALPHA_EPS)


# host-side timing of the last chained solve: seconds to enqueue all blocks, and to the end of the device work
last_timing: Dict[str, float] = {}
# CUDA graphs for the per-block launch sequences (False: host launches, e.g. to time single kernels with events)
use_graphs = True


def _priority(level: int) -> int:
    """Stream priority `level` steps above the default (clamped to the device's range): the VAMP chain is the
    critical path (2), the overlapped polish next (1); work on default-priority streams (such as the layer set-up
    of mpq_b200.pipeline) takes the SMs they leave."""
    lo, hi = torch.cuda.Stream.priority_range()
    return max(hi, lo - int(level))


def chain_supported(cfg: E8P12VampConfig) -> bool:
    """The chained path covers the default recipe: no best-iterate stop, polish 'block_cd' with the gram metric
    over the whole grid (or no polish)."""
    if bool(getattr(cfg, "best_iterate", False)):
        return False
    mode = _resolve_polish_mode(sweeps=max(int(cfg.polish_sweeps), 0), mode=str(getattr(cfg, "polish_mode", "block_cd")))
    if mode == "none":
        return True
    return (mode == "block_cd" and _resolve_e8p12_polish_metric(str(cfg.polish_metric or "gram")) == "gram"
            and int(getattr(cfg, "polish_max_blocks", 0) or 0) == 0)


def _row_err(L: E8Layer, Y_u: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """rowsum((Y_u - x Vs)^2) (mpq/linear.py:85-94) on the current stream."""
    C = ops.mm_nt(x, L.opVsT)
    out = torch.empty(x.shape[0], device=x.device, dtype=torch.float32)
    call("mpq_row_sqerr", ptr(Y_u), ptr(C), x.shape[0], C.shape[1], Y_u.stride(0), C.stride(0), ptr(out))
    return out


class _Graphable:
    """A launch sequence over static buffers that runs eagerly or as a captured CUDA graph."""

    def __init__(self):
        self.graph = None
        self.scratch = None
        self.nodes = 0

    def body(self) -> None:
        raise NotImplementedError

    def capture(self, stream: torch.cuda.Stream) -> None:
        """Capture body() on `stream` (idle, dedicated) into a graph with its own memory pool; unlike
        torch.cuda.graph this neither synchronises the device nor empties the allocator, so earlier work keeps
        running while the host captures."""
        g = torch.cuda.CUDAGraph()
        n0 = trace.launches()
        with ops.graph_scratch() as d:
            with torch.cuda.stream(stream):
                # thread_local: a set-up worker thread (mpq_b200.pipeline) may allocate or synchronise meanwhile
                g.capture_begin(capture_error_mode="thread_local")
                try:
                    self.body()
                finally:
                    g.capture_end()
        self.scratch = d
        self.nodes = trace.launches() - n0
        self.graph = g

    def run(self, use_graph: bool = True) -> None:
        if self.graph is None or not use_graph:
            self.body()
        else:
            self.graph.replay()
            trace.count_launch(self.nodes)


class _VampBlock(_Graphable):
    """One row block's VAMP iterations and final MAP decision (mpq/solver.py:961-1160)."""

    def __init__(self, L: E8Layer, cb, cfg: E8P12VampConfig, ctl: torch.Tensor, B: int, n: int, tau: float,
                 with_pscale: bool, em_active: bool):
        super().__init__()
        dev = L.dev
        nb = n // 8
        self.L, self.cb, self.cfg, self.ctl, self.tau, self.em_active = L, cb, cfg, ctl, tau, em_active
        self.W = torch.empty(B, n, device=dev)
        self.hat0 = torch.empty(B, n, device=dev)
        self.Y = torch.empty(B, L.R, device=dev)
        self.pscale = torch.empty(B, nb, device=dev) if with_pscale else None
        self.st = E8VampState(B, n, L.R, max(int(cfg.iters), 0), dev)
        self.obs_in = torch.empty(1, device=dev, dtype=torch.float64)
        self.vals = torch.empty(B, n, device=dev)
        self.idx = torch.empty(B, nb, device=dev, dtype=torch.int64)
        self.gstats = torch.empty(3, device=dev, dtype=torch.float64)  # gamma1 sum, min, max

    def body(self) -> None:
        from .e8p12 import e8p12_map_rows
        self.obs_in.copy_(self.ctl.view(torch.float64)[0:1])
        center = self.W if self.tau > 0.0 else None
        e8_vamp_device(self.st, self.ctl, self.L, Wr=self.W, hat0=self.hat0, center=center, pscale=self.pscale,
                       tau=self.tau, Y_u=self.Y, cfg=self.cfg, em_active=self.em_active)
        vals, idx32 = e8p12_map_rows(self.st.r1, self.cb, gamma=self.st.gamma1, center=center, pscale=self.pscale,
                                     prior_tau=self.tau)
        self.vals.copy_(vals)
        self.idx.copy_(idx32)
        g64 = self.st.gamma1.double()
        self.gstats[0:1].copy_(g64.sum().reshape(1))
        self.gstats[1:2].copy_(g64.min().reshape(1))
        self.gstats[2:3].copy_(g64.max().reshape(1))


class _PolishBlock(_Graphable):
    """The gram-metric greedy block CD of one row block (mpq/solver.py:1162-1215 with mpq/polish/block_cd.py)."""

    def __init__(self, L: E8Layer, gram, cb, B: int, n: int, sweeps: int):
        super().__init__()
        dev = L.dev
        nb = n // 8
        self.L, self.gram, self.cb, self.sweeps = L, gram, cb, sweeps
        self.stream = torch.cuda.Stream(dev, priority=_priority(1))
        self.x = torch.empty(B, n, device=dev)
        self.idx = torch.empty(B, nb, device=dev, dtype=torch.int64)
        self.Y = torch.empty(B, L.R, device=dev)
        self.x_out = torch.empty(B, n, device=dev)
        self.idx_out = torch.empty(B, nb, device=dev, dtype=torch.int64)
        # polish gain, final error mean, changed count, accepted updates, exact score evaluations, fails
        self.stats = torch.zeros(6, device=dev, dtype=torch.float64)
        self.trace = torch.zeros(max(sweeps, 0) + 1, device=dev, dtype=torch.float64)

    def body(self) -> None:
        from .e8p12 import gram_block_cd
        err_before = _row_err(self.L, self.Y, self.x)
        if self.sweeps > 0:
            x_out, idx_out, pst = gram_block_cd(x=self.x, Y_u=self.Y, Vs=self.L.Vs, cb=self.cb, sweeps=self.sweeps,
                                                idxs_init=self.idx, layer=self.gram, deferred=True)
            self.x_out.copy_(x_out)
            self.idx_out.copy_(idx_out)
            self.trace.copy_(pst["stabilized_objective_trace"])
            self.stats[3:4].copy_(pst["accepted_updates"].double())
            self.stats[4:5].copy_(pst["exact_score_evals"].double())
            self.stats[5:6].copy_(pst["_fails"].double())
        else:
            self.x_out.copy_(self.x)
            self.idx_out.copy_(self.idx)
        err_after = _row_err(self.L, self.Y, self.x_out)
        self.stats[0:1].copy_((err_before.double() - err_after.double()).mean().reshape(1))
        self.stats[1:2].copy_(err_after.double().mean().reshape(1))
        self.stats[2:3].copy_((self.idx != self.idx_out).sum().double().reshape(1))


class _ChainState:
    """Everything a chained solve of one shape keeps between calls: the static layer buffers, the control block, the
    block's VAMP graph and the polish streams' graphs (captured once, replayed for every block of every layer)."""

    def __init__(self, *, n, R, B, cb, cfg, tau, with_pscale, em_active, sweeps, polish_streams, dev):
        self.cb = cb  # keeps the codebook (and so its factor tables' key) alive
        self.L = E8Layer.static(n=n, R=R, cb=cb, device=dev)
        self.gram = self.L.gram() if sweeps > 0 else None
        self.ctl = vamp_ctl_new(dev)
        self.vamp = _VampBlock(self.L, cb, cfg, self.ctl, B, n, tau, with_pscale, em_active)
        self.polish = [_PolishBlock(self.L, self.gram, cb, B, n, sweeps) for _ in range(max(int(polish_streams), 1))]
        self.cap_stream = torch.cuda.Stream(dev)
        self.vamp_stream = torch.cuda.Stream(dev, priority=_priority(2))

    def capture(self):
        self.vamp.capture(self.cap_stream)
        for pb in self.polish:
            pb.capture(pb.stream)


_STATES: Dict[tuple, _ChainState] = {}
_WARM: set = set()  # devices whose kernels have run once in this process (launch attributes, tables, scratch)


@torch.inference_mode()
def e8p12_layer_chain(*, Wr: torch.Tensor, hat_init: torch.Tensor, cb, V: torch.Tensor, Vh: torch.Tensor,
                      S: torch.Tensor, Vs: torch.Tensor, cfg: E8P12VampConfig, block_rows: int, obs_init,
                      polish_streams: int = 6, graphs: Optional[bool] = None,
                      after_enqueue: Optional[Callable[[], None]] = None
                      ) -> Tuple[torch.Tensor, torch.Tensor, List[Dict[str, Any]]]:
    """Solve all rows of one E8P12 layer as the reference's serial chain of `block_rows`-row blocks.  graphs=False
    launches every kernel from the host (the same kernels and arguments as the graphs; per-launch timing works);
    None means the module default (use_graphs).  after_enqueue() runs once every block is enqueued, while the
    device works through them, with the VAMP stream current (e.g. to start the next layer's set-up after the VAMP
    chain, beside the last polish work, without competing for the host thread).

    Returns (hatWr (m, n), Qidxs int64 (m, n/8), per-block stats in the keys of solve_e8p12_rankspace_vamp plus
    the adapter's mechanism sums)."""
    from .e8p12 import prior_scale_from_center
    if graphs is None:
        graphs = use_graphs
    dev = Wr.device
    m, n = Wr.shape
    nb = n // 8
    R = int(S.numel())
    iters = max(int(cfg.iters), 0)
    tau = float(cfg.prior_tau)
    mode_scale = str(cfg.prior_tau_scale_mode or "absmax").strip().lower()
    sweeps = max(int(cfg.polish_sweeps), 0)
    polish_mode = _resolve_polish_mode(sweeps=sweeps, mode=str(getattr(cfg, "polish_mode", "block_cd")))
    if polish_mode == "none":
        sweeps = 0
    em_active = bool(cfg.em_obs_precision) and float(cfg.obs_precision) <= 0.0
    B = min(int(block_rows), m)
    key = (dev.index, n, R, B, id(cb), cfg, tau > 0.0, em_active, sweeps, int(polish_streams))
    cs = _STATES.get(key)
    if cs is None:
        cs = _ChainState(n=n, R=R, B=B, cb=cb, cfg=cfg, tau=tau, with_pscale=tau > 0.0, em_active=em_active,
                         sweeps=sweeps, polish_streams=polish_streams, dev=dev)
        _STATES[key] = cs
    L, ctl = cs.L, cs.ctl
    L.load(V=V, Vh=Vh, S=S, Vs=Vs)
    pscale_all = (prior_scale_from_center(Wr.reshape(m, nb, 8), mode_scale).reshape(m, nb).contiguous()
                  if tau > 0.0 else None)
    Y_u_all = ops.mm_nt(Wr, L.opVsT)  # FP32-faithful split product, all rows at once (rows are independent)
    fixed_obs = float(cfg.obs_precision) > 0.0
    obs0 = float(cfg.obs_precision) if fixed_obs else obs_init
    vamp_ctl_reset(ctl)
    if torch.is_tensor(obs0):  # the warm start computed on the device (no host read)
        ctl.view(torch.float64)[0:1].copy_(obs0.reshape(1).to(torch.float64))
    else:
        ctl.view(torch.float64)[0:1].fill_(float(obs0))
    final_hat = torch.empty_like(Wr)
    final_idx = torch.empty(m, nb, device=dev, dtype=torch.int64)
    starts = list(range(0, m, B))
    nblk = len(starts)
    # per-block statistics, read back once at the end
    b_ctl = torch.zeros(nblk, 16, device=dev, dtype=torch.int32)
    b_hist = torch.zeros(nblk, 3, max(iters, 1), device=dev, dtype=torch.float64)
    b_obs_in = torch.zeros(nblk, device=dev, dtype=torch.float64)
    b_g = torch.zeros(nblk, 3, device=dev, dtype=torch.float64)
    b_pol = torch.zeros(nblk, 6, device=dev, dtype=torch.float64)
    b_trace = torch.zeros(nblk, sweeps + 1, device=dev, dtype=torch.float64)
    main = torch.cuda.current_stream(dev)
    t_start = time.perf_counter()
    if graphs and cs.vamp.graph is None and dev.index in _WARM:
        cs.capture()
    # the VAMP chain runs on the state's high-priority stream, the polish on the polish streams; every tensor they
    # share with the caller was allocated above on the caller's stream, which waits for both before returning
    vs = cs.vamp_stream
    vs.wait_stream(main)
    tail = None  # a last block with fewer rows runs eagerly with its own buffers
    with torch.cuda.stream(vs):
        for bi, r0 in enumerate(starts):
            r1 = min(r0 + B, m)
            Bb = r1 - r0
            rb = slice(r0, r1)
            if Bb == B:
                vb, pb = cs.vamp, cs.polish[bi % len(cs.polish)]
            else:
                if tail is None:
                    tail = (_VampBlock(L, cb, cfg, ctl, Bb, n, tau, pscale_all is not None, em_active),
                            _PolishBlock(L, cs.gram, cb, Bb, n, sweeps))
                vb, pb = tail
            if graphs and bi > 0 and Bb == B and cs.vamp.graph is None:
                # first use in this process: block 0 ran eagerly (kernel attributes, tables, scratch set up)
                _WARM.add(dev.index)
                cs.capture()
            if bi > 0:
                vamp_ctl_reset(ctl)
                if fixed_obs:
                    ctl.view(torch.float64)[0:1].fill_(float(obs0))
            vb.W.copy_(Wr[rb])
            vb.hat0.copy_(hat_init[rb])
            vb.Y.copy_(Y_u_all[rb])
            if vb.pscale is not None:
                vb.pscale.copy_(pscale_all[rb])
            vb.run(graphs)
            final_hat[rb].copy_(vb.vals)
            final_idx[rb].copy_(vb.idx)
            b_ctl[bi].copy_(ctl)
            b_hist[bi, :, :iters].copy_(vb.st.hist[:, :iters])
            b_obs_in[bi:bi + 1].copy_(vb.obs_in)
            b_g[bi].copy_(vb.gstats)
            ev = torch.cuda.Event()
            ev.record(vs)
            pb.stream.wait_event(ev)
            with torch.cuda.stream(pb.stream):
                pb.x.copy_(final_hat[rb])
                pb.idx.copy_(final_idx[rb])
                pb.Y.copy_(Y_u_all[rb])
                pb.run(graphs)
                final_hat[rb].copy_(pb.x_out)
                final_idx[rb].copy_(pb.idx_out)
                b_pol[bi].copy_(pb.stats)
                b_trace[bi].copy_(pb.trace)
        if after_enqueue is not None:
            # called with the VAMP stream current: work it orders after the caller's stream (such as the next
            # layer's set-up) waits for the VAMP chain only, and overlaps the last blocks' polish
            after_enqueue()
    main.wait_stream(vs)
    for pb in cs.polish + ([tail[1]] if tail is not None else []):
        main.wait_stream(pb.stream)
    if not graphs or cs.vamp.graph is None:
        _WARM.add(dev.index)
    t_enq = time.perf_counter()
    ops.check_status(dev)  # synchronises: every block has finished
    last_timing.update(enqueue_s=t_enq - t_start, total_s=time.perf_counter() - t_start, blocks=float(nblk))
    ctl_h, hist_h, obs_in_h = b_ctl.cpu().numpy(), b_hist.cpu().tolist(), b_obs_in.cpu().tolist()
    g_h, pol_h, trace_h = b_g.cpu().tolist(), b_pol.cpu().tolist(), b_trace.cpu().tolist()
    out: List[Dict[str, Any]] = []
    for bi, r0 in enumerate(starts):
        rows = min(r0 + B, m) - r0
        cst = vamp_ctl_stats(ctl_h[bi], hist_h[bi][0], iters, hist_h[bi][1], hist_h[bi][2])
        if cst["fail"]:
            raise RuntimeError(f"alpha1 invalid: expected all in ({ALPHA_EPS}, 1-{ALPHA_EPS}).")
        gain, err_mean, changed, acc, evals, fails = pol_h[bi]
        if fails:
            raise RuntimeError("stabilize_cholesky failed for an E8P12 block gram")
        if sweeps > 0:
            tr = [float(v) for v in trace_h[bi]]
            pol = {"accepted_updates": float(acc), "exact_score_evals": int(evals), "stabilized_objective_trace": tr,
                   "stabilized_objective_nonincreasing": all(b <= a + max(1e-8, abs(a) * 1e-7)
                                                             for a, b in zip(tr, tr[1:]))}
        else:
            pol = {"accepted_updates": 0.0}
        obs_vals = cst["obs_values"]
        out.append({
            "solver": "e8p12_exact_vamp", "iters": iters, "rank": R, "nblocks": nb, "damping": float(cfg.damping),
            "prior_tau": tau, "prior_tau_scale_mode": mode_scale, "gamma_start": float(cfg.gamma_start),
            "gamma_retry_factor": max(float(cfg.gamma_retry_factor), 1.000001),
            "gamma_retry_steps": max(int(cfg.gamma_retry_steps), 0),
            "obs_precision_initial": float(obs_in_h[bi]), "obs_precision_final": cst["obs"],
            "obs_precision_mean": float(sum(obs_vals) / len(obs_vals)) if obs_vals else cst["obs"],
            "alpha1_retry_count": cst["alpha1_retry_count"], "alpha2_clip_count": cst["alpha2_clip_count"],
            "gamma2_invalid_count": cst["gamma2_invalid_count"], "alpha1_mean": cst["alpha1_mean"],
            "alpha2_mean": cst["alpha2_mean"], "mean_entropy": 0.0, "mean_margin": 0.0,
            "compile_prior": bool(getattr(cfg, "compile_prior", True)),
            "blocks_per_chunk": int(getattr(cfg, "blocks_per_chunk", 16)), "topk_k": int(getattr(cfg, "topk_k", 16)),
            "polish_sweeps": sweeps, "polish_mode": polish_mode,
            "polish_metric": _resolve_e8p12_polish_metric(str(cfg.polish_metric or "gram")),
            "polish_gain": float(gain), "polish_updates": float(pol.get("accepted_updates", 0.0)),
            "polish_trace": pol, "best_iterate_enabled": False, "best_iter": -1, "stop_iter": -1,
            "best_rankspace_error_mean": 0.0, "rankspace_error_mean": float(err_mean),
            "_gamma1_sum": float(g_h[bi][0]), "_gamma1_count": int(rows), "_gamma1_min": float(g_h[bi][1]),
            "_gamma1_max": float(g_h[bi][2]), "_changed_count": int(changed), "_changed_total": int(rows) * nb,
        })
    return final_hat, final_idx, out
