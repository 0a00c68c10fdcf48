#!/usr/bin/env python
"""Benchmark: seconds per 4096x4096 per-layer quantization solve (VAMP + 3 CD sweeps) on B200.

Workloads (seeded synthetic data with their shapes and distributions):
  e8p12  (configs[1], default)  W 4096x4096 ~ N(0, 0.02^2) (seed 0); X 16384x4096 with log-normal channel
         scales, H = X^T X / 16384 + 0.01 mean(diag H) I; randomized Hadamard on both dims (seeded +-1
         sign vectors), one global RMS scale; 2-bit E8P12 (2^16 codewords); RTN init; fp64 eigh of H;
         VAMP 16 iterations (tau 0.25) + 3 gram-metric block-CD sweeps.
  scalar  same W, H; internal block-Hadamard; 4-bit asym g128; RTN; fp32 eigh; VAMP 20
         iterations (tau 0.2) + 3 greedy scalar CD sweeps.
One step = one full layer solve from device-resident (W, H): rotation, eigendecomposition, RTN / grid,
warm start, VAMP, CD, audits.  Row blocking as the reference runs it: E8P12 in chained 128-row blocks (the QUIP#
adapter's default, mpq/adapters/quip_sharp.py:28); the scalar layer in the blocks the reference's GPTQ adapter
picks on a GPU (mpq/adapters/gptqmodel.py:313-327: 3640 + 456 rows at 4096 columns, 4 bits).

`--impl reference` times the CPU oracle (the reference algorithm restated in numpy) on the host cores: the
per-layer set-up (rotations, eigendecomposition) once, then every timed step solves a different slice of rows of
the same layer; the per-layer metric is the set-up plus the measured per-row time x 4096 rows.

Multi-GPU (torchrun): the layer's rows are sharded across ranks (each shard's VAMP starts from the
global warm start); rank 0 builds H and broadcasts it and W over NCCL; time = max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
import types
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

M_ROWS = 4096
N_COLS = 4096
T_CALIB = 16384
METRIC = "s per 4096^2 layer solve (VAMP+3 CD)"
WORKLOAD_DESC = {
    "model_e8": "config 3: Llama-3.2-1B-shaped decoder, random init, 128 x 2048 uniform-random calibration tokens, 2-bit "
                "E8P12 with randomized Hadamard on both sides, VAMP 16 it + 3 gram-CD sweeps, QUIP#-style float-model "
                "Hessians; layers solved round-robin over GPUs",
    "hessian": "calibration Hessian H = X^T X / T on the tensor cores (token-major activations X, T x n)",
    "model": "config 4: Llama-3-8B-shaped decoder, random init, 128 x 2048 uniform-random calibration tokens, 3-bit g128, "
             "internal Hadamard, VAMP 20 it + 3 CD sweeps, GPTQ sequential layer walk; rows of every linear sharded over GPUs",
    "e8p12": "config1: 4096x4096 layer, 2-bit E8P12, two-sided RHT, RTN init, fp64 eigh, VAMP 16 it + 3 gram-CD sweeps",
    "scalar": "config0: 4096x4096 layer, 4-bit asym g128, internal Hadamard, RTN init, VAMP 20 it + 3 CD sweeps",
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mpq", choices=["mpq", "reference"])
    ap.add_argument("--workload", default="e8p12", choices=sorted(WORKLOAD_DESC))
    ap.add_argument("--block-rows", type=int, default=0,
                    help="0: the reference's blocking (E8P12: 128-row chain; scalar: the GPTQ adapter's CUDA size)")
    ap.add_argument("--cpu-sample-rows", type=int, default=0,
                    help="rows of the CPU-baseline sample in the GPU arm's line (0: 16 for E8P12, 64 for scalar)")
    ap.add_argument("--ref-rows", type=int, default=0,
                    help="rows solved per timed step of the reference arm (0: 32 for E8P12, 64 for scalar)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--rows", type=int, default=0,
                    help="> 0: solve only this many rows per GPU (a small case for ncu; not a bench line)")
    ap.add_argument("--profile", action="store_true",
                    help="one warm-up + one timed step, no e2e / CPU legs (for an ncu launch list)")
    ap.add_argument("--model", default="llama3_8b", help="model workload: registered decoder shape")
    ap.add_argument("--model-layers", type=int, default=0, help="model workload: first N layers (0 = all)")
    ap.add_argument("--calib-seqs", type=int, default=128)
    ap.add_argument("--seq-len", type=int, default=2048)
    ap.add_argument("--bits", type=int, default=3)
    ap.add_argument("--preprocess", default="none", choices=["none", "awq"],
                    help="model workload: AWQ scaling before the walk (BASELINE config 2: --model qwen3_0p6b "
                         "--bits 4 --preprocess awq); timed with the walk and reported separately")
    ap.add_argument("--gemm-precision", default="", help="tf32x3 | f16x3 (FP32-faithful split products); default: "
                    "the library default")
    ap.add_argument("--hess-n", type=int, default=14336, help="hessian workload: features n")
    ap.add_argument("--hess-tokens", type=int, default=16384, help="hessian workload: tokens T per batch")
    ap.add_argument("--hess-dtype", default="bf16", choices=["bf16", "f32"])
    ap.add_argument("--schedule", default="auto", choices=["auto", "serial", "pipelined"],
                    help="e8p12: 'serial' sets up each step (rotations, eigendecomposition) before solving it; "
                         "'pipelined' (= 'auto') sets up step k+N on a worker stream once step k's VAMP chain is done, "
                         "beside its last polish work, and with N ranks computes each step's eigendecomposition on one "
                         "rank and copies it to the others")
    ap.add_argument("--polish-mode", default="block_cd", choices=["block_cd", "topk_block_cd"],
                    help="layer workloads: the polish recipe (block_cd is the reference's default)")
    a = ap.parse_args()
    if a.profile:
        a.steps, a.warmup, a.no_cpu_baseline, a.no_clocks = 1, 1, True, True
    if a.cpu_sample_rows <= 0:
        a.cpu_sample_rows = 16 if a.workload == "e8p12" else 64
    if a.ref_rows <= 0:
        a.ref_rows = 32 if a.workload == "e8p12" else 64
    return a


def bench_config(args, world: int) -> dict:
    """The workload description both arms print (identical keys and values at the same N)."""
    if args.workload == "e8p12":
        br = args.block_rows if args.block_rows > 0 else 128
    else:
        br = args.block_rows if args.block_rows > 0 else "reference CUDA size (3640 + 456)"
    return {"workload": WORKLOAD_DESC[args.workload], "rows": M_ROWS, "block_rows": br,
            "polish_mode": args.polish_mode, "parallelism": f"rows{world}",
            "l2": "256 MB buffer written between timed steps"}


# ----------------------------------------------------------------------------------------------
# synthetic inputs (same generator for the GPU arm and the CPU oracle)
# ----------------------------------------------------------------------------------------------

def synth_cpu():
    import torch
    g = torch.Generator(device="cpu").manual_seed(0)
    W = torch.randn(M_ROWS, N_COLS, generator=g) * 0.02
    s = torch.exp(torch.randn(N_COLS, generator=g))
    X = torch.randn(T_CALIB, N_COLS, generator=g) * s.sqrt()
    SU = (torch.randint(0, 2, (M_ROWS,), generator=g).float() * 2 - 1)
    SV = (torch.randint(0, 2, (N_COLS,), generator=g).float() * 2 - 1)
    return W, X, SU, SV


def hessian_device(X):
    """H = X^T X / T + 0.01 mean(diag) I on the GPU (tensor-core symmetric product, mpq_syrk_tc)."""
    import torch
    from mpq_b200.hessian import accumulate_xtx
    n = X.shape[1]
    H = torch.empty(n, n, device=X.device)
    accumulate_xtx(H, X, alpha=1.0 / X.shape[0], beta=0.0)
    H.add_(torch.eye(n, device=H.device) * (0.01 * float(H.diagonal().mean())))
    return H


def time_hessian(X, reps=3):
    """Device time of the X^T X accumulation (T x n fp32 calibration activations, 3xTF32 SYRK)."""
    import torch
    from mpq_b200.hessian import accumulate_xtx
    T, n = X.shape
    H = torch.zeros(n, n, device=X.device)
    accumulate_xtx(H, X, alpha=1.0 / T, beta=0.0)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        accumulate_xtx(H, X, alpha=1.0 / T, beta=0.0)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / reps
    flops = float(T) * n * (n + 1)  # algorithmic SYRK count
    return {"tokens": T, "n": n, "ms": ms, "tflops": flops / (ms * 1e-3) / 1e12,
            "what": "H = X^T X / T (split + 3xTF32 lower-triangle tcgen05 product), not part of the step time"}


# ----------------------------------------------------------------------------------------------
# clocks
# ----------------------------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, enabled: bool = True):
        self.proc = None
        # the raw samples go to MPQ_CLOCKS_DIR (default: the system temp directory); the JSON line carries the summary
        import tempfile
        self.path = Path(os.environ.get("MPQ_CLOCKS_DIR", tempfile.gettempdir())) / f"clocks_rank{index}.csv"
        if not enabled:
            return
        try:
            self.path.parent.mkdir(exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------------------------
# the measured steps
# ----------------------------------------------------------------------------------------------

class ScalarWorkload:
    dominant = "gemm_tc"

    def __init__(self, dev, block_rows, polish_mode="block_cd"):
        self.dev, self.block_rows, self.polish_mode = dev, block_rows, polish_mode

    def step(self, k, W, H, ahead=True):
        from mpq_b200.adapters.gptqmodel import GPTQAdapterConfig, run_mpq_quantization
        from mpq_b200.solver import UniformVampConfig
        if not W.is_cuda:
            W = W.to(self.dev, non_blocking=True)
            H = H.to(self.dev, non_blocking=True)
        qcfg = types.SimpleNamespace(bits=4, group_size=128, desc_act=False,
                                     mpq=types.SimpleNamespace(rotation_mode="internal_hadamard", solver="vamp"))
        out = run_mpq_quantization(W=W, H=2.0 * H, quantizer=None, qcfg=qcfg, module_name="bench.layer",
                                   vamp_cfg=UniformVampConfig(iters=20, prior_tau=0.2, damping=0.5, polish_sweeps=3, block_cd_backend="auto",
                                                              polish_mode=self.polish_mode),
                                   adapter_cfg=GPTQAdapterConfig(block_rows=self.block_rows or 128,
                                                                 grow_block_rows=self.block_rows <= 0))
        Q, q_int, scale, zero, g_idx, _, st = out
        return [q_int, scale, zero], {"raw_objective_mean": st["raw_objective_mean_final"],
                                      "obs_final": st["obs_precision_final"], "block_rows": st["block_rows"],
                                      "best_iters": [b["best_iter"] for b in st["block_stats"]]}

    def finish(self, k):
        return k

    def close(self):
        pass


class E8Workload:
    """One step = one 4096 x 4096 layer: its layer-wide set-up (two-sided RHT of W and H, the RMS scale, the fp64
    eigendecomposition of the rotated Hessian) and the chained solve of this rank's rows.

    Pipelined (the default): the set-up of step k + N is queued on the set-up pipeline's worker (mpq_b200.pipeline)
    once step k's blocks are enqueued.  With N ranks the eigendecomposition of step k is computed on rank k mod N
    only and the other ranks copy it from that rank's memory (mpq_b200.exchange) -- every step still carries one
    full set-up and one full solve of the layer across the job.  Serial: every rank sets up each step itself
    before solving it."""
    dominant = "e8p12_mmse"

    def __init__(self, dev, block_rows, SU, SV, rows, polish_mode="block_cd", rank=0, world=1, pipelined=True,
                 n=None):
        from mpq_b200.codebook import E8P12_codebook
        from mpq_b200.pipeline import SetupPipeline
        self.dev, self.block_rows, self.rows, self.polish_mode = dev, block_rows, rows, polish_mode
        self.rank, self.world = rank, world
        self.cb = E8P12_codebook()
        self.SU, self.SV = SU.to(dev), SV.to(dev)
        self.pipe = SetupPipeline(dev) if pipelined else None
        self.xchg = None
        if pipelined and world > 1:
            from mpq_b200.exchange import EigenExchange
            self.xchg = EigenExchange(n or N_COLS, dev)

    def owner(self, k: int) -> int:
        return k % self.world if self.pipe is not None else self.rank

    def setup(self, k, W, H):
        """Layer set-up of step k (W, H on the host are copied in first; the rotation and the scale are layer-wide,
        so every rank rotates the whole W and keeps its rows)."""
        from mpq_b200.adapters.gptqmodel import vamp_hessian_eigen
        from mpq_b200.rotation import rht_hessian, rht_weight
        if not W.is_cuda:
            W = W.to(self.dev, non_blocking=True)
            H = H.to(self.dev, non_blocking=True)
        m, n = W.shape
        Wr = rht_weight(W, self.SU, self.SV, m & -m, n & -n)
        Hr = rht_hessian(H, self.SV, n & -n)
        wscale = float(Wr.double().square().mean().sqrt())  # QUIP#'s global RMS scale, in float64
        r0, r1 = self.rows
        Wn = (Wr[r0:r1] / wscale).contiguous()
        eig = None
        if self.owner(k) == self.rank:
            eig = vamp_hessian_eigen(Hr, fp64=True)
            if self.xchg is not None:
                self.xchg.publish(k, eig)
        return {"Wn": Wn, "Hr": Hr, "wscale": wscale, "eig": eig}

    def queue(self, k, W, H):
        if self.pipe is not None and not self.pipe.pending(k):
            self.pipe.submit(k, self.setup, k, W, H)

    def step(self, k, W, H, ahead=True):
        """Solve step k (its set-up queued earlier, or run now); queue the set-up of step k + N once step k's device
        work is enqueued."""
        import torch
        from mpq_b200.adapters.quip_sharp import mpq_refine_codebook
        if self.pipe is not None:
            self.queue(k, W, H)
            P = self.pipe.get(k)
        else:
            P = self.setup(k, W, H)
        eig = P["eig"] if P["eig"] is not None else self.xchg.fetch(k)
        Wn = P["Wn"]
        m, n = Wn.shape
        args = types.SimpleNamespace(mpq_init="rtn", mpq_iters=16, mpq_prior_tau=0.25, mpq_polish_sweeps=3,
                                     mpq_block_rows=self.block_rows, quant_solver="vamp",
                                     quant_polish_mode=self.polish_mode, mpq_polish_metric="gram")
        nxt = (lambda: self.queue(k + self.world, W, H)) if (ahead and self.pipe is not None) else None
        hat, idx, st = mpq_refine_codebook(Wn, P["Hr"], Wn, torch.zeros(m, n // 8, dtype=torch.int64, device=self.dev),
                                           self.cb, args, module_name="bench.layer", eigen=eig, after_enqueue=nxt)
        from mpq_b200 import chain
        return [idx], {"surrogate_before": st["exact_surrogate_before_mean"],
                       "surrogate_after": st["exact_surrogate_after_mean"], "obs_final": st["obs_precision_final"],
                       "wscale": P["wscale"], "changed_fraction": st["mechanism"]["cleanup_changed_fraction"],
                       "block_rows": st["block_rows"], "chain_host_s": dict(chain.last_timing)}

    def settle(self):
        """Wait for the set-ups queued so far to complete (their results stay queued for their steps)."""
        if self.pipe is not None:
            for j in self.pipe.keys():
                self.pipe.wait(j)

    def finish(self, k):
        """Wait for the set-ups still queued (their work belongs to the steps that queued them) and drop them;
        returns the next step index (dropped steps' indices are not reused)."""
        if self.pipe is None:
            return k
        dropped = self.pipe.keys()
        self.pipe.drain()
        for j in dropped:
            if self.xchg is not None:
                self.xchg.skip(j)
        return max([k] + [j + 1 for j in dropped])

    def close(self):
        if self.pipe is not None:
            self.pipe.close()
        if self.xchg is not None:
            self.xchg.close()


def run_mpq(args):
    import torch
    import torch.distributed as dist
    from mpq_b200 import ops, trace
    from mpq_b200._lib import load
    load()
    if args.gemm_precision:
        ops.set_gemm_precision(args.gemm_precision)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    from mpq_b200.shard import broadcast_, row_shards
    Wc, Xc, SU, SV = synth_cpu()
    W = Wc.to(dev) if rank == 0 else torch.empty(M_ROWS, N_COLS, device=dev)
    hess = None
    if rank == 0:
        Xd = Xc.to(dev)
        H = hessian_device(Xd)
        hess = time_hessian(Xd)
        del Xd
    else:
        H = torch.empty(N_COLS, N_COLS, device=dev)
    del Xc
    broadcast_([W, H], src=0)  # W and H over NVLink (NCCL) to every rank
    r0, r1 = row_shards(M_ROWS, world, 128)[rank]
    if args.rows > 0:
        r1 = min(r1, r0 + args.rows)
    rows_per = r1 - r0
    if args.workload == "e8p12":
        block_rows = min(args.block_rows if args.block_rows > 0 else 128, rows_per)
    else:
        block_rows = min(args.block_rows, rows_per) if args.block_rows > 0 else 0
    pipelined = args.schedule != "serial"
    if args.workload == "e8p12":
        wl = E8Workload(dev, block_rows, SU, SV, (r0, r1), polish_mode=args.polish_mode, rank=rank, world=world,
                        pipelined=pipelined)
        Wr = W  # the rotation and scale are layer-wide; the workload solves rows r0:r1
    else:
        wl = ScalarWorkload(dev, block_rows, polish_mode=args.polish_mode)
        Wr = W[r0:r1].contiguous()
    flush = torch.empty(64 * 1024 * 1024, device=dev)  # 256 MB > 126 MB L2

    k = 0
    if hasattr(wl, "queue"):
        # fill the set-up pipeline: step j's set-up is queued N steps ahead of it (by step j - N, or here for the
        # first N steps), so no step of the timed region sets up inline however few warm-up steps there are
        for j in range(world):
            wl.queue(j, Wr, H)
    for _ in range(max(args.warmup, 0)):
        wl.step(k, Wr, H)
        k += 1
    torch.cuda.synchronize()

    # ---- device-resident timed region: K steps from one start event to one end event; the set-ups the timed
    # steps queued for later steps finish inside the region ----
    clocks = ClockSampler(local, enabled=not args.no_clocks)
    launches0 = trace.launches()
    stats = {}
    with trace.timing([wl.dominant]):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t_s = torch.cuda.Event(enable_timing=True)
        t_e = torch.cuda.Event(enable_timing=True)
        t_s.record()
        torch.cuda.nvtx.range_push("timed_steps")
        for _ in range(args.steps):
            flush.add_(1.0)
            outs, stats = wl.step(k, Wr, H)
            k += 1
        k = wl.finish(k)
        torch.cuda.nvtx.range_pop()
        t_e.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        dom = trace.summary(wl.dominant)
    launches = (trace.launches() - launches0) / max(args.steps, 1)
    dom_note = "CUDA events around every launch in the timed steps"
    if dom["launches"] == 0 and args.workload == "e8p12":
        # the chained solve replays CUDA graphs, whose kernel nodes events cannot bracket one by one: time the
        # dominant kernel's launches in one more step launched from the host (same kernels, arguments, stream)
        from mpq_b200 import chain
        chain.use_graphs = False
        with trace.timing([wl.dominant]):
            wl.step(k, Wr, H, ahead=False)
            k += 1
            torch.cuda.synchronize()
            dom = trace.summary(wl.dominant)
        chain.use_graphs = True
        dom_note = ("CUDA events around every launch of one extra step launched from the host (the timed steps replay "
                    "CUDA graphs of the same kernels with the same arguments)")
    clk = clocks.stop()
    ms = t_s.elapsed_time(t_e) / max(args.steps, 1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    if args.profile:
        wl.close()
        if world > 1:
            dist.destroy_process_group()
        return {"profile": True, "ms_per_step": ms, "gpu_launches": launches} if rank == 0 else None

    # ---- e2e through the public API with host buffers ----
    W_host = Wr.cpu().pin_memory()
    H_host = H.cpu().pin_memory()
    h2d = W_host.numel() * 4 + H_host.numel() * 4
    d2h = 0
    n_e2e = max(1, args.steps)  # as many steps as the timed region (a pipelined schedule drains once per region)
    if hasattr(wl, "queue"):
        for j in range(world):  # as in the timed region: each step's set-up queued N steps ahead
            wl.queue(k + j, W_host, H_host)
        # The set-ups queued here belong to the steps before the region (as the warm-up's do for the device-timed
        # region): they complete before the clock starts, and every timed step carries the one it queues for a
        # later step (finished inside the region by finish()).
        wl.settle()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        flush.add_(1.0)
        outs, _ = wl.step(k, W_host, H_host)  # the set-up copies this step's W and H from pinned host memory
        k += 1
        host = [o.cpu() for o in outs]
        d2h = sum(o.numel() * o.element_size() for o in host)
    k = wl.finish(k)
    torch.cuda.synchronize()
    e2e = (time.perf_counter() - t0) * 1e3 / n_e2e
    if world > 1:
        t = torch.tensor([e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e = float(t.item())

    result = None
    if rank == 0:
        pk = ROOT / "MEASURED_PEAKS.json"
        peaks = json.loads(pk.read_text()) if pk.exists() else {}
        roofline = dominant_roofline(wl.dominant, dom, peaks,
                                     1 if dom_note.startswith("CUDA events around every launch of one") else args.steps,
                                     sm_mhz=(clk or {}).get("sm_mhz"))
        roofline["timing"] = dom_note
        result = {
            "metric": METRIC, "value": ms / 1e3, "unit": "s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "gemm_precision": ops.gemm_precision(),
            "data": "synthetic (seeded W ~ N(0,0.02^2), X with log-normal channel scales)",
            "config": bench_config(args, world), "rows_per_gpu": rows_per,
            "e2e": {"value": e2e / 1e3, "unit": "s", "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": int(round(launches)),
            "roofline": roofline,
            "clocks": clk,
            "hessian": hess,
            "stats": stats,
        }
        if args.workload == "e8p12":
            result["schedule"] = ("serial: each step's layer set-up (rotations, fp64 eigendecomposition), then its solve"
                                  if not pipelined else
                                  "pipelined: the layer set-up of step k+N (rotations, fp64 eigendecomposition) runs on "
                                  "a low-priority worker stream after step k's VAMP chain, beside its polish; with N ranks the "
                                  "eigendecomposition of step k runs on rank k mod N and the others copy it over NVLink; "
                                  "the set-ups queued by the timed steps finish inside the timed region")
        if not args.no_cpu_baseline and world == 1:
            oracle = CpuOracle(args.workload, H=H.cpu())
            t_rows, ref_out = oracle.solve_rows(0, args.cpu_sample_rows)
            rows = args.cpu_sample_rows
            result["cpu_baseline"] = {
                "value": oracle.t_setup + t_rows * (M_ROWS / rows), "unit": "s", "cores": oracle.cores, "kind": "port",
                "sample": f"{rows} of {M_ROWS} rows solved as one block ({oracle.what}) in {t_rows:.1f} s, "
                          f"extrapolated x{M_ROWS // rows}; rotation + eigendecomposition once ({oracle.t_setup:.1f} s)"}
            result["parity_sample"] = gpu_vs_oracle(args.workload, oracle, ref_out, Wr, H, rows, dev)
    wl.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


# DRAM traffic per launch of the dominant kernels, from ncu captures (dram__bytes_read.sum +
# dram__bytes_write.sum) of the bench workload.
TRAFFIC = {
    # k_gemm_tc, one 4096 x 4096 x 4096 3xFP16 product
    "gemm_tc": {"bytes": 3.545e8 + 0.564e8, "launch": "4096x4096x4096 f16x3 product"},
    # k_e8p12<1> in the chained solve: one 128-row block x 512 8-blocks (ncu, VAMP iteration 8)
    "e8p12_mmse": {"bytes": 4.527e6 + 0.0, "launch": "128 rows x 512 blocks (one block of the chain)",
                   "warp_instructions": 1.586e8},
}


def dominant_roofline(name, dom, peaks, steps, sm_mhz=None):
    """roofline object of the dominant kernel from its CUDA-event launch times and algorithmic work."""
    secs = dom["ms_avg"] * 1e-3
    common = {"launches_per_step": dom["launches"] / max(steps, 1), "ms_per_step": dom["ms_total"] / max(steps, 1),
              "traffic": TRAFFIC[name]["bytes"], "traffic_launch": TRAFFIC[name]["launch"]}
    if name == "gemm_tc":
        peak = float(peaks.get("bf16_tflops_sustained", 1394.3))
        achieved = dom["work_avg"] / secs / 1e12 if secs > 0 else 0.0
        return {"bound": "tensor", "kernel": "k_gemm_tc (tcgen05 FP32-faithful split rank-space products)",
                "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "peak_source": "MEASURED_PEAKS.json bf16_tflops_sustained (measured)" if peaks else "fallback",
                "achieved_counts": "algorithmic 2MNK per product (the f16x3 split issues 3 fp16 MMAs per FLOP, so "
                                   "its ceiling is 1/3 of the dense fp16/bf16 peak)", **common}
    peak = float(peaks.get("hbm_gbs", 6650.0))
    achieved = dom["work_avg"] / secs / 1e9 if secs > 0 else 0.0
    # the binding roof is instruction issue (4 warp instructions per SM per cycle): the ncu instruction count of the
    # same launch shape over the live CUDA-event duration, against 148 SMs x 4 x the measured SM clock
    clk_ghz = float(sm_mhz or peaks.get("sm_max_mhz", 1965.0)) / 1e3
    issue_peak = 148 * 4 * clk_ghz
    issue_achieved = TRAFFIC[name]["warp_instructions"] / secs / 1e9 if secs > 0 else 0.0
    # the reference algorithm's arithmetic (512 components x ~104 FP32/MUFU ops per 8-vector, no pruning) at the same
    # rate, against the FP32 CUDA-core peak (148 SMs x 128 lanes x 2 FLOP x clock)
    items = dom["work_avg"] / 12.0 / 8.0
    ref_ops = items * 512 * 104
    fp32_peak = 148 * 128 * 2 * clk_ghz / 1e3
    return {"bound": "hbm", "kernel": "k_e8p12<1> (E8P12 factorized posterior)", "achieved": achieved, "peak": peak,
            "unit": "GB/s", "frac": achieved / peak,
            "peak_source": "MEASURED_PEAKS.json hbm_gbs (measured)" if peaks else "fallback",
            "achieved_counts": "algorithmic bytes: r1, prior centre and x1 (12 B per coordinate) + per-row scalars",
            "compute_roofline": {
                "bound": "instruction issue", "achieved": issue_achieved, "peak": issue_peak,
                "unit": "G warp-instructions/s", "frac": issue_achieved / issue_peak,
                "counts": f"{TRAFFIC[name]['warp_instructions']:.3g} warp instructions per launch (ncu, same shape)",
                "reference_equivalent_fp32": {"achieved_tflops": ref_ops / secs / 1e12 if secs > 0 else 0.0,
                                              "peak_tflops": fp32_peak,
                                              "frac": (ref_ops / secs / 1e12) / fp32_peak if secs > 0 else 0.0,
                                              "counts": "512 components x 104 ops per 8-vector (the unpruned "
                                                        "reference arithmetic) over the measured launch time"}},
            **common}


# ----------------------------------------------------------------------------------------------
# CPU oracle (the reference algorithm restated in numpy) on a bounded sample
# ----------------------------------------------------------------------------------------------

class CpuOracle:
    """The reference algorithm restated in numpy/torch-CPU (oracle/) on all host cores: per-layer set-up once
    (rotations, eigendecomposition), then row slices of the same layer solved as blocks."""

    def __init__(self, workload: str, H=None):
        import torch
        from oracle import layer as OL
        self.workload = workload
        self.cores = os.cpu_count() or 1
        torch.set_num_threads(self.cores)
        Wc, Xc, SU, SV = synth_cpu()
        W = Wc.numpy()
        SU, SV = SU.numpy(), SV.numpy()
        if H is None:
            H = OL.hessian_from_calibration(Xc.numpy())
        else:
            H = H.numpy() if hasattr(H, "numpy") else np.asarray(H)
        del Xc
        t0 = time.perf_counter()
        if workload == "e8p12":
            from oracle import e8p12 as OE
            self.cb = OE.E8P12_codebook()
            Hr = OL.right_block_hadamard(np.ascontiguousarray(H.T), SV, N_COLS).T.copy()
            self.Hr = OL.right_block_hadamard(Hr, SV, N_COLS)
            lam, self.V, _ = OL.vamp_hessian_eigen(self.Hr, fp64=True)
            self.S = np.sqrt(lam).astype(np.float32)
            self.Vs = (self.V * self.S[None, :]).astype(np.float32)
            Wr = OL.right_block_hadamard(W, SV, N_COLS)
            Wr = OL.right_block_hadamard(np.ascontiguousarray(Wr.T), SU, M_ROWS).T.copy()
            self.Wn = (Wr / np.sqrt((Wr.astype(np.float64) ** 2).mean())).astype(np.float32)
            self.mcache = OE.block_metric_cache(self.Vs, self.cb)
            self.what = "VAMP 16 it + 3 gram-CD sweeps"
        else:
            Hw = (np.float32(0.5) * (2.0 * H)).astype(np.float32)
            lam, V, _ = OL.vamp_hessian_eigen(Hw)
            signs = OL.rademacher_signs_torch(N_COLS, "bench.layer:full", 0)
            self.Wr = OL.right_block_hadamard(W, signs, N_COLS)
            Hm = OL.right_block_hadamard(np.ascontiguousarray(Hw.T), signs, N_COLS).T.copy()
            self.Hm = OL.right_block_hadamard(Hm, signs, N_COLS)
            self.V = OL.right_block_hadamard(np.ascontiguousarray(V.T), signs, N_COLS).T.copy()
            self.S = np.sqrt(lam).astype(np.float32)
            self.Vs = (self.V * self.S[None, :]).astype(np.float32)
            self.what = "VAMP 20 it + 3 CD sweeps"
        self.t_setup = time.perf_counter() - t0

    def solve_rows(self, r0: int, r1: int):
        """Solve rows [r0, r1) as one block; returns (seconds, codes)."""
        from oracle import layer as OL
        t0 = time.perf_counter()
        if self.workload == "e8p12":
            from oracle import e8p12 as OE
            Wb = self.Wn[r0:r1]
            hat0, _ = OE.rtn_init(Wb, self.cb)
            out = OE.solve_e8p12_rankspace_vamp(Wr=Wb, hatWr_init=hat0, cb=self.cb, V=self.V,
                                                Vh=np.ascontiguousarray(self.V.T), S=self.S, Vs=self.Vs,
                                                cfg=OE.E8P12VampConfig(iters=16, prior_tau=0.25, polish_sweeps=3),
                                                metric_cache=self.mcache)
            codes = (out[0], out[1])
        else:
            from oracle import uniform_vamp as OU
            G = 128
            Wb = self.Wr[r0:r1]
            rows = Wb.shape[0]
            sg = np.empty((rows, N_COLS // G), np.float32)
            zg = np.empty_like(sg)
            for gi in range(N_COLS // G):
                a, b = OL.find_params_minmax(Wb[:, gi * G:(gi + 1) * G], 15)
                sg[:, gi], zg[:, gi] = a[:, 0], b[:, 0]
            sf, zf = np.repeat(sg, G, 1), np.repeat(zg, G, 1)
            q = np.clip(np.round(Wb / sf) + zf, 0, 15).astype(np.float32)
            xr = (sf * (q - zf)).astype(np.float32)
            out = OU.solve_uniform_rankspace_vamp(W=Wb, x_rtn=xr, scale_full=sf, zero_full=zf, maxq=15, V=self.V,
                                                  Vh=np.ascontiguousarray(self.V.T), S=self.S, Vs=self.Vs,
                                                  cfg=OU.UniformVampConfig(iters=20, prior_tau=0.2, damping=0.5,
                                                                           polish_sweeps=3), gram_full=self.Hm)
            codes = (out[1], out[0], sg, zg, xr)
        return time.perf_counter() - t0, codes


def gpu_vs_oracle(workload, oracle, ref_out, Wd, Hd, rows, dev):
    """The CUDA solve of the oracle sample's rows (same rows, one block, same H) against the oracle's result: code
    agreement and the relative proxy-loss difference tr((W - Q) H (W - Q)^T)."""
    import torch
    from mpq_b200 import solver as S
    from mpq_b200.adapters.gptqmodel import vamp_hessian_eigen
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    if workload == "e8p12":
        from mpq_b200.codebook import E8P12_codebook
        from mpq_b200.e8p12 import e8p12_nearest
        Hr = t(oracle.Hr)
        lam, V, _ = vamp_hessian_eigen(Hr, fp64=True)
        Sv = torch.sqrt(lam).contiguous()
        Vs = (V * Sv.unsqueeze(0)).contiguous()
        Wb = t(oracle.Wn[:rows])
        cb = E8P12_codebook()
        hat0, _ = e8p12_nearest(Wb.reshape(-1, 8), cb)
        hat, idx, _, _ = S.solve_e8p12_rankspace_vamp(Wr=Wb, hatWr_init=hat0.reshape(rows, -1), cb=cb, V=V,
                                                      Vh=V.T.contiguous(), S=Sv, Vs=Vs,
                                                      cfg=S.E8P12VampConfig(iters=16, prior_tau=0.25, polish_sweeps=3))
        ref_hat, ref_idx = ref_out
        agree = float((idx.cpu().numpy() == ref_idx).mean())
        Hm64 = oracle.Hr.astype(np.float64)
        W64 = oracle.Wn[:rows].astype(np.float64)
        got, want = hat.cpu().numpy().astype(np.float64), ref_hat.astype(np.float64)
    else:
        ref_x, ref_q, sg, zg, xr = ref_out
        Hm = t(oracle.Hm)
        V = t(oracle.V)
        Sv = t(oracle.S)
        Vs = t(oracle.Vs)
        Wb = t(oracle.Wr[:rows])
        q, x, _, _, _ = S.solve_uniform_rankspace_vamp(
            W=Wb, x_rtn=t(xr), scale_full=t(sg), zero_full=t(zg), maxq=15, V=V, Vh=V.T.contiguous(), S=Sv, Vs=Vs,
            cfg=S.UniformVampConfig(iters=20, prior_tau=0.2, damping=0.5, polish_sweeps=3, block_cd_backend="auto"),
            gram_full=Hm)
        agree = float((q.cpu().numpy() == ref_q).mean())
        Hm64 = oracle.Hm.astype(np.float64)
        W64 = oracle.Wr[:rows].astype(np.float64)
        got, want = x.cpu().numpy().astype(np.float64), ref_x.astype(np.float64)
    pg = float((((W64 - got) @ Hm64) * (W64 - got)).sum())
    pw = float((((W64 - want) @ Hm64) * (W64 - want)).sum())
    return {"rows": int(rows), "code_agreement": agree, "proxy_rel_delta": (pg - pw) / pw,
            "what": "the oracle's CPU solve of the CPU-baseline rows (one block, the same inputs) vs the CUDA solve"}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    if args.workload in ("model", "model_e8"):
        return {"impl": "reference", "unavailable": "the whole-model CPU run (about 46 h for the 8B shape) is not "
                "timed; the per-layer CPU baseline is the --workload e8p12 / scalar reference arm"}
    oracle = CpuOracle(args.workload)
    R = max(int(args.ref_rows), 1)
    for w in range(max(args.warmup, 0)):  # warm-up: thread pools, allocator, page cache (one row each)
        oracle.solve_rows(M_ROWS - 1 - w, M_ROWS - w)
    step_s, rows_done = [], 0
    for k in range(max(args.steps, 1)):
        r0 = (k * R) % M_ROWS
        r1 = min(r0 + R, M_ROWS)
        secs, _ = oracle.solve_rows(r0, r1)
        step_s.append(secs)
        rows_done += r1 - r0
    per_row = float(np.sum(step_s)) / max(rows_done, 1)
    per_row_steps = [s_ / R for s_ in step_s]
    v = oracle.t_setup + per_row * M_ROWS
    sample = (f"{rows_done} of {M_ROWS} rows measured ({len(step_s)} steps, a different {R}-row slice solved as one "
              f"block each: {oracle.what}); per-row time {per_row:.3f} s (steps {min(per_row_steps):.3f}-"
              f"{max(per_row_steps):.3f} s), x {M_ROWS} rows = extrapolation x{M_ROWS / rows_done:.1f} of the measured "
              f"rows; set-up (rotation + eigendecomposition) measured once, {oracle.t_setup:.1f} s; per-row work does "
              f"not depend on the blocking")
    return {"impl": "reference", "metric": METRIC, "value": v, "unit": "s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": float(np.mean(step_s)) * 1e3, "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "gemm_precision": "fp32 (CPU)",
            "data": "synthetic (seeded W ~ N(0,0.02^2), X with log-normal channel scales)",
            "config": bench_config(args, world),
            "cpu_baseline": {"value": v, "unit": "s", "cores": oracle.cores, "kind": "port", "sample": sample},
            "measured": {"rows": rows_done, "seconds": float(np.sum(step_s)), "per_row_s": per_row,
                         "per_row_s_min": min(per_row_steps), "per_row_s_max": max(per_row_steps),
                         "setup_s": oracle.t_setup, "extrapolation": M_ROWS / rows_done,
                         "ms_per_step_is": "wall time of one timed step (one row slice); value is the per-layer metric"},
            "e2e": {"value": v, "unit": "s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_model(args):
    """Whole-model quantization time (one timed run; a full 8B-shape run takes minutes, so no warm-up steps)."""
    import datetime
    import torch
    import torch.distributed as dist
    from mpq_b200 import trace
    from mpq_b200._lib import load
    from mpq_b200.model import ModelQuantConfig, build_synthetic_decoder, calibration_ids, quantize_model
    load()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=dev)
    layers = args.model_layers if args.model_layers > 0 else None
    e8 = args.workload == "model_e8"
    name = ("llama32_1b" if args.model == "llama3_8b" else args.model) if e8 else args.model
    model = build_synthetic_decoder(name, device=dev, seed=0, num_layers=layers)
    ids = calibration_ids(args.calib_seqs, args.seq_len, model.config.vocab_size, seed=0)
    cfg = ModelQuantConfig(bits=args.bits, group_size=128, iters=20, prior_tau=0.2, damping=0.5, polish_sweeps=3)
    clocks = ClockSampler(local, enabled=not args.no_clocks)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = trace.launches()
    t0 = time.perf_counter()
    awq_s = None
    if args.preprocess == "awq" and not e8:
        from mpq_b200.awq import apply_awq_scaling
        apply_awq_scaling(model, ids, bits=args.bits, group_size=128, sym=False, batch_size=32)
        torch.cuda.synchronize()
        awq_s = time.perf_counter() - t0
    if e8:
        from mpq_b200.model import QuipModelConfig, quantize_model_quip
        out = quantize_model_quip(model, ids, QuipModelConfig(iters=16, prior_tau=0.25, polish_sweeps=3,
                                                               keep_attrs=False))
    else:
        out = quantize_model(model, ids, cfg)
    torch.cuda.synchronize()
    secs = time.perf_counter() - t0
    clk = clocks.stop()
    if world > 1:
        t = torch.tensor([secs], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        secs = float(t.item())
    res = None
    if rank == 0 and e8:
        groups = out["groups"]
        res = {"metric": f"s per {name}-shape full-model quantization", "value": secs, "unit": "s", "n_gpus": world,
               "steps": 1, "warmup": 0, "ms_per_step": secs * 1e3, "higher_is_better": False, "scaling": "strong",
               "vs_baseline": None, "dtype": "f32 solve / bf16 model", "data": "synthetic",
               "config": {"workload": WORKLOAD_DESC["model_e8"], "model": name,
                          "layers": model.config.num_hidden_layers, "calibration": [args.calib_seqs, args.seq_len],
                          "parallelism": f"layers{world}+calib{world}"},
               "timings_rank0_s": out["timings"], "gpu_launches": trace.launches() - launches0, "clocks": clk,
               "groups": len(groups),
               "proxy_error_mean": float(np.mean([g["proxy_error"] for g in groups.values()]))}
    elif rank == 0:
        mods = out["modules"]
        res = {"metric": f"s per {args.model}-shape full-model quantization", "value": secs, "unit": "s",
               "n_gpus": world, "steps": 1, "warmup": 0, "ms_per_step": secs * 1e3, "higher_is_better": False,
               "scaling": "strong", "vs_baseline": None, "dtype": "f32 solve / bf16 model", "data": "synthetic",
               "config": {"workload": WORKLOAD_DESC["model"], "model": args.model, "layers": model.config.num_hidden_layers,
                          "calibration": [args.calib_seqs, args.seq_len], "bits": args.bits, "group_size": 128,
                          "preprocess": args.preprocess, "parallelism": f"rows{world}+calib{world}"},
               "awq_s_rank0": awq_s,
               "timings_rank0_s": out["timings"], "gpu_launches": trace.launches() - launches0, "clocks": clk,
               "linears": len(mods),
               "solve_s_by_projection_rank0": {k: round(sum(m["solve_s"] for n, m in mods.items() if n.endswith(k)), 3)
                                               for k in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj",
                                                         "down_proj")},
               "rankspace_error_over_rtn": float(np.mean([m["rankspace_error_mean"] / max(m["rtn_rankspace_error_mean"], 1e-30)
                                                          for m in mods.values() if m.get("rankspace_error_mean")]))}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return res


def run_hessian(args):
    """Device time of one X^T X accumulation (the Hessian hooks' work per calibration batch)."""
    import torch
    from mpq_b200._lib import load
    from mpq_b200.hessian import accumulate_xtx
    load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n, T = args.hess_n, args.hess_tokens
    g = torch.Generator(device=dev).manual_seed(0)
    X = torch.randn(T, n, device=dev, generator=g).to(torch.bfloat16 if args.hess_dtype == "bf16" else torch.float32)
    H = torch.zeros(n, n, device=dev)
    for _ in range(max(args.warmup, 1)):
        accumulate_xtx(H, X, alpha=1.0 / T, beta=0.0)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        accumulate_xtx(H, X, alpha=1.0 / T, beta=1.0)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / max(args.steps, 1)
    tf = float(T) * n * (n + 1) / (ms * 1e-3) / 1e12
    pk = ROOT / "MEASURED_PEAKS.json"
    peaks = json.loads(pk.read_text()) if pk.exists() else {}
    peak = float(peaks.get("bf16_tflops", 1590.0))
    return {"metric": "ms per X^T X accumulation", "value": ms, "unit": "ms", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": False, "dtype": args.hess_dtype, "data": "synthetic",
            "config": {"workload": WORKLOAD_DESC["hessian"], "n": n, "tokens": T},
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                         "achieved_counts": "algorithmic T n (n + 1) (symmetric product)",
                         "peak_source": "MEASURED_PEAKS.json bf16_tflops (measured)" if peaks else "fallback"}}


def main():
    args = parse()
    if args.impl == "reference":
        res = run_reference(args)
    elif args.workload in ("model", "model_e8"):
        res = run_model(args)
    elif args.workload == "hessian":
        res = run_hessian(args)
    else:
        res = run_mpq(args)
    if res is not None:
        print(json.dumps(res))


if __name__ == "__main__":
    main()
