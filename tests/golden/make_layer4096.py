"""Golden outputs of the reference at the benchmark's width: 256 rows x 4096 columns of BASELINE configs 0 and 1,
solved by the reference's own per-linear drivers with its 128-row block chain.

    python tests/golden/make_layer4096.py --reference <reference source tree>

Writes tests/golden/layer4096.npz: the reference's codes (E8P12 indices, 4-bit codes, scales, zeros), its proxy
losses tr((W - Q) H (W - Q)^T) and the obs-precision chain.  The inputs are not stored: layer4096_inputs.py
rebuilds them bit for bit on any machine.  Third-party pieces the reference calls but does not vendor are passed
as the restatements the oracle and the product use (the min-max grid for GPTQModel's find_params, the restated
E8P12 grid for QUIP#'s codebook, the raw-Hessian greedy CD dispatch of the CUDA polish); make_golden.py has them.
"""
from __future__ import annotations

import argparse
import json
import sys
import time
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROWS = 256
BLOCK_ROWS = 128


def e8p12_case(W, H, SU, SV):
    from mpq.adapters.quip_sharp import mpq_refine_codebook
    from mpq.rotation import apply_right_block_hadamard
    from make_golden import _reference_codebook
    from layer4096_inputs import rms_scale
    n = W.shape[1]
    t = apply_right_block_hadamard(W, signs=SV, had_dim=n)
    Wr = apply_right_block_hadamard(t.T.contiguous(), signs=SU, had_dim=W.shape[0]).T.contiguous()
    Hr = apply_right_block_hadamard(H.T.contiguous(), signs=SV, had_dim=n)
    Hr = apply_right_block_hadamard(Hr.T.contiguous(), signs=SV, had_dim=n)
    wscale = rms_scale(Wr)
    Wn = (Wr[:ROWS] / wscale).contiguous()
    cb = _reference_codebook()
    hat0, q0 = cb.quantize(Wn.reshape(-1, 8))
    args = types.SimpleNamespace(mpq_init="rtn", mpq_iters=16, mpq_prior_tau=0.25, mpq_polish_sweeps=3,
                                 mpq_block_rows=BLOCK_ROWS, mpq_blocks_per_chunk=1 << 20, mpq_compile_prior=False,
                                 quant_solver="vamp", quant_polish_mode="block_cd", mpq_polish_metric="gram")
    t0 = time.time()
    hatWr, Qidxs, st = mpq_refine_codebook(Wn, Hr, hat0.view(ROWS, n), q0.view(ROWS, n // 8), cb, args,
                                           module_name="layer4096.e8p12")
    secs = time.time() - t0
    d = (Wn - hatWr).double()
    proxy = float(((d @ Hr.double()) * d).sum())
    d0 = (Wn - hat0.view(ROWS, n)).double()
    proxy_rtn = float(((d0 @ Hr.double()) * d0).sum())
    # stage by stage: the same chain without the polish (the VAMP-stage codes), and one polish sweep started from
    # those codes (mpq/solver.py:369-423 on each row block, the reference's eigendecomposition)
    args_v = types.SimpleNamespace(**{**vars(args), "quant_polish_mode": "none", "mpq_polish_sweeps": 0})
    _, Q_vamp, _ = mpq_refine_codebook(Wn, Hr, hat0.view(ROWS, n), q0.view(ROWS, n // 8), cb, args_v,
                                       module_name="layer4096.e8p12")
    from mpq.adapters.quip_sharp import _vamp_hessian_eigen
    from mpq.solver import polish_e8p12_rankspace
    lam, V, _, _ = _vamp_hessian_eigen(Hr)
    Vs = V * lam.sqrt().unsqueeze(0)
    grid = cb.grid

    def polish(codes, sweeps):
        x = grid.index_select(0, codes.reshape(-1)).reshape(codes.shape[0], n)
        _, idx, _, _ = polish_e8p12_rankspace(x_init=x, idxs_init=codes, Y_u=Wn[rb].matmul(Vs), Vs=Vs, cb=cb,
                                              sweeps=sweeps, polish_mode="block_cd", polish_metric="gram")
        return idx

    sweep1, flipped = [], None
    for r0 in range(0, ROWS, BLOCK_ROWS):
        rb = slice(r0, r0 + BLOCK_ROWS)
        sweep1.append(polish(Q_vamp[rb], 1))
        if r0 == 0:
            # sensitivity of the reference's own polish: two of the block's 65,536 starting codes changed to a
            # neighbouring codeword (index ^ 1), three sweeps, compared with the unperturbed three-sweep result
            base = polish(Q_vamp[rb], 3)
            qp = Q_vamp[rb].clone()
            qp[5, 100] ^= 1
            qp[77, 300] ^= 1
            pert = polish(qp, 3)
            flipped = dict(changed_inputs=2, agreement=float((pert == base).double().mean()),
                           rows_equal=int((pert == base).all(1).sum()), matches_chain=float((base == Qidxs[rb]).double().mean()))
    meta = dict(rows=ROWS, block_rows=BLOCK_ROWS, iters=16, wscale=wscale, proxy=proxy, proxy_rtn=proxy_rtn,
                obs_init=st["obs_precision_initial"], obs_final=st["obs_precision_final"],
                surrogate_after=st["exact_surrogate_after_mean"], seconds=secs, polish_sensitivity=flipped)
    print("e8p12", json.dumps(meta))
    return {"e8/Qidxs": Qidxs.numpy().astype(np.int32), "e8/Qidxs_vamp": Q_vamp.numpy().astype(np.int32),
            "e8/Qidxs_sweep1": torch.cat(sweep1).numpy().astype(np.int32), "e8/meta": np.array(json.dumps(meta))}


def scalar_case(W, H):
    from make_golden import MinMaxQuantizer, _install_gpu_polish_semantics
    _install_gpu_polish_semantics()
    from mpq.adapters.gptqmodel import GPTQAdapterConfig, run_mpq_quantization
    from mpq.rotation import apply_right_block_hadamard
    from mpq.solver import UniformVampConfig
    qcfg = types.SimpleNamespace(bits=4, group_size=128, desc_act=False,
                                 mpq=types.SimpleNamespace(rotation_mode="internal_hadamard", solver="vamp"))
    cfg = UniformVampConfig(iters=20, prior_tau=0.2, damping=0.5, polish_sweeps=3, block_cd_backend="auto")
    Wb = W[:ROWS].contiguous()
    t0 = time.time()
    Q, q_int, scale, zero, g_idx, _, st = run_mpq_quantization(
        W=Wb, H=2.0 * H, quantizer=MinMaxQuantizer(4), qcfg=qcfg, module_name="layer4096.scalar", vamp_cfg=cfg,
        adapter_cfg=GPTQAdapterConfig(block_rows=BLOCK_ROWS))
    secs = time.time() - t0
    d = (Wb - Q).double()
    proxy = float(((d @ H.double()) * d).sum())
    # stage by stage: the chain without the polish (the VAMP stage with its best-iterate stop) and with one sweep
    stages = {}
    for sweeps, key in ((0, "sc/q_vamp"), (1, "sc/q_sweep1")):
        cfg_s = UniformVampConfig(iters=20, prior_tau=0.2, damping=0.5, polish_sweeps=sweeps, block_cd_backend="auto")
        _, q_s, _, _, _, _, _ = run_mpq_quantization(
            W=Wb, H=2.0 * H, quantizer=MinMaxQuantizer(4), qcfg=qcfg, module_name="layer4096.scalar", vamp_cfg=cfg_s,
            adapter_cfg=GPTQAdapterConfig(block_rows=BLOCK_ROWS))
        stages[key] = q_s.numpy().astype(np.uint8)
    meta = dict(rows=ROWS, block_rows=BLOCK_ROWS, iters=20, proxy=proxy, raw_objective=st["raw_objective_mean_final"],
                obs_init=st["obs_precision_initial"], obs_final=st["obs_precision_final"],
                best_iters=[b["best_iter"] for b in st["block_stats"]], seconds=secs)
    print("scalar", json.dumps(meta))
    return {"sc/q_int": q_int.numpy().astype(np.uint8), "sc/scale": scale.numpy(), "sc/zero": zero.numpy(),
            "sc/meta": np.array(json.dumps(meta)), **stages}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference source tree (poseidonchan/MPQ)")
    ap.add_argument("--threads", type=int, default=8)
    ap.add_argument("--only", default="", choices=["", "scalar", "e8p12"], help="regenerate one case, keep the rest")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    sys.path.insert(0, str(HERE))
    torch.set_num_threads(args.threads)
    from layer4096_inputs import synth
    W, H, SU, SV = synth("cpu")
    out = HERE / "layer4096.npz"
    cases = dict(np.load(out)) if (args.only and out.exists()) else {}
    if args.only in ("", "scalar"):
        cases.update(scalar_case(W, H))
    if args.only in ("", "e8p12"):
        cases.update(e8p12_case(W, H, SU, SV))
    np.savez_compressed(out, **cases)
    print("wrote", HERE / "layer4096.npz")


if __name__ == "__main__":
    main()
