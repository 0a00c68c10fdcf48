"""Parity at the benchmark's width: 256 rows x 4096 columns of BASELINE configs 0 and 1, solved by the CUDA drivers
with the reference's own blocking (chained 128-row blocks), against the reference's outputs on the same inputs
(tests/golden/layer4096.npz, written by tests/golden/make_layer4096.py running the reference on the CPU).

Stage by stage:
  * VAMP stage (the chain without the polish): >= 99.9 % code agreement;
  * one polish sweep started from the reference's own VAMP-stage codes: >= 99.9 % code agreement;
  * the full solve (VAMP + 3 polish sweeps): proxy loss tr((W - Q) H (W - Q)^T) within 0.5 % of the reference's,
    with the reference's chained 128-row blocks and with the same rows as one 256-row block.
The full solve's codes are not held to 99.9 %: the greedy polish orders the blocks of a sweep by gains averaged
over the block's rows, so a single changed code of one row reorders near-tied blocks of the next sweep for every
row.  The reference itself shows it (the fixture's meta records its own polish with 2 of 65,536 starting codes
changed), and float32 rounding differences between any two implementations change a few VAMP-stage codes."""
import json
import sys
import types

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def layer(golden_dir, cuda_dev):
    sys.path.insert(0, str(golden_dir))
    from layer4096_inputs import synth
    W, H, SU, SV = synth(device=str(cuda_dev))
    z = np.load(golden_dir / "layer4096.npz")
    return {"W": W.to(cuda_dev), "H": H.to(cuda_dev), "SU": SU.to(cuda_dev), "SV": SV.to(cuda_dev), "z": z}


def _proxy(Wb, Q, H):
    d = (Wb - Q).double()
    return float(((d @ H.double()) * d).sum())


@pytest.fixture(scope="module")
def e8(layer):
    """Rotated, RMS-normalised rows and the rotated Hessian (the QUIP# flow), RTN start, codebook."""
    from layer4096_inputs import rms_scale
    from mpq_b200.codebook import E8P12_codebook
    from mpq_b200.e8p12 import e8p12_nearest
    from mpq_b200.rotation import rht_hessian, rht_weight
    W, H = layer["W"], layer["H"]
    meta = json.loads(str(layer["z"]["e8/meta"]))
    rows, n = meta["rows"], W.shape[1]
    Wr = rht_weight(W, layer["SU"], layer["SV"], W.shape[0], n)
    Hr = rht_hessian(H, layer["SV"], n)
    wscale = rms_scale(Wr)
    assert abs(wscale - meta["wscale"]) <= 1e-12 * meta["wscale"]
    Wn = (Wr[:rows] / wscale).contiguous()
    cb = E8P12_codebook()
    hat0, q0 = e8p12_nearest(Wn.reshape(-1, 8), cb)
    return {"Wn": Wn, "Hr": Hr, "cb": cb, "hat0": hat0.view(rows, n), "q0": q0.view(rows, n // 8), "meta": meta}


def _refine(e8, *, block_rows, sweeps):
    from mpq_b200.adapters.quip_sharp import mpq_refine_codebook
    args = types.SimpleNamespace(mpq_init="rtn", mpq_iters=e8["meta"]["iters"], mpq_prior_tau=0.25,
                                 mpq_polish_sweeps=sweeps, mpq_block_rows=block_rows, quant_solver="vamp",
                                 quant_polish_mode="block_cd" if sweeps else "none", mpq_polish_metric="gram")
    return mpq_refine_codebook(e8["Wn"], e8["Hr"], e8["hat0"], e8["q0"], e8["cb"], args,
                               module_name="layer4096.e8p12")


def test_e8p12_layer4096_vamp_stage(layer, e8):
    hat, idx, st = _refine(e8, block_rows=e8["meta"]["block_rows"], sweeps=0)
    agree = float((idx.cpu().numpy() == layer["z"]["e8/Qidxs_vamp"]).mean())
    assert agree >= 0.999, agree
    assert abs(st["obs_precision_final"] - e8["meta"]["obs_final"]) <= 1e-4 * e8["meta"]["obs_final"]


def test_e8p12_layer4096_polish_sweep_from_reference_codes(layer, e8):
    """One gram-metric polish sweep per 128-row block, started from the reference's own VAMP-stage codes."""
    from mpq_b200 import ops
    from mpq_b200.adapters.gptqmodel import vamp_hessian_eigen
    from mpq_b200.solver import polish_e8p12_rankspace
    z = layer["z"]
    lam, V, _ = vamp_hessian_eigen(e8["Hr"], fp64=True)
    Vs = (V * torch.sqrt(lam).unsqueeze(0)).contiguous()
    grid = e8["cb"].grid.to(e8["Wn"].device)
    codes = torch.from_numpy(z["e8/Qidxs_vamp"].astype(np.int64)).to(e8["Wn"].device)
    br, out = e8["meta"]["block_rows"], []
    for r0 in range(0, codes.shape[0], br):
        c = codes[r0:r0 + br]
        Y_u = ops.mm_nt(e8["Wn"][r0:r0 + br].contiguous(), ops.Operand(Vs.t().contiguous()), precision="fp32")
        x0 = grid.index_select(0, c.reshape(-1)).reshape(c.shape[0], -1)
        _, idx, _, _ = polish_e8p12_rankspace(x_init=x0, idxs_init=c, Y_u=Y_u, Vs=Vs, cb=e8["cb"], sweeps=1,
                                              polish_mode="block_cd", polish_metric="gram")
        out.append(idx.cpu().numpy())
    agree = float((np.concatenate(out) == z["e8/Qidxs_sweep1"]).mean())
    assert agree >= 0.999, agree


@pytest.mark.parametrize("block_rows", [128, 256])
def test_e8p12_layer4096_proxy_loss(layer, e8, block_rows):
    hat, idx, st = _refine(e8, block_rows=block_rows, sweeps=3)
    torch.cuda.synchronize()
    meta = e8["meta"]
    proxy = _proxy(e8["Wn"], hat, e8["Hr"])
    rel = abs(proxy - meta["proxy"]) / meta["proxy"]
    assert rel <= 0.005, (proxy, meta["proxy"], rel)
    assert proxy < meta["proxy_rtn"]
    print(f"block_rows {block_rows}: proxy {proxy:.3f} vs reference {meta['proxy']:.3f} ({rel:.2e}); code agreement "
          f"{float((idx.cpu().numpy() == layer['z']['e8/Qidxs']).mean()):.4f}")


def _scalar(layer, *, block_rows, sweeps):
    from mpq_b200.adapters.gptqmodel import GPTQAdapterConfig, run_mpq_quantization
    from mpq_b200.solver import UniformVampConfig
    meta = json.loads(str(layer["z"]["sc/meta"]))
    Wb = layer["W"][:meta["rows"]].contiguous()
    qcfg = types.SimpleNamespace(bits=4, group_size=128, desc_act=False,
                                 mpq=types.SimpleNamespace(rotation_mode="internal_hadamard", solver="vamp"))
    cfg = UniformVampConfig(iters=meta["iters"], prior_tau=0.2, damping=0.5, polish_sweeps=sweeps,
                            block_cd_backend="auto")
    out = run_mpq_quantization(W=Wb, H=2.0 * layer["H"], quantizer=None, qcfg=qcfg, module_name="layer4096.scalar",
                               vamp_cfg=cfg, adapter_cfg=GPTQAdapterConfig(block_rows=block_rows, grow_block_rows=False))
    return Wb, meta, out


def test_scalar_layer4096_vamp_stage(layer):
    """The VAMP stage (with its best-iterate stop) of the chained 128-row blocks."""
    z = layer["z"]
    Wb, meta, (Q, q_int, scale, zero, g_idx, _, st) = _scalar(layer, block_rows=json.loads(str(z["sc/meta"]))["block_rows"],
                                                              sweeps=0)
    np.testing.assert_allclose(scale.cpu().numpy(), z["sc/scale"], rtol=1e-6)
    np.testing.assert_array_equal(zero.cpu().numpy(), z["sc/zero"])
    agree = float((q_int.cpu().numpy() == z["sc/q_vamp"]).mean())
    assert agree >= 0.999, agree
    assert [b["best_iter"] for b in st["block_stats"]] == meta["best_iters"]


def test_scalar_layer4096_polish_sweep_from_reference_codes(layer):
    """One raw-Hessian greedy CD sweep per 128-row block started from the reference's own VAMP-stage codes, then the
    row-wise keep-if-better merge (mpq/solver.py:749-754), against the reference's one-sweep chain."""
    from mpq_b200 import ops
    from mpq_b200._lib import call, ptr
    from mpq_b200.adapters.gptqmodel import vamp_hessian_eigen
    from mpq_b200.rotation import apply_right_block_hadamard, resolve_block_hadamard_plan, sample_rademacher_signs
    from mpq_b200.solver import polish_uniform_rankspace
    z = layer["z"]
    meta = json.loads(str(z["sc/meta"]))
    dev = layer["W"].device
    n, rows, br = layer["W"].shape[1], meta["rows"], meta["block_rows"]
    _, had = resolve_block_hadamard_plan(n)
    signs = sample_rademacher_signs(width=n, key="layer4096.scalar:full", seed=0, device=dev)
    Hw = 0.5 * (2.0 * layer["H"])
    lam, V, _ = vamp_hessian_eigen(Hw)
    Wr = apply_right_block_hadamard(layer["W"][:rows].contiguous(), signs=signs, had_dim=had)
    Hm = apply_right_block_hadamard(Hw.T.contiguous(), signs=signs, had_dim=had).T.contiguous()
    Hm = apply_right_block_hadamard(Hm, signs=signs, had_dim=had)
    V = apply_right_block_hadamard(V.T.contiguous(), signs=signs, had_dim=had).T.contiguous()
    Vs = (V * torch.sqrt(lam).unsqueeze(0)).contiguous()
    sg = torch.from_numpy(z["sc/scale"]).to(dev)
    zg = torch.from_numpy(z["sc/zero"]).to(dev)
    q_v = torch.from_numpy(z["sc/q_vamp"].astype(np.float32)).to(dev)
    x_v = sg.repeat_interleave(128, 1) * (q_v - zg.repeat_interleave(128, 1))
    VsT = ops.Operand(Vs.t().contiguous())
    out = []
    for r0 in range(0, rows, br):
        rb = slice(r0, r0 + br)
        Y_u = ops.mm_nt(Wr[rb].contiguous(), VsT, precision="fp32")
        q_p, x_p, err_p, _ = polish_uniform_rankspace(x_init=x_v[rb].contiguous(), Y_u=Y_u, Vs=Vs,
                                                      scale_full=sg[rb].contiguous(), zero_full=zg[rb].contiguous(),
                                                      maxq=15, sweeps=1, polish_mode="block_cd",
                                                      block_cd_backend="auto", gram_full=Hm)
        C = ops.mm_nt(x_v[rb].contiguous(), VsT)
        err_v = torch.empty(br, device=dev)
        call("mpq_row_sqerr", ptr(Y_u), ptr(C), br, C.shape[1], Y_u.stride(0), C.stride(0), ptr(err_v))
        keep = (err_p + 1e-12) < err_v
        q = torch.where(keep[:, None], q_p.to(torch.float32), q_v[rb])
        out.append(q.to(torch.uint8).cpu().numpy())
    agree = float((np.concatenate(out) == z["sc/q_sweep1"]).mean())
    assert agree >= 0.999, agree


@pytest.mark.parametrize("block_rows", [128, 256])
def test_scalar_layer4096_proxy_loss(layer, block_rows):
    Wb, meta, (Q, q_int, scale, zero, g_idx, _, st) = _scalar(layer, block_rows=block_rows, sweeps=3)
    torch.cuda.synchronize()
    proxy = _proxy(Wb, Q, layer["H"])
    rel = abs(proxy - meta["proxy"]) / meta["proxy"]
    assert rel <= 0.005, (proxy, meta["proxy"], rel)
    print(f"block_rows {block_rows}: proxy {proxy:.4f} vs reference {meta['proxy']:.4f} ({rel:.2e}); code agreement "
          f"{float((q_int.cpu().numpy() == layer['z']['sc/q_int']).mean()):.4f}")
