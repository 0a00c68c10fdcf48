"""Generate golden input/output vectors by running the REFERENCE implementation (poseidonchan/MPQ).

Run in a container where the reference source tree is importable (pass its path with
``--reference``).  The outputs are small ``.npz`` fixtures committed next to this script;
tests read only the fixtures, never the reference tree.

Where the reference calls into third-party code that is not vendored (GPTQModel's
``Quantizer.find_params``; the CUDA dispatch of the uniform polish), this script passes the
same restatements the oracle and the product use, and says so in the fixture metadata.
"""
from __future__ import annotations

import argparse
import json
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _np(t):
    return t.detach().cpu().numpy()


class MinMaxQuantizer:
    """Asymmetric per-row min-max grid: the restatement of GPTQModel's find_params."""

    def __init__(self, bits: int):
        self.maxq = 2 ** bits - 1

    def find_params(self, x, weight=True):
        zero = torch.zeros(x.shape[0], dtype=x.dtype)
        xmin = torch.minimum(x.min(1)[0], zero)
        xmax = torch.maximum(x.max(1)[0], zero)
        tmp = (xmin == 0) & (xmax == 0)
        xmin[tmp] = -1
        xmax[tmp] = 1
        self.scale = ((xmax - xmin) / self.maxq).unsqueeze(1)
        self.zero = torch.round(-xmin / self.scale.squeeze(1)).unsqueeze(1)


def synth_layer(m, n, seed, calib_mult=4):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(m, n, generator=g) * 0.02
    s = torch.exp(torch.randn(n, generator=g))
    X = torch.randn(calib_mult * n, n, generator=g) * s.sqrt()
    H = X.T @ X / X.shape[0]
    H = H + 0.01 * H.diagonal().mean() * torch.eye(n)
    return W, H


def gen_uniform_denoise(out):
    from mpq.priors.uniform import discrete_uniform_mmse, nearest_atom_idx, dequant_from_q
    g = torch.Generator().manual_seed(11)
    cases = {}
    for name, (B, n, maxq, tau) in {"q4": (6, 256, 15, 0.2), "q3": (5, 128, 7, 0.25), "q4_noprior": (4, 128, 15, 0.0)}.items():
        W = torch.randn(B, n, generator=g) * 0.02
        scale = (torch.rand(B, n // 64, generator=g) * 0.01 + 0.002).repeat_interleave(64, 1)
        zero = torch.randint(0, maxq + 1, (B, n // 64), generator=g).float().repeat_interleave(64, 1)
        r1 = W + torch.randn(B, n, generator=g) * 0.01
        # exact ties: r1 halfway between two atoms, center far away
        r1[0, :16] = scale[0, :16] * (torch.arange(16).float() % maxq + 0.5 - zero[0, :16])
        gamma = torch.rand(B, 1, generator=g) * 2e4 + 1e3
        post = discrete_uniform_mmse(r1=r1, gamma1=gamma, scale_full=scale, zero_full=zero, maxq=maxq,
                                     prior_center=W, prior_tau=tau, need_stats=False, vamp_backend="eager")
        q = nearest_atom_idx(x=post["map_value"], scale_full=scale, zero_full=zero, maxq=maxq)
        x = dequant_from_q(q_int=q, scale_full=scale, zero_full=zero)
        for k, v in dict(r1=r1, W=W, scale=scale, zero=zero, gamma=gamma, mean=post["mean"], var=post["var"],
                         map_idx=post["map_idx"], map_value=post["map_value"], alpha1=post["alpha1"], q=q, x=x).items():
            cases[f"{name}/{k}"] = _np(v)
        cases[f"{name}/maxq"] = np.array(maxq)
        cases[f"{name}/tau"] = np.array(tau, dtype=np.float64)
    # rounding ties of nearest_atom_idx: x/scale + zero exactly k + 0.5
    scale = torch.full((2, 32), 0.5)
    zero = torch.full((2, 32), 3.0)
    x = (torch.arange(64).float().view(2, 32) * 0.25 - 4.0)
    cases["ties/x"] = _np(x)
    cases["ties/scale"] = _np(scale)
    cases["ties/zero"] = _np(zero)
    cases["ties/q"] = _np(nearest_atom_idx(x=x, scale_full=scale, zero_full=zero, maxq=7))
    np.savez_compressed(out / "uniform_denoise.npz", **cases)


def gen_linear(out):
    from mpq.linear import linear_mmse_exact, em_update_obs_precision_rankspace, vamp_rankspace_error
    W, H = synth_layer(8, 64, 3)
    lam, V = torch.linalg.eigh(H)
    lam = lam.flip(0).clamp_min(1e-6 * float(lam.max()))
    V = V.flip(1).contiguous()
    S = lam.sqrt()
    Vs = V * S
    g = torch.Generator().manual_seed(5)
    r2 = W + torch.randn(W.shape, generator=g) * 0.005
    gamma2 = torch.rand(8, 1, generator=g) * 1e4 + 1e3
    Y_u = W @ Vs
    obs = 1234.5
    x2, a2, res = linear_mmse_exact(r2, gamma2, Y_u=Y_u, V=V, Vh=V.T.contiguous(), S=S, obs_precision=obs)
    beta = em_update_obs_precision_rankspace(residual_u=res, gamma2=gamma2, S=S, obs_precision=obs, num_obs=64)
    err = vamp_rankspace_error(Y_u=Y_u, x=r2, Vs=Vs)
    np.savez_compressed(out / "linear_mmse.npz", r2=_np(r2), gamma2=_np(gamma2), Y_u=_np(Y_u), V=_np(V), S=_np(S),
                        Vs=_np(Vs), obs=np.array(obs), x2=_np(x2), alpha2=_np(a2), residual=_np(res),
                        beta=np.array(beta), err=_np(err))


def gen_scalar_cd(out):
    from mpq.polish.triton_scalar_cd import uniform_scalar_diag_greedy_cd
    W, H = synth_layer(12, 128, 7)
    lam, V = torch.linalg.eigh(H)
    lam = lam.flip(0).clamp_min(1e-6 * float(lam.max()))
    V = V.flip(1).contiguous()
    Vs = V * lam.sqrt()
    maxq = 15
    Wg = W.view(12, 2, 64)
    mn, mx = Wg.amin(-1).clamp(max=0), Wg.amax(-1).clamp(min=0)
    scale = ((mx - mn) / maxq).repeat_interleave(64, 1)
    zero = torch.round(-mn / ((mx - mn) / maxq)).repeat_interleave(64, 1)
    q = torch.clamp(torch.round(W / scale) + zero, 0, maxq)
    x = scale * (q - zero)
    Y_u = W @ Vs
    xp, st = uniform_scalar_diag_greedy_cd(x=x, Y_u=Y_u, Vs=Vs, gram_full=H, scale=scale, zero=zero, maxq=maxq,
                                           sweeps=3, update_backend="torch")
    np.savez_compressed(out / "scalar_cd.npz", x=_np(x), Y_u=_np(Y_u), Vs=_np(Vs), H=_np(H), scale=_np(scale),
                        zero=_np(zero), x_out=_np(xp), accepted=np.array(st["accepted_updates"]))


def _install_gpu_polish_semantics():
    """Route the uniform polish through the raw-H greedy CD (the reference's CUDA dispatch,
    mpq/solver.py:299-333) with the torch twin, since CUDA is absent in this container."""
    import mpq.solver as S
    from mpq.polish.triton_scalar_cd import uniform_scalar_diag_greedy_cd
    from mpq.priors.uniform import nearest_atom_idx, dequant_from_q
    from mpq.linear import vamp_rankspace_error

    def polish(*, x_init, Y_u, Vs, scale_full, zero_full, maxq, sweeps, polish_mode, gram_full=None, **kw):
        xp, st = uniform_scalar_diag_greedy_cd(x=x_init.float(), Y_u=Y_u, Vs=Vs, gram_full=gram_full,
                                               scale=scale_full, zero=zero_full, maxq=maxq, sweeps=int(sweeps),
                                               accept_tol=0.0, update_backend="torch")
        q = nearest_atom_idx(x=xp, scale_full=scale_full, zero_full=zero_full, maxq=maxq).to(torch.int32)
        xo = dequant_from_q(q_int=q, scale_full=scale_full, zero_full=zero_full)
        return q, xo, vamp_rankspace_error(Y_u=Y_u, x=xo, Vs=Vs), dict(st, block_cd_backend="triton")

    S.polish_uniform_rankspace = polish


def gen_scalar_layer(out):
    _install_gpu_polish_semantics()
    from mpq.adapters.gptqmodel import run_mpq_quantization, GPTQAdapterConfig
    from mpq.solver import UniformVampConfig
    cases = {}
    # (m, n, bits, block_rows, iters, desc_act, final_decision); "c" activation order, "d" round-mean decision
    layers = {"a": (48, 256, 4, 16, 20, False, "map"), "b": (32, 128, 3, 32, 16, False, "map"),
              "c": (40, 256, 4, 16, 16, True, "map"), "d": (32, 256, 3, 16, 12, False, "round_mean")}
    for name, (m, n, bits, block_rows, iters, desc_act, decision) in layers.items():
        W, H = synth_layer(m, n, 100 + m)
        qcfg = types.SimpleNamespace(bits=bits, group_size=64, desc_act=desc_act,
                                     mpq=types.SimpleNamespace(rotation_mode="internal_hadamard", solver="vamp"))
        cfg = UniformVampConfig(iters=iters, prior_tau=0.2, damping=0.5, polish_sweeps=3, block_cd_backend="auto",
                                final_decision=decision)
        acfg = GPTQAdapterConfig(block_rows=block_rows)
        Q, q_int, scale, zero, g_idx, _, st = run_mpq_quantization(
            W=W, H=2.0 * H, quantizer=MinMaxQuantizer(bits), qcfg=qcfg, module_name=f"golden.{name}",
            vamp_cfg=cfg, adapter_cfg=acfg)
        for k, v in dict(W=W, H=H, Q=Q, q_int=q_int, scale=scale, zero=zero, g_idx=g_idx).items():
            cases[f"{name}/{k}"] = _np(v)
        cases[f"{name}/meta"] = np.array(json.dumps(dict(bits=bits, group_size=64, block_rows=block_rows, iters=iters,
                                                          desc_act=desc_act, final_decision=decision,
                                                          obs_init=st["obs_precision_initial"],
                                                          obs_final=st["obs_precision_final"],
                                                          raw_objective=st["raw_objective_mean_final"],
                                                          best_iters=[b["best_iter"] for b in st["block_stats"]],
                                                          stop_iters=[b["stop_iter"] for b in st["block_stats"]],
                                                          polish_updates=[b["polish_updates"] for b in st["block_stats"]])))
    np.savez_compressed(out / "scalar_layer.npz", **cases)


def gen_rotation(out):
    from mpq.rotation import apply_right_block_hadamard, apply_right_block_hadamard_inverse, sample_rademacher_signs
    from mpq.utils import stable_seed
    g = torch.Generator().manual_seed(9)
    M = torch.randn(6, 256, generator=g)
    signs = sample_rademacher_signs(width=256, key="golden.rot:full", seed=0, device=torch.device("cpu"))
    R = apply_right_block_hadamard(M, signs=signs, had_dim=64)
    Ri = apply_right_block_hadamard_inverse(R, signs=signs, had_dim=64)
    seeds = np.array([stable_seed(k, base_seed=b) for k, b in [("a", 0), ("model.layers.0.q_proj:full", 0), ("x", 7)]])
    np.savez_compressed(out / "rotation.npz", M=_np(M), signs=_np(signs), R=_np(R), Ri=_np(Ri), seeds=seeds)


def _reference_codebook():
    """Torch wrapper of the restated E8P12 grid with the attributes the reference reads; its quantize()
    is the reference's own factorized MAP at unit precision (nearest codeword)."""
    sys.path.insert(0, str(HERE.parents[1]))
    from oracle.e8p12 import E8P12_codebook as NpCB
    from mpq.priors.e8p12 import vamp_vector_map_e8p12

    class E8P12_codebook:
        codesz = 8
        idx_dtype = torch.int64

        def __init__(self):
            self.grid = torch.from_numpy(NpCB().grid.copy())
            self.grid_packed_abs = torch.arange(256, dtype=torch.int64)

        def quantize(self, X, return_idx=True, **kw):
            X = X.reshape(-1, 8).float()
            out = vamp_vector_map_e8p12(r1_blocks=X.view(1, -1, 8), gamma1=torch.ones(1, 1), cb=self,
                                        blocks_per_chunk=1 << 30)
            idx = out["map_idxs"].view(-1)
            vals = self.grid.index_select(0, idx)
            return (vals, idx) if return_idx else vals

    return E8P12_codebook()


def gen_e8p12(out):
    from mpq.priors.e8p12 import vamp_vector_discrete_mmse_e8p12, vamp_vector_map_e8p12, prior_scale_from_center
    from mpq.polish.block_cd import _cd_gram_step_impl
    from mpq.linear import stabilize_cholesky
    cb = _reference_codebook()
    g = torch.Generator().manual_seed(21)
    cases = {}
    B, nb = 12, 40
    W = torch.randn(B, nb, 8, generator=g) * 0.8
    r1 = W + torch.randn(B, nb, 8, generator=g) * 0.3
    ps = prior_scale_from_center(W, "absmax")
    for name, gam in {"lo": torch.rand(B, 1, generator=g) * 4 + 1, "hi": torch.rand(B, 1, generator=g) * 40 + 10,
                      "snap": torch.full((B, 1), 1500.0)}.items():
        post = vamp_vector_discrete_mmse_e8p12(r1_blocks=r1, gamma1=gam, cb=cb, blocks_per_chunk=nb,
                                               prior_center_blocks=W, prior_scale_blocks=ps, prior_tau=0.25,
                                               compile_prior=False)
        mp = vamp_vector_map_e8p12(r1_blocks=r1, gamma1=gam, cb=cb, blocks_per_chunk=nb, prior_center_blocks=W,
                                   prior_scale_blocks=ps, prior_tau=0.25)
        for k in ("x1_blocks", "var1", "map_idxs", "alpha1"):
            cases[f"{name}/{k}"] = _np(post[k])
        cases[f"{name}/map_only_idxs"] = _np(mp["map_idxs"])
        cases[f"{name}/gamma"] = _np(gam)
    cases["r1"] = _np(r1)
    cases["W"] = _np(W)
    # nearest codeword (RTN) of unscaled Gaussian blocks
    X = torch.randn(2048, 8, generator=g)
    _, qi = cb.quantize(X)
    cases["rtn/X"] = _np(X)
    cases["rtn/idx"] = _np(qi)
    # one gram-metric CD step (mpq/polish/block_cd.py:212-246)
    n, R, Bc = 64, 64, 48
    Vs = torch.randn(n, R, generator=g) / 8
    resid = torch.randn(Bc, R, generator=g) * 0.5
    xb = cb.grid[torch.randint(0, 65536, (Bc,), generator=g)]
    vb = Vs[8:16]
    gram = vb @ vb.T
    chol = stabilize_cholesky(gram)
    ginv = torch.cholesky_inverse(chol)
    rn = resid.square().sum(1)
    new_x, best, acc, rupd, nn_, na = _cd_gram_step_impl(resid, xb, vb.T.contiguous(), ginv, chol, cb.grid, gram, vb,
                                                         rn, 0.0)
    for k, v in dict(Vs=Vs, resid=resid, xb=xb, chol=chol, ginv=ginv, best=best, accept=acc, new_x=new_x).items():
        cases[f"gram/{k}"] = _np(v)
    np.savez_compressed(out / "e8p12_prior.npz", **cases)


def gen_e8p12_stats(out):
    """The posterior's diagnostics (need_stats): per-block log-partition, entropy and top-2 log-score margin."""
    from mpq.priors.e8p12 import vamp_vector_discrete_mmse_e8p12, prior_scale_from_center
    cb = _reference_codebook()
    g = torch.Generator().manual_seed(33)
    cases = {}
    B, nb = 6, 24
    W = torch.randn(B, nb, 8, generator=g) * 0.8
    r1 = W + torch.randn(B, nb, 8, generator=g) * 0.3
    ps = prior_scale_from_center(W, "absmax")
    gams = {"lo": torch.rand(B, 1, generator=g) * 4 + 0.5, "hi": torch.rand(B, 1, generator=g) * 40 + 10,
            "snap": torch.full((B, 1), 1500.0)}
    for name, gam in gams.items():
        for tau in (0.0, 0.25):
            post = vamp_vector_discrete_mmse_e8p12(r1_blocks=r1, gamma1=gam, cb=cb, blocks_per_chunk=nb,
                                                   need_stats=True, prior_center_blocks=W if tau else None,
                                                   prior_scale_blocks=ps if tau else None, prior_tau=tau,
                                                   compile_prior=False, return_logZ_blocks=True,
                                                   return_margin_blocks=True, return_entropy_blocks=True)
            key = f"{name}_t{int(tau * 100)}"
            for k in ("logZ_blocks", "margin_blocks", "entropy_blocks", "x1_blocks", "var1"):
                cases[f"{key}/{k}"] = _np(post[k])
            cases[f"{key}/entropy"] = np.array(post["entropy"])
            cases[f"{key}/margin"] = np.array(post["margin"])
        cases[f"{name}/gamma"] = _np(gam)
    cases["r1"] = _np(r1)
    cases["W"] = _np(W)
    cases["ps"] = _np(ps)
    np.savez_compressed(out / "e8p12_stats.npz", **cases)


def gen_e8p12_layer(out):
    from mpq.adapters.quip_sharp import mpq_refine_codebook
    cb = _reference_codebook()
    cases = {}
    for name, (m, n, block_rows, iters) in {"a": (32, 256, 16, 16), "b": (24, 128, 24, 8)}.items():
        W, H = synth_layer(m, n, 300 + m)
        Wr = W / W.square().mean().sqrt() * 0.9  # unit-scale weights as QUIP# feeds the codebook
        args = types.SimpleNamespace(mpq_init="rtn", mpq_iters=iters, mpq_prior_tau=0.25, mpq_polish_sweeps=3,
                                     mpq_block_rows=block_rows, mpq_blocks_per_chunk=1 << 20, mpq_compile_prior=False,
                                     quant_solver="vamp", quant_polish_mode="block_cd", mpq_polish_metric="gram")
        hat0, q0 = cb.quantize(Wr.reshape(-1, 8))
        hatWr, Qidxs, st = mpq_refine_codebook(Wr, H, hat0.view(m, n), q0.view(m, n // 8), cb, args,
                                               module_name=f"golden.e8.{name}")
        for k, v in dict(Wr=Wr, H=H, hatWr=hatWr, Qidxs=Qidxs).items():
            cases[f"{name}/{k}"] = _np(v)
        cases[f"{name}/meta"] = np.array(json.dumps(dict(block_rows=block_rows, iters=iters,
                                                          obs_init=st["obs_precision_initial"],
                                                          obs_final=st["obs_precision_final"],
                                                          surrogate_before=st["exact_surrogate_before_mean"],
                                                          surrogate_after=st["exact_surrogate_after_mean"],
                                                          changed=st["mechanism"]["cleanup_changed_count"])))
    np.savez_compressed(out / "e8p12_layer.npz", **cases)


def gen_e8p12_topk_layer(out):
    """mpq_refine_codebook with the top-k polish recipe (quant_polish_mode "topk_block_cd")."""
    from mpq.adapters.quip_sharp import mpq_refine_codebook
    cb = _reference_codebook()
    cases = {}
    m, n, block_rows, iters, k = 24, 128, 24, 8, 12
    W, H = synth_layer(m, n, 777)
    Wr = W / W.square().mean().sqrt() * 0.9
    args = types.SimpleNamespace(mpq_init="rtn", mpq_iters=iters, mpq_prior_tau=0.25, mpq_polish_sweeps=3,
                                 mpq_block_rows=block_rows, mpq_blocks_per_chunk=1 << 20, mpq_compile_prior=False,
                                 quant_solver="vamp", quant_polish_mode="topk_block_cd", mpq_polish_metric="gram",
                                 mpq_topk_k=k)
    hat0, q0 = cb.quantize(Wr.reshape(-1, 8))
    hatWr, Qidxs, st = mpq_refine_codebook(Wr, H, hat0.view(m, n), q0.view(m, n // 8), cb, args,
                                           module_name="golden.e8.topk")
    for kk, v in dict(Wr=Wr, H=H, hatWr=hatWr, Qidxs=Qidxs).items():
        cases[f"t/{kk}"] = _np(v)
    cases["t/meta"] = np.array(json.dumps(dict(block_rows=block_rows, iters=iters, k=k,
                                                surrogate_after=st["exact_surrogate_after_mean"])))
    np.savez_compressed(out / "e8p12_topk_layer.npz", **cases)


def _tiny_llama(seed, dtype=torch.float64):
    from transformers import AutoModelForCausalLM, LlamaConfig
    cfg = LlamaConfig(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=2,
                      num_key_value_heads=2, head_dim=32, vocab_size=128, initializer_range=0.02,
                      attn_implementation="sdpa", max_position_embeddings=256)
    torch.manual_seed(seed)
    model = AutoModelForCausalLM.from_config(cfg, dtype=dtype).eval()
    with torch.no_grad():  # log-normal channel gains: activation outliers for the scale search to find
        for layer in model.model.layers:
            layer.input_layernorm.weight.copy_(torch.exp(1.5 * torch.randn(cfg.hidden_size)))
            layer.post_attention_layernorm.weight.copy_(torch.exp(1.5 * torch.randn(cfg.hidden_size)))
    return model


def gen_awq(out):
    """mpq/awq_scale.py apply_awq_scaling on a tiny Llama (4-bit g32, asymmetric), in float64: with float32 weights
    on the CPU the reference's saved copies (`.to(float32).cpu().contiguous()`) alias the live weights, so its
    per-ratio restore is a no-op; in float64 (as in bf16 on the GPU) the copy is real."""
    from mpq.awq_scale import apply_awq_scaling
    from mpq.dense_decoder_adapter import resolve_dense_decoder_adapter_for_model
    model = _tiny_llama(5)
    before = {k: v.clone() for k, v in model.state_dict().items()}
    g = torch.Generator().manual_seed(9)
    ids = torch.randint(0, 128, (4, 32), generator=g)
    blocks = [{"input_ids": ids[i:i + 1]} for i in range(ids.shape[0])]
    adapter = resolve_dense_decoder_adapter_for_model(model)
    dbg = apply_awq_scaling(model, adapter, blocks, bits=4, group_size=32, sym=False, batch_size=2, device="cpu")
    # the starting weights are rebuilt by the test from the same seeded CPU initialisation (a checksum pins them);
    # the scaled weights are stored in float32 (the test's tolerance is 1e-5)
    cases = {"ids": _np(ids), "before_checksum": np.array([float(v.double().abs().sum()) for v in before.values()])}
    for k, v in model.state_dict().items():
        if not torch.equal(v, before[k]):
            cases[f"after/{k}"] = _np(v.float())
    cases["meta"] = np.array(json.dumps(dbg))
    np.savez_compressed(out / "awq.npz", **cases)


def _block_cd_problem(B, n, R, seed, scale_rows=0.02):
    """A rank-space least-squares problem Y_u = W Vs with Vs from a random Hessian's eigenbasis."""
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(B, n, generator=g) * scale_rows
    s = torch.exp(torch.randn(n, generator=g))
    X = torch.randn(4 * n, n, generator=g) * s.sqrt()
    H = X.T @ X / X.shape[0] + 0.01 * torch.eye(n)
    lam, V = torch.linalg.eigh(H.double())
    lam, V = lam.flip(0)[:R].clamp_min(1e-6), V.flip(1)[:, :R]
    Vs = (V * lam.sqrt()).float().contiguous()
    return W, H, Vs


def gen_block_cd(out):
    """The reference's generic rank-space block CD (plugin engine) with its own providers, eager steps."""
    from mpq.polish.block_cd import BlockCDConfig, E8P12Provider, UniformScalarProvider, block_coordinate_descent_rankspace
    cases = {}
    # scalar provider, block_size 1, diag metric, three orders
    for name, order in {"s_greedy": "greedy_gain", "s_static": "static", "s_cyclic": "cyclic"}.items():
        B, n, maxq = 12, 64, 15
        W, H, Vs = _block_cd_problem(B, n, n, 41)
        q = MinMaxQuantizer(4)
        q.find_params(W)
        scale = q.scale.expand(B, n).contiguous()
        zero = q.zero.expand(B, n).contiguous()
        x0 = scale * (torch.clamp(torch.round(W / scale) + zero, 0, maxq) - zero)
        Y_u = W @ Vs
        cfg = BlockCDConfig(sweeps=2, metric="diag", order_mode=order, compile_steps=False)
        prov = UniformScalarProvider(scale=scale, zero=zero, maxq=maxq)
        q0 = torch.clamp(torch.round(x0 / scale + zero), 0, maxq).to(torch.int32)  # as polish_uniform_rankspace
        xo, qo, st = block_coordinate_descent_rankspace(x=x0, Y_u=Y_u, Vs=Vs, block_size=1, provider=prov, cfg=cfg,
                                                        idxs_init=q0, raw_target=W, raw_gram=H)
        for k, v in dict(W=W, H=H, Vs=Vs, scale=scale, zero=zero, x0=x0, q0=q0, Y_u=Y_u, x=xo, q=qo).items():
            cases[f"{name}/{k}"] = _np(v)
        cases[f"{name}/meta"] = np.array(json.dumps({"order": order, "sweeps": 2, "maxq": maxq, "stats": st}))
    # E8P12 provider, block_size 8: gram metric (eager generic path) and isotropic metric, capped blocks
    cb = _reference_codebook()
    for name, (metric, max_blocks) in {"e_gram": ("gram", 0), "e_iso": ("diag", 0), "e_gram_cap": ("gram", 5)}.items():
        B, n = 10, 64
        W, H, Vs = _block_cd_problem(B, n, n, 53, scale_rows=1.0)
        x0, i0 = cb.quantize(W.reshape(-1, 8))
        x0, i0 = x0.reshape(B, n), i0.reshape(B, n // 8)
        Y_u = W @ Vs
        cfg = BlockCDConfig(sweeps=2, metric=metric, order_mode="greedy_gain", max_blocks_per_sweep=max_blocks,
                            compile_steps=False)
        xo, io, st = block_coordinate_descent_rankspace(x=x0, Y_u=Y_u, Vs=Vs, block_size=8, provider=E8P12Provider(cb=cb),
                                                        cfg=cfg, idxs_init=i0)
        for k, v in dict(W=W, Vs=Vs, x0=x0, i0=i0, Y_u=Y_u, x=xo, idx=io).items():
            cases[f"{name}/{k}"] = _np(v)
        cases[f"{name}/meta"] = np.array(json.dumps({"metric": metric, "max_blocks": max_blocks, "sweeps": 2,
                                                     "stats": st}))
    np.savez_compressed(out / "block_cd.npz", **cases)


def gen_topk(out):
    """Top-k candidate sets (uniform and E8P12) and the generic block CD with the top-k providers."""
    from mpq.priors.uniform import uniform_map_topk
    from mpq.priors.e8p12 import vamp_vector_map_topk_e8p12, prior_scale_from_center
    from mpq.polish.block_cd import BlockCDConfig, E8P12TopKProvider, UniformTopKProvider, block_coordinate_descent_rankspace
    cases = {}
    g = torch.Generator().manual_seed(71)
    for name, (bits, tau, k) in {"u4p": (4, 0.25, 5), "u4": (4, 0.0, 16), "u2p": (2, 0.5, 16)}.items():
        B, n, maxq = 6, 48, 2 ** bits - 1
        W = torch.randn(B, n, generator=g) * 0.05
        q = MinMaxQuantizer(bits)
        q.find_params(W)
        scale = q.scale.expand(B, n).contiguous()
        zero = q.zero.expand(B, n).contiguous()
        r1 = W + torch.randn(B, n, generator=g) * 0.01
        gam = torch.rand(B, 1, generator=g) * 2e4 + 1e3
        o = uniform_map_topk(r1=r1, gamma1=gam, scale_full=scale, zero_full=zero, maxq=maxq, prior_center=W,
                             prior_tau=tau, k=k)
        for kk, v in dict(W=W, scale=scale, zero=zero, r1=r1, gamma=gam, q=o["topk_q"], values=o["topk_values"],
                          scores=o["topk_scores"]).items():
            cases[f"{name}/{kk}"] = _np(v)
        cases[f"{name}/meta"] = np.array(json.dumps({"maxq": maxq, "tau": tau, "k": k}))
    cb = _reference_codebook()
    B, nb = 8, 24
    W = torch.randn(B, nb, 8, generator=g) * 0.8
    r1 = W + torch.randn(B, nb, 8, generator=g) * 0.3
    ps = prior_scale_from_center(W, "absmax")
    for name, (lo, hi, tau, k) in {"e_lo_p": (1.0, 5.0, 0.25, 16), "e_hi": (10.0, 50.0, 0.0, 40),
                                   "e_lo": (0.5, 2.0, 0.0, 7)}.items():
        gam = torch.rand(B, 1, generator=g) * (hi - lo) + lo
        o = vamp_vector_map_topk_e8p12(r1_blocks=r1, gamma1=gam, cb=cb, k=k, blocks_per_chunk=nb,
                                       prior_center_blocks=W if tau > 0 else None,
                                       prior_scale_blocks=ps if tau > 0 else None, prior_tau=tau)
        cases[f"{name}/gamma"] = _np(gam)
        cases[f"{name}/idxs"] = _np(o["topk_idxs"])
        cases[f"{name}/scores"] = _np(o["topk_scores"])
        cases[f"{name}/meta"] = np.array(json.dumps({"tau": tau, "k": k}))
    cases["e/r1"] = _np(r1)
    cases["e/W"] = _np(W)
    # generic block CD with the top-k providers (eager steps)
    B, n, maxq = 12, 64, 15
    W, H, Vs = _block_cd_problem(B, n, n, 83)
    q = MinMaxQuantizer(4)
    q.find_params(W)
    scale = q.scale.expand(B, n).contiguous()
    zero = q.zero.expand(B, n).contiguous()
    r1 = W + torch.randn(B, n, generator=g) * 0.004
    gam = torch.full((B, 1), 3e4)
    tk = uniform_map_topk(r1=r1, gamma1=gam, scale_full=scale, zero_full=zero, maxq=maxq, prior_center=W,
                          prior_tau=0.0, k=4)
    x0 = tk["topk_values"][:, :, 0].contiguous()
    q0 = tk["topk_q"][:, :, 0].to(torch.int32)
    Y_u = W @ Vs
    cfg = BlockCDConfig(sweeps=2, metric="diag", order_mode="greedy_gain", compile_steps=False)
    xo, qo, st = block_coordinate_descent_rankspace(
        x=x0, Y_u=Y_u, Vs=Vs, block_size=1, provider=UniformTopKProvider(topk_values=tk["topk_values"], topk_q=tk["topk_q"]),
        cfg=cfg, idxs_init=q0, raw_target=W, raw_gram=H)
    for kk, v in dict(W=W, H=H, Vs=Vs, Y_u=Y_u, x0=x0, q0=q0, tq=tk["topk_q"], tv=tk["topk_values"], x=xo, q=qo).items():
        cases[f"cd_u/{kk}"] = _np(v)
    cases["cd_u/meta"] = np.array(json.dumps({"stats": st}))
    for name, metric in {"cd_eg": "gram", "cd_ed": "diag"}.items():
        B, n = 10, 64
        W, H, Vs = _block_cd_problem(B, n, n, 97, scale_rows=1.0)
        r1 = (W + torch.randn(B, n, generator=g) * 0.2).view(B, n // 8, 8)
        gam = torch.rand(B, 1, generator=g) * 4 + 2
        tk = vamp_vector_map_topk_e8p12(r1_blocks=r1, gamma1=gam, cb=cb, k=12, blocks_per_chunk=1 << 20)
        i0 = tk["topk_idxs"][:, :, 0].contiguous()
        x0 = cb.grid[i0].reshape(B, n)
        Y_u = W @ Vs
        cfg = BlockCDConfig(sweeps=2, metric=metric, order_mode="greedy_gain", compile_steps=False)
        xo, io, st = block_coordinate_descent_rankspace(
            x=x0, Y_u=Y_u, Vs=Vs, block_size=8, provider=E8P12TopKProvider(cb=cb, topk_idxs=tk["topk_idxs"]), cfg=cfg,
            idxs_init=i0)
        for kk, v in dict(W=W, Vs=Vs, Y_u=Y_u, r1=r1, gamma=gam, ti=tk["topk_idxs"], x0=x0, i0=i0, x=xo,
                          idx=io).items():
            cases[f"{name}/{kk}"] = _np(v)
        cases[f"{name}/meta"] = np.array(json.dumps({"metric": metric, "stats": st}))
    np.savez_compressed(out / "topk.npz", **cases)


def gen_postprocess(out):
    """postprocess_gptq_quantization (the MPQ polish of a GPTQ solution), block_cd and topk_block_cd."""
    from mpq.adapters.gptqmodel import postprocess_gptq_quantization, GPTQAdapterConfig
    cases = {}
    for name, (m, n, bits, gs, mode, k) in {"pp_cd": (24, 128, 4, 32, "block_cd", 16),
                                            "pp_topk": (20, 128, 3, 64, "topk_block_cd", 3)}.items():
        W, H = synth_layer(m, n, 500 + m)
        maxq = 2 ** bits - 1
        sg = torch.empty(m, n // gs)
        zg = torch.empty(m, n // gs)
        for gi in range(n // gs):
            q = MinMaxQuantizer(bits)
            q.find_params(W[:, gi * gs:(gi + 1) * gs])
            sg[:, gi], zg[:, gi] = q.scale[:, 0], q.zero[:, 0]
        g_idx = torch.arange(n, dtype=torch.int32) // gs
        sf, zf = sg[:, g_idx.long()], zg[:, g_idx.long()]
        Q0 = sf * (torch.clamp(torch.round(W / sf) + zf, 0, maxq) - zf)
        qcfg = types.SimpleNamespace(bits=bits, group_size=gs, mpq=types.SimpleNamespace(
            polish_mode=mode, polish_sweeps=3, topk_k=k, iters=10, prior_tau=0.2, block_cd_backend=""))
        Q, qf, _, _, _, _, st = postprocess_gptq_quantization(W=W, H=H, Q_init=Q0, scale_groups=sg, zero_groups=zg,
                                                               g_idx=g_idx, qcfg=qcfg, module_name=f"golden.pp.{name}",
                                                               adapter_cfg=GPTQAdapterConfig(block_rows=m))
        for kk, v in dict(W=W, H=H, Q0=Q0, sg=sg, zg=zg, g_idx=g_idx, Q=Q, q=qf).items():
            cases[f"{name}/{kk}"] = _np(v)
        keep = {k2: st[k2] for k2 in ("rankspace_error_mean_before", "rankspace_error_mean_final", "polish_updates",
                                       "module_fail_closed", "polish_assignment_changes", "raw_objective_mean_final")}
        keep["fp"] = st["input_fingerprint"]
        cases[f"{name}/meta"] = np.array(json.dumps(dict(bits=bits, gs=gs, mode=mode, k=k, stats=keep)))
    np.savez_compressed(out / "postprocess.npz", **cases)


GENERATORS = {"uniform_denoise": gen_uniform_denoise, "linear": gen_linear, "scalar_cd": gen_scalar_cd,
              "scalar_layer": gen_scalar_layer, "rotation": gen_rotation, "e8p12": gen_e8p12,
              "e8p12_layer": gen_e8p12_layer, "block_cd": gen_block_cd, "topk": gen_topk,
              "postprocess": gen_postprocess, "e8p12_topk_layer": gen_e8p12_topk_layer, "awq": gen_awq,
              "e8p12_stats": gen_e8p12_stats}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference source tree (poseidonchan/MPQ)")
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    torch.set_num_threads(8)
    for name, fn in GENERATORS.items():
        if args.only and name not in args.only.split(","):
            continue
        fn(HERE)
        print("wrote", name)


if __name__ == "__main__":
    main()
