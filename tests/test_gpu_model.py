"""Whole-model driver on a tiny random-init Llama-shaped decoder (GPU)."""
import numpy as np
import pytest
import torch

from oracle import gptq_pack as OP


@pytest.mark.gpu
def test_quantize_tiny_llama(cuda_dev):
    from mpq_b200.model import ModelQuantConfig, build_synthetic_decoder, calibration_ids, quantize_model
    model = build_synthetic_decoder("tiny_llama", device=cuda_dev, seed=0)
    ids = calibration_ids(8, 64, model.config.vocab_size, seed=1)
    before = {n: p.detach().clone() for n, p in model.named_parameters() if "proj" in n}
    with torch.inference_mode():
        ref_logits = model(ids[:2].to(cuda_dev)).logits.float()
    cfg = ModelQuantConfig(bits=4, group_size=64, iters=6, polish_sweeps=1, batch_size=4, keep_codes=True,
                           export_gptq=True)
    out = quantize_model(model, ids, cfg)
    mods = out["modules"]
    assert len(mods) == 2 * 7
    for name, st in mods.items():
        assert st["rankspace_error_mean"] <= st["rtn_rankspace_error_mean"] * (1 + 1e-6), name
        assert st["q_int"].dtype == torch.uint8 and int(st["q_int"].max()) <= 15
        assert st["scale"].shape == (st["rows"], st["cols"] // 64)
        g = st["gptq"]
        assert g["qweight"].dtype == torch.int32 and g["qweight"].shape == (st["cols"] * 4 // 32, st["rows"])
        assert g["qzeros"].shape == (st["cols"] // 64, st["rows"] * 4 // 32)
        assert g["scales"].dtype == torch.float16 and g["scales"].shape == (st["cols"] // 64, st["rows"])
        np.testing.assert_array_equal(OP.unpack_rows(g["qweight"].numpy(), 4, st["cols"]).T, st["q_int"].numpy())
    changed = [n for n, p in model.named_parameters() if "proj" in n and not torch.equal(p, before[n])]
    assert len(changed) == 2 * 7
    with torch.inference_mode():
        logits = model(ids[:2].to(cuda_dev)).logits.float()
    assert torch.isfinite(logits).all()
    # 4-bit weights keep the random model's function close
    rel = (logits - ref_logits).norm() / ref_logits.norm()
    assert rel < 0.5, rel
    assert set(out["timings"]) >= {"forward_hessian", "solve", "forward_out"}


@pytest.mark.gpu
def test_quantize_tiny_llama_e8p12(cuda_dev):
    from mpq_b200.model import QuipModelConfig, build_synthetic_decoder, calibration_ids, quantize_model_quip
    model = build_synthetic_decoder("tiny_llama", device=cuda_dev, seed=0)
    ids = calibration_ids(8, 64, model.config.vocab_size, seed=2)
    cfg = QuipModelConfig(iters=6, polish_sweeps=1, batch_size=4)
    out = quantize_model_quip(model, ids, cfg)
    groups = out["groups"]
    assert sorted(groups) == sorted(f"{l}_{g}" for l in range(2) for g in ("qkv", "o", "up", "down"))
    for key, g in groups.items():
        rows = sum(s[0] for s in g["shapes"])
        cols = g["shapes"][0][1]
        assert g["Qidxs"].shape == (rows, cols // 8) and g["Qidxs"].dtype == torch.int16
        assert g["SU"].shape == (rows,) and g["SV"].shape == (cols,)
        assert g["surrogate_after"] <= g["surrogate_before"] * (1 + 1e-6), key
        assert g["proxy_error"] < 0.5, key
        assert g["fused"] == (len(g["shapes"]) > 1)
    with torch.inference_mode():
        logits = model(ids[:2].to(cuda_dev)).logits.float()
    assert torch.isfinite(logits).all()


@pytest.mark.gpu
@pytest.mark.parametrize("walk", ["gptq", "quip"])
def test_quantize_tiny_llama_topk_polish(cuda_dev, walk):
    """Both whole-model walks with the top-k polish recipe."""
    from mpq_b200.model import (ModelQuantConfig, QuipModelConfig, build_synthetic_decoder, calibration_ids,
                                quantize_model, quantize_model_quip)
    model = build_synthetic_decoder("tiny_llama", device=cuda_dev, seed=0)
    ids = calibration_ids(8, 64, model.config.vocab_size, seed=3)
    if walk == "gptq":
        out = quantize_model(model, ids, ModelQuantConfig(bits=3, group_size=64, iters=6, polish_sweeps=1, batch_size=4,
                                                          polish_mode="topk_block_cd", topk_k=4))
        for name, st in out["modules"].items():
            assert st["rankspace_error_mean"] <= st["rtn_rankspace_error_mean"] * (1 + 1e-6), name
    else:
        out = quantize_model_quip(model, ids, QuipModelConfig(iters=6, polish_sweeps=1, batch_size=4,
                                                              polish_mode="topk_block_cd", topk_k=8))
        for key, g in out["groups"].items():
            assert g["surrogate_after"] <= g["surrogate_before"] * (1 + 1e-6), key
    with torch.inference_mode():
        logits = model(ids[:2].to(cuda_dev)).logits.float()
    assert torch.isfinite(logits).all()


@pytest.mark.gpu
@pytest.mark.parametrize("walk", ["gptq", "quip"])
def test_tiny_llama_walk_matches_oracle_per_linear(cuda_dev, walk):
    """Each linear (GPTQ walk) or projection group (QUIP# walk) of a 2-layer tiny decoder, solved inside the
    whole-model walk, against the CPU oracle solving the same inputs (the walk's own float W and Hessian), stage by
    stage as at full width:
      * VAMP stage (the walk run without polish): codes of every linear >= 99.9 %;
      * polish (GPTQ walk): one sweep started from the oracle's own VAMP-stage codes, CUDA vs oracle >= 99.9 %;
      * full solve (one polish sweep): the model's total proxy loss within 0.5 %.
    The full solve is not held per linear: the polish orders its columns / blocks by gains averaged over all rows,
    so a handful of different starting codes reorders the sweep for every row (in this model, 4 of 65,536 VAMP-stage
    codes of one linear move 7.5 % of its polished codes and its proxy loss by 3 %; the oracle started from the
    CUDA solve's codes reproduces the CUDA result).  QUIP#: the first 128-row block of each group's chain (the
    oracle's warm start is the whole group's, as in the walk)."""
    from oracle import e8p12 as OE
    from oracle import layer as OL
    from oracle import uniform_vamp as OU
    from oracle.uniform_vamp import UniformVampConfig
    from mpq_b200.model import (ModelQuantConfig, QuipModelConfig, build_synthetic_decoder, calibration_ids,
                                quantize_model, quantize_model_quip)
    from mpq_b200.solver import polish_uniform_rankspace
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_dev)
    for sweeps in (0, 1):
        model = build_synthetic_decoder("tiny_llama", device=cuda_dev, seed=0)
        ids = calibration_ids(8, 64, model.config.vocab_size, seed=4)
        agree, losses, polish_agree = [], [], []
        if walk == "gptq":
            out = quantize_model(model, ids, ModelQuantConfig(bits=4, group_size=64, iters=6, polish_sweeps=sweeps,
                                                              batch_size=4, keep_codes=True, keep_inputs=True))
            for name, st in out["modules"].items():
                W, H = st["inputs"]["W"].numpy(), st["inputs"]["H"].numpy()
                ref = OL.run_scalar_layer(W=W, H=H, bits=4, group_size=64, block_rows=W.shape[0], module_name=name,
                                          vamp_cfg=UniformVampConfig(iters=6, prior_tau=0.2, damping=0.5,
                                                                     polish_sweeps=sweeps))
                agree.append(float((st["q_int"].numpy() == ref["q_int"]).mean()))
                # the walk writes Q back into the bf16 model: compare both losses on bf16-rounded weights
                Q = model.get_submodule(name).weight.detach().float().cpu().numpy()
                Qr = torch.from_numpy(np.ascontiguousarray(ref["Q"])).bfloat16().float().numpy()
                losses.append((OL.proxy_loss(W, Q, H), OL.proxy_loss(W, Qr, H)))
                if sweeps == 0:
                    # one polish sweep from the oracle's own VAMP-stage codes, CUDA vs oracle
                    sf = np.repeat(ref["scale"], 64, 1).astype(np.float32)
                    zf = np.repeat(ref["zero"], 64, 1).astype(np.float32)
                    x0 = ref["Q_work"].astype(np.float32)
                    Y_u = (ref["W_work"] @ ref["Vs"]).astype(np.float32)
                    q_o, _, _, _ = OU.polish_uniform_gpu_semantics(x_init=x0, Y_u=Y_u, Vs=ref["Vs"], scale_full=sf,
                                                                   zero_full=zf, maxq=15, sweeps=1,
                                                                   gram_full=ref["H_metric"])
                    q_g, _, _, _ = polish_uniform_rankspace(x_init=t(x0), Y_u=t(Y_u), Vs=t(ref["Vs"]),
                                                            scale_full=t(sf), zero_full=t(zf), maxq=15, sweeps=1,
                                                            polish_mode="block_cd", block_cd_backend="auto",
                                                            gram_full=t(ref["H_metric"]))
                    polish_agree.append(float((q_g.cpu().numpy() == q_o).mean()))
        else:
            out = quantize_model_quip(model, ids, QuipModelConfig(iters=6, polish_sweeps=sweeps, batch_size=4,
                                                                  polish_mode="block_cd" if sweeps else "none",
                                                                  keep_inputs=True))
            cb = OE.E8P12_codebook()
            for key, g in out["groups"].items():
                Wn, Hr = g["inputs"]["Wn"].numpy(), g["inputs"]["Hr"].numpy()
                ref = OE.refine_codebook(Wr=Wn, Hr=Hr, cb=cb, block_rows=128, max_blocks=1,
                                         cfg=OE.E8P12VampConfig(iters=6, prior_tau=0.25, polish_sweeps=sweeps))
                r = min(128, Wn.shape[0])
                got = g["Qidxs"].numpy().astype(np.int64)[:r] & 0xFFFF
                agree.append(float((got == ref["Qidxs"][:r]).mean()))
                losses.append((OL.proxy_loss(Wn[:r], cb.grid[got].reshape(r, -1), Hr),
                               OL.proxy_loss(Wn[:r], ref["hatWr"][:r], Hr)))
        print(walk, "sweeps", sweeps, "agreement per linear", [round(a, 4) for a in agree],
              "polish from oracle codes", [round(a, 4) for a in polish_agree])
        if sweeps == 0:
            assert min(agree) >= 0.999, agree
            assert all(a >= 0.999 for a in polish_agree), polish_agree
        got_total, ref_total = sum(a for a, _ in losses), sum(b for _, b in losses)
        assert abs(got_total - ref_total) <= 0.005 * ref_total, (sweeps, got_total, ref_total)


@pytest.mark.gpu
def test_quip_ckpt_hfize_round_trip(cuda_dev, tmp_path):
    """QUIP# ckpt -> dense Hugging Face model (hfize): a fresh float model with the ckpt applied matches the walk's
    quantized model (the ckpt stores SV with the RMS scale folded in as fp16, QUIP#'s format, so a decoded weight
    is at most one bf16 step from the in-memory one), and the saved directory loads back bit for bit."""
    from transformers import AutoModelForCausalLM
    from mpq_b200.export import export_dense_hf_from_ckpt, save_quip_config
    from mpq_b200.model import QuipModelConfig, build_synthetic_decoder, calibration_ids, quantize_model_quip
    model = build_synthetic_decoder("tiny_llama", device=cuda_dev, seed=0)
    ids = calibration_ids(8, 64, model.config.vocab_size, seed=5)
    ckpt = tmp_path / "ckpt"
    quantize_model_quip(model, ids, QuipModelConfig(iters=4, polish_sweeps=1, batch_size=4, keep_attrs=False,
                                                    checkpoint_dir=str(ckpt)))
    save_quip_config(ckpt, model, {"bits": 2})
    fresh = build_synthetic_decoder("tiny_llama", device=cuda_dev, seed=0)
    export_dense_hf_from_ckpt(ckpt, tmp_path / "hf", model=fresh)
    want = {n: p.detach().float() for n, p in model.named_parameters()}
    for n, p in fresh.named_parameters():
        a = p.detach().float()
        # at most one bf16 step apart (the fp16 scale moves a few values across a bf16 rounding boundary), and
        # values that cancel to ~0 in the inverse Hadamard may differ by its rounding (~1e-9 here)
        tol = 2.0 ** -7 * torch.maximum(a.abs(), want[n].abs()) + 1e-6 * float(want[n].abs().max())
        bad = (a - want[n]).abs() > tol
        assert not bad.any(), (n, int(bad.sum()), a[bad][:4].tolist(), want[n][bad][:4].tolist())
    decoded = {n: p.detach() for n, p in fresh.named_parameters()}
    loaded = AutoModelForCausalLM.from_pretrained(str(tmp_path / "hf"), torch_dtype=torch.bfloat16)
    for n, p in loaded.named_parameters():
        assert torch.equal(p.detach().to(cuda_dev), decoded[n]), n
