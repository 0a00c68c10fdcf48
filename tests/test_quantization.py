"""The public QuantizationConfig / quantize API: recipe resolution as the reference's mpq/quantization.py
(CPU) and one end-to-end run per backend on a tiny model with its artifacts and per-layer resume (GPU)."""
import json

import numpy as np
import pytest
import torch

from mpq_b200.quantization import QuantizationConfig


def test_scalar_recipe_resolves_to_paper_defaults():
    r = QuantizationConfig(bits=3).resolve()
    assert (r.backend, r.codebook, r.preprocess, r.rotation, r.solver, r.polish_mode) == \
        ("gptqmodel", "grid_g128", "awq", "internal_hadamard", "vamp", "block_cd")
    assert (r.init, r.iters, r.prior_tau, r.symmetric, r.group_size) == ("rtn", 16, 0.2, False, 128)


def test_e8p12_recipe_selects_quip_backend():
    r = QuantizationConfig(bits=2).resolve()
    assert (r.backend, r.codebook, r.preprocess, r.rotation, r.polish_mode, r.init, r.prior_tau) == \
        ("quip", "e8p12", "none", "had", "block_cd", "rtn", 0.2)
    assert r.symmetric is None


@pytest.mark.parametrize("bits", [0, 1, 5, 8])
def test_unsupported_bits(bits):
    with pytest.raises(ValueError, match="bits must be one of"):
        QuantizationConfig(bits=bits).resolve()


@pytest.mark.parametrize("kw,msg", [(dict(group_size=0), "group_size"), (dict(damping=1.5), "damping"),
                                    (dict(iters=0), "iters"), (dict(polish_sweeps=-1), "polish_sweeps"),
                                    (dict(preprocess="gptq"), "preprocess"), (dict(init="zero"), "init"),
                                    (dict(calibration_samples=0), "calibration_samples")])
def test_invalid_configs(kw, msg):
    with pytest.raises(ValueError, match=msg):
        QuantizationConfig(**kw).resolve()


def test_polish_sweeps_zero_disables_polish_and_overrides():
    r = QuantizationConfig(bits=4, polish_sweeps=0, preprocess="none", prior_tau=0.3, symmetric=True).resolve()
    assert (r.polish_mode, r.preprocess, r.prior_tau, r.symmetric) == ("none", "none", 0.3, True)


def test_unbuilt_options_fail_loudly(tmp_path):
    from mpq_b200 import quantize
    for cfg, msg in ((QuantizationConfig(bits=4, evaluate=True), "evaluate"),
                     (QuantizationConfig(bits=4, init="ldlq"), "init"),
                     (QuantizationConfig(bits=4, symmetric=True), "symmetric")):
        with pytest.raises(ValueError, match=msg):
            quantize("tiny_llama", tmp_path, cfg)


def test_text_calibration_needs_ids():
    from mpq_b200.quantization import _calibration
    r = QuantizationConfig(bits=4).resolve()
    with pytest.raises(ValueError, match="calibration"):
        _calibration(r, 100, None)
    ids = _calibration(QuantizationConfig(bits=4, calibration_dataset="random", calibration_samples=3,
                                          calibration_seqlen=5).resolve(), 100, None)
    assert ids.shape == (3, 5) and int(ids.max()) < 100


@pytest.mark.gpu
def test_quantize_gptq_backend_end_to_end(cuda_dev, tmp_path):
    from safetensors.torch import load_file

    from mpq_b200 import quantize
    from oracle import gptq_pack as OP
    cfg = QuantizationConfig(bits=4, group_size=64, iters=4, polish_sweeps=1, calibration_dataset="random",
                             calibration_samples=8, calibration_seqlen=64)
    out = quantize("tiny_llama", tmp_path, cfg)
    assert out["backend"] == "gptqmodel" and "awq" in out and len(out["modules"]) == 14
    res = json.loads((tmp_path / "backend_results.json").read_text())
    assert res["config"]["preprocess"] == "awq"
    qc = json.loads((tmp_path / "gptq" / "quantize_config.json").read_text())
    assert qc["bits"] == 4 and qc["group_size"] == 64 and qc["mpq"]["rotation_mode"] == "internal_hadamard"
    t = load_file(str(tmp_path / "gptq" / "model.safetensors"))
    qw = t["model.layers.0.self_attn.q_proj.qweight"]
    assert qw.dtype == torch.int32 and qw.shape == (256 * 4 // 32, 256)
    assert "model.layers.0.self_attn.q_proj.weight" not in t and "model.embed_tokens.weight" in t
    codes = OP.unpack_rows(qw.numpy(), 4, 256)
    assert codes.max() <= 15
    assert sorted(p.name for p in (tmp_path / "layers").iterdir()) == ["layer_0.pt", "layer_1.pt"]
    # a second run resumes every layer from the saved state and writes the same tensors
    out2 = quantize("tiny_llama", tmp_path, cfg)
    assert "quantize_solve" not in out2["timings"]
    t2 = load_file(str(tmp_path / "gptq" / "model.safetensors"))
    np.testing.assert_array_equal(t2["model.layers.1.mlp.down_proj.qweight"].numpy(),
                                  t["model.layers.1.mlp.down_proj.qweight"].numpy())


@pytest.mark.gpu
def test_quantize_quip_backend_end_to_end(cuda_dev, tmp_path):
    from mpq_b200 import quantize
    cfg = QuantizationConfig(bits=2, iters=4, polish_sweeps=1, calibration_dataset="random", calibration_samples=8,
                             calibration_seqlen=64)
    out = quantize("tiny_llama", tmp_path, cfg)
    assert out["backend"] == "quip" and len(out["groups"]) == 8
    ck = tmp_path / "quip_ckpt"
    names = sorted(p.name for p in ck.iterdir())
    assert "config.pt" in names and "0_qkv.pt" in names and "1_down.pt" in names and "1_layernorm.pt" in names
    a = torch.load(ck / "0_qkv.pt", weights_only=False)
    assert a["Qidxs"].dtype == torch.int16 and a["fused"] and len(a["shapes"]) == 3 and a["packed"] is False
    assert a["rotation_family"] == "had" and a["left_stage_signs"].shape == (4, 256) and "mpq_stats" in a
    conf = torch.load(ck / "config.pt", weights_only=False)
    assert conf["model_config"].quip_params["codebook"] == "E8P12"
    assert (tmp_path / "hf" / "config.json").is_file()
    # resume: every group loads from the ckpt and decodes to the same weights
    from mpq_b200.model import build_synthetic_decoder
    m = build_synthetic_decoder("tiny_llama", device=cuda_dev, seed=0)
    out2 = quantize(m, tmp_path, cfg)
    assert all(g.get("resumed") for g in out2["groups"].values())
    w = m.model.layers[0].self_attn.q_proj.weight.float()
    assert torch.isfinite(w).all()
    # the decoded weights match the first run's dense model (fp16 SU / SV in the ckpt, bf16 weights)
    from safetensors.torch import load_file
    dense = load_file(str(tmp_path / "hf" / "model.safetensors"))
    ref = dense["model.layers.0.self_attn.q_proj.weight"].float().to(w.device)
    assert ((w - ref).norm() / ref.norm()).item() < 1e-2
