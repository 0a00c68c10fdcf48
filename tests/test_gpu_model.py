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
