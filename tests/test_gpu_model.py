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
