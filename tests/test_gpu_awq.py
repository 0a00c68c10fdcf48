"""AWQ scaling (the 3/4-bit preprocess) against the reference's apply_awq_scaling run on the same tiny model
(float64, so that both searches see the same losses to far below the gaps between ratios)."""
import json

import numpy as np
import pytest
import torch


def _tiny_llama(dev, dtype=torch.float64, seed=None):
    """The golden run's model: seeded CPU initialisation (as tests/golden/make_golden.py builds it), then moved."""
    from transformers import AutoModelForCausalLM, LlamaConfig
    cfg = LlamaConfig(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=2,
                      num_key_value_heads=2, head_dim=32, vocab_size=128, initializer_range=0.02,
                      attn_implementation="sdpa", max_position_embeddings=256)
    if seed is not None:
        torch.manual_seed(seed)
    model = AutoModelForCausalLM.from_config(cfg, dtype=dtype).eval()
    if seed is not None:
        with torch.no_grad():
            for layer in model.model.layers:
                layer.input_layernorm.weight.copy_(torch.exp(1.5 * torch.randn(cfg.hidden_size)))
                layer.post_attention_layernorm.weight.copy_(torch.exp(1.5 * torch.randn(cfg.hidden_size)))
    return model.to(dev)


@pytest.mark.gpu
def test_awq_matches_reference(cuda_dev, golden_dir):
    from mpq_b200.awq import apply_awq_scaling
    z = np.load(golden_dir / "awq.npz")
    ref = json.loads(str(z["meta"]))
    model = _tiny_llama(cuda_dev, seed=5)
    sums = np.array([float(v.double().abs().sum()) for v in model.state_dict().values()])
    np.testing.assert_allclose(sums, z["before_checksum"], rtol=1e-12, err_msg="seeded initialisation drifted")
    with torch.no_grad():
        ref_logits = model(torch.from_numpy(z["ids"]).to(cuda_dev)).logits
    dbg = apply_awq_scaling(model, torch.from_numpy(z["ids"]), bits=4, group_size=32, sym=False, batch_size=2)
    mine = [(g["name"], g["best_ratio"]) for l in dbg["layers"] for g in l["groups"]]
    theirs = [(g["name"], g["best_ratio"]) for l in ref["layers"] for g in l["groups"]]
    assert [n for n, _ in mine] == [n for n, _ in theirs]
    assert mine == theirs
    errs = [g["best_error"] for l in dbg["layers"] for g in l["groups"]]
    ref_errs = [g["best_error"] for l in ref["layers"] for g in l["groups"]]
    np.testing.assert_allclose(errs, ref_errs, rtol=1e-5)
    after = model.state_dict()
    for k in z.files:
        if k.startswith("after/"):
            np.testing.assert_allclose(after[k[len("after/"):]].float().cpu().numpy(), z[k], rtol=1e-5, atol=1e-6,
                                       err_msg=k)
    # the folded scales leave the float model's function unchanged
    with torch.no_grad():
        logits = model(torch.from_numpy(z["ids"]).to(cuda_dev)).logits
    torch.testing.assert_close(logits, ref_logits, rtol=1e-6, atol=1e-8)


def test_awq_requires_gpu():
    from mpq_b200.awq import apply_awq_scaling
    with pytest.raises(ValueError, match="GPU"):
        apply_awq_scaling(_tiny_llama("cpu"), torch.zeros(1, 4, dtype=torch.long), bits=4, group_size=32)
