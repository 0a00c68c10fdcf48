"""Checkpoint directory writers on the CPU (layouts and keys; the packed tensors themselves are tested on the GPU)."""
import json

import torch

from mpq_b200.export import quip_group_attrs, save_gptq_checkpoint, save_quip_config, save_quip_layer


def _tiny():
    from transformers import AutoModelForCausalLM, LlamaConfig
    cfg = LlamaConfig(hidden_size=64, intermediate_size=128, num_hidden_layers=1, num_attention_heads=2,
                      num_key_value_heads=2, head_dim=32, vocab_size=64)
    return AutoModelForCausalLM.from_config(cfg)


def test_gptq_directory_layout(tmp_path):
    from safetensors.torch import load_file
    model = _tiny()
    mods = {}
    for name in ("self_attn.q_proj", "mlp.down_proj"):
        w = model.model.layers[0].get_submodule(name).weight
        out_f, in_f = w.shape
        mods[f"model.layers.0.{name}"] = {"gptq": {
            "qweight": torch.zeros(in_f * 4 // 32, out_f, dtype=torch.int32),
            "qzeros": torch.zeros(in_f // 32, out_f * 4 // 32, dtype=torch.int32),
            "scales": torch.ones(in_f // 32, out_f, dtype=torch.float16),
            "g_idx": torch.arange(in_f, dtype=torch.int32) // 32}}
    save_gptq_checkpoint(model, mods, tmp_path, bits=4, group_size=32)
    t = load_file(str(tmp_path / "model.safetensors"))
    assert "model.layers.0.self_attn.q_proj.qweight" in t and "model.layers.0.self_attn.q_proj.weight" not in t
    assert "model.layers.0.self_attn.k_proj.weight" in t and "model.embed_tokens.weight" in t
    qc = json.loads((tmp_path / "quantize_config.json").read_text())
    assert qc["bits"] == 4 and qc["group_size"] == 32 and qc["desc_act"] is False and qc["sym"] is False
    assert qc["mpq"]["rotation_effective"] == "internal_block_hadamard"
    assert json.loads((tmp_path / "config.json").read_text())["hidden_size"] == 64


def test_quip_ckpt_layout(tmp_path):
    model = _tiny()
    entry = {"Qidxs": torch.zeros(64 + 64 + 64, 8, dtype=torch.int16), "SU": torch.ones(192, dtype=torch.float16),
             "SV": torch.ones(64, dtype=torch.float16), "fused": True, "shapes": [(64, 64)] * 3,
             "scales": [1.0, 1.0, 1.0], "mpq_stats": {"obs_precision_final": 3.0}}
    save_quip_layer(tmp_path, 0, model.model.layers[0], {"qkv": entry})
    save_quip_config(tmp_path, model, {"bits": 2})
    a = torch.load(tmp_path / "0_qkv.pt", weights_only=False)
    assert a["packed"] is False and a["codesz"] == 8 and a["rotation_family"] == "had"
    assert a["left_stage_signs"].shape == (4, 64) and a["right_stage_perms"].shape == (3, 192)
    ln = torch.load(tmp_path / "0_layernorm.pt", weights_only=False)
    assert set(ln) >= {"input_layernorm", "post_attention_layernorm"}
    cfg = torch.load(tmp_path / "config.pt", weights_only=False)
    assert cfg["model_config"].quip_params["codesz"] == 8 and cfg["quant_args"]["bits"] == 2
    assert quip_group_attrs({"fused": False})["scaleWH"] is None
