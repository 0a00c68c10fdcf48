"""Export of quantized linears in the GPTQ checkpoint format (qweight / qzeros / scales / g_idx).

The reference returns the solver's integer codes, group scales/zeros and g_idx
(mpq/adapters/gptqmodel.py:650-1163) and GPTQModel packs them (patches/gptqmodel.patch:370-395; the packer is
not vendored).  The format restated here is GPTQ's "v1" layout:

* qweight int32 (in_features * bits / 32, out_features): the codes of each output column as a little-endian
  bit stream along the input dimension (3-bit codes straddle word boundaries);
* qzeros int32 (groups, out_features * bits / 32): (zero - 1) masked to `bits`, packed along the output dimension;
* scales float16 (groups, out_features); g_idx int32 (in_features).
With the internal Hadamard rotation the codes live in the rotated input basis; the model applies the rotation to
its inputs at load time (the reference installs input hooks, patches/gptqmodel.patch:478-491).
"""
from __future__ import annotations

from typing import Dict

import torch

from ._lib import call, ptr


def _pack(codes: torch.Tensor, sp: int, so: int, n_pack: int, n_other: int, bits: int, offset: int) -> torch.Tensor:
    rows = n_pack * bits // 32
    out = torch.empty(rows, n_other, device=codes.device, dtype=torch.int32)
    call("mpq_pack_bits", ptr(codes), sp, so, n_pack, n_other, int(bits), int(offset), ptr(out), out.stride(0))
    return out


@torch.inference_mode()
def pack_gptq(q_int: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor, g_idx: torch.Tensor, bits: int
              ) -> Dict[str, torch.Tensor]:
    """q_int (out, in) uint8 codes, scale / zero (out, groups), g_idx (in,) -> GPTQ v1 tensors (on q_int's device)."""
    if q_int.dtype != torch.uint8 or not q_int.is_cuda:
        raise ValueError("q_int must be a CUDA uint8 tensor")
    out_f, in_f = q_int.shape
    if (in_f * bits) % 32 or (out_f * bits) % 32:
        raise ValueError(f"in_features and out_features times bits must be multiples of 32 (bits={bits})")
    q = q_int.contiguous()
    qweight = _pack(q, 1, q.stride(0), in_f, out_f, bits, 0)
    z8 = zero.to(torch.float32).round().clamp(0, 255).to(torch.uint8).contiguous()  # (out, groups)
    groups = z8.shape[1]
    qzeros = _pack(z8, z8.stride(0), 1, out_f, groups, bits, 1).t().contiguous()
    return {"qweight": qweight, "qzeros": qzeros, "scales": scale.to(torch.float16).t().contiguous(),
            "g_idx": g_idx.to(torch.int32).contiguous()}


# ---------------------------------------------------------------------------------------------------------------
# checkpoint directories
# ---------------------------------------------------------------------------------------------------------------

def save_gptq_checkpoint(model, modules: Dict[str, Dict], out_dir, *, bits: int, group_size: int,
                         rotation: str = "internal_hadamard", rotation_seed: int = 0, extra: Dict = None) -> str:
    """A GPTQ-format model directory: ``model.safetensors`` with every packed linear's ``<name>.qweight``,
    ``.qzeros``, ``.scales``, ``.g_idx`` (+ ``.bias``) and all other parameters as they are, ``config.json`` and
    ``quantize_config.json`` (GPTQ v1, asymmetric, no act-order).  With the internal Hadamard rotation the codes
    are in the solver basis: a loader installs the input hooks
    (``mpq_b200.adapters.gptqmodel.install_internal_hadamard_input_hooks``), as the reference's load path does.
    ``modules`` is ``quantize_model(...)["modules"]`` run with ``export_gptq=True``.  Returns the directory."""
    import json
    import os

    from safetensors.torch import save_file
    os.makedirs(out_dir, exist_ok=True)
    tensors: Dict[str, torch.Tensor] = {}
    packed = set()
    for name, entry in modules.items():
        g = entry.get("gptq")
        if g is None:
            raise ValueError(f"module {name!r} has no packed tensors (run quantize_model with export_gptq=True)")
        for k in ("qweight", "qzeros", "scales", "g_idx"):
            tensors[f"{name}.{k}"] = g[k].detach().cpu().contiguous()
        packed.add(name)
    for pname, p in model.state_dict().items():
        mod = pname.rsplit(".", 1)[0]
        if mod in packed:
            if pname.endswith(".bias"):
                tensors[pname] = p.detach().cpu().contiguous()
            continue
        tensors[pname] = p.detach().cpu().contiguous()
    # tied embeddings share storage: safetensors stores each tensor once
    seen: Dict[int, str] = {}
    for k in list(tensors):
        ptr_ = tensors[k].data_ptr()
        if ptr_ in seen and tensors[k].numel() and tensors[seen[ptr_]].shape == tensors[k].shape:
            tensors[k] = tensors[k].clone()
        seen[ptr_] = k
    save_file(tensors, os.path.join(out_dir, "model.safetensors"), metadata={"format": "pt"})
    model.config.to_json_file(os.path.join(out_dir, "config.json"))
    qc = {"bits": int(bits), "group_size": int(group_size), "desc_act": False, "sym": False, "true_sequential": True,
          "quant_method": "gptq", "checkpoint_format": "gptq",
          "mpq": {"rotation_mode": str(rotation), "rotation_seed": int(rotation_seed),
                  "rotation_effective": "internal_block_hadamard" if rotation == "internal_hadamard" else rotation}}
    if extra:
        qc["mpq"].update(extra)
    with open(os.path.join(out_dir, "quantize_config.json"), "w") as f:
        json.dump(qc, f, indent=2, sort_keys=True)
    return str(out_dir)


def _rotation_state_keys(prefix: str, width: int) -> Dict:
    """The serialized rotation state of the randomized Hadamard ("had") rotation, whose structured-state fields
    are all zero (patches/quip_sharp.patch:153-165, 453-462)."""
    return {f"{prefix}rotation_code": torch.tensor(0), f"{prefix}block_size": torch.tensor(0),
            f"{prefix}depth": torch.tensor(0), f"{prefix}householder_count": torch.tensor(0),
            f"{prefix}stage_signs": torch.zeros(4, width), f"{prefix}stage_perms": torch.zeros(3, width, dtype=torch.int64),
            f"{prefix}stage_inv_perms": torch.zeros(3, width, dtype=torch.int64),
            f"{prefix}householder": torch.zeros(1, width)}


def quip_group_attrs(entry: Dict) -> Dict:
    """The saved attribute dict of one QUIP# group (mpq/quip_generic.py:398-426, patches/quip_sharp.patch:440-475):
    Qidxs, SU, SV (fp16, the RMS scale folded into SV), scaleWH, the rotation state of both sides ("had"), fused,
    shapes, scales, mpq_stats and, when computed, input_fingerprint.  Qidxs are stored unpacked (int16,
    rows x cols / 8): the packed layout of QUIP#'s decode kernels belongs to QUIP#'s codebook class, which is not part
    of the reference tree."""
    keep = ("Qidxs", "SU", "SV", "fused", "shapes", "scales", "proxy_error", "surrogate_before", "surrogate_after",
            "mpq_stats", "input_fingerprint")
    out = {k: entry[k] for k in keep if k in entry}
    out.update(packed=False, codebook="E8P12", codesz=8, scaleWH=None, rotation_family="had",
               left_rotation_family="had", right_rotation_family="had", left_rotation_fallback_reason="",
               right_rotation_fallback_reason="")
    if "Qidxs" in entry:
        m, nb = entry["Qidxs"].shape
        out.update(_rotation_state_keys("left_", nb * 8))
        out.update(_rotation_state_keys("right_", m))
    return out


def save_quip_layer(out_dir, li: int, layer, groups: Dict[str, Dict]) -> None:
    """``{li}_{group}.pt`` for each quantized group of layer li and ``{li}_layernorm.pt`` (mpq/quip_generic.py:
    650-734)."""
    import os
    os.makedirs(out_dir, exist_ok=True)
    for name, entry in groups.items():
        torch.save(quip_group_attrs(entry), os.path.join(out_dir, f"{li}_{name}.pt"))
    payload = {"input_layernorm": layer.input_layernorm.weight.detach().cpu(),
               "post_attention_layernorm": layer.post_attention_layernorm.weight.detach().cpu()}
    torch.save(payload, os.path.join(out_dir, f"{li}_layernorm.pt"))


def save_quip_config(out_dir, model, quant_args: Dict) -> None:
    """``config.pt``: the quantization arguments and the model config with its ``quip_params``
    (mpq/quip_generic.py:936-953)."""
    import copy
    import os
    os.makedirs(out_dir, exist_ok=True)
    cfg = copy.deepcopy(model.config)
    cfg.update({"quip_params": {"lora_rank": 0, "rescale_WH": False, "codebook": "E8P12", "codebook_version": 1,
                                "codesz": 8, "idx_dtype": "torch.int16", "packsz": 1, "resid_scale_override": -1,
                                "adapter_name": "llama_like_dense_decoder"}})
    torch.save({"quant_args": dict(quant_args), "model_config": cfg, "adapter_name": "llama_like_dense_decoder"},
               os.path.join(out_dir, "config.pt"))


def apply_quip_ckpt(model, ckpt_dir, cb=None) -> int:
    """Write every quantized group of a QUIP# ckpt directory into ``model`` (decoded dense weights) and load the
    saved layernorms (mpq/quip_generic.py apply_quantized_ckpt_to_model, the step before hfize's save).
    Returns the number of groups applied."""
    import os
    from .codebook import E8P12_codebook
    from .model import QUIP_GROUPS, _quip_load_group
    cb = cb or E8P12_codebook()
    layers = model.model.layers
    applied = 0
    with torch.inference_mode():
        for li, layer in enumerate(layers):
            for name, mods in QUIP_GROUPS:
                if os.path.exists(os.path.join(ckpt_dir, f"{li}_{name}.pt")):
                    _quip_load_group(str(ckpt_dir), f"{li}_{name}", layer, mods, cb, True)
                    applied += 1
            ln = os.path.join(ckpt_dir, f"{li}_layernorm.pt")
            if os.path.exists(ln):
                payload = torch.load(ln, map_location="cpu", weights_only=False)
                for key in ("input_layernorm", "post_attention_layernorm"):
                    w = getattr(layer, key).weight
                    w.copy_(payload[key].to(device=w.device, dtype=w.dtype))
    return applied


def export_dense_hf_from_ckpt(quantized_path, hf_output_path, model=None, cb=None):
    """A dense Hugging Face model from a QUIP# ckpt directory (mpq/quip_generic.py:1047-1069): the float model named
    by ``config.pt`` (or the given ``model``; with no network a local checkpoint or an in-memory model is
    needed), every group's decoded E8P12 weights applied, then ``save_pretrained``."""
    import os
    saved = torch.load(os.path.join(quantized_path, "config.pt"), map_location="cpu", weights_only=False)
    if model is None:
        from transformers import AutoModelForCausalLM
        mc = saved["model_config"]
        model = AutoModelForCausalLM.from_pretrained(mc._name_or_path, torch_dtype="auto", low_cpu_mem_usage=True,
                                                     config=mc)
    n = apply_quip_ckpt(model, quantized_path, cb=cb)
    if n == 0:
        raise ValueError(f"no quantized groups found in {quantized_path}")
    model.save_pretrained(str(hf_output_path), safe_serialization=True)
    return model
