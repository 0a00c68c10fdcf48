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
