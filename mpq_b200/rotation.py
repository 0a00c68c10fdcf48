"""Input rotations on the CUDA block-Hadamard kernel.

Reference: mpq/rotation.py:17-47 (plans), :325-340 (Rademacher signs), :404-441 (block Hadamard).
"""
from __future__ import annotations

import hashlib

import torch

from ._lib import call, ptr


def stable_seed(key: str, *, base_seed: int = 0) -> int:
    """mpq/utils.py:10-21."""
    digest = hashlib.sha256(str(key).encode("utf-8")).digest()
    extra = int.from_bytes(digest[:4], byteorder="little", signed=False)
    return int((int(base_seed) + int(extra)) % (2**31 - 1))


def largest_pow2_factor(n: int) -> int:
    n = int(n)
    if n <= 0:
        raise ValueError(f"expected positive n, got {n}.")
    return int(n & -n)


def resolve_block_hadamard_plan(width: int) -> tuple[str, int]:
    """mpq/rotation.py:40-45."""
    had_dim = largest_pow2_factor(int(width))
    if had_dim >= 2:
        return "block", int(had_dim)
    return "none", 1


@torch.inference_mode()
def sample_rademacher_signs(*, width: int, key: str, seed: int = 0, device: torch.device,
                            dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """mpq/rotation.py:325-340: the sign stream is torch's seeded CPU generator (bit-compatible)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(stable_seed(str(key), base_seed=int(seed)))
    s = torch.randint(0, 2, (int(width),), generator=g, dtype=torch.int64)
    return s.to(torch.float32).mul_(2.0).sub_(1.0).to(device=device, dtype=dtype)


def _apply(matrix: torch.Tensor, signs, had_dim: int, mode: int) -> torch.Tensor:
    m = matrix.to(torch.float32).contiguous()
    if not m.is_cuda:
        raise ValueError("block Hadamard requires CUDA tensors (there is no CPU path)")
    shape = m.shape
    m2 = m.reshape(-1, shape[-1])
    out = torch.empty_like(m2)
    n = int(shape[-1])
    had = int(had_dim)
    if had <= 1:
        if signs is None:
            return m.clone()
        return (m2 * signs.view(1, -1)).reshape(shape)
    s = None if signs is None else signs.to(device=m.device, dtype=torch.float32).contiguous()
    rows = m2.shape[0]
    for r0 in range(0, rows, 65535):
        r1 = min(rows, r0 + 65535)
        call("mpq_block_hadamard", ptr(m2[r0:r1]), m2.stride(0), ptr(out[r0:r1]), out.stride(0), r1 - r0, n, had,
             ptr(s), mode)
    return out.reshape(shape)


def apply_block_hadamard(matrix: torch.Tensor, *, had_dim: int) -> torch.Tensor:
    return _apply(matrix, None, had_dim, 0)


def apply_right_block_hadamard(matrix: torch.Tensor, *, signs: torch.Tensor, had_dim: int) -> torch.Tensor:
    """(M * signs) then normalized block Hadamard of the last dim (mpq/rotation.py:432-434)."""
    return _apply(matrix, signs, had_dim, 0)


def apply_right_block_hadamard_inverse(matrix: torch.Tensor, *, signs: torch.Tensor, had_dim: int) -> torch.Tensor:
    """block Hadamard then * signs (mpq/rotation.py:437-439)."""
    return _apply(matrix, signs, had_dim, 1)


@torch.inference_mode()
def rht_weight(W: torch.Tensor, SU: torch.Tensor, SV: torch.Tensor, had_out: int, had_in: int) -> torch.Tensor:
    """Two-sided randomized Hadamard of a weight (QUIP# incoherence processing, restated):
    Wr = Had_out diag(SU) W diag(SV) Had_in  (normalized block Hadamard on each side)."""
    t = apply_right_block_hadamard(W, signs=SV, had_dim=had_in)
    t = apply_right_block_hadamard(t.T.contiguous(), signs=SU, had_dim=had_out)
    return t.T.contiguous()


@torch.inference_mode()
def rht_weight_inverse(Wr: torch.Tensor, SU: torch.Tensor, SV: torch.Tensor, had_out: int, had_in: int) -> torch.Tensor:
    t = apply_right_block_hadamard_inverse(Wr.T.contiguous(), signs=SU, had_dim=had_out)
    return apply_right_block_hadamard_inverse(t.T.contiguous(), signs=SV, had_dim=had_in)


@torch.inference_mode()
def rht_hessian(H: torch.Tensor, SV: torch.Tensor, had_in: int) -> torch.Tensor:
    """Hr = Had_in diag(SV) H diag(SV) Had_in (the input-side rotation of the Hessian)."""
    t = apply_right_block_hadamard(H.T.contiguous(), signs=SV, had_dim=had_in)
    return apply_right_block_hadamard(t.T.contiguous(), signs=SV, had_dim=had_in)
