"""E8P12 codebook: construction and the factor tables the CUDA kernels read.

``factor_tables(cb)`` accepts any object with the QUIP# ``E8P12_codebook`` attribute surface (``grid``
65536 x 8, ``codesz`` 8) and derives, like mpq/priors/e8p12.py:83-151, the 256 abs patterns, their sign
parities and squared norms, and the (branch, abs, sign) -> index table, with the same structural checks.

``E8P12_codebook`` builds the grid from the published E8P construction (QUIP# paper): the 227 abs
patterns of the half-integer E8 coset with norm^2 <= 10 plus 29 of norm^2 12 (five 3/2, three 1/2; the
first 29 in lexicographic order), each with every even-parity sign flip of its signed base pattern and a
+-1/4 shift.  Index = (abs << 8) | s, shift by the parity of s, flip mask s ^ parity(s).  The real QUIP#
table (lib/codebook/latticee8_padded12.py @ 1d8f873) is not vendored, so the index order and the 29
padding patterns are this construction's own; pass a QUIP# codebook object to use its indices.
"""
from __future__ import annotations

from typing import Dict

import numpy as np
import torch


def _abs_patterns() -> np.ndarray:
    vals = np.array([0.5, 1.5, 2.5, 3.5])
    allp = np.stack(np.meshgrid(*([vals] * 8), indexing="ij"), axis=-1).reshape(-1, 8)
    small = sorted(map(tuple, allp[(allp ** 2).sum(axis=1) <= 10]))
    two = np.array([0.5, 1.5])
    c12 = np.stack(np.meshgrid(*([two] * 8), indexing="ij"), axis=-1).reshape(-1, 8)
    pad = sorted(map(tuple, c12[(c12 ** 2).sum(axis=1) == 12]))
    if len(small) != 227 or len(pad) != 56:
        raise RuntimeError("E8P12 abs-pattern enumeration failed")
    return np.asarray(small + pad[:29], dtype=np.float64)


class E8P12_codebook:
    """E8P12 codebook with the attributes the reference reads (grid, grid_packed_abs, codesz, idx_dtype)."""

    codesz = 8
    idx_dtype = torch.int64

    def __init__(self, device: torch.device | str = "cpu"):
        base = _abs_patterns()
        odd = (np.rint(base.sum(axis=1)).astype(np.int64) % 2) == 1
        base[odd, 7] *= -1.0
        s = np.arange(256, dtype=np.int64)
        par = np.zeros_like(s)
        for k in range(8):
            par ^= (s >> k) & 1
        flips = 1.0 - 2.0 * (((s ^ par)[:, None] >> np.arange(8)[None, :]) & 1)
        off = np.where(par == 1, -0.25, 0.25)
        grid = base[:, None, :] * flips[None, :, :] + off[None, :, None]
        self.grid = torch.from_numpy(grid.reshape(65536, 8).astype(np.float32)).to(device)
        self.grid_packed_abs = torch.arange(256, dtype=torch.int64)

    def quantize(self, X: torch.Tensor, return_idx: bool = True, **kw):
        """Nearest codeword (the factorized MAP at unit precision, lowest index on ties)."""
        from .e8p12 import e8p12_nearest
        vals, idx = e8p12_nearest(X.reshape(-1, 8), self)
        return (vals, idx) if return_idx else vals


_TABLES: Dict[tuple, Dict[str, torch.Tensor]] = {}


def factor_tables(cb, device: torch.device) -> Dict[str, torch.Tensor]:
    """Device tables for the kernels: base_abs (256x8 f32), base_sqnorm (256 f32), base_parity (256 i32),
    idx_lut (2x256x256 i32), grid (65536x8 f32) and sign_id (65536 u8: sign bits of grid - offset).
    Cached per (codebook, device)."""
    key = (id(cb), device.type, device.index)
    t = _TABLES.get(key)
    if t is not None:
        return t
    grid = cb.grid.detach().to(device="cpu", dtype=torch.float32).numpy()
    if grid.shape != (65536, 8) or int(getattr(cb, "codesz", 8)) != 8:
        raise ValueError(f"expected a 65536 x 8 E8P12 grid, got {grid.shape}")
    base_template = grid[np.arange(256) << 8] - np.float32(0.25)
    sign_mask = (base_template < 0).astype(np.int64)
    parity = sign_mask.sum(axis=1) & 1
    base_abs = np.abs(base_template).astype(np.float32)
    sqnorm = np.zeros(256, np.float32)
    for k in range(8):  # sequential order, as the kernels use
        sqnorm = sqnorm + base_abs[:, k] * base_abs[:, k]
    full = np.arange(65536, dtype=np.int64)
    raw = full & 255
    br = np.zeros_like(raw)
    for k in range(8):
        br ^= (raw >> k) & 1
    offset = np.where(br == 1, np.float32(-0.25), np.float32(0.25)).astype(np.float32)
    resid = grid - offset[:, None]
    sid = ((resid < 0).astype(np.int64) << np.arange(8)[None, :]).sum(axis=1)
    lut = np.full((2, 256, 256), -1, dtype=np.int64)
    lut[br, full >> 8, sid] = full
    if not np.allclose(np.abs(resid), base_abs[full >> 8], atol=1e-6, rtol=1e-6):
        raise RuntimeError("failed to reconstruct E8P12 abs base patterns from current codebook grid.")
    spar = np.zeros(256, np.int64)
    for k in range(8):
        spar ^= (np.arange(256) >> k) & 1
    valid = np.broadcast_to(spar[None, None, :] == parity[None, :, None], lut.shape)
    if not (np.all(lut[valid] >= 0) and np.all(lut[~valid] < 0)):
        raise RuntimeError("E8P12 codebook does not have the (branch, abs, parity-valid sign) structure.")
    if not np.isin(base_abs, np.array([0.5, 1.5, 2.5], np.float32)).all():
        # the posterior/MAP kernels tabulate the per-coordinate terms for these three magnitudes
        raise RuntimeError("E8P12 abs patterns must have coordinates 1/2, 3/2 or 5/2.")
    t = {
        "base_abs": torch.from_numpy(base_abs).to(device),
        "base_sqnorm": torch.from_numpy(sqnorm).to(device),
        "base_parity": torch.from_numpy(parity.astype(np.int32)).to(device),
        "idx_lut": torch.from_numpy(lut.astype(np.int32)).to(device),
        "grid": torch.from_numpy(np.ascontiguousarray(grid)).to(device),
        "sign_id": torch.from_numpy(sid.astype(np.uint8)).to(device),
    }
    _TABLES[key] = t
    return t
