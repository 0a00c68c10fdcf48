"""Deterministic 4096-column layer inputs shared by the fixture generator (make_layer4096.py, which runs the
reference on the CPU) and the GPU parity tests (which run the CUDA path on the same inputs).

The construction follows BASELINE configs 0 and 1: W 4096 x 4096 ~ N(0, 0.02^2) (torch generator seed 0),
X 16384 x 4096 with log-normal channel scales, H = X^T X / 16384 + 0.01 mean(diag H) I, and for E8P12 +-1 sign
vectors of the randomized Hadamard transform on both sides.  To make H bit-identical on every machine, X^T X is
accumulated in float64 (any summation order) and rounded once to float32, and the regulariser is formed from the
float64 diagonal mean; the RMS scale of the rotated weights is likewise taken in float64.
"""
from __future__ import annotations

import torch

M_ROWS = 4096
N_COLS = 4096
T_CALIB = 16384


def synth(device: str = "cpu"):
    """(W fp32 m x n, H fp32 n x n, SU +-1 (m), SV +-1 (n)); X^T X on `device` in float64."""
    g = torch.Generator(device="cpu").manual_seed(0)
    W = torch.randn(M_ROWS, N_COLS, generator=g) * 0.02
    s = torch.exp(torch.randn(N_COLS, generator=g))
    X = torch.randn(T_CALIB, N_COLS, generator=g) * s.sqrt()
    SU = (torch.randint(0, 2, (M_ROWS,), generator=g).float() * 2 - 1)
    SV = (torch.randint(0, 2, (N_COLS,), generator=g).float() * 2 - 1)
    Xd = X.to(device=device, dtype=torch.float64)
    H64 = (Xd.T @ Xd) / float(T_CALIB)
    del Xd
    reg = 0.01 * float(H64.diagonal().mean())
    H = H64.float()
    del H64
    H.diagonal().add_(torch.tensor(reg, dtype=torch.float32, device=H.device))
    return W, H.cpu(), SU, SV


def rms_scale(Wr: torch.Tensor) -> float:
    """sqrt(mean(Wr^2)) in float64 (QUIP#'s global Wscale of the rotated weights)."""
    return float(Wr.double().square().mean().sqrt())
