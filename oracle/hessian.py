"""CPU restatement of the calibration-Hessian hooks the MPQ drivers consume (TEST INFRASTRUCTURE ONLY).

QUIP# utils.register_H_hook / done() and regularize_H (QUIP# @ 1d8f873, un-vendored; finalised at
mpq/quip_generic.py:906-918, re-centred and regularised at mpq/quip_generic.py:373-378) and GPTQModel
GPTQ.add_batch (GPTQModel @ ed96f2e, un-vendored; feeds mpq/adapters/gptqmodel.py:650-679), restated
from their published sources in float64.  Parity against the third-party code itself is unpinned.
"""
import numpy as np


def quip_hook(batches, n):
    """H = sum x^T x, mu = sum x, ct = tokens; finalised as H / ct - (mu / ct)(mu / ct)^T."""
    H = np.zeros((n, n))
    mu = np.zeros(n)
    ct = 0
    for b in batches:
        x = np.asarray(b, np.float64).reshape(-1, n)
        H += x.T @ x
        mu += x.sum(axis=0)
        ct += x.shape[0]
    mu = mu / ct
    return H / ct - np.outer(mu, mu), mu, ct


def gptq_add_batch(batches, n):
    """H <- H ns / (ns + b) + (2 / (ns + b)) x^T x, b = leading dimension of a 3-D input (1 for 2-D)."""
    H = np.zeros((n, n))
    ns = 0
    for b in batches:
        a = np.asarray(b, np.float64)
        tmp = a.shape[0] if a.ndim == 3 else 1
        x = a.reshape(-1, n)
        H *= ns / (ns + tmp)
        ns += tmp
        H += (2.0 / ns) * (x.T @ x)
    return H


def regularize_H(H, n, sigma_reg):
    """H / mean(diag H) + sigma_reg I."""
    H = H / np.diag(H).mean()
    H[np.arange(n), np.arange(n)] += sigma_reg
    return H
