"""ctypes binding of ``libmpq_b200.so`` (the C-ABI declared in ``include/mpq_b200.h``).

The library is the product: there is no CPU or library fallback.  Importing a kernel entry
point when the shared object is missing raises immediately.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Any, Dict, Tuple

import torch

from . import trace as _trace

LIB_PATH = Path(__file__).resolve().parent / "libmpq_b200.so"

P = ctypes.c_void_p
I = ctypes.c_int
L = ctypes.c_int64
F = ctypes.c_float
D = ctypes.c_double

# name -> argtypes (every entry returns int status; `stream` is the trailing c_void_p)
SIGNATURES: Dict[str, Tuple[Any, ...]] = {
    "mpq_uniform_mmse": (P, L, P, L, P, P, L, I, P, I, I, I, F, P, L, P, P, P, P, P),
    "mpq_uniform_map_decision": (P, L, P, L, P, P, L, I, P, I, I, I, F, P, P, L, P),
    "mpq_uniform_nearest": (P, L, P, P, L, I, I, I, I, P, P, L, P),
    "mpq_group_minmax": (P, L, I, I, I, I, P, P, L, P),
    "mpq_uniform_rtn": (P, L, P, P, L, I, I, I, I, P, P, L, P),
    "mpq_block_hadamard": (P, L, P, L, I, I, I, P, I, P),
    "mpq_e8p12_mmse": (P, L, P, L, P, L, P, F, I, I, P, P, P, P, P, P, L, P, L, P, L, P, L, P, P),
    "mpq_e8p12_mmse_rows": (P, L, P, L, P, L, P, F, I, I, P, P, P, P, P, P, L, P, I, P, P, P),
    "mpq_e8p12_mmse_rows_round_ctl": (P, L, P, L, P, L, P, F, I, I, P, P, P, P, P, P, L, P, I, P, P,
                                      P, P, P, P, P, P, P, P, P, P, P, P, P, I, I, F, I, P, F, P, P),
    "mpq_e8p12_map": (P, L, P, L, P, L, P, F, F, I, I, P, P, P, P, P, P, L, P, L, P),
    "mpq_e8p12_stats": (P, L, P, L, P, L, P, F, I, I, P, P, P, P, P, P, P, P, L, P),
    "mpq_e8p12_topk": (P, L, P, L, P, L, P, F, I, I, P, P, P, P, P, I, P, P, P, P),
    "mpq_uniform_topk": (P, L, P, L, P, P, L, I, P, I, I, I, F, I, P, P, P, P),
    "mpq_topk_pick": (P, L, P, L, P, L, I, I, I, P, P, L, P, P),
    "mpq_gram_meta": (P, L, I, I, P, P, P),
    "mpq_gram_gain": (P, L, I, I, P, P, P),
    "mpq_gram_gather": (P, L, I, P, L, P, I, I, P, P, P, P),
    "mpq_gram_gather_split": (P, L, I, P, L, P, I, I, P, P, L, P, P, P, L, P, P, P, P, P, L, P, P),
    "mpq_gram_gather_sweep": (P, L, I, P, L, P, I, P, P, L, P, P, P, L, P, P, P, P, L, P, P),
    "mpq_gram_chunk_planes": (P, L, P, L, I, L, P, P, P, I, I, P, P, P, P, P, P, L, P, P, P, L, P, P, P, I, F, P),
    "mpq_gram_chunk": (P, L, P, L, P, P, P, I, I, P, P, P, P, P, P, L, P, P, P, I, F, P),
    "mpq_gram_search": (P, I, P, F, F, P, P, P, P, P, P),
    "mpq_vamp_rows": (P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, F, F, I, P),
    "mpq_gamma_retry": (P, P, I, I, F, P),
    "mpq_vamp_r2": (P, P, P, P, P, P, P, I, I, L, F, P),
    "mpq_linear_epilogue": (P, P, P, P, F, I, I, L, P, P, P),
    "mpq_vamp_r1": (P, P, P, P, P, P, I, I, L, F, P),
    "mpq_row_sqerr": (P, P, I, I, L, L, P, P),
    "mpq_residual": (P, P, I, I, L, P, P),
    "mpq_mean_rows": (P, P, I, P, P),
    "mpq_polish_merge": (P, P, P, P, P, P, P, I, I, L, P, P),
    "mpq_gamma_init": (P, P, I, I, L, F, P, P),
    "mpq_row_dot": (P, L, P, L, I, I, P, P),
    "mpq_sub": (P, P, P, I, I, L, P),
    "mpq_peer_alloc": (ctypes.c_size_t, P, P, P),
    "mpq_peer_open": (P, P, P),
    "mpq_peer_close": (P, P),
    "mpq_peer_free": (P, P),
    "mpq_copy_bytes": (P, P, ctypes.c_size_t, P),
    "mpq_gemm_f32": (I, I, I, I, F, P, L, P, L, F, P, L, P),
    "mpq_gemm_tc": (I, I, I, I, F, P, L, P, L, F, P, L, P, P),
    "mpq_split_tf32": (P, L, P, P, L, I, I, P),
    "mpq_gemm_f16x3": (I, I, I, F, P, P, L, P, P, P, L, P, F, P, L, P, P),
    "mpq_gemm_f16x3_splitk": (I, I, I, F, P, P, L, P, P, P, L, P, F, P, L, I, P, L, P, P),
    "mpq_split_f16": (P, L, I, I, P, P, L, P, P),
    "mpq_gemm_tf32x3_noalloc": (I, I, I, F, P, L, P, L, F, P, L, P, P),
    "mpq_syrk_tc": (I, I, I, F, P, P, L, F, P, L, P, P),
    "mpq_split_tf32_t": (P, I, L, I, I, P, P, L, P),
    "mpq_col_sum": (P, I, L, I, I, F, F, P, P),
    "mpq_syrk_bf16": (I, I, F, P, L, F, P, L, I, P, P),
    "mpq_syrk_bf16_acc": (I, I, F, P, L, F, P, L, I, P, P),
    "mpq_syrk_tc_acc": (I, I, I, F, P, P, L, F, P, L, I, P, P),
    "mpq_transpose_bf16": (P, L, I, I, P, L, P),
    "mpq_cd_target": (P, L, P, L, I, I, P, P, P, L, P),
    "mpq_pack_bits": (P, L, L, I, I, I, I, P, L, P),
    "mpq_cd_accept": (P, L, P, L, P, L, P, P, I, I, F, P, L, P, P, L, P, P),
    "mpq_cd_diag": (P, I, I, L, P, P, P),
    "mpq_cd_gain": (P, I, I, L, P, P, P),
    "mpq_argsort_desc": (P, I, P, P),
    "mpq_cd_gather": (P, L, I, P, I, I, P, P, P),
    "mpq_cd_block": (P, L, P, L, P, P, L, I, P, P, P, I, I, P, P, P, P, I, I, F, P),
    "mpq_cd_block_topk": (P, L, P, L, P, P, L, I, P, L, P, P, P, I, I, P, P, P, P, I, F, P),
    "mpq_vamp_ctl_size": (),
    "mpq_vamp_ctl_begin": (P, P, P, I, P, P),
    "mpq_vamp_ctl_round": (P, P, P, P, I, I, F, I, P),
    "mpq_vamp_ctl_commit": (P, P, P, P, P, P, P, I, I, I, D, D, D, P, P, P, P, P, I, P, P, P),
    "mpq_vamp_ctl_best": (P, P, I, I, P, P, P, P, P, P, P, P, P, P, P, L, I, P, P),
    "mpq_vamp_rows_ctl": (P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, F, I, P, P),
    "mpq_vamp_rows_round_ctl": (P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, F, I, P, F, P, P),
    "mpq_vamp_r2_ctl": (P, P, P, P, P, P, P, I, I, L, F, P, P),
    "mpq_linear_epilogue_ctl": (P, P, P, P, I, I, L, P, P, P, P),
    "mpq_vamp_r1_ctl": (P, P, P, P, P, P, I, I, L, F, P, P, P),
    "mpq_vamp_r2_split_ctl": (P, P, P, P, P, P, P, I, I, L, F, P, P, L, P, P, P),
    "mpq_linear_epilogue_parts_ctl": (P, I, P, L, P, P, I, I, P, P, P, L, P, P, P, P),
    "mpq_vamp_r1_parts_ctl": (P, I, P, P, P, P, P, I, I, L, F, P, P, P),
    "mpq_gemm_f16x3_parts": (I, I, I, P, P, L, P, P, P, L, P, I, P, L, P, P),
    "mpq_gram_chunk_topk": (P, L, P, L, P, P, P, I, I, P, P, I, I, P, P, L, P, P, P, I, F, P),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load the CUDA library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"libmpq_b200.so not found at {LIB_PATH}; build it with `python -m mpq_b200.build` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = list(argtypes)
        fn.restype = ctypes.c_int
    lib.mpq_last_error.restype = ctypes.c_char_p
    lib.mpq_last_error.argtypes = []
    lib.mpq_abi_version.restype = ctypes.c_int
    _lib = lib
    return lib


def ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def call(name: str, *args) -> None:
    """Invoke a C-ABI entry point on the current torch stream; raise RuntimeError on failure."""
    lib = load()
    fn = getattr(lib, name)
    status = fn(*args, stream_ptr())
    _trace.count_launch()
    if status != 0:
        msg = lib.mpq_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed with status {status}: {msg}")
