"""MPQ per-layer quantization solve on NVIDIA B200 (sm_100a).

Public surface mirrors the reference (poseidonchan/MPQ): ``mpq_b200.solver`` holds
``solve_uniform_rankspace_vamp`` / ``polish_uniform_rankspace`` and the config dataclasses,
``mpq_b200.adapters.gptqmodel.run_mpq_quantization`` is the per-linear scalar driver.
Every numerical step runs in ``libmpq_b200.so`` (C-ABI, ``include/mpq_b200.h``).
"""
from .quantization import QuantizationConfig, quantize
from .solver import E8P12VampConfig, UniformVampConfig, polish_uniform_rankspace, solve_uniform_rankspace_vamp

__version__ = "0.1.0"
__all__ = ["QuantizationConfig", "quantize", "UniformVampConfig", "E8P12VampConfig", "solve_uniform_rankspace_vamp",
           "polish_uniform_rankspace"]
