"""Solver variants built on the baseline solvers of ``mpq_b200.solver`` (mpq/solvers/)."""
from .vamp_topk_polish import solve_e8p12_rankspace_vamp_topk_polish

__all__ = ["solve_e8p12_rankspace_vamp_topk_polish"]
