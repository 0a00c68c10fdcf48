"""Generic rank-space block CD (plugin engine): the CPU oracle against the reference's golden vectors, and
the CUDA engine (through the C-ABI kernels) against both."""
import json

import numpy as np
import pytest
import torch

from oracle import block_cd as OB
from oracle import e8p12 as OE

SCALAR = ["s_greedy", "s_static", "s_cyclic"]
E8 = ["e_gram", "e_iso", "e_gram_cap"]


@pytest.fixture(scope="module")
def gz(golden_dir):
    return np.load(golden_dir / "block_cd.npz")


def _meta(gz, c):
    return json.loads(str(gz[f"{c}/meta"]))


def _objectives(stats):
    return [t["stabilized_objective_mean"] for t in stats["sweep_trace"]]


@pytest.mark.parametrize("case", SCALAR)
def test_oracle_scalar_provider_matches_reference(gz, case):
    m = _meta(gz, case)
    x, q, st = OB.block_coordinate_descent_rankspace(
        x=gz[f"{case}/x0"], Y_u=gz[f"{case}/Y_u"], Vs=gz[f"{case}/Vs"], block_size=1,
        propose=OB.scalar_provider(gz[f"{case}/scale"], gz[f"{case}/zero"], m["maxq"]), sweeps=m["sweeps"],
        metric="diag", order_mode=m["order"], idxs_init=gz[f"{case}/q0"], raw_target=gz[f"{case}/W"],
        raw_gram=gz[f"{case}/H"])
    np.testing.assert_array_equal(x, gz[f"{case}/x"])
    np.testing.assert_array_equal(q, gz[f"{case}/q"])
    assert st["accepted_updates"] == m["stats"]["accepted_updates"]
    np.testing.assert_allclose(_objectives(st), _objectives(m["stats"]), rtol=1e-6)
    np.testing.assert_allclose([t["raw_objective_mean"] for t in st["sweep_trace"]],
                               [t["raw_objective_mean"] for t in m["stats"]["sweep_trace"]], rtol=1e-5)


@pytest.mark.parametrize("case", E8)
def test_oracle_e8p12_provider_matches_reference(gz, case):
    m = _meta(gz, case)
    x, idx, st = OB.block_coordinate_descent_rankspace(
        x=gz[f"{case}/x0"], Y_u=gz[f"{case}/Y_u"], Vs=gz[f"{case}/Vs"], block_size=8,
        propose=OB.e8p12_provider(OE.E8P12_codebook()), sweeps=m["sweeps"], metric=m["metric"],
        max_blocks_per_sweep=m["max_blocks"], idxs_init=gz[f"{case}/i0"])
    np.testing.assert_array_equal(idx, gz[f"{case}/idx"])
    assert st["accepted_updates"] == m["stats"]["accepted_updates"]
    assert [t["assignment_changes_from_cd0"] for t in st["sweep_trace"]] == \
        [t["assignment_changes_from_cd0"] for t in m["stats"]["sweep_trace"]]


def _d(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("case", SCALAR)
def test_engine_scalar_provider(cuda_dev, gz, case):
    from mpq_b200.block_cd import BlockCDConfig, UniformScalarProvider, block_coordinate_descent_rankspace
    m = _meta(gz, case)
    prov = UniformScalarProvider(scale=_d(gz[f"{case}/scale"], cuda_dev), zero=_d(gz[f"{case}/zero"], cuda_dev),
                                 maxq=m["maxq"])
    x, q, st = block_coordinate_descent_rankspace(
        x=_d(gz[f"{case}/x0"], cuda_dev), Y_u=_d(gz[f"{case}/Y_u"], cuda_dev), Vs=_d(gz[f"{case}/Vs"], cuda_dev),
        block_size=1, provider=prov, cfg=BlockCDConfig(sweeps=m["sweeps"], metric="diag", order_mode=m["order"]),
        idxs_init=_d(gz[f"{case}/q0"], cuda_dev), raw_target=_d(gz[f"{case}/W"], cuda_dev),
        raw_gram=_d(gz[f"{case}/H"], cuda_dev))
    agree = (x.cpu().numpy() == gz[f"{case}/x"]).mean()
    assert agree >= 0.99, agree
    assert q.dtype == torch.int32
    assert (q.cpu().numpy() == gz[f"{case}/q"]).mean() >= 0.99
    np.testing.assert_allclose(_objectives(st), _objectives(m["stats"]), rtol=2e-4)
    assert st["stabilized_objective_nonincreasing"]


@pytest.mark.gpu
@pytest.mark.parametrize("case", E8)
def test_engine_e8p12_provider(cuda_dev, gz, case):
    from mpq_b200.block_cd import BlockCDConfig, E8P12Provider, block_coordinate_descent_rankspace
    from mpq_b200.codebook import E8P12_codebook
    m = _meta(gz, case)
    x, idx, st = block_coordinate_descent_rankspace(
        x=_d(gz[f"{case}/x0"], cuda_dev), Y_u=_d(gz[f"{case}/Y_u"], cuda_dev), Vs=_d(gz[f"{case}/Vs"], cuda_dev),
        block_size=8, provider=E8P12Provider(cb=E8P12_codebook()),
        cfg=BlockCDConfig(sweeps=m["sweeps"], metric=m["metric"], max_blocks_per_sweep=m["max_blocks"]),
        idxs_init=_d(gz[f"{case}/i0"], cuda_dev))
    assert idx.dtype == torch.int64
    agree = (idx.cpu().numpy() == gz[f"{case}/idx"]).mean()
    assert agree >= 0.99, agree
    np.testing.assert_allclose(_objectives(st), _objectives(m["stats"]), rtol=1e-3)
    assert len(st["sweep_trace"]) == m["sweeps"] + 1


@pytest.mark.gpu
def test_engine_generic_path_matches_fused_gram_path(cuda_dev, gz):
    """The same gram-metric problem through the fused chunked kernels and through the per-block loop (a
    provider that is not an E8P12Provider instance takes the generic path)."""
    from mpq_b200.block_cd import BlockCDConfig, E8P12Provider, block_coordinate_descent_rankspace
    from mpq_b200.codebook import E8P12_codebook
    cb = E8P12_codebook()

    class Wrapped:
        def __init__(self):
            self.inner = E8P12Provider(cb=cb)

        def propose(self, **kw):
            return self.inner.propose(**kw)

    c = "e_gram"
    args = dict(x=_d(gz[f"{c}/x0"], cuda_dev), Y_u=_d(gz[f"{c}/Y_u"], cuda_dev), Vs=_d(gz[f"{c}/Vs"], cuda_dev),
                block_size=8, cfg=BlockCDConfig(sweeps=2, metric="gram"), idxs_init=_d(gz[f"{c}/i0"], cuda_dev))
    _, i_fused, s_fused = block_coordinate_descent_rankspace(provider=E8P12Provider(cb=cb), **args)
    _, i_gen, s_gen = block_coordinate_descent_rankspace(provider=Wrapped(), **args)
    assert (i_fused.cpu() == i_gen.cpu()).float().mean().item() >= 0.99
    np.testing.assert_allclose(_objectives(s_fused), _objectives(s_gen), rtol=1e-4)
