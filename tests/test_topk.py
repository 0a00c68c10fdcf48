"""Top-k polish ("topk_block_cd"): candidate sets and providers.  The CPU oracle against the reference's golden
vectors, then the CUDA kernels (mpq_uniform_topk, mpq_e8p12_topk, mpq_topk_pick) and the engine against both."""
import json

import numpy as np
import pytest
import torch

from oracle import block_cd as OB
from oracle import e8p12 as OE
from oracle import topk as OT

UNI = ["u4p", "u4", "u2p"]
E8 = ["e_lo_p", "e_hi", "e_lo"]


@pytest.fixture(scope="module")
def gz(golden_dir):
    return np.load(golden_dir / "topk.npz")


def _meta(gz, c):
    return json.loads(str(gz[f"{c}/meta"]))


def assert_topk_match(idx_a, sc_a, idx_b, sc_b, rtol=1e-6, atol=1e-6, min_agree=0.995):
    """Same scores position by position; where the chosen candidates differ the two scores are tied."""
    idx_a, idx_b = np.asarray(idx_a), np.asarray(idx_b)
    sc_a, sc_b = np.asarray(sc_a, np.float64), np.asarray(sc_b, np.float64)
    assert idx_a.shape == idx_b.shape
    np.testing.assert_allclose(sc_a, sc_b, rtol=rtol, atol=atol)
    diff = idx_a != idx_b
    assert 1.0 - diff.mean() >= min_agree, diff.mean()
    if diff.any():
        tol = atol + rtol * np.abs(sc_b[diff])
        assert np.all(np.abs(sc_a[diff] - sc_b[diff]) <= tol)


# ---------------------------------------------------------------- oracle vs reference

@pytest.mark.parametrize("case", UNI)
def test_oracle_uniform_topk_matches_reference(gz, case):
    m = _meta(gz, case)
    o = OT.uniform_map_topk(r1=gz[f"{case}/r1"], gamma1=gz[f"{case}/gamma"], scale_full=gz[f"{case}/scale"],
                            zero_full=gz[f"{case}/zero"], maxq=m["maxq"], prior_center=gz[f"{case}/W"],
                            prior_tau=m["tau"], k=m["k"])
    assert o["topk_q"].shape == gz[f"{case}/q"].shape
    np.testing.assert_array_equal(o["topk_q"], gz[f"{case}/q"])
    np.testing.assert_array_equal(o["topk_values"], gz[f"{case}/values"])
    np.testing.assert_array_equal(o["topk_scores"], gz[f"{case}/scores"])


@pytest.mark.parametrize("case", E8)
def test_oracle_e8p12_topk_matches_reference(gz, case):
    m = _meta(gz, case)
    W = gz["e/W"]
    ps = OE.prior_scale_from_center(W, "absmax") if m["tau"] > 0 else None
    o = OT.vamp_vector_map_topk_e8p12(r1_blocks=gz["e/r1"], gamma1=gz[f"{case}/gamma"], cb=OE.E8P12_codebook(),
                                      k=m["k"], prior_center_blocks=W if m["tau"] > 0 else None,
                                      prior_scale_blocks=ps, prior_tau=m["tau"])
    assert_topk_match(o["topk_idxs"], o["topk_scores"], gz[f"{case}/idxs"], gz[f"{case}/scores"], min_agree=0.999)


def test_oracle_uniform_topk_provider_cd_matches_reference(gz):
    c = "cd_u"
    m = _meta(gz, c)
    x, q, st = OB.block_coordinate_descent_rankspace(
        x=gz[f"{c}/x0"], Y_u=gz[f"{c}/Y_u"], Vs=gz[f"{c}/Vs"], block_size=1,
        propose=OT.uniform_topk_provider(gz[f"{c}/tv"], gz[f"{c}/tq"]), sweeps=2, metric="diag",
        order_mode="greedy_gain", idxs_init=gz[f"{c}/q0"], raw_target=gz[f"{c}/W"], raw_gram=gz[f"{c}/H"])
    np.testing.assert_array_equal(x, gz[f"{c}/x"])
    np.testing.assert_array_equal(q, gz[f"{c}/q"])
    assert st["accepted_updates"] == m["stats"]["accepted_updates"]


@pytest.mark.parametrize("case", ["cd_eg", "cd_ed"])
def test_oracle_e8p12_topk_provider_cd_matches_reference(gz, case):
    m = _meta(gz, case)
    x, idx, st = OB.block_coordinate_descent_rankspace(
        x=gz[f"{case}/x0"], Y_u=gz[f"{case}/Y_u"], Vs=gz[f"{case}/Vs"], block_size=8,
        propose=OT.e8p12_topk_provider(gz[f"{case}/ti"], OE.E8P12_codebook().grid), sweeps=2, metric=m["metric"],
        order_mode="greedy_gain", idxs_init=gz[f"{case}/i0"])
    np.testing.assert_array_equal(idx, gz[f"{case}/idx"])
    assert st["accepted_updates"] == m["stats"]["accepted_updates"]


def test_oracle_topk_tie_order():
    """Equal scores keep the lower grid level / the lower flat candidate first (a planted exact tie)."""
    scale = np.full((1, 1), 0.5, np.float32)
    zero = np.full((1, 1), 1.0, np.float32)
    # r1 halfway between atoms 0 (q=1) and 0.5 (q=2): q=1 and q=2 tie for the best score
    o = OT.uniform_map_topk(r1=np.full((1, 1), 0.25, np.float32), gamma1=np.ones((1, 1), np.float32),
                            scale_full=scale, zero_full=zero, maxq=3, prior_center=None, prior_tau=0.0, k=4)
    assert o["topk_q"][0, 0].tolist() == [1, 2, 0, 3]


# ---------------------------------------------------------------- CUDA vs oracle / reference

def _d(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("case", UNI)
def test_gpu_uniform_topk_matches_reference(cuda_dev, gz, case):
    from mpq_b200.topk import uniform_map_topk
    m = _meta(gz, case)
    o = uniform_map_topk(r1=_d(gz[f"{case}/r1"], cuda_dev), gamma1=_d(gz[f"{case}/gamma"], cuda_dev),
                         scale_full=_d(gz[f"{case}/scale"], cuda_dev), zero_full=_d(gz[f"{case}/zero"], cuda_dev),
                         maxq=m["maxq"], prior_center=_d(gz[f"{case}/W"], cuda_dev), prior_tau=m["tau"], k=m["k"])
    assert o["topk_q"].dtype == torch.int64
    np.testing.assert_array_equal(o["topk_q"].cpu().numpy(), gz[f"{case}/q"])
    np.testing.assert_array_equal(o["topk_values"].cpu().numpy(), gz[f"{case}/values"])
    np.testing.assert_array_equal(o["topk_scores"].cpu().numpy(), gz[f"{case}/scores"])


@pytest.mark.gpu
@pytest.mark.parametrize("bits,k,group", [(4, 16, 0), (3, 5, 64), (2, 7, 32), (5, 9, 32), (8, 40, 64)])
def test_gpu_uniform_topk_matches_oracle(cuda_dev, bits, k, group):
    from mpq_b200.topk import uniform_map_topk
    rng = np.random.default_rng(bits * 31 + k)
    B, n, maxq = 96, 512, 2 ** bits - 1
    W = (rng.standard_normal((B, n)) * 0.05).astype(np.float32)
    G = n // group if group else n
    s = (rng.random((B, G)) * 0.02 + 0.005).astype(np.float32)
    z = rng.integers(0, maxq + 1, (B, G)).astype(np.float32)
    sf = np.repeat(s, n // G, axis=1) if group else s
    zf = np.repeat(z, n // G, axis=1) if group else z
    r1 = (W + rng.standard_normal((B, n)) * 0.01).astype(np.float32)
    gam = (rng.random((B, 1)) * 2e4 + 1e3).astype(np.float32)
    ref = OT.uniform_map_topk(r1=r1, gamma1=gam, scale_full=sf, zero_full=zf, maxq=maxq, prior_center=W,
                              prior_tau=0.25, k=k)
    o = uniform_map_topk(r1=_d(r1, cuda_dev), gamma1=_d(gam, cuda_dev), scale_full=_d(s, cuda_dev),
                         zero_full=_d(z, cuda_dev), maxq=maxq, prior_center=_d(W, cuda_dev), prior_tau=0.25, k=k)
    np.testing.assert_array_equal(o["topk_q"].cpu().numpy(), ref["topk_q"])
    np.testing.assert_array_equal(o["topk_values"].cpu().numpy(), ref["topk_values"])
    np.testing.assert_array_equal(o["topk_scores"].cpu().numpy(), ref["topk_scores"])


@pytest.mark.gpu
@pytest.mark.parametrize("case", E8)
def test_gpu_e8p12_topk_matches_reference(cuda_dev, gz, case):
    from mpq_b200.codebook import E8P12_codebook
    from mpq_b200.topk import vamp_vector_map_topk_e8p12
    m = _meta(gz, case)
    W = gz["e/W"]
    ps = OE.prior_scale_from_center(W, "absmax") if m["tau"] > 0 else None
    cb = E8P12_codebook()
    o = vamp_vector_map_topk_e8p12(r1_blocks=_d(gz["e/r1"], cuda_dev), gamma1=_d(gz[f"{case}/gamma"], cuda_dev),
                                   cb=cb, k=m["k"], prior_center_blocks=_d(W, cuda_dev) if m["tau"] > 0 else None,
                                   prior_scale_blocks=_d(ps, cuda_dev) if ps is not None else None,
                                   prior_tau=m["tau"])
    assert o["topk_idxs"].dtype == torch.int64
    assert_topk_match(o["topk_idxs"].cpu().numpy(), o["topk_scores"].cpu().numpy(), gz[f"{case}/idxs"],
                      gz[f"{case}/scores"], min_agree=0.999)
    grid = cb.grid.cpu().numpy()
    np.testing.assert_array_equal(o["topk_vals"].cpu().numpy(), grid[o["topk_idxs"].cpu().numpy()])


@pytest.mark.gpu
@pytest.mark.parametrize("k,tau,glo,ghi", [(16, 0.25, 1.0, 6.0), (64, 0.0, 20.0, 200.0), (1024, 0.0, 0.3, 1.0)])
def test_gpu_e8p12_topk_matches_oracle(cuda_dev, k, tau, glo, ghi):
    from mpq_b200.codebook import E8P12_codebook
    from mpq_b200.topk import vamp_vector_map_topk_e8p12
    rng = np.random.default_rng(k)
    B, nb = (16, 16) if k == 1024 else (48, 64)
    W = (rng.standard_normal((B, nb, 8)) * 0.8).astype(np.float32)
    r1 = (W + rng.standard_normal((B, nb, 8)) * 0.3).astype(np.float32)
    gam = (rng.random((B, 1)) * (ghi - glo) + glo).astype(np.float32)
    ps = OE.prior_scale_from_center(W, "absmax") if tau > 0 else None
    ref = OT.vamp_vector_map_topk_e8p12(r1_blocks=r1, gamma1=gam, cb=OE.E8P12_codebook(), k=k,
                                        prior_center_blocks=W if tau > 0 else None, prior_scale_blocks=ps,
                                        prior_tau=tau)
    o = vamp_vector_map_topk_e8p12(r1_blocks=_d(r1, cuda_dev), gamma1=_d(gam, cuda_dev), cb=E8P12_codebook(), k=k,
                                   prior_center_blocks=_d(W, cuda_dev) if tau > 0 else None,
                                   prior_scale_blocks=_d(ps, cuda_dev) if ps is not None else None, prior_tau=tau)
    # identical float32 operation order: bit-exact scores and indices
    np.testing.assert_array_equal(o["topk_scores"].cpu().numpy(), ref["topk_scores"])
    np.testing.assert_array_equal(o["topk_idxs"].cpu().numpy(), ref["topk_idxs"])


@pytest.mark.gpu
def test_gpu_uniform_topk_provider_cd_matches_reference(cuda_dev, gz):
    from mpq_b200.block_cd import BlockCDConfig, UniformTopKProvider, block_coordinate_descent_rankspace
    c = "cd_u"
    m = _meta(gz, c)
    prov = UniformTopKProvider(topk_values=_d(gz[f"{c}/tv"], cuda_dev), topk_q=_d(gz[f"{c}/tq"], cuda_dev))
    x, q, st = block_coordinate_descent_rankspace(
        x=_d(gz[f"{c}/x0"], cuda_dev), Y_u=_d(gz[f"{c}/Y_u"], cuda_dev), Vs=_d(gz[f"{c}/Vs"], cuda_dev), block_size=1,
        provider=prov, cfg=BlockCDConfig(sweeps=2, metric="diag"), idxs_init=_d(gz[f"{c}/q0"], cuda_dev),
        raw_target=_d(gz[f"{c}/W"], cuda_dev), raw_gram=_d(gz[f"{c}/H"], cuda_dev))
    assert (q.cpu().numpy() == gz[f"{c}/q"]).mean() >= 0.99
    assert (x.cpu().numpy() == gz[f"{c}/x"]).mean() >= 0.99
    assert abs(st["accepted_updates"] - m["stats"]["accepted_updates"]) <= 0.01 * max(m["stats"]["accepted_updates"], 1)


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["cd_eg", "cd_ed"])
def test_gpu_e8p12_topk_provider_cd_matches_reference(cuda_dev, gz, case):
    from mpq_b200.block_cd import BlockCDConfig, E8P12TopKProvider, block_coordinate_descent_rankspace
    from mpq_b200.codebook import E8P12_codebook
    m = _meta(gz, case)
    x, idx, st = block_coordinate_descent_rankspace(
        x=_d(gz[f"{case}/x0"], cuda_dev), Y_u=_d(gz[f"{case}/Y_u"], cuda_dev), Vs=_d(gz[f"{case}/Vs"], cuda_dev),
        block_size=8, provider=E8P12TopKProvider(cb=E8P12_codebook(), topk_idxs=_d(gz[f"{case}/ti"], cuda_dev)),
        cfg=BlockCDConfig(sweeps=2, metric=m["metric"]), idxs_init=_d(gz[f"{case}/i0"], cuda_dev))
    assert idx.dtype == torch.int64
    assert (idx.cpu().numpy() == gz[f"{case}/idx"]).mean() >= 0.99
    assert abs(st["accepted_updates"] - m["stats"]["accepted_updates"]) <= 0.02 * max(m["stats"]["accepted_updates"], 1)


@pytest.mark.gpu
def test_gpu_topk_pick_matches_oracle(cuda_dev):
    """mpq_topk_pick with and without the metric factor against the oracle providers' selection."""
    from mpq_b200._lib import call, ptr
    rng = np.random.default_rng(5)
    grid = OE.E8P12_codebook().grid
    B, nb, k = 512, 3, 24
    ti = rng.integers(0, 65536, (B, nb, k)).astype(np.int64)
    target = rng.standard_normal((B, 8)).astype(np.float32)
    L = np.tril(rng.standard_normal((8, 8))).astype(np.float32) + 3 * np.eye(8, dtype=np.float32)
    for metric in ("gram", "diag"):
        ref_v, ref_i = OT.e8p12_topk_provider(ti, grid)(block_idx=1, target=target, metric=metric, gram_chol=L)
        vals = _d(grid[ti].astype(np.float32), cuda_dev)
        idx = _d(ti, cuda_dev, torch.int32)
        tg = _d(target, cuda_dev)
        out_v = torch.empty(B, 8, device=cuda_dev)
        out_i = torch.empty(B, device=cuda_dev, dtype=torch.int32)
        chol = _d(L, cuda_dev) if metric == "gram" else None
        call("mpq_topk_pick", ptr(tg), 8, ptr(vals[:, 1]), nb * k * 8, ptr(idx[:, 1]), nb * k, B, k, 8, ptr(chol),
             ptr(out_v), 8, ptr(out_i))
        np.testing.assert_array_equal(out_i.cpu().numpy(), ref_i)
        np.testing.assert_array_equal(out_v.cpu().numpy(), ref_v)


class _Wrapped:
    """A provider that is not one of the built-in classes: the engine takes its generic per-block loop."""

    def __init__(self, inner):
        self.inner = inner

    def propose(self, **kw):
        return self.inner.propose(**kw)


@pytest.mark.gpu
def test_gpu_fused_uniform_topk_engine_matches_generic(cuda_dev, gz):
    from mpq_b200.block_cd import BlockCDConfig, UniformTopKProvider, block_coordinate_descent_rankspace
    c = "cd_u"
    args = dict(x=_d(gz[f"{c}/x0"], cuda_dev), Y_u=_d(gz[f"{c}/Y_u"], cuda_dev), Vs=_d(gz[f"{c}/Vs"], cuda_dev),
                block_size=1, cfg=BlockCDConfig(sweeps=3, metric="diag"), idxs_init=_d(gz[f"{c}/q0"], cuda_dev))
    mk = lambda: UniformTopKProvider(topk_values=_d(gz[f"{c}/tv"], cuda_dev), topk_q=_d(gz[f"{c}/tq"], cuda_dev))
    x_f, q_f, s_f = block_coordinate_descent_rankspace(provider=mk(), **args)
    x_g, q_g, s_g = block_coordinate_descent_rankspace(provider=_Wrapped(mk()), **args)
    assert (q_f.cpu() == q_g.cpu()).float().mean() >= 0.99
    assert abs(s_f["accepted_updates"] - s_g["accepted_updates"]) <= 0.01 * s_g["accepted_updates"] + 2
    np.testing.assert_allclose([t["stabilized_objective_mean"] for t in s_f["sweep_trace"]],
                               [t["stabilized_objective_mean"] for t in s_g["sweep_trace"]], rtol=2e-3)
    assert s_f["stabilized_objective_nonincreasing"]


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["cd_eg"])
def test_gpu_fused_e8p12_topk_engine_matches_generic(cuda_dev, gz, case):
    from mpq_b200.block_cd import BlockCDConfig, E8P12TopKProvider, block_coordinate_descent_rankspace
    from mpq_b200.codebook import E8P12_codebook
    cb = E8P12_codebook()
    args = dict(x=_d(gz[f"{case}/x0"], cuda_dev), Y_u=_d(gz[f"{case}/Y_u"], cuda_dev),
                Vs=_d(gz[f"{case}/Vs"], cuda_dev), block_size=8, cfg=BlockCDConfig(sweeps=3, metric="gram"),
                idxs_init=_d(gz[f"{case}/i0"], cuda_dev))
    mk = lambda: E8P12TopKProvider(cb=cb, topk_idxs=_d(gz[f"{case}/ti"], cuda_dev))
    _, i_f, s_f = block_coordinate_descent_rankspace(provider=mk(), **args)
    _, i_g, s_g = block_coordinate_descent_rankspace(provider=_Wrapped(mk()), **args)
    assert i_f.dtype == torch.int64
    assert (i_f.cpu() == i_g.cpu()).float().mean() >= 0.99
    assert abs(s_f["accepted_updates"] - s_g["accepted_updates"]) <= 0.02 * s_g["accepted_updates"] + 2


@pytest.mark.gpu
def test_gpu_fused_topk_engines_large(cuda_dev):
    """A 512 x 1024 problem through the fused top-k engines against the oracle engine."""
    from mpq_b200.block_cd import BlockCDConfig, UniformTopKProvider, block_coordinate_descent_rankspace
    rng = np.random.default_rng(17)
    B, n, maxq, k = 96, 512, 15, 6
    A = rng.standard_normal((2 * n, n)).astype(np.float32) * np.exp(rng.standard_normal(n)).astype(np.float32) ** 0.5
    H = (A.T @ A / (2 * n)).astype(np.float32) + 0.01 * np.eye(n, dtype=np.float32)
    lam, V = np.linalg.eigh(H.astype(np.float64))
    Vs = (V[:, ::-1] * np.sqrt(lam[::-1])).astype(np.float32)
    W = (rng.standard_normal((B, n)) * 0.02).astype(np.float32)
    s = np.full((B, n), 0.006, np.float32)
    z = np.full((B, n), 8.0, np.float32)
    r1 = (W + rng.standard_normal((B, n)).astype(np.float32) * 0.002).astype(np.float32)
    tk = OT.uniform_map_topk(r1=r1, gamma1=np.full((B, 1), 5e4, np.float32), scale_full=s, zero_full=z, maxq=maxq,
                             prior_center=W, prior_tau=0.2, k=k)
    q0 = tk["topk_q"][:, :, 0].astype(np.int32)
    x0 = tk["topk_values"][:, :, 0].copy()
    Y_u = (W @ Vs).astype(np.float32)
    _, rq, rst = OB.block_coordinate_descent_rankspace(
        x=x0, Y_u=Y_u, Vs=Vs, block_size=1, propose=OT.uniform_topk_provider(tk["topk_values"], tk["topk_q"]),
        sweeps=2, metric="diag", order_mode="greedy_gain", idxs_init=q0)
    x, q, st = block_coordinate_descent_rankspace(
        x=_d(x0, cuda_dev), Y_u=_d(Y_u, cuda_dev), Vs=_d(Vs, cuda_dev), block_size=1,
        provider=UniformTopKProvider(topk_values=_d(tk["topk_values"], cuda_dev), topk_q=_d(tk["topk_q"], cuda_dev)),
        cfg=BlockCDConfig(sweeps=2, metric="diag"), idxs_init=_d(q0, cuda_dev))
    assert (q.cpu().numpy() == rq).mean() >= 0.99
    assert abs(st["accepted_updates"] - rst["accepted_updates"]) <= 0.01 * rst["accepted_updates"] + 2
