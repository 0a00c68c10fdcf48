"""The set-up pipeline (mpq_b200.pipeline): layer set-up on a worker thread and low-priority stream ahead of the
solves gives the same results as the serial order, in the per-layer adapter and in the QUIP# model walk."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _layers(dev, count, m=256, n=1024):
    g = torch.Generator().manual_seed(5)
    out = []
    for _ in range(count):
        W = torch.randn(m, n, generator=g) * 0.02
        X = torch.randn(2 * n, n, generator=g) * torch.exp(torch.randn(n, generator=g)).sqrt()
        H = X.T @ X / X.shape[0]
        H += torch.eye(n) * 0.01 * H.diagonal().mean()
        SU = torch.randint(0, 2, (m,), generator=g).float() * 2 - 1
        SV = torch.randint(0, 2, (n,), generator=g).float() * 2 - 1
        out.append(tuple(t.to(dev) for t in (W, H, SU, SV)))
    return out


def _setup(W, H, SU, SV, eigen):
    from mpq_b200.adapters.gptqmodel import vamp_hessian_eigen
    from mpq_b200.rotation import rht_hessian, rht_weight
    m, n = W.shape
    Wr = rht_weight(W, SU, SV, m, n)
    Hr = rht_hessian(H, SV, n)
    Wn = (Wr / float(Wr.double().square().mean().sqrt())).contiguous()
    return {"Wn": Wn, "Hr": Hr, "eig": vamp_hessian_eigen(Hr, fp64=True) if eigen else None}


def _solve(P, cb, after=None):
    import types
    from mpq_b200.adapters.quip_sharp import mpq_refine_codebook
    args = types.SimpleNamespace(mpq_init="rtn", mpq_iters=8, mpq_prior_tau=0.25, mpq_polish_sweeps=2,
                                 mpq_block_rows=128, quant_solver="vamp", quant_polish_mode="block_cd",
                                 mpq_polish_metric="gram")
    Wn = P["Wn"]
    m, n = Wn.shape
    return mpq_refine_codebook(Wn, P["Hr"], Wn, torch.zeros(m, n // 8, dtype=torch.int64, device=Wn.device), cb, args,
                               module_name="pipeline.test", eigen=P["eig"], after_enqueue=after)


def test_pipelined_setup_matches_serial(cuda_dev):
    from mpq_b200.codebook import E8P12_codebook
    from mpq_b200.pipeline import SetupPipeline
    cb = E8P12_codebook()
    layers = _layers(cuda_dev, 3)
    serial = [_solve(_setup(*L, eigen=False), cb) for L in layers]  # the adapter's own eigendecomposition
    got = []
    with SetupPipeline(cuda_dev) as pipe:
        pipe.submit(0, _setup, *layers[0], eigen=True)
        for k in range(len(layers)):
            P = pipe.get(k)
            nxt = (lambda j=k + 1: pipe.submit(j, _setup, *layers[j], eigen=True)) if k + 1 < len(layers) else None
            got.append(_solve(P, cb, after=nxt))
    torch.cuda.synchronize()
    for (h0, i0, s0), (h1, i1, s1) in zip(serial, got):
        assert torch.equal(i0, i1)
        assert torch.equal(h0, h1)
        assert s0["obs_precision_final"] == s1["obs_precision_final"]
        assert s0["eigen_floor"] == s1["eigen_floor"]


def test_pipeline_reraises_setup_errors(cuda_dev):
    from mpq_b200.pipeline import SetupPipeline

    def bad():
        raise ValueError("set-up failed")

    with SetupPipeline(cuda_dev) as pipe:
        pipe.submit("x", bad)
        with pytest.raises(ValueError, match="set-up failed"):
            pipe.get("x")
        pipe.submit("y", lambda: None)
        with pytest.raises(KeyError):
            pipe.submit("y", lambda: None)


def test_eigen_argument_is_checked(cuda_dev):
    from mpq_b200.codebook import E8P12_codebook
    P = _setup(*_layers(cuda_dev, 1, m=128, n=256)[0], eigen=True)
    lam, V, floor = P["eig"]
    P["eig"] = (lam[:-1], V, floor)
    with pytest.raises(ValueError, match="eigen"):
        _solve(P, E8P12_codebook())


def test_quip_walk_pipelined_matches_serial(cuda_dev):
    from mpq_b200.model import QuipModelConfig, build_synthetic_decoder, calibration_ids, quantize_model_quip
    outs = []
    for pipelined in (False, True):
        model = build_synthetic_decoder("tiny_llama", device=cuda_dev, seed=0)
        ids = calibration_ids(8, 64, model.config.vocab_size, seed=2)
        out = quantize_model_quip(model, ids, QuipModelConfig(iters=6, polish_sweeps=1, batch_size=4,
                                                              pipelined=pipelined))
        outs.append((out["groups"], {n: p.detach().clone() for n, p in model.named_parameters() if "proj" in n}))
    (g0, w0), (g1, w1) = outs
    assert sorted(g0) == sorted(g1)
    for key in g0:
        assert torch.equal(g0[key]["Qidxs"], g1[key]["Qidxs"]), key
    for name in w0:
        assert torch.equal(w0[name], w1[name]), name


def test_wait_completes_a_setup_and_keeps_it_queued(cuda_dev):
    """wait(key) blocks until the set-up's device work is done; the result stays queued and get() returns it."""
    from mpq_b200.pipeline import SetupPipeline
    (W, H, SU, SV), = _layers(cuda_dev, 1)
    with SetupPipeline(cuda_dev) as pipe:
        pipe.submit(7, _setup, W, H, SU, SV, eigen=True)
        pipe.wait(7)
        assert pipe.pending(7) and pipe.keys() == [7]
        P = pipe.get(7)
        assert not pipe.pending(7)
    want = _setup(W, H, SU, SV, eigen=True)
    torch.cuda.synchronize()
    assert torch.equal(P["Wn"], want["Wn"]) and torch.equal(P["Hr"], want["Hr"])
    assert torch.equal(P["eig"][0], want["eig"][0])
