"""Edge cases: empty inputs through the C-ABI and the Python entry points, and run-to-run determinism."""
import numpy as np
import pytest
import torch

from oracle import e8p12 as OE
from oracle import layer as OL


@pytest.mark.gpu
def test_empty_inputs_are_no_ops(cuda_dev):
    from mpq_b200 import ops
    from mpq_b200._lib import call, ptr
    from mpq_b200.codebook import E8P12_codebook, factor_tables
    from mpq_b200.e8p12 import _tab_ptrs
    t = factor_tables(E8P12_codebook(), cuda_dev)
    dummy = torch.zeros(8, device=cuda_dev)
    # zero rows / zero blocks: success without a launch
    call("mpq_e8p12_mmse", ptr(dummy), 8, None, 0, None, 0, ptr(dummy), 0.0, 0, 1, *_tab_ptrs(t), ptr(dummy), 8,
         None, 0, None, 0, None, 0, ptr(dummy))
    call("mpq_e8p12_map", ptr(dummy), 8, None, 0, None, 0, None, 1.0, 0.0, 3, 0, *_tab_ptrs(t), None, 0, None, 0)
    call("mpq_uniform_mmse", ptr(dummy), 8, ptr(dummy), 8, ptr(dummy), ptr(dummy), 1, 0, ptr(dummy), 0, 8, 15, 0.0,
         ptr(dummy), 8, None, None, None, ptr(dummy))
    call("mpq_uniform_mmse", None, 8, None, 8, None, None, 1, 0, None, 0, 8, 15, 0.0, None, 8, None, None, None, None)
    # top-k entries: empty shapes succeed, bad k is rejected with a message
    call("mpq_e8p12_topk", None, 8, None, 0, None, 0, None, 0.0, 0, 4, *_tab_ptrs(t), 16, None, None, None)
    call("mpq_uniform_topk", None, 8, None, 0, None, None, 1, 0, None, 0, 8, 15, 0.0, 4, None, None, None)
    call("mpq_topk_pick", None, 8, None, 8, None, 8, 0, 4, 8, None, None, 8, None)
    with pytest.raises(RuntimeError, match="k must be in"):
        call("mpq_e8p12_topk", ptr(dummy), 8, None, 0, None, 0, ptr(dummy), 0.0, 1, 1, *_tab_ptrs(t), 2000,
             ptr(dummy), None, None)
    with pytest.raises(RuntimeError, match="k must be in"):
        call("mpq_uniform_topk", ptr(dummy), 8, None, 0, ptr(dummy), ptr(dummy), 1, 0, ptr(dummy), 1, 8, 3, 0.0, 5,
             ptr(dummy), ptr(dummy), None)
    from mpq_b200.topk import uniform_map_topk, vamp_vector_map_topk_e8p12
    e = torch.zeros(0, 16, device=cuda_dev)
    o = uniform_map_topk(r1=e, gamma1=torch.zeros(0, 1, device=cuda_dev), scale_full=e, zero_full=e, maxq=15,
                         prior_center=e, prior_tau=0.2, k=4)
    assert o["topk_q"].shape == (0, 16, 4)
    o = vamp_vector_map_topk_e8p12(r1_blocks=torch.zeros(0, 2, 8, device=cuda_dev),
                                   gamma1=torch.zeros(0, 1, device=cuda_dev), cb=E8P12_codebook(), k=8)
    assert o["topk_idxs"].shape == (0, 2, 8)
    A = torch.zeros(0, 64, device=cuda_dev)
    B = torch.randn(32, 64, device=cuda_dev)
    for prec in ("f16x3", "tf32x3", "fp32"):
        C = ops.mm_nt(A, ops.Operand(B, prec), precision=prec)
        assert C.shape == (0, 32)
    torch.cuda.synchronize()
    ops.check_status(cuda_dev)


@pytest.mark.gpu
def test_e8p12_posterior_is_deterministic(cuda_dev):
    from mpq_b200 import e8p12 as PE
    from mpq_b200.codebook import E8P12_codebook
    cb = E8P12_codebook()
    g = torch.Generator(device="cpu").manual_seed(4)
    r1 = (torch.randn(64, 96, 8, generator=g) * 0.9).to(cuda_dev)
    gam = (torch.rand(64, 1, generator=g) * 20 + 2).to(cuda_dev)
    a = PE.vamp_vector_discrete_mmse_e8p12(r1_blocks=r1, gamma1=gam, cb=cb)
    b = PE.vamp_vector_discrete_mmse_e8p12(r1_blocks=r1, gamma1=gam, cb=cb)
    for k in ("x1_blocks", "var1", "map_idxs", "alpha1"):
        assert torch.equal(a[k], b[k]), k


@pytest.mark.gpu
def test_e8p12_solve_is_deterministic(cuda_dev):
    """A 256 x 1024 E8P12 solve twice: identical codes and errors (fixed-order reductions throughout)."""
    from mpq_b200 import solver as S
    from mpq_b200.codebook import E8P12_codebook
    rng = np.random.default_rng(12)
    m, n = 256, 1024
    W = rng.standard_normal((m, n)).astype(np.float32)
    s = np.exp(rng.standard_normal(n)).astype(np.float32)
    X = (rng.standard_normal((2 * n, n)) * np.sqrt(s)).astype(np.float32)
    H = OL.hessian_from_calibration(X)
    lam, V, _ = OL.vamp_hessian_eigen(H, fp64=True)
    Sv = np.sqrt(lam).astype(np.float32)
    Vs = (V * Sv[None, :]).astype(np.float32)
    cb = E8P12_codebook()
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_dev)
    hat0, _ = OE.rtn_init(W, OE.E8P12_codebook())
    outs = []
    for _ in range(2):
        hat, idx, err, st = S.solve_e8p12_rankspace_vamp(Wr=d(W), hatWr_init=d(hat0), cb=cb, V=d(V), Vh=d(V.T.copy()),
                                                         S=d(Sv), Vs=d(Vs), cfg=S.E8P12VampConfig(iters=8, polish_sweeps=2))
        outs.append((idx.cpu(), err.cpu()))
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])
    assert outs[0][0].min() >= 0 and outs[0][0].max() < 65536
