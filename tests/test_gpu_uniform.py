"""GPU parity of the grouped-scalar kernels against the CPU oracle (all calls go through the C-ABI)."""
import numpy as np
import pytest
import torch

from oracle import layer as OL
from oracle import uniform_vamp as OU

pytestmark = pytest.mark.gpu


def _rng(seed):
    return np.random.default_rng(seed)


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _uniform_case(seed, B, n, maxq, group):
    r = _rng(seed)
    W = (r.standard_normal((B, n)) * 0.02).astype(np.float32)
    G = n // group
    scale_g = (r.random((B, G)) * 0.01 + 0.002).astype(np.float32)
    zero_g = r.integers(0, maxq + 1, (B, G)).astype(np.float32)
    r1 = (W + r.standard_normal((B, n)).astype(np.float32) * 0.01).astype(np.float32)
    sf = np.repeat(scale_g, group, 1)
    zf = np.repeat(zero_g, group, 1)
    # exact ties between neighbouring atoms
    r1[0, :16] = sf[0, :16] * (np.arange(16, dtype=np.float32) % maxq + np.float32(0.5) - zf[0, :16])
    gamma = (r.random((B, 1)) * 2e4 + 1e3).astype(np.float32)
    return W, scale_g, zero_g, sf, zf, r1, gamma


@pytest.mark.parametrize("maxq,tau,grouped", [(15, 0.2, True), (15, 0.2, False), (7, 0.25, True), (3, 0.0, True),
                                              (1, 0.2, True), (31, 0.2, True)])
def test_uniform_mmse_matches_oracle(cuda_dev, maxq, tau, grouped):
    from mpq_b200._lib import call, ptr
    B, n, group = 9, 384, 64
    W, sg, zg, sf, zf, r1, gamma = _uniform_case(1 + maxq, B, n, maxq, group)
    ref = OU.discrete_uniform_mmse(r1=r1, gamma1=gamma, scale_full=sf, zero_full=zf, maxq=maxq, prior_center=W,
                                   prior_tau=tau)
    d = lambda a: _t(a, cuda_dev)
    s_in, z_in = (d(sg), d(zg)) if grouped else (d(sf), d(zf))
    gshift = 6 if grouped else 0
    mean = torch.empty(B, n, device=cuda_dev)
    var = torch.empty(B, n, device=cuda_dev)
    mapv = torch.empty(B, n, device=cuda_dev)
    mapi = torch.empty(B, n, device=cuda_dev, dtype=torch.uint8)
    vsum = torch.empty(B, device=cuda_dev)
    r1d, Wd, gd = d(r1), d(W), d(gamma[:, 0])
    call("mpq_uniform_mmse", ptr(r1d), n, ptr(Wd), n, ptr(s_in), ptr(z_in), s_in.stride(0), gshift, ptr(gd), B, n,
         maxq, tau, ptr(mean), n, ptr(var), ptr(mapv), ptr(mapi), ptr(vsum))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(mapi.cpu().numpy(), ref["map_idx"])          # bit-exact codes
    np.testing.assert_array_equal(mapv.cpu().numpy(), ref["map_value"])
    np.testing.assert_allclose(mean.cpu().numpy(), ref["mean"], rtol=2e-5, atol=1e-8)
    # var = E[x^2] - mean^2 cancels: its error is a few ulps of E[x^2], not of var
    v, rv = var.cpu().numpy(), ref["var"]
    second = rv + ref["mean"].astype(np.float64) ** 2
    assert np.all(np.abs(v - rv) <= 2e-3 * np.abs(rv) + 16 * np.finfo(np.float32).eps * second)
    np.testing.assert_allclose(gamma[:, 0] * vsum.cpu().numpy() / n, ref["alpha1"][:, 0], rtol=1e-4)
    # the MAP hard decision
    q = torch.empty(B, n, device=cuda_dev, dtype=torch.uint8)
    x = torch.empty(B, n, device=cuda_dev)
    call("mpq_uniform_map_decision", ptr(r1d), n, ptr(Wd), n, ptr(s_in), ptr(z_in), s_in.stride(0), gshift, ptr(gd),
         B, n, maxq, tau, ptr(q), ptr(x), n)
    rq, rx = OU.uniform_hard_decision(x_mean=ref["mean"], x_map=ref["map_value"], scale_full=sf, zero_full=zf,
                                      maxq=maxq)
    np.testing.assert_array_equal(q.cpu().numpy(), rq)
    np.testing.assert_array_equal(x.cpu().numpy(), rx)


def test_uniform_mmse_golden_reference_vectors(cuda_dev, golden_dir):
    """The kernel against vectors produced by the reference itself."""
    from mpq_b200._lib import call, ptr
    z = np.load(golden_dir / "uniform_denoise.npz")
    for case in ("q4", "q3", "q4_noprior"):
        g = lambda k: z[f"{case}/{k}"]
        B, n = g("r1").shape
        d = lambda a: _t(a.astype(np.float32), cuda_dev)
        mean = torch.empty(B, n, device=cuda_dev)
        mapi = torch.empty(B, n, device=cuda_dev, dtype=torch.uint8)
        vsum = torch.empty(B, device=cuda_dev)
        # keep every device input alive until the launch is enqueued
        sc, ze, r1d, Wd, gd = d(g("scale")), d(g("zero")), d(g("r1")), d(g("W")), d(g("gamma")[:, 0])
        call("mpq_uniform_mmse", ptr(r1d), n, ptr(Wd), n, ptr(sc), ptr(ze), n, 0, ptr(gd), B, n, int(g("maxq")),
             float(g("tau")), ptr(mean), n, None, None, ptr(mapi), ptr(vsum))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(mapi.cpu().numpy().astype(np.int64), g("map_idx"))
        np.testing.assert_allclose(mean.cpu().numpy(), g("mean"), rtol=2e-5, atol=1e-8)


def test_nearest_rtn_minmax_hadamard_bit_exact(cuda_dev):
    from mpq_b200._lib import call, ptr
    r = _rng(5)
    B, n, group, maxq = 7, 512, 128, 15
    W = (r.standard_normal((B, n)) * 0.03).astype(np.float32)
    W[2, :128] = 0.0  # all-zero group -> [-1, 1] grid
    sg_ref = np.empty((B, n // group), np.float32)
    zg_ref = np.empty_like(sg_ref)
    for g in range(n // group):
        s, z = OL.find_params_minmax(W[:, g * group:(g + 1) * group], maxq)
        sg_ref[:, g], zg_ref[:, g] = s[:, 0], z[:, 0]
    Wd = _t(W, cuda_dev)
    sg = torch.empty(B, n // group, device=cuda_dev)
    zg = torch.empty_like(sg)
    call("mpq_group_minmax", ptr(Wd), n, B, n, group, maxq, ptr(sg), ptr(zg), sg.stride(0))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(sg.cpu().numpy(), sg_ref)
    np.testing.assert_array_equal(zg.cpu().numpy(), zg_ref)
    sf, zf = np.repeat(sg_ref, group, 1), np.repeat(zg_ref, group, 1)
    # RTN: round(W/s) + z
    x = torch.empty(B, n, device=cuda_dev)
    q = torch.empty(B, n, device=cuda_dev, dtype=torch.uint8)
    call("mpq_uniform_rtn", ptr(Wd), n, ptr(sg), ptr(zg), sg.stride(0), 7, B, n, maxq, ptr(q), ptr(x), n)
    qr = np.clip(np.round(W / sf) + zf, 0, maxq).astype(np.float32)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(q.cpu().numpy(), qr.astype(np.uint8))
    np.testing.assert_array_equal(x.cpu().numpy(), (sf * (qr - zf)).astype(np.float32))
    # nearest_atom_idx with round-half-even ties
    xt = (np.arange(B * n, dtype=np.float32).reshape(B, n) % 37 - 18) * np.float32(0.25) * sf
    xtd = _t(xt, cuda_dev)
    call("mpq_uniform_nearest", ptr(xtd), n, ptr(sg), ptr(zg), sg.stride(0), 7, B, n, maxq, ptr(q), ptr(x), n)
    rq = OU.nearest_atom_idx(x=xt, scale_full=sf, zero_full=zf, maxq=maxq)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(q.cpu().numpy(), rq.astype(np.uint8))
    # block Hadamard rotation and its inverse (bit-exact against the reference butterfly order)
    from mpq_b200.rotation import apply_right_block_hadamard, apply_right_block_hadamard_inverse
    signs = OL.rademacher_signs_torch(n, "test:full", 0)
    for had in (64, 512):
        R = apply_right_block_hadamard(Wd, signs=_t(signs, cuda_dev), had_dim=had)
        np.testing.assert_array_equal(R.cpu().numpy(), OL.right_block_hadamard(W, signs, had))
        Ri = apply_right_block_hadamard_inverse(R, signs=_t(signs, cuda_dev), had_dim=had)
        np.testing.assert_array_equal(Ri.cpu().numpy(), OL.right_block_hadamard_inverse(R.cpu().numpy(), signs, had))


@pytest.mark.parametrize("M,N,K", [(128, 256, 512), (37, 91, 300), (1, 5, 7)])
def test_gemm_f32(cuda_dev, M, N, K):
    from mpq_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(M + N + K)
    A = torch.randn(M, K, generator=g)
    Bt = torch.randn(N, K, generator=g)
    Bn = torch.randn(K, N, generator=g)
    C = ops.gemm_nt(A.to(cuda_dev), Bt.to(cuda_dev)).cpu()
    torch.testing.assert_close(C, A.double().matmul(Bt.double().T).float(), rtol=1e-5, atol=1e-4)
    C0 = torch.randn(M, N, generator=g)
    C2 = ops.gemm_nn(A.to(cuda_dev), Bn.to(cuda_dev), out=C0.clone().to(cuda_dev), alpha=-1.0, beta=1.0).cpu()
    torch.testing.assert_close(C2, (C0.double() - A.double() @ Bn.double()).float(), rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("M,N,K", [(256, 512, 1024), (300, 200, 196), (128, 256, 32), (1000, 4096, 4096),
                                   (128, 4096, 4096), (128, 128, 4096), (96, 200, 1000), (128, 4096, 128)])
@pytest.mark.parametrize("prec", ["tf32x3", "f16x3", "tf32"])
def test_gemm_tensor_core(cuda_dev, M, N, K, prec):
    """tcgen05 TF32 GEMM (3xTF32 split or single product) against an fp64 product."""
    from mpq_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N + K)
    A = torch.randn(M, K, generator=g)
    Bt = torch.randn(N, K, generator=g)
    C0 = torch.randn(M, N, generator=g)
    ref = (A.double() @ Bt.double().T)
    out = ops.mm_nt(A.to(cuda_dev), ops.Operand(Bt.to(cuda_dev), prec), precision=prec)
    torch.cuda.synchronize()
    ops.check_status(cuda_dev)
    err = (out.cpu().double() - ref).abs().max().item()
    scale = (A.double().abs() @ Bt.double().abs().T).max().item()
    # 3xTF32 is FP32-class (the tensor core's FP32 accumulation is not round-to-nearest, so it sits
    # ~10x above an FP32 FMA chain but ~1000x below a single TF32 product)
    tol = 2e-3 if prec == "tf32" else 1e-5
    assert err <= tol * scale, (err, scale)
    out2 = ops.mm_nt(A.to(cuda_dev), ops.Operand(Bt.to(cuda_dev), prec), out=C0.to(cuda_dev), alpha=-0.5, beta=2.0,
                     precision=prec)
    err2 = (out2.cpu().double() - (2.0 * C0.double() - 0.5 * ref)).abs().max().item()
    assert err2 <= tol * scale + 1e-5


@pytest.mark.parametrize("M,N,K", [(128, 4096, 4096), (512, 768, 1000)])
def test_gemm_splitk_matches_single_pass(cuda_dev, M, N, K):
    """The split-K form of the f16x3 product (chosen for small M) against the single-pass kernel and fp64: same
    bound, deterministic across calls."""
    from mpq_b200 import ops
    from mpq_b200._lib import call, ptr
    g = torch.Generator(device="cpu").manual_seed(M + 3 * K)
    A = torch.randn(M, K, generator=g).to(cuda_dev)
    Bt = torch.randn(N, K, generator=g).to(cuda_dev)
    opB = ops.Operand(Bt, "f16x3")
    Ah, Al, Ai = ops.split_f16(A)
    Bh, Bl, Bi = opB.f16
    st = ops.status_word(cuda_dev)
    outs = []
    for splits in (1, 5, 5, 24):
        C = torch.full((M, N), 3.0, device=cuda_dev)
        ws = torch.empty(splits * M * N, device=cuda_dev)
        call("mpq_gemm_f16x3_splitk", M, N, K, -0.5, ptr(Ah), ptr(Al), Ah.stride(0), ptr(Ai), ptr(Bh), ptr(Bl),
             Bh.stride(0), ptr(Bi), 2.0, ptr(C), C.stride(0), splits, ptr(ws), ws.numel(), ptr(st))
        outs.append(C)
    torch.cuda.synchronize()
    ops.check_status(cuda_dev)
    ref = 6.0 - 0.5 * (A.double() @ Bt.double().T)
    scale = 0.5 * (A.double().abs() @ Bt.double().abs().T).max().item()
    for C in outs:
        assert (C.double() - ref).abs().max().item() <= 1e-5 * scale + 1e-5
    assert torch.equal(outs[1], outs[2])  # fixed reduction order


@pytest.mark.parametrize("N", [128, 100, 40])
def test_gemm_parts_narrow_tiles_match_splitk(cuda_dev, N):
    """Split-K partial planes of a narrow product (N <= 128 runs on 128-wide tiles) added in plane order equal the
    split-K product's own reduction (256-wide tiles) bit for bit: the tile width does not change any element."""
    from mpq_b200 import ops
    from mpq_b200._lib import call, ptr
    M, K, splits = 128, 4096, 24
    g = torch.Generator(device="cpu").manual_seed(N)
    A = torch.randn(M, K, generator=g).to(cuda_dev)
    Bt = (torch.randn(N, K, generator=g) * torch.exp(torch.randn(N, 1, generator=g))).to(cuda_dev)
    Ah, Al, Ai = ops.split_f16(A)
    Bh, Bl, Bi = ops.Operand(Bt, "f16x3").f16
    st = ops.status_word(cuda_dev)
    C = torch.zeros(M, N, device=cuda_dev)
    ws = torch.empty(splits * M * N, device=cuda_dev)
    call("mpq_gemm_f16x3_splitk", M, N, K, 1.0, ptr(Ah), ptr(Al), Ah.stride(0), ptr(Ai), ptr(Bh), ptr(Bl),
         Bh.stride(0), ptr(Bi), 0.0, ptr(C), C.stride(0), splits, ptr(ws), ws.numel(), ptr(st))
    planes = torch.empty(splits * M * N, device=cuda_dev)
    call("mpq_gemm_f16x3_parts", M, N, K, ptr(Ah), ptr(Al), Ah.stride(0), ptr(Ai), ptr(Bh), ptr(Bl), Bh.stride(0),
         ptr(Bi), splits, ptr(planes), planes.numel(), ptr(st))
    torch.cuda.synchronize()
    ops.check_status(cuda_dev)
    P = planes.view(splits, M, N)
    acc = P[0].clone()
    for s_ in range(1, splits):
        acc = acc + P[s_]
    assert torch.equal(acc, C)
    ref = A.double() @ Bt.double().T
    scale = (A.double().abs() @ Bt.double().abs().T).max().item()
    assert (C.double() - ref).abs().max().item() <= 1e-5 * scale


@pytest.mark.parametrize("rows,cols,ldx", [(128, 4096, 4096), (37, 100, 104), (5, 98, 98), (300, 4100, 4100)])
def test_split_f16_bits_match_definition(cuda_dev, rows, cols, ldx):
    """mpq_split_f16 (16-byte path for rows of 4k floats at 4k-aligned strides, the warp-per-row path otherwise) bit
    for bit against its definition: s = 2^(15 - e) with max|row| < 2^e, hi = fp16_rn(x s), lo = fp16_rn(x s - hi),
    inverse scale 2^(e - 15); zero rows and rows spanning 2^±6 magnitudes included."""
    from mpq_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(rows + cols)
    base = torch.randn(rows, ldx, generator=g) * torch.exp(3.0 * torch.randn(rows, 1, generator=g))
    base[0] = 0.0
    x = base.to(cuda_dev)[:, :cols]
    hi, lo, inv = ops.split_f16(x)
    torch.cuda.synchronize()
    mx = x.abs().amax(1)
    e = torch.where(mx > 0, torch.frexp(mx).exponent, torch.zeros_like(mx, dtype=torch.int32))
    one = torch.ones_like(mx)
    y = x * torch.ldexp(one, 15 - e)[:, None]
    h = y.half()
    lo_want = (y - h.float()).half()
    assert torch.equal(hi[:, :cols].view(torch.int16), h.view(torch.int16))
    assert torch.equal(lo[:, :cols].view(torch.int16), lo_want.view(torch.int16))
    assert torch.equal(inv, torch.ldexp(one, e - 15))


def test_gemm_f16x3_wide_dynamic_range(cuda_dev):
    """f16x3 on rows whose entries span 2^20 (log-uniform magnitudes, as Vs rows under log-normal channel scales
    and small eigenvalues): every entry within 1e-5 of its own |A||B|^T scale plus the split's absolute floor
    (entries below 2^-18 of their row maximum keep an absolute error of at most 2^-38 of that maximum)."""
    from mpq_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(5)
    M, N, K = 256, 384, 2048
    A = torch.randn(M, K, generator=g, dtype=torch.float64) * torch.exp2(-20.0 * torch.rand(M, K, generator=g,
                                                                                              dtype=torch.float64))
    Bt = torch.randn(N, K, generator=g, dtype=torch.float64) * torch.exp2(-20.0 * torch.rand(N, K, generator=g,
                                                                                               dtype=torch.float64))
    A32, B32 = A.float(), Bt.float()
    out = ops.mm_nt(A32.to(cuda_dev), ops.Operand(B32.to(cuda_dev), "f16x3"), precision="f16x3").cpu().double()
    ops.check_status(cuda_dev)
    Ad, Bd = A32.double(), B32.double()
    ref = Ad @ Bd.T
    per_entry = Ad.abs() @ Bd.abs().T
    floor = 2.0 ** -36 * (Ad.abs().amax(1, keepdim=True) * Bd.abs().sum(1)[None, :]
                          + Ad.abs().sum(1, keepdim=True) * Bd.abs().amax(1)[None, :])
    excess = ((out - ref).abs() - (1e-5 * per_entry + floor)).max().item()
    assert excess <= 0.0, excess


def _layer_fixture(m, n, seed):
    r = _rng(seed)
    W = (r.standard_normal((m, n)) * 0.02).astype(np.float32)
    s = np.exp(r.standard_normal(n)).astype(np.float32)
    X = (r.standard_normal((4 * n, n)) * np.sqrt(s)).astype(np.float32)
    H = OL.hessian_from_calibration(X)
    return W, H


def _eig(H):
    lam, V, _ = OL.vamp_hessian_eigen(H)
    S = np.sqrt(lam).astype(np.float32)
    return V, S, (V * S[None, :]).astype(np.float32)


def _rtn(W, maxq, group):
    sg = np.empty((W.shape[0], W.shape[1] // group), np.float32)
    zg = np.empty_like(sg)
    for g in range(W.shape[1] // group):
        s, z = OL.find_params_minmax(W[:, g * group:(g + 1) * group], maxq)
        sg[:, g], zg[:, g] = s[:, 0], z[:, 0]
    sf, zf = np.repeat(sg, group, 1), np.repeat(zg, group, 1)
    q = np.clip(np.round(W / sf) + zf, 0, maxq).astype(np.float32)
    return sg, zg, sf, zf, (sf * (q - zf)).astype(np.float32)


def test_scalar_cd_matches_oracle(cuda_dev):
    from mpq_b200 import solver as S
    W, H = _layer_fixture(24, 320, 21)
    V, Sv, Vs = _eig(H)
    maxq, group = 15, 64
    sg, zg, sf, zf, x0 = _rtn(W, maxq, group)
    Y_u = W @ Vs
    ref_x, ref_st = OU.uniform_scalar_diag_greedy_cd(x=x0, Y_u=Y_u, Vs=Vs, gram_full=H, scale=sf, zero=zf, maxq=maxq,
                                                     sweeps=3)
    d = lambda a: _t(a, cuda_dev)
    q, x, err, st = S.polish_uniform_rankspace(x_init=d(x0), Y_u=d(Y_u), Vs=d(Vs), scale_full=d(sg), zero_full=d(zg),
                                               maxq=maxq, sweeps=3, polish_mode="block_cd", gram_full=d(H))
    ref_q = OU.nearest_atom_idx(x=ref_x, scale_full=sf, zero_full=zf, maxq=maxq)
    agree = (q.cpu().numpy() == ref_q).mean()
    assert agree >= 0.999, agree
    assert abs(st["accepted_updates"] - ref_st["accepted_updates"]) <= 0.01 * ref_st["accepted_updates"] + 2


@pytest.mark.parametrize("m,n,iters,maxq,group", [(64, 256, 20, 15, 64), (40, 192, 16, 7, 64), (1, 128, 10, 15, 128),
                                                   (48, 256, 16, 3, 128)])
def test_solve_uniform_vamp_matches_oracle(cuda_dev, m, n, iters, maxq, group):
    from mpq_b200 import solver as S
    W, H = _layer_fixture(m, n, 3 + m)
    V, Sv, Vs = _eig(H)
    sg, zg, sf, zf, x_rtn = _rtn(W, maxq, group)
    ocfg = OU.UniformVampConfig(iters=iters, prior_tau=0.2, damping=0.5, polish_sweeps=3)
    rq, rx, rerr, rrtn, rst = OU.solve_uniform_rankspace_vamp(W=W, x_rtn=x_rtn, scale_full=sf, zero_full=zf,
                                                              maxq=maxq, V=V, Vh=V.T.copy(), S=Sv, Vs=Vs, cfg=ocfg,
                                                              gram_full=H)
    d = lambda a: _t(a, cuda_dev)
    cfg = S.UniformVampConfig(iters=iters, prior_tau=0.2, damping=0.5, polish_sweeps=3, block_cd_backend="auto")
    q, x, err, rtn_err, st = S.solve_uniform_rankspace_vamp(W=d(W), x_rtn=d(x_rtn), scale_full=d(sg), zero_full=d(zg),
                                                            maxq=maxq, V=d(V), Vh=d(V.T.copy()), S=d(Sv), Vs=d(Vs),
                                                            cfg=cfg, gram_full=d(H))
    agree = (q.cpu().numpy() == rq).mean()
    assert agree >= 0.999, (agree, st["best_iter"], rst["best_iter"])
    loss = OL.proxy_loss(W, x.cpu().numpy(), H)
    rloss = OL.proxy_loss(W, rx, H)
    assert abs(loss - rloss) <= 0.005 * rloss
    np.testing.assert_allclose(rtn_err.cpu().numpy(), rrtn, rtol=1e-3)


@pytest.mark.parametrize("m,n,iters,maxq,group,k", [(48, 256, 12, 15, 64, 4), (32, 192, 10, 3, 64, 16)])
def test_solve_uniform_vamp_topk_matches_oracle(cuda_dev, m, n, iters, maxq, group, k):
    """polish_mode "topk_block_cd": top-k atoms from the final message, generic engine with the top-k provider."""
    from mpq_b200 import solver as S
    W, H = _layer_fixture(m, n, 70 + m)
    V, Sv, Vs = _eig(H)
    sg, zg, sf, zf, x_rtn = _rtn(W, maxq, group)
    ocfg = OU.UniformVampConfig(iters=iters, prior_tau=0.2, damping=0.5, polish_sweeps=2, polish_mode="topk_block_cd",
                                topk_k=k)
    rq, rx, rerr, _, rst = OU.solve_uniform_rankspace_vamp(W=W, x_rtn=x_rtn, scale_full=sf, zero_full=zf, maxq=maxq,
                                                           V=V, Vh=V.T.copy(), S=Sv, Vs=Vs, cfg=ocfg, gram_full=H)
    d = lambda a: _t(a, cuda_dev)
    cfg = S.UniformVampConfig(iters=iters, prior_tau=0.2, damping=0.5, polish_sweeps=2, polish_mode="topk_block_cd",
                              topk_k=k)
    q, x, err, _, st = S.solve_uniform_rankspace_vamp(W=d(W), x_rtn=d(x_rtn), scale_full=d(sg), zero_full=d(zg),
                                                      maxq=maxq, V=d(V), Vh=d(V.T.copy()), S=d(Sv), Vs=d(Vs), cfg=cfg,
                                                      gram_full=d(H))
    agree = (q.cpu().numpy() == rq).mean()
    assert agree >= 0.995, (agree, st["polish_updates"], rst["polish_updates"])
    loss, rloss = OL.proxy_loss(W, x.cpu().numpy(), H), OL.proxy_loss(W, rx, H)
    assert abs(loss - rloss) <= 0.005 * rloss
    assert st["polish_updates"] > 0
    # every final level is one of the coordinate's top-k candidates or the pre-polish MAP level
    np.testing.assert_array_equal(x.cpu().numpy(), (sf * (q.cpu().numpy().astype(np.float32) - zf)))


def test_polish_uniform_topk_entry(cuda_dev):
    """polish_uniform_rankspace(polish_mode="topk_block_cd") against the oracle engine with the top-k provider."""
    from mpq_b200 import solver as S
    from oracle import block_cd as OB
    from oracle import topk as OT
    W, H = _layer_fixture(40, 256, 91)
    V, Sv, Vs = _eig(H)
    maxq, group = 7, 64
    sg, zg, sf, zf, x0 = _rtn(W, maxq, group)
    Y_u = (W @ Vs).astype(np.float32)
    r1 = (W + _rng(4).standard_normal(W.shape).astype(np.float32) * 0.003).astype(np.float32)
    gam = np.full((W.shape[0], 1), 2e4, np.float32)
    tk = OT.uniform_map_topk(r1=r1, gamma1=gam, scale_full=sf, zero_full=zf, maxq=maxq, prior_center=W,
                             prior_tau=0.2, k=3)
    q0 = OU.nearest_atom_idx(x=x0, scale_full=sf, zero_full=zf, maxq=maxq)
    _, rq, rst = OB.block_coordinate_descent_rankspace(
        x=x0, Y_u=Y_u, Vs=Vs, block_size=1, propose=OT.uniform_topk_provider(tk["topk_values"], tk["topk_q"]),
        sweeps=2, metric="diag", order_mode="greedy_gain", idxs_init=q0)
    d = lambda a: _t(a, cuda_dev)
    q, x, err, st = S.polish_uniform_rankspace(x_init=d(x0), Y_u=d(Y_u), Vs=d(Vs), scale_full=d(sg), zero_full=d(zg),
                                               maxq=maxq, sweeps=2, polish_mode="topk_block_cd",
                                               topk_values=d(tk["topk_values"]), topk_q=d(tk["topk_q"]))
    assert q.dtype == torch.int32
    assert (q.cpu().numpy() == rq).mean() >= 0.995
    assert abs(st["accepted_updates"] - rst["accepted_updates"]) <= 0.01 * rst["accepted_updates"] + 2
    with pytest.raises(ValueError, match="topk_values"):
        S.polish_uniform_rankspace(x_init=d(x0), Y_u=d(Y_u), Vs=d(Vs), scale_full=d(sg), zero_full=d(zg), maxq=maxq,
                                   sweeps=2, polish_mode="topk_block_cd")


@pytest.mark.parametrize("case", ["a", "b", "c", "d"])
def test_run_mpq_quantization_matches_reference_golden(cuda_dev, golden_dir, case):
    """The full per-linear driver against the reference's own output (tests/golden/scalar_layer.npz): a/b the default
    recipe, c activation order (desc_act), d the round-mean final decision."""
    import json
    import types
    from mpq_b200.adapters.gptqmodel import GPTQAdapterConfig, run_mpq_quantization
    from mpq_b200.solver import UniformVampConfig
    z = np.load(golden_dir / "scalar_layer.npz")
    g = lambda k: z[f"{case}/{k}"]
    meta = json.loads(str(g("meta")))
    qcfg = types.SimpleNamespace(bits=meta["bits"], group_size=meta["group_size"],
                                 desc_act=bool(meta.get("desc_act", False)),
                                 mpq=types.SimpleNamespace(rotation_mode="internal_hadamard", solver="vamp"))
    cfg = UniformVampConfig(iters=meta["iters"], prior_tau=0.2, damping=0.5, polish_sweeps=3, block_cd_backend="auto",
                            final_decision=meta.get("final_decision", "map"))
    acfg = GPTQAdapterConfig(block_rows=meta["block_rows"], grow_block_rows=False)
    Q, q_int, scale, zero, g_idx, _, st = run_mpq_quantization(
        W=_t(g("W"), cuda_dev), H=_t(2.0 * g("H"), cuda_dev), quantizer=None, qcfg=qcfg, module_name=f"golden.{case}",
        vamp_cfg=cfg, adapter_cfg=acfg)
    np.testing.assert_allclose(scale.cpu().numpy(), g("scale"), rtol=1e-6)
    np.testing.assert_array_equal(zero.cpu().numpy(), g("zero"))
    np.testing.assert_array_equal(g_idx.cpu().numpy(), g("g_idx"))
    assert st["desc_act"] == bool(meta.get("desc_act", False))
    agree = (q_int.cpu().numpy() == g("q_int")).mean()
    assert agree >= 0.999, agree
    rel = abs(st["raw_objective_mean_final"] - meta["raw_objective"]) / meta["raw_objective"]
    assert rel <= 0.005, rel
    np.testing.assert_allclose(Q.cpu().numpy(), g("Q"), rtol=0, atol=2e-3 * np.abs(g("Q")).max())
