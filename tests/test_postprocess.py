"""GPTQ postprocess (the MPQ polish of a finished GPTQ solution, mpq/adapters/gptqmodel.py:1250-1470): the CPU
oracle against the reference's golden vectors, and the CUDA driver against both."""
import json
import types

import numpy as np
import pytest
import torch

from oracle import layer as OL
from oracle.uniform_vamp import UniformVampConfig

CASES = ["pp_cd", "pp_topk"]


@pytest.fixture(scope="module")
def gz(golden_dir):
    return np.load(golden_dir / "postprocess.npz")


def _meta(gz, c):
    return json.loads(str(gz[f"{c}/meta"]))


@pytest.mark.parametrize("case", CASES)
def test_oracle_postprocess_matches_reference(gz, case):
    m = _meta(gz, case)
    o = OL.postprocess_gptq(W=gz[f"{case}/W"], H=gz[f"{case}/H"], Q_init=gz[f"{case}/Q0"],
                            scale_groups=gz[f"{case}/sg"], zero_groups=gz[f"{case}/zg"], g_idx=gz[f"{case}/g_idx"],
                            bits=m["bits"], polish_mode=m["mode"], polish_sweeps=3, topk_k=m["k"],
                            vamp_cfg=UniformVampConfig(iters=10, prior_tau=0.2))
    st = m["stats"]
    agree = (o["q"] == gz[f"{case}/q"]).mean()
    assert agree >= 0.999, agree
    assert o["fail_closed"] == st["module_fail_closed"]
    np.testing.assert_allclose(float(o["err_final"].mean()), st["rankspace_error_mean_final"], rtol=1e-4)
    np.testing.assert_allclose(float(o["err_before"].mean()), st["rankspace_error_mean_before"], rtol=1e-5)


def _d(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_gpu_postprocess_matches_reference(cuda_dev, gz, case):
    from mpq_b200.adapters.gptqmodel import GPTQAdapterConfig, postprocess_gptq_quantization
    m = _meta(gz, case)
    qcfg = types.SimpleNamespace(bits=m["bits"], group_size=m["gs"], mpq=types.SimpleNamespace(
        polish_mode=m["mode"], polish_sweeps=3, topk_k=m["k"], iters=10, prior_tau=0.2, block_cd_backend=""))
    W = gz[f"{case}/W"]
    Q, q, sg, zg, g_idx, secs, st = postprocess_gptq_quantization(
        W=_d(W, cuda_dev), H=_d(gz[f"{case}/H"], cuda_dev), Q_init=_d(gz[f"{case}/Q0"], cuda_dev),
        scale_groups=_d(gz[f"{case}/sg"], cuda_dev), zero_groups=_d(gz[f"{case}/zg"], cuda_dev),
        g_idx=_d(gz[f"{case}/g_idx"], cuda_dev), qcfg=qcfg, module_name=f"golden.pp.{case}",
        adapter_cfg=GPTQAdapterConfig(block_rows=W.shape[0]))
    ref = m["stats"]
    assert q.dtype == torch.int32 and g_idx.dtype == torch.int32
    agree = (q.cpu().numpy() == gz[f"{case}/q"]).mean()
    assert agree >= 0.995, agree
    assert st["module_fail_closed"] == ref["module_fail_closed"]
    np.testing.assert_allclose(st["rankspace_error_mean_final"], ref["rankspace_error_mean_final"], rtol=2e-3)
    np.testing.assert_allclose(st["rankspace_error_mean_before"], ref["rankspace_error_mean_before"], rtol=1e-4)
    assert st["rankspace_error_mean_final"] <= st["rankspace_error_mean_before"]
    assert st["input_fingerprint"]["w_sha256"] == ref["fp"]["w_sha256"]
    # Q is the dequantized q on the GPTQ grid
    sf = gz[f"{case}/sg"][:, gz[f"{case}/g_idx"]]
    zf = gz[f"{case}/zg"][:, gz[f"{case}/g_idx"]]
    np.testing.assert_array_equal(Q.cpu().numpy(), (sf * (q.cpu().numpy().astype(np.float32) - zf)))
