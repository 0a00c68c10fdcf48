"""Internal block-Hadamard rotation plan, GPTQ prepare/finalize and the load-time input hooks (GPU)."""
import types

import numpy as np
import pytest
import torch

from oracle import layer as OL


class _PackedLinear(torch.nn.Module):
    """A stand-in for a GPTQ QuantLinear: packed tensors plus a forward over the dequantized solver-basis codes."""

    def __init__(self, q_int, scale, zero, group, bits):
        super().__init__()
        from mpq_b200.export import pack_gptq
        rows, cols = q_int.shape
        g_idx = torch.arange(cols, device=q_int.device, dtype=torch.int32) // group
        packed = pack_gptq(q_int, scale, zero, g_idx, bits)
        self.qweight, self.qzeros, self.scales = packed["qweight"], packed["qzeros"], packed["scales"]
        self.bits, self.in_features = bits, cols
        sf = scale.repeat_interleave(group, dim=1)
        zf = zero.repeat_interleave(group, dim=1)
        self.register_buffer("w_solver", sf * (q_int.float() - zf))

    def forward(self, x):
        return x @ self.w_solver.T


@pytest.mark.gpu
def test_prepare_finalize_roundtrip(cuda_dev):
    from mpq_b200.adapters.gptqmodel import finalize_gptq_internal_hadamard, prepare_gptq_internal_hadamard
    rng = np.random.default_rng(0)
    W = torch.from_numpy(rng.standard_normal((32, 384)).astype(np.float32)).to(cuda_dev)
    A = rng.standard_normal((600, 384)).astype(np.float32)
    H = torch.from_numpy(A.T @ A / 600).to(cuda_dev)
    qcfg = types.SimpleNamespace(mpq=types.SimpleNamespace(rotation_mode="internal_hadamard"))
    Ww, Hw, plan = prepare_gptq_internal_hadamard(W=W, H=H, qcfg=qcfg, module_name="m.q_proj")
    assert plan["internal"] and plan["block_dim"] == 128 and plan["effective"] == "internal_block_hadamard"
    # the rotation is orthogonal: the proxy objective is unchanged
    np.testing.assert_allclose(float((Ww @ Hw * Ww).sum()), float((W @ H * W).sum()), rtol=1e-4)
    back = finalize_gptq_internal_hadamard(Q_work=Ww, rotation_plan=plan)
    torch.testing.assert_close(back, W, rtol=1e-5, atol=1e-5)
    # the oracle's rotation (the reference's torch butterfly) gives the same solver-basis weights
    ref = OL.right_block_hadamard(W.cpu().numpy(), plan["signs"].cpu().numpy(), 128)
    np.testing.assert_allclose(Ww.cpu().numpy(), ref, rtol=1e-6, atol=1e-6)
    plan_none = prepare_gptq_internal_hadamard(W=W, H=H, qcfg=types.SimpleNamespace(mpq=types.SimpleNamespace(
        rotation_mode="none")), module_name="m.q_proj")[2]
    assert not plan_none["internal"]
    with pytest.raises(ValueError):
        prepare_gptq_internal_hadamard(W=W, H=H, qcfg=types.SimpleNamespace(mpq=types.SimpleNamespace(
            rotation_mode="spin")), module_name="m")


@pytest.mark.gpu
def test_input_hooks_reproduce_dense_weights(cuda_dev):
    """Packed solver-basis codes + the input pre-hook give the same outputs as the dense inverse-rotated Q."""
    from mpq_b200.adapters.gptqmodel import GPTQAdapterConfig, install_internal_hadamard_input_hooks, run_mpq_quantization
    from mpq_b200.solver import UniformVampConfig
    rng = np.random.default_rng(1)
    rows, cols, group, bits = 48, 256, 64, 4
    W = torch.from_numpy((rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)).to(cuda_dev)
    A = (rng.standard_normal((4 * cols, cols)) * np.exp(rng.standard_normal(cols))).astype(np.float32)
    H = torch.from_numpy(2.0 * A.T @ A / A.shape[0]).to(cuda_dev)
    qcfg = types.SimpleNamespace(bits=bits, group_size=group, desc_act=False,
                                 mpq=types.SimpleNamespace(rotation_mode="internal_hadamard", solver="vamp"))
    Q, q_int, scale, zero, g_idx, _, st = run_mpq_quantization(
        W=W, H=H, quantizer=None, qcfg=qcfg, module_name="model.layers.0.mlp.up_proj",
        vamp_cfg=UniformVampConfig(iters=4, polish_sweeps=1), adapter_cfg=GPTQAdapterConfig(block_rows=rows))
    assert st["rotation_internal"]
    model = torch.nn.Module()
    model.layers = torch.nn.Module()
    model.layers.add_module("0", torch.nn.Module())
    getattr(model.layers, "0").mlp = torch.nn.Module()
    getattr(model.layers, "0").mlp.up_proj = _PackedLinear(q_int, scale, zero, group, bits)
    # under a top-level wrapper the module is named "model.layers.0.mlp.up_proj", the key the solve used
    wrapper = torch.nn.Module()
    wrapper.model = model
    assert install_internal_hadamard_input_hooks(wrapper) == 1
    assert install_internal_hadamard_input_hooks(wrapper) == 0  # idempotent
    x = torch.from_numpy(rng.standard_normal((5, cols)).astype(np.float32)).to(cuda_dev)
    y = getattr(wrapper.model.layers, "0").mlp.up_proj(x)
    torch.testing.assert_close(y, x @ Q.T, rtol=1e-4, atol=1e-5)
    with pytest.raises(RuntimeError, match="width mismatch"):
        getattr(wrapper.model.layers, "0").mlp.up_proj(x[:, :128])
