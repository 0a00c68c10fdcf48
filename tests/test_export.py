"""GPTQ-format export: the word-by-word restatement (CPU) and the CUDA bit-stream packer against it."""
import numpy as np
import pytest
import torch

from oracle import gptq_pack as OP


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
def test_oracle_pack_roundtrip(bits):
    r = np.random.default_rng(bits)
    codes = r.integers(0, 1 << bits, size=(64, 5))
    words = OP.pack_rows(codes, bits)
    assert words.shape == (64 * bits // 32, 5)
    np.testing.assert_array_equal(OP.unpack_rows(words, bits, 64), codes)


@pytest.mark.gpu
@pytest.mark.parametrize("bits,group", [(2, 64), (3, 128), (4, 128), (8, 32)])
def test_pack_gptq_matches_oracle(cuda_dev, bits, group):
    from mpq_b200.export import pack_gptq
    r = np.random.default_rng(10 + bits)
    out_f, in_f = 96, 256
    q = r.integers(0, 1 << bits, size=(out_f, in_f)).astype(np.uint8)
    ng = in_f // group
    scale = r.random((out_f, ng)).astype(np.float32) + 0.01
    zero = r.integers(0, 1 << bits, size=(out_f, ng)).astype(np.float32)  # includes zero = 0 (masked to all ones)
    g_idx = (np.arange(in_f) // group).astype(np.int32)
    got = pack_gptq(torch.from_numpy(q).to(cuda_dev), torch.from_numpy(scale).to(cuda_dev),
                    torch.from_numpy(zero).to(cuda_dev), torch.from_numpy(g_idx).to(cuda_dev), bits)
    want = OP.pack_gptq(q, scale, zero, g_idx, bits)
    for k in ("qweight", "qzeros", "g_idx"):
        np.testing.assert_array_equal(got[k].cpu().numpy(), want[k], err_msg=k)
    np.testing.assert_array_equal(got["scales"].cpu().numpy(), want["scales"])
    np.testing.assert_array_equal(OP.unpack_rows(got["qweight"].cpu().numpy(), bits, in_f).T, q)
