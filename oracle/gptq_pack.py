"""GPTQ v1 packing restated word by word (TEST INFRASTRUCTURE ONLY; the format of GPTQModel's packer, which is not
vendored in the reference tree: parity against GPTQModel itself is unpinned)."""
import numpy as np


def pack_rows(intw, bits):
    """intw (n_pack, n_other) non-negative codes < 2**bits -> (n_pack * bits // 32, n_other) uint32 words.  Codes are
    written in order into a little-endian bit stream per column; 32 // bits codes per word for 2/4/8 bits, and for
    3 bits the 10-codes-per-word pattern with the 11th and 22nd codes split across words."""
    intw = intw.astype(np.uint64)
    n_pack, n_other = intw.shape
    out = np.zeros((n_pack * bits // 32, n_other), np.uint64)
    if bits in (2, 4, 8):
        per = 32 // bits
        for row in range(out.shape[0]):
            for k in range(per):
                out[row] |= intw[row * per + k] << np.uint64(bits * k)
    elif bits == 3:
        i = 0
        row = 0
        while row < out.shape[0]:
            for k in range(10):
                out[row] |= intw[i + k] << np.uint64(3 * k)
            i += 10
            out[row] |= (intw[i] << np.uint64(30)) & np.uint64(0xFFFFFFFF)
            row += 1
            out[row] |= (intw[i] >> np.uint64(2)) & np.uint64(1)
            i += 1
            for k in range(10):
                out[row] |= intw[i + k] << np.uint64(3 * k + 1)
            i += 10
            out[row] |= (intw[i] << np.uint64(31)) & np.uint64(0xFFFFFFFF)
            row += 1
            out[row] |= (intw[i] >> np.uint64(1)) & np.uint64(3)
            i += 1
            for k in range(10):
                out[row] |= intw[i + k] << np.uint64(3 * k + 2)
            i += 10
            row += 1
    else:
        raise ValueError(bits)
    return (out & np.uint64(0xFFFFFFFF)).astype(np.uint32)


def pack_gptq(q_int, scale, zero, g_idx, bits):
    """q_int (out, in), scale / zero (out, groups) -> qweight, qzeros, scales, g_idx (numpy)."""
    mask = (1 << bits) - 1
    qweight = pack_rows(q_int.T.astype(np.int64), bits).view(np.int32)
    z = ((np.rint(zero).astype(np.int64) - 1) & mask)  # (out, groups)
    qzeros = pack_rows(z, bits).T.copy().view(np.int32)
    return {"qweight": qweight, "qzeros": qzeros, "scales": scale.T.astype(np.float16), "g_idx": g_idx.astype(np.int32)}


def unpack_rows(words, bits, n_pack):
    """Inverse of pack_rows through the bit stream."""
    w = words.view(np.uint32).astype(np.uint64)
    n_other = w.shape[1]
    out = np.zeros((n_pack, n_other), np.int64)
    for j in range(n_pack):
        b = j * bits
        r, s = divmod(b, 32)
        v = w[r] >> np.uint64(s)
        if s + bits > 32:
            v |= w[r + 1] << np.uint64(32 - s)
        out[j] = (v & np.uint64((1 << bits) - 1)).astype(np.int64)
    return out
