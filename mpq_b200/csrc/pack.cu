// GPTQ-format packing of integer codes (the export of the scalar path).
//
// GPTQ checkpoints store b-bit codes as a little-endian bit stream inside int32 words: code j of a packed
// line sits at stream bits [b j, b j + b), 32 codes fill b words (3-bit codes straddle word boundaries).
// qweight packs along the input dimension (word row w of column o holds codes of inputs 32w/b ...), qzeros
// along the output dimension.  Reference: the export after mpq/adapters/gptqmodel.py:650-1163 through
// GPTQModel's packer (patches/gptqmodel.patch:370-395), which is not vendored.
#include "common.cuh"

namespace mpq {

// out[w, c] (words along the packed axis) for codes src laid out with the packed axis strided by `sp` and the
// other axis by `so`: word w covers stream bits [32 w, 32 w + 32).  `offset` is subtracted from every code and the
// result masked to b bits (the v1 format stores zero - 1).
__global__ void k_pack_bits(const uint8_t* __restrict__ src, int64_t sp, int64_t so, int n_pack, int n_other, int bits,
                            int offset, int32_t* __restrict__ out, int64_t ld_out, int out_packed_rows) {
  const int64_t total = (int64_t)out_packed_rows * n_other;
  const uint32_t mask = (1u << bits) - 1u;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % n_other), w = (int)(i / n_other);
    const int64_t b0 = 32LL * w;
    const int j0 = (int)(b0 / bits), j1 = (int)((b0 + 31) / bits);
    uint64_t acc = 0;
    for (int j = j0; j <= j1; ++j) {
      if (j >= n_pack) break;
      const uint32_t v = (uint32_t)((int)src[(int64_t)j * sp + (int64_t)c * so] - offset) & mask;
      const int64_t pos = (int64_t)j * bits - b0;  // may be negative for the code straddling into this word
      if (pos >= 0) acc |= (uint64_t)v << pos;
      else acc |= (uint64_t)(v >> (-pos));
    }
    out[(int64_t)w * ld_out + c] = (int32_t)(uint32_t)(acc & 0xffffffffull);
  }
}

}  // namespace mpq

using namespace mpq;

// Pack codes along one axis: src element (p, o) at src[p * sp + o * so] (p: packed axis, n_pack codes; o: other axis,
// n_other), output (n_pack * bits / 32) x n_other int32 words (leading dimension ld_out).  n_pack * bits must be a
// multiple of 32.  bits in {2, 3, 4, 8}.
MPQ_API int mpq_pack_bits(const uint8_t* src, int64_t sp, int64_t so, int n_pack, int n_other, int bits, int offset,
                          int32_t* out, int64_t ld_out, void* stream) {
  MPQ_CHECK_ARG(src && out, "mpq_pack_bits: null pointer");
  MPQ_CHECK_ARG(bits == 2 || bits == 3 || bits == 4 || bits == 8, "mpq_pack_bits: bits must be 2, 3, 4 or 8");
  MPQ_CHECK_ARG(n_pack >= 0 && n_other >= 0 && ((int64_t)n_pack * bits) % 32 == 0,
                "mpq_pack_bits: n_pack * bits must be a multiple of 32");
  MPQ_CHECK_ARG(ld_out >= n_other, "mpq_pack_bits: ld_out < n_other");
  const int rows = (int)((int64_t)n_pack * bits / 32);
  const int64_t total = (int64_t)rows * n_other;
  if (total == 0) return MPQ_OK;
  int64_t g = (total + 255) / 256;
  if (g > 148 * 32) g = 148 * 32;
  k_pack_bits<<<(int)g, 256, 0, (cudaStream_t)stream>>>(src, sp, so, n_pack, n_other, bits, offset, out, ld_out, rows);
  return launch_status("mpq_pack_bits");
}
