// Block Walsh-Hadamard transform of the last dimension (the internal input rotation).
//
// Reference: mpq/rotation.py:404-441 (apply_block_hadamard / apply_right_block_hadamard[_inverse])
// with the torch butterfly of mpq/rotation.py:135-157 as the numerical definition: stages with
// stride h = 1, 2, 4, ... combine (x[p], x[p+h]) -> (x[p]+x[p+h], x[p]-x[p+h]), then divide by
// sqrt(had_dim) in float32.  Same stage order, so results are bit-identical to that definition.
//
// One CTA per (row, block); the block (had_dim <= 16384 floats) is staged in shared memory.
#include "common.cuh"

namespace mpq {

// mode 0: y = FWHT(x * signs) / sqrt(h)      (right rotation)
// mode 1: y = (FWHT(x) / sqrt(h)) * signs    (inverse right rotation)
__global__ void __launch_bounds__(1024) k_block_hadamard(const float* __restrict__ x, int64_t ldx, float* __restrict__ y,
                                                         int64_t ldy, int n, int had, const float* __restrict__ signs,
                                                         int mode) {
  extern __shared__ float sh[];
  const int row = blockIdx.y;
  const int c0 = blockIdx.x * had;
  const float* src = x + row * ldx + c0;
  for (int i = threadIdx.x; i < had; i += blockDim.x) {
    float v = src[i];
    if (mode == 0 && signs) v = fmul(v, signs[c0 + i]);
    sh[i] = v;
  }
  __syncthreads();
  for (int h = 1; h < had; h <<= 1) {
    for (int t = threadIdx.x; t < (had >> 1); t += blockDim.x) {
      const int p = ((t & ~(h - 1)) << 1) | (t & (h - 1));
      const float a = sh[p], b = sh[p + h];
      sh[p] = fadd(a, b);
      sh[p + h] = fsub(a, b);
    }
    __syncthreads();
  }
  const float s = sqrtf((float)had);
  float* dst = y + row * ldy + c0;
  for (int i = threadIdx.x; i < had; i += blockDim.x) {
    float v = fdiv(sh[i], s);
    if (mode == 1 && signs) v = fmul(v, signs[c0 + i]);
    dst[i] = v;
  }
}

}  // namespace mpq

using namespace mpq;

MPQ_API int mpq_block_hadamard(const float* x, int64_t ldx, float* y, int64_t ldy, int rows, int n, int had,
                               const float* signs, int mode, void* stream) {
  MPQ_CHECK_ARG(x && y, "mpq_block_hadamard: null pointer");
  MPQ_CHECK_ARG(had >= 1 && (had & (had - 1)) == 0 && had <= 16384, "mpq_block_hadamard: had_dim %d must be a power of two <= 16384", had);
  MPQ_CHECK_ARG(n % had == 0, "mpq_block_hadamard: width %d not divisible by had_dim %d", n, had);
  MPQ_CHECK_ARG(mode == 0 || mode == 1, "mpq_block_hadamard: mode must be 0 or 1");
  MPQ_CHECK_ARG(rows <= 65535, "mpq_block_hadamard: at most 65535 rows per call");
  if (rows == 0 || n == 0) return MPQ_OK;
  const size_t smem = (size_t)had * sizeof(float);
  {
    const int ast = smem_opt_in((const void*)k_block_hadamard, smem, "mpq_block_hadamard");
    if (ast) return ast;
  }
  dim3 grid(n / had, rows);
  int threads = had / 2 < 1024 ? (had / 2 > 32 ? had / 2 : 32) : 1024;
  k_block_hadamard<<<grid, threads, smem, (cudaStream_t)stream>>>(x, ldx, y, ldy, n, had, signs, mode);
  return launch_status("mpq_block_hadamard");
}
