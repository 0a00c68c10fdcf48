// Calibration-Hessian accumulation helpers: the transposing TF32 split that turns token-major
// activations X (T x n) into the K-major operands of the tensor-core SYRK (n x T), and the column sums
// of X (the QUIP# hook's running mean).  The SYRK itself is mpq_syrk_tc (gemm_tc.cu).
//
// Reference: the Hessian hooks the MPQ drivers consume (QUIP# utils.register_H_hook, finalised at
// mpq/quip_generic.py:906-918 and re-centred at :373-375; GPTQModel GPTQ.add_batch feeding
// mpq/adapters/gptqmodel.py:650-679) — both third-party, not part of the reference tree.
#include <cuda_bf16.h>
#include "common.cuh"

namespace mpq {

template <typename T>
__device__ __forceinline__ float load_f32(const T* p);
template <>
__device__ __forceinline__ float load_f32<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float load_f32<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// hi[j, t] = tf32_rna(X[t, j]), lo[j, t] = X[t, j] - hi[j, t]  (lo may be null); 32 x 32 tiles through shared
// memory so that both the reads (along j) and the writes (along t) are coalesced.
template <typename T>
__global__ void __launch_bounds__(256) k_split_tf32_t(const T* __restrict__ x, int64_t ldx, int tokens, int n,
                                                      float* __restrict__ hi, float* __restrict__ lo, int64_t ldo) {
  __shared__ float tile[32][33];
  const int t0 = blockIdx.x * 32, j0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  #pragma unroll
  for (int r = ty; r < 32; r += 8) {
    const int t = t0 + r, j = j0 + tx;
    tile[r][tx] = (t < tokens && j < n) ? load_f32<T>(x + (int64_t)t * ldx + j) : 0.f;
  }
  __syncthreads();
  #pragma unroll
  for (int r = ty; r < 32; r += 8) {
    const int j = j0 + r, t = t0 + tx;
    if (j < n && t < tokens) {
      const float v = tile[tx][r];
      uint32_t h;
      asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
      hi[(int64_t)j * ldo + t] = __uint_as_float(h);
      if (lo) lo[(int64_t)j * ldo + t] = fsub(v, __uint_as_float(h));
    }
  }
}

// out[j, t] = X[t, j] for bf16 activations (the K-major operand of the bf16 symmetric product), 32 x 32 tiles.
__global__ void __launch_bounds__(256) k_transpose_bf16(const __nv_bfloat16* __restrict__ x, int64_t ldx, int tokens,
                                                        int n, __nv_bfloat16* __restrict__ out, int64_t ldo) {
  __shared__ __nv_bfloat16 tile[32][34];
  const int t0 = blockIdx.x * 32, j0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  #pragma unroll
  for (int r = ty; r < 32; r += 8) {
    const int t = t0 + r, j = j0 + tx;
    tile[r][tx] = (t < tokens && j < n) ? x[(int64_t)t * ldx + j] : __float2bfloat16(0.f);
  }
  __syncthreads();
  #pragma unroll
  for (int r = ty; r < 32; r += 8) {
    const int j = j0 + r, t = t0 + tx;
    if (j < n && t < tokens) out[(int64_t)j * ldo + t] = tile[tx][r];
  }
}

// out[j] = beta * out[j] + alpha * sum_t X[t, j]: each CTA owns 32 columns; 8 row-partial sums per column
// combined in a fixed order.
template <typename T>
__global__ void __launch_bounds__(256) k_col_sum(const T* __restrict__ x, int64_t ldx, int tokens, int n, float alpha,
                                                 float beta, float* __restrict__ out) {
  __shared__ float part[8][32];
  const int j = blockIdx.x * 32 + (threadIdx.x & 31), ty = threadIdx.x >> 5;
  float acc = 0.f;
  if (j < n)
    for (int t = ty; t < tokens; t += 8) acc += load_f32<T>(x + (int64_t)t * ldx + j);
  part[ty][threadIdx.x & 31] = acc;
  __syncthreads();
  if (ty == 0 && j < n) {
    float s = 0.f;
    #pragma unroll
    for (int r = 0; r < 8; ++r) s += part[r][threadIdx.x];
    out[j] = (beta != 0.f ? beta * out[j] : 0.f) + alpha * s;
  }
}

}  // namespace mpq

using namespace mpq;

// dtype: 0 = float32, 1 = bfloat16 activations.  hi/lo: n x round_up(T, 4) (leading dimension ldo, a multiple of 4).
MPQ_API int mpq_split_tf32_t(const void* x, int dtype, int64_t ldx, int tokens, int n, float* hi, float* lo,
                             int64_t ldo, void* stream) {
  MPQ_CHECK_ARG(x && hi, "mpq_split_tf32_t: null pointer");
  MPQ_CHECK_ARG(dtype == 0 || dtype == 1, "mpq_split_tf32_t: dtype must be 0 (f32) or 1 (bf16)");
  MPQ_CHECK_ARG(tokens >= 0 && n >= 0 && ldx >= n && ldo >= tokens, "mpq_split_tf32_t: bad shape");
  if (tokens == 0 || n == 0) return MPQ_OK;
  dim3 grid((tokens + 31) / 32, (n + 31) / 32);
  if (dtype == 0)
    k_split_tf32_t<float><<<grid, 256, 0, (cudaStream_t)stream>>>((const float*)x, ldx, tokens, n, hi, lo, ldo);
  else
    k_split_tf32_t<__nv_bfloat16><<<grid, 256, 0, (cudaStream_t)stream>>>((const __nv_bfloat16*)x, ldx, tokens, n,
                                                                          hi, lo, ldo);
  return launch_status("mpq_split_tf32_t");
}

MPQ_API int mpq_transpose_bf16(const void* x, int64_t ldx, int tokens, int n, void* out, int64_t ldo, void* stream) {
  MPQ_CHECK_ARG(x && out, "mpq_transpose_bf16: null pointer");
  MPQ_CHECK_ARG(tokens >= 0 && n >= 0 && ldx >= n && ldo >= tokens, "mpq_transpose_bf16: bad shape");
  if (tokens == 0 || n == 0) return MPQ_OK;
  dim3 grid((tokens + 31) / 32, (n + 31) / 32);
  k_transpose_bf16<<<grid, 256, 0, (cudaStream_t)stream>>>((const __nv_bfloat16*)x, ldx, tokens, n,
                                                          (__nv_bfloat16*)out, ldo);
  return launch_status("mpq_transpose_bf16");
}

MPQ_API int mpq_col_sum(const void* x, int dtype, int64_t ldx, int tokens, int n, float alpha, float beta, float* out,
                        void* stream) {
  MPQ_CHECK_ARG(x && out, "mpq_col_sum: null pointer");
  MPQ_CHECK_ARG(dtype == 0 || dtype == 1, "mpq_col_sum: dtype must be 0 (f32) or 1 (bf16)");
  MPQ_CHECK_ARG(tokens >= 0 && n >= 0 && ldx >= n, "mpq_col_sum: bad shape");
  if (n == 0) return MPQ_OK;
  const int grid = (n + 31) / 32;
  if (dtype == 0)
    k_col_sum<float><<<grid, 256, 0, (cudaStream_t)stream>>>((const float*)x, ldx, tokens, n, alpha, beta, out);
  else
    k_col_sum<__nv_bfloat16><<<grid, 256, 0, (cudaStream_t)stream>>>((const __nv_bfloat16*)x, ldx, tokens, n, alpha,
                                                                      beta, out);
  return launch_status("mpq_col_sum");
}
