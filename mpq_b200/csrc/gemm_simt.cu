// FP32 CUDA-core GEMM:  C = alpha * A * op(B) + beta * C
//   A: M x K row-major (K-major).   op(B) = B^T with B: N x K row-major ("NT"), or
//                                   op(B) = B   with B: K x N row-major ("NN").
// Used for the small-K column-block updates of the scalar CD and as the exact-FP32 path of
// the rank-space products.  128x128 CTA tile, BK = 8, 256 threads, 8x8 outputs per thread,
// double-buffered shared memory.
#include "common.cuh"

namespace mpq {

template <bool B_IS_NT>
__global__ void __launch_bounds__(256) k_gemm_f32(int M, int N, int K, float alpha, const float* __restrict__ A,
                                                  int64_t lda, const float* __restrict__ B, int64_t ldb, float beta,
                                                  float* __restrict__ C, int64_t ldc) {
  constexpr int BM = 128, BN = 128, BK = 8;
  __shared__ float As[2][BK][BM + 4];
  __shared__ float Bs[2][BK][BN + 4];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int tr = tid / 16, tc = tid % 16;  // 16 x 16 thread grid, 8x8 each (strided by 16)
  float acc[8][8];
  #pragma unroll
  for (int i = 0; i < 8; ++i)
    #pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  // A tile: 128 rows x 8 k -> each thread loads 4 (row = tid/2, k = (tid%2)*4 + 0..3)
  auto load_tile = [&](int buf, int k0) {
    {
      const int r = tid >> 1, kk = (tid & 1) * 4;
      const int gm = m0 + r;
      #pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int gk = k0 + kk + t;
        As[buf][kk + t][r] = (gm < M && gk < K) ? A[(int64_t)gm * lda + gk] : 0.f;
      }
    }
    if (B_IS_NT) {
      const int r = tid >> 1, kk = (tid & 1) * 4;
      const int gn = n0 + r;
      #pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int gk = k0 + kk + t;
        Bs[buf][kk + t][r] = (gn < N && gk < K) ? B[(int64_t)gn * ldb + gk] : 0.f;
      }
    } else {
      // B: K x N row-major; 8 k-rows x 128 n -> each thread loads 4 consecutive n
      const int kk = tid >> 5, c = (tid & 31) * 4;
      const int gk = k0 + kk;
      #pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int gn = n0 + c + t;
        Bs[buf][kk][c + t] = (gn < N && gk < K) ? B[(int64_t)gk * ldb + gn] : 0.f;
      }
    }
  };

  int buf = 0;
  load_tile(0, 0);
  __syncthreads();
  for (int k0 = 0; k0 < K; k0 += BK) {
    if (k0 + BK < K) load_tile(buf ^ 1, k0 + BK);
    #pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[8], bv[8];
      #pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = As[buf][kk][tr + 16 * i];
      #pragma unroll
      for (int j = 0; j < 8; ++j) bv[j] = Bs[buf][kk][tc + 16 * j];
      #pragma unroll
      for (int i = 0; i < 8; ++i)
        #pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], bv[j], acc[i][j]);
    }
    __syncthreads();
    buf ^= 1;
  }
  #pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int gm = m0 + tr + 16 * i;
    if (gm >= M) continue;
    #pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + tc + 16 * j;
      if (gn >= N) continue;
      float* cp = C + (int64_t)gm * ldc + gn;
      *cp = beta == 0.f ? alpha * acc[i][j] : alpha * acc[i][j] + beta * (*cp);
    }
  }
}

}  // namespace mpq

using namespace mpq;

// layout: 0 = "NT" (B is N x K row-major), 1 = "NN" (B is K x N row-major)
MPQ_API int mpq_gemm_f32(int layout, int M, int N, int K, float alpha, const float* A, int64_t lda, const float* B,
                         int64_t ldb, float beta, float* C, int64_t ldc, void* stream) {
  MPQ_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "mpq_gemm_f32: negative shape");
  MPQ_CHECK_ARG(layout == 0 || layout == 1, "mpq_gemm_f32: layout must be 0 (NT) or 1 (NN)");
  if (M == 0 || N == 0) return MPQ_OK;  // empty tensors may carry null pointers
  MPQ_CHECK_ARG(A && B && C, "mpq_gemm_f32: null pointer");
  dim3 grid((N + 127) / 128, (M + 127) / 128);
  MPQ_CHECK_ARG(grid.y <= 65535, "mpq_gemm_f32: M too large");
  if (layout == 0)
    k_gemm_f32<true><<<grid, 256, 0, (cudaStream_t)stream>>>(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
  else
    k_gemm_f32<false><<<grid, 256, 0, (cudaStream_t)stream>>>(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
  return launch_status("mpq_gemm_f32");
}
