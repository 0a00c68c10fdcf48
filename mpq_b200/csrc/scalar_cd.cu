// Scalar greedy coordinate descent over the grouped-scalar grid (the uniform polish).
//
// Reference: mpq/polish/triton_scalar_cd.py:164-307 (uniform_scalar_diag_greedy_cd) and its
// persistent Triton sweep :28-110.  The reference streams the whole B x n right-hand side once
// per column (a rank-1 update against the raw Hessian row).  Here each sweep visits the greedy
// order in column blocks J of up to 128 columns:
//   1. k_cd_block: per row (one warp), the 128 sequential column decisions run in registers
//      against H[J, J] held in shared memory; the accepted steps delta[b, k] are written out.
//   2. one GEMM  rhs[:, :] -= delta(B x |J|) * H[J, :]  applies the block's updates to all
//      columns (the deferred "lazy" form of the reference's per-column rank-1 updates).
// Within a block the decisions see exactly the updates the reference applies; only the
// floating-point summation order of earlier blocks' updates differs.
#include "common.cuh"

namespace mpq {

constexpr int kCdBlock = 128;

// diag[j] = max(sum_r Vs[j, r]^2, 1e-12); diag_inv = 1 / diag  (triton_scalar_cd.py:198-199)
__global__ void k_cd_diag(const float* __restrict__ Vs, int n, int R, int64_t ld, float* __restrict__ diag,
                          float* __restrict__ diag_inv) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= n) return;
  float acc = 0.f;
  for (int r = lane; r < R; r += 32) {
    const float v = Vs[warp * ld + r];
    acc += v * v;
  }
  acc = warp_sum(acc);
  if (lane == 0) {
    const float d = fmaxf(acc, 1e-12f);
    diag[warp] = d;
    diag_inv[warp] = fdiv(1.f, d);
  }
}

// gain[j] = sum_b (rhs[b,j]^2 * diag_inv[j]) / B  (triton_scalar_cd.py:242); fixed row order.
__global__ void k_cd_gain(const float* __restrict__ rhs, int B, int n, int64_t ld, const float* __restrict__ diag_inv,
                          float* __restrict__ gain) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  const float di = diag_inv[j];
  float acc = 0.f;
  for (int b = 0; b < B; ++b) {
    const float v = rhs[b * ld + j];
    acc = fadd(acc, fmul(fmul(v, v), di));
  }
  gain[j] = fdiv(acc, (float)(B > 0 ? B : 1));
}

// Single-CTA bitonic argsort, descending by key, ties by ascending index.  NaN keys sort last.
__global__ void __launch_bounds__(1024) k_argsort_desc(const float* __restrict__ key, int n, int npow2,
                                                       int* __restrict__ order) {
  extern __shared__ unsigned char smem_raw[];
  float* k = reinterpret_cast<float*>(smem_raw);
  int* v = reinterpret_cast<int*>(k + npow2);
  for (int i = threadIdx.x; i < npow2; i += blockDim.x) {
    float x = i < n ? key[i] : -INFINITY;
    if (isnan(x)) x = -INFINITY;
    k[i] = x;
    v[i] = i < n ? i : 0x7fffffff;
  }
  __syncthreads();
  for (int size = 2; size <= npow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < npow2; i += blockDim.x) {
        const int p = i ^ stride;
        if (p > i) {
          const bool up = (i & size) == 0;  // "up" segments sort in the target (descending) order
          const float ki = k[i], kp = k[p];
          const int vi = v[i], vp = v[p];
          const bool p_first = (kp > ki) || (kp == ki && vp < vi);  // p should precede i
          if (p_first == up) {
            k[i] = kp; k[p] = ki;
            v[i] = vp; v[p] = vi;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) order[i] = v[i];
}

// HJT[j, k] = H[J[k], j] (n x 128, transposed through shared-memory tiles so both the read of
// H's rows and the write are coalesced) and Hsub[k, l] = H[J[k], J[l]] for J = order[c0 : c0 + K].
__global__ void __launch_bounds__(256) k_cd_gather(const float* __restrict__ H, int64_t ldh, int n,
                                                   const int* __restrict__ order, int c0, int K,
                                                   float* __restrict__ HJT, float* __restrict__ Hsub) {
  __shared__ float tile[32][33];
  const int j0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  for (int kk = ty; kk < 32; kk += 8) {
    const int k = k0 + kk, j = j0 + tx;
    float v = 0.f;
    if (k < K && j < n) v = H[(int64_t)order[c0 + k] * ldh + j];
    tile[kk][tx] = v;
  }
  __syncthreads();
  for (int jj = ty; jj < 32; jj += 8) {
    const int j = j0 + jj, k = k0 + tx;
    if (j < n) HJT[(int64_t)j * kCdBlock + k] = tile[tx][jj];
  }
  if (blockIdx.x == 0) {
    for (int i = threadIdx.x; i < 32 * kCdBlock; i += blockDim.x) {
      const int k = k0 + i / kCdBlock, l = i % kCdBlock;
      if (k < kCdBlock) Hsub[k * kCdBlock + l] = (k < K && l < K) ? H[(int64_t)order[c0 + k] * ldh + order[c0 + l]] : 0.f;
    }
  }
}

struct CdArgs {
  float* x; int64_t ldx;
  const float* rhs; int64_t ldr;
  const float* scale; const float* zero; int64_t ld_p; int gshift;
  // top-k candidate mode: per (row, column) kc <= 32 candidate values (and their grid levels), row stride ld_cand;
  // the chosen level of an accepted step is written to qout
  const float* cand; const int* cand_q; int64_t ld_cand; int kc;
  int* qout; int64_t ldq;
  const float* diag; const float* diag_inv;
  const int* order; int c0; int K;
  const float* Hsub;
  float* res;        // (B) residual norm, read and written
  float* delta;      // (B x 128) accepted steps of this block
  int* accepted;     // (1) accepted-update counter
  int B; int maxq; float accept_tol;
};

// One warp per row: the sequential decisions of one column block (triton_scalar_cd.py:59-107).  TOPK: the
// candidate of a column is the nearest of its precomputed top-k values to the target (first minimum of the
// squared distance, mpq/polish/block_cd.py:657-685) instead of the rounded grid level.
template <bool TOPK>
__global__ void __launch_bounds__(256) k_cd_block(CdArgs a) {
  extern __shared__ float Hs[];  // kCdBlock x kCdBlock
  __shared__ float s_diag[kCdBlock], s_dinv[kCdBlock];
  __shared__ int s_col[kCdBlock];
  for (int i = threadIdx.x; i < kCdBlock * kCdBlock; i += blockDim.x) Hs[i] = a.Hsub[i];
  for (int i = threadIdx.x; i < kCdBlock; i += blockDim.x) {
    const int col = i < a.K ? a.order[a.c0 + i] : 0;
    s_col[i] = col;
    s_diag[i] = i < a.K ? a.diag[col] : 1.f;
    s_dinv[i] = i < a.K ? a.diag_inv[col] : 1.f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (b >= a.B) return;
  float rhs[4], xv[4], sv[4], zv[4], dl[4];
  #pragma unroll
  for (int t = 0; t < 4; ++t) {
    const int l = t * 32 + lane;
    dl[t] = 0.f;
    if (l < a.K) {
      const int col = s_col[l];
      rhs[t] = a.rhs[b * a.ldr + col];
      xv[t] = a.x[b * a.ldx + col];
      if constexpr (TOPK) {
        sv[t] = 1.f; zv[t] = 0.f;
      } else {
        sv[t] = a.scale[b * a.ld_p + (col >> a.gshift)];
        zv[t] = a.zero[b * a.ld_p + (col >> a.gshift)];
      }
    } else {
      rhs[t] = 0.f; xv[t] = 0.f; sv[t] = 1.f; zv[t] = 0.f;
    }
  }
  float res = a.res[b];
  const float tol1 = 1.f + a.accept_tol;
  int acc_count = 0;
  const float* crow = TOPK ? a.cand + (int64_t)b * a.ld_cand : nullptr;
  // this lane's candidate of the next four columns (loads issued four decisions ahead)
  float c0 = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
  if constexpr (TOPK) {
    if (lane < a.kc) {
      c0 = crow[(int64_t)s_col[0] * a.kc + lane];
      if (a.K > 1) c1 = crow[(int64_t)s_col[1] * a.kc + lane];
      if (a.K > 2) c2 = crow[(int64_t)s_col[2] * a.kc + lane];
      if (a.K > 3) c3 = crow[(int64_t)s_col[3] * a.kc + lane];
    }
  }
  #pragma unroll
  for (int t = 0; t < 4; ++t) {
    for (int lk = 0; lk < 32; ++lk) {
      const int k = t * 32 + lk;
      if (k >= a.K) break;
      const float rk = __shfl_sync(0xffffffffu, rhs[t], lk);
      const float xk = __shfl_sync(0xffffffffu, xv[t], lk);
      const float target = fadd(xk, fmul(rk, s_dinv[k]));
      float xq;
      int pick = 0;
      if constexpr (TOPK) {
        const float cv = c0;
        c0 = c1;
        c1 = c2;
        c2 = c3;
        if (k + 4 < a.K && lane < a.kc) c3 = crow[(int64_t)s_col[k + 4] * a.kc + lane];
        float key = INFINITY;
        int ci = 0x7fffffff;
        if (lane < a.kc) {
          const float dd = fsub(cv, target);
          key = fmul(dd, dd);
          if (key != key) key = INFINITY;
          ci = lane;
        }
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) {  // first minimum: smaller distance, then smaller candidate index
          const float ok = __shfl_xor_sync(0xffffffffu, key, o);
          const int oc = __shfl_xor_sync(0xffffffffu, ci, o);
          if (oc != 0x7fffffff && (ci == 0x7fffffff || ok < key || (ok == key && oc < ci))) { key = ok; ci = oc; }
        }
        pick = ci;
        xq = __shfl_sync(0xffffffffu, cv, pick);
      } else {
        const float sk = fmaxf(__shfl_sync(0xffffffffu, sv[t], lk), 1e-12f);
        const float zk = __shfl_sync(0xffffffffu, zv[t], lk);
        float qf = rintf(fadd(fdiv(target, sk), zk));
        qf = fminf(fmaxf(qf, 0.f), (float)a.maxq);
        xq = fmul(sk, fsub(qf, zk));
      }
      const float d = fsub(xq, xk);
      const float cand = fmaxf(fsub(fadd(res, fmul(fmul(d, d), s_diag[k])), fmul(fmul(2.f, rk), d)), 0.f);
      if (fadd(cand, 1e-12f) < fmul(res, tol1)) {
        res = cand;
        ++acc_count;
        if (lane == lk) { xv[t] = xq; dl[t] = d; }
        if constexpr (TOPK) {
          if (lane == 0 && a.qout && a.cand_q)
            a.qout[b * a.ldq + s_col[k]] = a.cand_q[(int64_t)b * a.ld_cand + (int64_t)s_col[k] * a.kc + pick];
        }
        const float* hrow = Hs + k * kCdBlock;
        #pragma unroll
        for (int u = 0; u < 4; ++u) rhs[u] = fsub(rhs[u], fmul(d, hrow[u * 32 + lane]));
      }
    }
  }
  #pragma unroll
  for (int t = 0; t < 4; ++t) {
    const int l = t * 32 + lane;
    if (l < a.K) a.x[b * a.ldx + s_col[l]] = xv[t];
    a.delta[(int64_t)b * kCdBlock + l] = dl[t];
  }
  if (lane == 0) {
    a.res[b] = res;
    if (acc_count) atomicAdd(a.accepted, acc_count);
  }
}

}  // namespace mpq

using namespace mpq;

MPQ_API int mpq_cd_diag(const float* Vs, int n, int R, int64_t ld, float* diag, float* diag_inv, void* stream) {
  MPQ_CHECK_ARG(Vs && diag && diag_inv, "mpq_cd_diag: null pointer");
  if (n == 0) return MPQ_OK;
  k_cd_diag<<<(n * 32 + 255) / 256, 256, 0, (cudaStream_t)stream>>>(Vs, n, R, ld, diag, diag_inv);
  return launch_status("mpq_cd_diag");
}

MPQ_API int mpq_cd_gain(const float* rhs, int B, int n, int64_t ld, const float* diag_inv, float* gain, void* stream) {
  MPQ_CHECK_ARG(rhs && diag_inv && gain, "mpq_cd_gain: null pointer");
  if (n == 0) return MPQ_OK;
  k_cd_gain<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(rhs, B, n, ld, diag_inv, gain);
  return launch_status("mpq_cd_gain");
}

MPQ_API int mpq_argsort_desc(const float* key, int n, int* order, void* stream) {
  MPQ_CHECK_ARG(key && order, "mpq_argsort_desc: null pointer");
  MPQ_CHECK_ARG(n >= 0 && n <= 16384, "mpq_argsort_desc: n must be in [0, 16384], got %d", n);
  if (n == 0) return MPQ_OK;
  int np2 = 1;
  while (np2 < n) np2 <<= 1;
  if (np2 < 2) np2 = 2;
  const size_t smem = (size_t)np2 * 8;
  {
    const int ast = smem_opt_in((const void*)k_argsort_desc, smem, "mpq_argsort_desc");
    if (ast) return ast;
  }
  k_argsort_desc<<<1, 1024, smem, (cudaStream_t)stream>>>(key, n, np2, order);
  return launch_status("mpq_argsort_desc");
}

MPQ_API int mpq_cd_gather(const float* H, int64_t ldh, int n, const int* order, int c0, int K, float* HJT, float* Hsub,
                          void* stream) {
  MPQ_CHECK_ARG(H && order && HJT && Hsub, "mpq_cd_gather: null pointer");
  MPQ_CHECK_ARG(K >= 1 && K <= kCdBlock && c0 >= 0 && c0 + K <= n, "mpq_cd_gather: bad block [%d, %d)", c0, c0 + K);
  dim3 grid((n + 31) / 32, kCdBlock / 32);
  k_cd_gather<<<grid, 256, 0, (cudaStream_t)stream>>>(H, ldh, n, order, c0, K, HJT, Hsub);
  return launch_status("mpq_cd_gather");
}

MPQ_API int mpq_cd_block(float* x, int64_t ldx, const float* rhs, int64_t ldr, const float* scale, const float* zero,
                         int64_t ld_p, int gshift, const float* diag, const float* diag_inv, const int* order, int c0,
                         int K, const float* Hsub, float* res, float* delta, int* accepted, int B, int maxq,
                         float accept_tol, void* stream) {
  MPQ_CHECK_ARG(x && rhs && scale && zero && diag && diag_inv && order && Hsub && res && delta && accepted,
                "mpq_cd_block: null pointer");
  MPQ_CHECK_ARG(K >= 1 && K <= kCdBlock, "mpq_cd_block: K must be in [1, %d]", kCdBlock);
  MPQ_CHECK_ARG(maxq >= 1 && maxq <= 255, "mpq_cd_block: bad maxq");
  if (B == 0) return MPQ_OK;
  CdArgs a{x, ldx, rhs, ldr, scale, zero, ld_p, gshift, nullptr, nullptr, 0, 0, nullptr, 0, diag, diag_inv, order, c0,
           K, Hsub, res, delta, accepted, B, maxq, accept_tol};
  const size_t smem = (size_t)kCdBlock * kCdBlock * sizeof(float);
  {
    const int ast = smem_opt_in((const void*)k_cd_block<false>, smem, "mpq_cd_block");
    if (ast) return ast;
  }
  k_cd_block<false><<<(B + 7) / 8, 256, smem, (cudaStream_t)stream>>>(a);
  return launch_status("mpq_cd_block");
}

MPQ_API int mpq_cd_block_topk(float* x, int64_t ldx, const float* rhs, int64_t ldr, const float* cand,
                              const int* cand_q, int64_t ld_cand, int kc, int* qout, int64_t ldq, const float* diag,
                              const float* diag_inv, const int* order, int c0, int K, const float* Hsub, float* res,
                              float* delta, int* accepted, int B, float accept_tol, void* stream) {
  MPQ_CHECK_ARG(K >= 1 && K <= kCdBlock, "mpq_cd_block_topk: K must be in [1, %d]", kCdBlock);
  MPQ_CHECK_ARG(kc >= 1 && kc <= 32, "mpq_cd_block_topk: kc must be in [1, 32]");
  if (B == 0) return MPQ_OK;
  MPQ_CHECK_ARG(x && rhs && cand && diag && diag_inv && order && Hsub && res && delta && accepted,
                "mpq_cd_block_topk: null pointer");
  CdArgs a{x, ldx, rhs, ldr, nullptr, nullptr, 0, 0, cand, cand_q, ld_cand, kc, qout, ldq, diag, diag_inv, order, c0,
           K, Hsub, res, delta, accepted, B, 1, accept_tol};
  const size_t smem = (size_t)kCdBlock * kCdBlock * sizeof(float);
  {
    const int ast = smem_opt_in((const void*)k_cd_block<true>, smem, "mpq_cd_block_topk");
    if (ast) return ast;
  }
  k_cd_block<true><<<(B + 7) / 8, 256, smem, (cudaStream_t)stream>>>(a);
  return launch_status("mpq_cd_block_topk");
}
