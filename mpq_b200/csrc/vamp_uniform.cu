// VAMP message updates in rank space: the per-row scalar algebra and the fused element-wise
// passes around the three rank-space GEMMs of each iteration.
//
// Reference: mpq/solver.py:553-699 (the scalar VAMP loop; the E8P12 loop :961-1122 shares
// the algebra), mpq/linear.py:10-82 (linear_mmse_exact, em_update_obs_precision_rankspace),
// mpq/linear.py:85-94 (vamp_rankspace_error), mpq/utils.py:24-57 (damping, validity masks).
//
// Row state lives in small device vectors of length B.  Flags that steer the host control
// flow (retry / skip / best-iterate) are counted with integer atomics (order independent).
#include "common.cuh"
#include "vamp_rows.cuh"

namespace mpq {

__global__ void __launch_bounds__(kRowThreads) k_vamp_rows(RowState st, const float* __restrict__ S, int B, int n,
                                                          int n_var, int R, float obs, float damping, int final_retry,
                                                          const VampCtl* __restrict__ ctl, RoundCtl rc) {
  __shared__ float red[2][kRowThreads / 32];
  const int b = blockIdx.x;
  if (b >= B) return;
  vamp_row_stage<false>(st, S, b, B, n, n_var, R, obs, damping, final_retry, ctl, rc, red);
}

// gamma retry (mpq/solver.py:593-596): divide/multiply the work precision of invalid rows.
__global__ void k_gamma_retry(float* gamma1_work, const float* alpha1_raw_src_var, const float* var_rowsum, int B,
                              int n, float factor) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  float g = gamma1_work[b];
  const float a = fmul(g, fdiv(var_rowsum[b], (float)n));
  if (a <= kAlphaEps) g = fdiv(g, factor);
  if (a >= kOneMinusAlphaEps) g = fmul(g, factor);
  gamma1_work[b] = fmaxf(g, 1e-12f);
}

// r2 = damp(r2_prev, (eta1*x1 - gamma1w*r1)/gamma2_new)          (mpq/solver.py:605-612)
__global__ void k_vamp_r2(const float* __restrict__ x1, const float* __restrict__ r1, const float* __restrict__ r2_prev,
                          float* __restrict__ r2, const float* __restrict__ eta1, const float* __restrict__ g1w,
                          const float* __restrict__ g2n, int B, int n, int64_t ld, float damping,
                          const VampCtl* __restrict__ ctl) {
  if (ctl) {
    if (ctl->skip) return;
    if (!ctl->have_prev) r2_prev = nullptr;
  }
  const int64_t total = (int64_t)B * n;
  const float omd = (float)(1.0 - (double)damping);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / n), j = (int)(i % n);
    const int64_t o = b * ld + j;
    const float rn = fdiv(fsub(fmul(eta1[b], x1[o]), fmul(g1w[b], r1[o])), g2n[b]);
    r2[o] = r2_prev ? fadd(fmul(omd, r2_prev[o]), fmul(damping, rn)) : rn;
  }
}

// Linear-module epilogue over P = r2 @ V  (mpq/linear.py:46-55):
//   rb = Y_u - P*s;  u = rb * (obs*s/denom);  rowsum((rb*gamma2/denom)^2)
// One CTA per row; the row sum is reduced in a fixed order.
__global__ void __launch_bounds__(256) k_linear_epilogue(const float* __restrict__ P, const float* __restrict__ Y_u,
                                                         const float* __restrict__ S, const float* __restrict__ g2,
                                                         float obs, int R, int64_t ld, float* __restrict__ u,
                                                         float* __restrict__ resid_rowsum,
                                                         const VampCtl* __restrict__ ctl) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  if (ctl) {
    if (ctl->skip) return;
    obs = (float)ctl->obs;
  }
  const float gb = g2[b];
  float acc = 0.f;
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    const float s = S[r];
    const float den = fadd(fmul(obs, fmul(s, s)), gb);
    const float rb = fsub(Y_u[b * ld + r], fmul(P[b * ld + r], s));
    const float coeff = fdiv(fmul(obs, s), den);
    u[b * ld + r] = fmul(rb, coeff);
    const float ra = fmul(rb, fdiv(gb, den));
    acc += ra * ra;
  }
  const float t = block_sum(acc, red);
  if (threadIdx.x == 0) resid_rowsum[b] = t;
}

// r1 update from D = u @ V^T  (mpq/linear.py:51-52, mpq/solver.py:645-653):
//   x2 = r2 + D;  r1_new = (eta2*x2 - gamma2*r2)/gamma1_new;  r1 = (1-d) r1 + d r1_new
// ctl (optional): nothing happens on a skipped iteration; r2_keep (optional) receives a copy of r2 (the next
// iteration's r2_prev).
__global__ void k_vamp_r1(const float* __restrict__ D, const float* __restrict__ r2, float* __restrict__ r1,
                          const float* __restrict__ eta2, const float* __restrict__ g2, const float* __restrict__ g1n,
                          int B, int n, int64_t ld, float damping, const VampCtl* __restrict__ ctl,
                          float* __restrict__ r2_keep) {
  if (ctl && ctl->skip) return;
  const int64_t total = (int64_t)B * n;
  const float omd = (float)(1.0 - (double)damping);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / n), j = (int)(i % n);
    const int64_t o = b * ld + j;
    if (r2_keep) r2_keep[o] = r2[o];
    const float x2 = fadd(r2[o], D[o]);
    const float rn = fdiv(fsub(fmul(eta2[b], x2), fmul(g2[b], r2[o])), g1n[b]);
    r1[o] = damping >= 1.f ? rn : fadd(fmul(omd, r1[o]), fmul(damping, rn));
  }
}

// ---- fused forms for the device-resident loop: the products' split-K partial planes are added by the consumer (in
// plane order, as the split-K reduction does), and the producers of the next product's A operand write it already
// split (row-scaled fp16 halves, as mpq_split_f16) ----

__device__ __forceinline__ float sum_parts(const float* __restrict__ parts, int splits, int64_t plane, int64_t o) {
  float acc = parts[o];
  for (int s = 1; s < splits; ++s) acc += parts[(int64_t)s * plane + o];
  return acc;
}

// r2 (as k_vamp_r2) plus its row-scaled fp16 split; one CTA per row: pass 1 writes r2 and finds the row maximum,
// pass 2 re-reads the row (this thread's own writes) and stores the halves.
__global__ void __launch_bounds__(256) k_vamp_r2_split(const float* __restrict__ x1, const float* __restrict__ r1,
                                                       const float* __restrict__ r2_prev, float* __restrict__ r2,
                                                       const float* __restrict__ eta1, const float* __restrict__ g1w,
                                                       const float* __restrict__ g2n, int n, int64_t ld, float damping,
                                                       unsigned short* __restrict__ hi, unsigned short* __restrict__ lo,
                                                       int64_t ldo, float* __restrict__ inv_scale,
                                                       const VampCtl* __restrict__ ctl) {
  __shared__ float red[32];
  if (ctl) {
    if (ctl->skip) return;
    if (!ctl->have_prev) r2_prev = nullptr;
  }
  const int b = blockIdx.x;
  const float omd = (float)(1.0 - (double)damping);
  const float e1 = eta1[b], gw = g1w[b], gn = g2n[b];
  float mx = 0.f;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const int64_t o = b * ld + j;
    const float rn = fdiv(fsub(fmul(e1, x1[o]), fmul(gw, r1[o])), gn);
    const float v = r2_prev ? fadd(fmul(omd, r2_prev[o]), fmul(damping, rn)) : rn;
    r2[o] = v;
    mx = fmaxf(mx, fabsf(v));
  }
  __shared__ float s_scale[2];
  const float m = block_max(mx, red);
  if (threadIdx.x == 0) {
    split_f16_scale(m, s_scale[0], s_scale[1]);
    inv_scale[b] = s_scale[1];
  }
  __syncthreads();
  const float sc = s_scale[0];
  for (int j = threadIdx.x; j < n; j += blockDim.x)
    split_f16_store(r2[b * ld + j], sc, hi + b * ldo + j, lo + b * ldo + j);
}

// Linear-module epilogue (as k_linear_epilogue) over P given as split-K partial planes, with u written as its
// row-scaled fp16 split (u itself goes to `u` as scratch for the second pass).
__global__ void __launch_bounds__(256) k_linear_epilogue_parts(const float* __restrict__ parts, int splits,
                                                               int64_t plane, const float* __restrict__ Y_u,
                                                               int64_t ldy, const float* __restrict__ S,
                                                               const float* __restrict__ g2, int R,
                                                               float* __restrict__ u, unsigned short* __restrict__ hi,
                                                               unsigned short* __restrict__ lo, int64_t ldo,
                                                               float* __restrict__ inv_scale,
                                                               float* __restrict__ resid_rowsum,
                                                               const VampCtl* __restrict__ ctl) {
  __shared__ float red[32];
  if (ctl && ctl->skip) return;
  const float obs = (float)ctl->obs;
  const int b = blockIdx.x;
  const float gb = g2[b];
  float acc = 0.f, mx = 0.f;
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    const float s = S[r];
    const float den = fadd(fmul(obs, fmul(s, s)), gb);
    const float P = sum_parts(parts, splits, plane, (int64_t)b * R + r);
    const float rb = fsub(Y_u[b * ldy + r], fmul(P, s));
    const float coeff = fdiv(fmul(obs, s), den);
    const float uv = fmul(rb, coeff);
    u[(int64_t)b * R + r] = uv;
    mx = fmaxf(mx, fabsf(uv));
    const float ra = fmul(rb, fdiv(gb, den));
    acc += ra * ra;
  }
  const float t = block_sum(acc, red);
  if (threadIdx.x == 0) resid_rowsum[b] = t;
  __shared__ float s_scale[2];
  const float m = block_max(mx, red);
  if (threadIdx.x == 0) {
    split_f16_scale(m, s_scale[0], s_scale[1]);
    inv_scale[b] = s_scale[1];
  }
  __syncthreads();
  const float sc = s_scale[0];
  for (int r = threadIdx.x; r < R; r += blockDim.x)
    split_f16_store(u[(int64_t)b * R + r], sc, hi + b * ldo + r, lo + b * ldo + r);
}

// r1 update (as k_vamp_r1) with D given as split-K partial planes (B x n each).
__global__ void k_vamp_r1_parts(const float* __restrict__ parts, int splits, int64_t plane,
                                const float* __restrict__ r2, float* __restrict__ r1, const float* __restrict__ eta2,
                                const float* __restrict__ g2, const float* __restrict__ g1n, int B, int n, int64_t ld,
                                float damping, const VampCtl* __restrict__ ctl, float* __restrict__ r2_keep) {
  if (ctl && ctl->skip) return;
  const int64_t total = (int64_t)B * n;
  const float omd = (float)(1.0 - (double)damping);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / n), j = (int)(i % n);
    const int64_t o = b * ld + j;
    if (r2_keep) r2_keep[o] = r2[o];
    const float x2 = fadd(r2[o], sum_parts(parts, splits, plane, (int64_t)b * n + j));
    const float rn = fdiv(fsub(fmul(eta2[b], x2), fmul(g2[b], r2[o])), g1n[b]);
    r1[o] = damping >= 1.f ? rn : fadd(fmul(omd, r1[o]), fmul(damping, rn));
  }
}

// rowsum((Y - C)^2) (vamp_rankspace_error), optionally rowsum((Y - C)^2) + add[b]; one CTA per row.
__global__ void __launch_bounds__(256) k_row_sqerr(const float* __restrict__ Y, const float* __restrict__ C, int R,
                                                   int64_t ldy, int64_t ldc, float* __restrict__ out) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  float acc = 0.f;
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    const float d = fsub(Y[b * ldy + r], C[b * ldc + r]);
    acc += d * d;
  }
  const float t = block_sum(acc, red);
  if (threadIdx.x == 0) out[b] = t;
}

// residual = Y - C (in place into C), and rowsum(residual^2)
__global__ void __launch_bounds__(256) k_residual(const float* __restrict__ Y, float* __restrict__ C, int R,
                                                  int64_t ld, float* __restrict__ rowsum) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  float acc = 0.f;
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    const float d = fsub(Y[b * ld + r], C[b * ld + r]);
    C[b * ld + r] = d;
    acc += d * d;
  }
  const float t = block_sum(acc, red);
  if (threadIdx.x == 0 && rowsum) rowsum[b] = t;
}

// mean over B of (a[b] + (c ? c[b] : 0)) in a fixed order (single CTA).
__global__ void __launch_bounds__(1024) k_mean_rows(const float* __restrict__ a, const float* __restrict__ c, int B,
                                                    float* __restrict__ out) {
  __shared__ float red[32];
  float acc = 0.f;
  for (int b = threadIdx.x; b < B; b += blockDim.x) acc += c ? fadd(a[b], c[b]) : a[b];
  const float t = block_sum(acc, red);
  if (threadIdx.x == 0) *out = B > 0 ? t / (float)B : 0.f;
}

// Row-wise selection:  dst[b,:] = mask[b] ? src[b,:] : dst[b,:]  for f32 and u8 payloads, and
// the polish merge mask improve = err_after + 1e-12 < err_before (mpq/solver.py:749-754).
__global__ void k_polish_merge(const float* __restrict__ err_after, float* __restrict__ err_final,
                               const float* __restrict__ err_before, const float* __restrict__ x_src,
                               float* __restrict__ x_dst, const uint8_t* __restrict__ q_src, uint8_t* __restrict__ q_dst,
                               int B, int n, int64_t ld, int* improved_count) {
  const int b = blockIdx.x;
  const bool imp = fadd(err_after[b], 1e-12f) < err_before[b];
  if (!imp) return;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    x_dst[b * ld + j] = x_src[b * ld + j];
    q_dst[b * ld + j] = q_src[b * ld + j];
  }
  if (threadIdx.x == 0) {
    err_final[b] = err_after[b];
    atomicAdd(improved_count, 1);
  }
}

// gamma1 = 0.25 * gamma_start / max(mean_j (W - x_rtn)^2, 1e-12)  (mpq/solver.py:481, :86-87)
__global__ void __launch_bounds__(256) k_gamma_init(const float* __restrict__ W, const float* __restrict__ x, int n,
                                                    int64_t ld, float gamma_start, float* __restrict__ gamma1) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  float acc = 0.f;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float d = fsub(W[b * ld + j], x[b * ld + j]);
    acc += d * d;
  }
  const float t = block_sum(acc, red);
  if (threadIdx.x == 0) {
    const float mse = fmaxf(t / (float)n, 1e-12f);
    gamma1[b] = fmul(gamma_start, fdiv(0.25f, mse));
  }
}

static inline int ew_grid(int64_t total) {
  int64_t g = (total + 255) / 256;
  if (g > 148 * 16) g = 148 * 16;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace mpq

using namespace mpq;

MPQ_API int mpq_vamp_rows(const float* var_rowsum, float* gamma1, float* gamma1_work, float* alpha1, float* eta1,
                          float* gamma2_new, float* gamma2, const float* gamma2_prev, float* alpha2, float* eta2,
                          float* gamma1_new, float* gamma1_next, float* trace, int* flags, const float* S, int B,
                          int n, int n_var, int R, float obs, float damping, int final_retry, void* stream) {
  MPQ_CHECK_ARG(var_rowsum && gamma1 && gamma1_work && alpha1 && eta1 && gamma2_new && gamma2 && alpha2 && eta2 &&
                    gamma1_new && gamma1_next && trace && flags && S,
                "mpq_vamp_rows: null pointer");
  if (B == 0) return MPQ_OK;
  RowState st{var_rowsum, gamma1, gamma1_work, alpha1, eta1, gamma2_new, gamma2, gamma2_prev,
              alpha2, eta2, gamma1_new, gamma1_next, trace, flags};
  MPQ_CHECK_ARG(n_var >= 1, "mpq_vamp_rows: n_var must be >= 1");
  k_vamp_rows<<<B, kRowThreads, 0, (cudaStream_t)stream>>>(st, S, B, n, n_var, R, obs, damping, final_retry, nullptr,
                                                            RoundCtl{});
  return launch_status("mpq_vamp_rows");
}

// mpq_vamp_rows under device-side control (ctl: VampCtl): runs only while ctl.active, obs from ctl, gamma2_prev
// (always given) used once ctl.have_prev.
MPQ_API int mpq_vamp_rows_ctl(const float* var_rowsum, float* gamma1, float* gamma1_work, float* alpha1, float* eta1,
                              float* gamma2_new, float* gamma2, const float* gamma2_prev, float* alpha2, float* eta2,
                              float* gamma1_new, float* gamma1_next, float* trace, int* flags, const float* S, int B,
                              int n, int n_var, int R, float damping, int final_retry, const void* ctl, void* stream) {
  MPQ_CHECK_ARG(var_rowsum && gamma1 && gamma1_work && alpha1 && eta1 && gamma2_new && gamma2 && gamma2_prev &&
                    alpha2 && eta2 && gamma1_new && gamma1_next && trace && flags && S && ctl,
                "mpq_vamp_rows_ctl: null pointer");
  MPQ_CHECK_ARG(n_var >= 1, "mpq_vamp_rows_ctl: n_var must be >= 1");
  if (B == 0) return MPQ_OK;
  RowState st{var_rowsum, gamma1, gamma1_work, alpha1, eta1, gamma2_new, gamma2, damping < 1.f ? gamma2_prev : nullptr,
              alpha2, eta2, gamma1_new, gamma1_next, trace, flags};
  k_vamp_rows<<<B, kRowThreads, 0, (cudaStream_t)stream>>>(st, S, B, n, n_var, R, 0.f, damping, final_retry,
                                                            static_cast<const VampCtl*>(ctl), RoundCtl{});
  return launch_status("mpq_vamp_rows_ctl");
}

// mpq_vamp_rows_ctl followed by the end of the retry round (mpq_vamp_ctl_round), taken by the last row CTA to
// finish: one launch per round.  counter: caller-owned device word, zero before the first launch (every launch
// leaves it at zero).
MPQ_API int mpq_vamp_rows_round_ctl(const float* var_rowsum, float* gamma1, float* gamma1_work, float* alpha1,
                                    float* eta1, float* gamma2_new, float* gamma2, const float* gamma2_prev,
                                    float* alpha2, float* eta2, float* gamma1_new, float* gamma1_next, float* trace,
                                    int* flags, const float* S, int B, int n, int n_var, int R, float damping,
                                    int final_retry, void* ctl, float factor, unsigned* counter, void* stream) {
  MPQ_CHECK_ARG(var_rowsum && gamma1 && gamma1_work && alpha1 && eta1 && gamma2_new && gamma2 && gamma2_prev &&
                    alpha2 && eta2 && gamma1_new && gamma1_next && trace && flags && S && ctl && counter,
                "mpq_vamp_rows_round_ctl: null pointer");
  MPQ_CHECK_ARG(n_var >= 1, "mpq_vamp_rows_round_ctl: n_var must be >= 1");
  if (B == 0) return MPQ_OK;
  RowState st{var_rowsum, gamma1, gamma1_work, alpha1, eta1, gamma2_new, gamma2, damping < 1.f ? gamma2_prev : nullptr,
              alpha2, eta2, gamma1_new, gamma1_next, trace, flags};
  RoundCtl rc{static_cast<VampCtl*>(ctl), counter, factor, n_var};
  k_vamp_rows<<<B, kRowThreads, 0, (cudaStream_t)stream>>>(st, S, B, n, n_var, R, 0.f, damping, final_retry,
                                                            static_cast<const VampCtl*>(ctl), rc);
  return launch_status("mpq_vamp_rows_round_ctl");
}

MPQ_API int mpq_gamma_retry(float* gamma1_work, const float* var_rowsum, int B, int n, float factor, void* stream) {
  MPQ_CHECK_ARG(gamma1_work && var_rowsum, "mpq_gamma_retry: null pointer");
  if (B == 0) return MPQ_OK;
  k_gamma_retry<<<(B + 255) / 256, 256, 0, (cudaStream_t)stream>>>(gamma1_work, nullptr, var_rowsum, B, n, factor);
  return launch_status("mpq_gamma_retry");
}

MPQ_API int mpq_vamp_r2(const float* x1, const float* r1, const float* r2_prev, float* r2, const float* eta1,
                        const float* gamma1_work, const float* gamma2_new, int B, int n, int64_t ld, float damping,
                        void* stream) {
  MPQ_CHECK_ARG(x1 && r1 && r2 && eta1 && gamma1_work && gamma2_new, "mpq_vamp_r2: null pointer");
  if ((int64_t)B * n == 0) return MPQ_OK;
  k_vamp_r2<<<ew_grid((int64_t)B * n), 256, 0, (cudaStream_t)stream>>>(x1, r1, r2_prev, r2, eta1, gamma1_work,
                                                                       gamma2_new, B, n, ld, damping, nullptr);
  return launch_status("mpq_vamp_r2");
}

// mpq_vamp_r2 under device-side control: nothing on a skipped iteration; r2_prev (always given) used once
// ctl.have_prev.
MPQ_API int mpq_vamp_r2_ctl(const float* x1, const float* r1, const float* r2_prev, float* r2, const float* eta1,
                            const float* gamma1_work, const float* gamma2_new, int B, int n, int64_t ld, float damping,
                            const void* ctl, void* stream) {
  MPQ_CHECK_ARG(x1 && r1 && r2_prev && r2 && eta1 && gamma1_work && gamma2_new && ctl, "mpq_vamp_r2_ctl: null pointer");
  if ((int64_t)B * n == 0) return MPQ_OK;
  k_vamp_r2<<<ew_grid((int64_t)B * n), 256, 0, (cudaStream_t)stream>>>(
      x1, r1, damping < 1.f ? r2_prev : nullptr, r2, eta1, gamma1_work, gamma2_new, B, n, ld, damping,
      static_cast<const VampCtl*>(ctl));
  return launch_status("mpq_vamp_r2_ctl");
}

MPQ_API int mpq_linear_epilogue(const float* P, const float* Y_u, const float* S, const float* gamma2, float obs,
                                int B, int R, int64_t ld, float* u, float* resid_rowsum, void* stream) {
  MPQ_CHECK_ARG(P && Y_u && S && gamma2 && u && resid_rowsum, "mpq_linear_epilogue: null pointer");
  if (B == 0) return MPQ_OK;
  k_linear_epilogue<<<B, 256, 0, (cudaStream_t)stream>>>(P, Y_u, S, gamma2, obs, R, ld, u, resid_rowsum, nullptr);
  return launch_status("mpq_linear_epilogue");
}

// mpq_linear_epilogue under device-side control: nothing on a skipped iteration, obs from ctl.
MPQ_API int mpq_linear_epilogue_ctl(const float* P, const float* Y_u, const float* S, const float* gamma2, int B,
                                    int R, int64_t ld, float* u, float* resid_rowsum, const void* ctl, void* stream) {
  MPQ_CHECK_ARG(P && Y_u && S && gamma2 && u && resid_rowsum && ctl, "mpq_linear_epilogue_ctl: null pointer");
  if (B == 0) return MPQ_OK;
  k_linear_epilogue<<<B, 256, 0, (cudaStream_t)stream>>>(P, Y_u, S, gamma2, 0.f, R, ld, u, resid_rowsum,
                                                         static_cast<const VampCtl*>(ctl));
  return launch_status("mpq_linear_epilogue_ctl");
}

MPQ_API int mpq_vamp_r1(const float* D, const float* r2, float* r1, const float* eta2, const float* gamma2,
                        const float* gamma1_new, int B, int n, int64_t ld, float damping, void* stream) {
  MPQ_CHECK_ARG(D && r2 && r1 && eta2 && gamma2 && gamma1_new, "mpq_vamp_r1: null pointer");
  if ((int64_t)B * n == 0) return MPQ_OK;
  k_vamp_r1<<<ew_grid((int64_t)B * n), 256, 0, (cudaStream_t)stream>>>(D, r2, r1, eta2, gamma2, gamma1_new, B, n, ld,
                                                                       damping, nullptr, nullptr);
  return launch_status("mpq_vamp_r1");
}

// mpq_vamp_r1 under device-side control: nothing on a skipped iteration; r2_keep (optional) receives r2.
MPQ_API int mpq_vamp_r1_ctl(const float* D, const float* r2, float* r1, const float* eta2, const float* gamma2,
                            const float* gamma1_new, int B, int n, int64_t ld, float damping, float* r2_keep,
                            const void* ctl, void* stream) {
  MPQ_CHECK_ARG(D && r2 && r1 && eta2 && gamma2 && gamma1_new && ctl, "mpq_vamp_r1_ctl: null pointer");
  if ((int64_t)B * n == 0) return MPQ_OK;
  k_vamp_r1<<<ew_grid((int64_t)B * n), 256, 0, (cudaStream_t)stream>>>(D, r2, r1, eta2, gamma2, gamma1_new, B, n, ld,
                                                                       damping, static_cast<const VampCtl*>(ctl),
                                                                       r2_keep);
  return launch_status("mpq_vamp_r1_ctl");
}

MPQ_API int mpq_row_sqerr(const float* Y, const float* C, int B, int R, int64_t ldy, int64_t ldc, float* out,
                          void* stream) {
  MPQ_CHECK_ARG(Y && C && out, "mpq_row_sqerr: null pointer");
  if (B == 0) return MPQ_OK;
  k_row_sqerr<<<B, 256, 0, (cudaStream_t)stream>>>(Y, C, R, ldy, ldc, out);
  return launch_status("mpq_row_sqerr");
}

MPQ_API int mpq_residual(const float* Y, float* C, int B, int R, int64_t ld, float* rowsum, void* stream) {
  MPQ_CHECK_ARG(Y && C, "mpq_residual: null pointer");
  if (B == 0) return MPQ_OK;
  k_residual<<<B, 256, 0, (cudaStream_t)stream>>>(Y, C, R, ld, rowsum);
  return launch_status("mpq_residual");
}

MPQ_API int mpq_mean_rows(const float* a, const float* c, int B, float* out, void* stream) {
  MPQ_CHECK_ARG(a && out, "mpq_mean_rows: null pointer");
  k_mean_rows<<<1, 1024, 0, (cudaStream_t)stream>>>(a, c, B, out);
  return launch_status("mpq_mean_rows");
}

MPQ_API int mpq_polish_merge(const float* err_after, float* err_final, const float* err_before, const float* x_src,
                             float* x_dst, const uint8_t* q_src, uint8_t* q_dst, int B, int n, int64_t ld,
                             int* improved_count, void* stream) {
  MPQ_CHECK_ARG(err_after && err_final && err_before && x_src && x_dst && q_src && q_dst && improved_count,
                "mpq_polish_merge: null pointer");
  if (B == 0) return MPQ_OK;
  k_polish_merge<<<B, 256, 0, (cudaStream_t)stream>>>(err_after, err_final, err_before, x_src, x_dst, q_src, q_dst, B,
                                                      n, ld, improved_count);
  return launch_status("mpq_polish_merge");
}

MPQ_API int mpq_gamma_init(const float* W, const float* x, int B, int n, int64_t ld, float gamma_start, float* gamma1,
                           void* stream) {
  MPQ_CHECK_ARG(W && x && gamma1, "mpq_gamma_init: null pointer");
  if (B == 0) return MPQ_OK;
  k_gamma_init<<<B, 256, 0, (cudaStream_t)stream>>>(W, x, n, ld, gamma_start, gamma1);
  return launch_status("mpq_gamma_init");
}

// out[b] = sum_j A[b,j] * C[b,j]   (row-wise dot, e.g. the raw Hessian audit (d H) . d)
namespace mpq {
__global__ void __launch_bounds__(256) k_row_dot(const float* __restrict__ A, int64_t lda, const float* __restrict__ C,
                                                 int64_t ldc, int n, float* __restrict__ out) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  float acc = 0.f;
  for (int j = threadIdx.x; j < n; j += blockDim.x) acc += A[b * lda + j] * C[b * ldc + j];
  const float t = block_sum(acc, red);
  if (threadIdx.x == 0) out[b] = t;
}

// D = A - C  (elementwise, e.g. delta = W - x)
__global__ void k_sub(const float* __restrict__ A, const float* __restrict__ C, float* __restrict__ D, int B, int n,
                      int64_t ld) {
  const int64_t total = (int64_t)B * n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / n), j = (int)(i % n);
    D[b * ld + j] = fsub(A[b * ld + j], C[b * ld + j]);
  }
}
}  // namespace mpq

MPQ_API int mpq_row_dot(const float* A, int64_t lda, const float* C, int64_t ldc, int B, int n, float* out,
                        void* stream) {
  MPQ_CHECK_ARG(A && C && out, "mpq_row_dot: null pointer");
  if (B == 0) return MPQ_OK;
  k_row_dot<<<B, 256, 0, (cudaStream_t)stream>>>(A, lda, C, ldc, n, out);
  return launch_status("mpq_row_dot");
}

MPQ_API int mpq_sub(const float* A, const float* C, float* D, int B, int n, int64_t ld, void* stream) {
  MPQ_CHECK_ARG(A && C && D, "mpq_sub: null pointer");
  if ((int64_t)B * n == 0) return MPQ_OK;
  k_sub<<<ew_grid((int64_t)B * n), 256, 0, (cudaStream_t)stream>>>(A, C, D, B, n, ld);
  return launch_status("mpq_sub");
}

// ---- entry points of the fused forms (device-resident loop) ----

// r2 = damp(r2_prev, (eta1 x1 - gamma1w r1) / gamma2_new) and its row-scaled fp16 split (hi, lo: B x ldo halves,
// inv_scale: B) under device control: nothing on a skipped iteration, r2_prev used once ctl.have_prev.
MPQ_API int mpq_vamp_r2_split_ctl(const float* x1, const float* r1, const float* r2_prev, float* r2, const float* eta1,
                                  const float* gamma1_work, const float* gamma2_new, int B, int n, int64_t ld,
                                  float damping, void* hi, void* lo, int64_t ldo, float* inv_scale, const void* ctl,
                                  void* stream) {
  MPQ_CHECK_ARG(x1 && r1 && r2_prev && r2 && eta1 && gamma1_work && gamma2_new && hi && lo && inv_scale && ctl,
                "mpq_vamp_r2_split_ctl: null pointer");
  MPQ_CHECK_ARG(ldo >= n && ld >= n, "mpq_vamp_r2_split_ctl: bad leading dimension");
  if ((int64_t)B * n == 0) return MPQ_OK;
  k_vamp_r2_split<<<B, 256, 0, (cudaStream_t)stream>>>(x1, r1, damping < 1.f ? r2_prev : nullptr, r2, eta1,
                                                       gamma1_work, gamma2_new, n, ld, damping,
                                                       static_cast<unsigned short*>(hi), static_cast<unsigned short*>(lo),
                                                       ldo, inv_scale, static_cast<const VampCtl*>(ctl));
  return launch_status("mpq_vamp_r2_split_ctl");
}

// Linear-module epilogue over P = sum of `splits` partial planes (B x R each, plane stride B R) with u written split
// (u: B x R fp32 scratch; hi, lo: B x ldo halves; inv_scale: B) and rowsum(residual_after^2), under device control.
MPQ_API int mpq_linear_epilogue_parts_ctl(const float* parts, int splits, const float* Y_u, int64_t ldy, const float* S,
                                          const float* gamma2, int B, int R, float* u, void* hi, void* lo, int64_t ldo,
                                          float* inv_scale, float* resid_rowsum, const void* ctl, void* stream) {
  MPQ_CHECK_ARG(parts && Y_u && S && gamma2 && u && hi && lo && inv_scale && resid_rowsum && ctl,
                "mpq_linear_epilogue_parts_ctl: null pointer");
  MPQ_CHECK_ARG(splits >= 1 && ldo >= R && ldy >= R, "mpq_linear_epilogue_parts_ctl: bad argument");
  if (B == 0) return MPQ_OK;
  k_linear_epilogue_parts<<<B, 256, 0, (cudaStream_t)stream>>>(parts, splits, (int64_t)B * R, Y_u, ldy, S, gamma2, R, u,
                                                               static_cast<unsigned short*>(hi),
                                                               static_cast<unsigned short*>(lo), ldo, inv_scale,
                                                               resid_rowsum, static_cast<const VampCtl*>(ctl));
  return launch_status("mpq_linear_epilogue_parts_ctl");
}

// r1 update with D = sum of `splits` partial planes (B x n each, plane stride B n), under device control.
MPQ_API int mpq_vamp_r1_parts_ctl(const float* parts, int splits, const float* r2, float* r1, const float* eta2,
                                  const float* gamma2, const float* gamma1_new, int B, int n, int64_t ld, float damping,
                                  float* r2_keep, const void* ctl, void* stream) {
  MPQ_CHECK_ARG(parts && r2 && r1 && eta2 && gamma2 && gamma1_new && ctl, "mpq_vamp_r1_parts_ctl: null pointer");
  MPQ_CHECK_ARG(splits >= 1, "mpq_vamp_r1_parts_ctl: splits must be >= 1");
  if ((int64_t)B * n == 0) return MPQ_OK;
  k_vamp_r1_parts<<<ew_grid((int64_t)B * n), 256, 0, (cudaStream_t)stream>>>(
      parts, splits, (int64_t)B * n, r2, r1, eta2, gamma2, gamma1_new, B, n, ld, damping,
      static_cast<const VampCtl*>(ctl), r2_keep);
  return launch_status("mpq_vamp_r1_parts_ctl");
}
