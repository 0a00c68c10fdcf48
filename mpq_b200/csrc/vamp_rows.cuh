// The per-row scalar stage of a VAMP iteration (alpha1 / gamma2 / alpha2 / gamma1 algebra and the EM trace term),
// shared by the row-stage kernel (vamp_uniform.cu) and the E8P12 posterior's fused row stage (e8p12.cu).
//
// Reference: mpq/solver.py:559-631 (up to the linear module, plus the gamma-only parts of linear_mmse_exact,
// mpq/linear.py:10-56), mpq/utils.py:24-57 (damping, validity masks).
#pragma once
#include "common.cuh"

namespace mpq {

constexpr float kAlphaEps = 1e-7f;
// float32(1.0 - 1e-7), the comparison constant torch uses for `1.0 - alpha_eps`
constexpr float kOneMinusAlphaEps = 0.99999988079071044921875f;

__device__ __forceinline__ bool alpha_valid(float a) { return isfinite(a) && a > kAlphaEps && a < kOneMinusAlphaEps; }
__device__ __forceinline__ bool precision_valid(float g) { return isfinite(g) && g > 1e-12f; }
__device__ __forceinline__ float clip_alpha(float a) {
  a = nan_to_num(a, 0.5f, kOneMinusAlphaEps, kAlphaEps);
  return fminf(fmaxf(a, kAlphaEps), kOneMinusAlphaEps);
}

// flags[0] = #rows with invalid alpha1, flags[1] = #rows non-finite alpha1,
// flags[2] = #rows invalid gamma2_new, flags[3] = #rows invalid damped gamma2, flags[4] = #alpha2 clipped
struct RowState {
  const float* var_rowsum;  // (B) sum_j var1
  float* gamma1;            // (B) committed gamma1
  float* gamma1_work;       // (B) gamma1 used by the current denoiser call
  float* alpha1;            // (B)
  float* eta1;              // (B)
  float* gamma2_new;        // (B)
  float* gamma2;            // (B) damped (current)
  const float* gamma2_prev; // (B) previous damped gamma2 or null
  float* alpha2;            // (B) clipped
  float* eta2;              // (B)
  float* gamma1_new;        // (B)
  float* gamma1_next;       // (B) damped gamma1 for the next iteration
  float* trace;             // (B) sum_r s^2 / (obs s^2 + gamma2)
  int* flags;               // (8)
};

// Stage A+B of one VAMP iteration (mpq/solver.py:559-631 up to the linear module, plus the
// gamma-only parts of linear_mmse_exact and the EM trace term).  One CTA of kRowThreads threads per row; the
// rank-space sums over S are thread-strided and reduced in a fixed tree order.
constexpr int kRowThreads = 128;

// ctl (optional): device-side control -- the launch does nothing unless a retry round is open, obs is read from the
// control block, and gamma2_prev is used only once an iteration has been committed.
// Optional fused end of the retry round: the last row CTA to finish takes the round's decision (ctl_round_serial).
struct RoundCtl {
  VampCtl* ctl;          // the control block (writable)
  unsigned* counter;     // arrival counter, zero between launches
  float factor;
  int n_var;
};

// The row stage of row b, run by threads 0 .. kRowThreads - 1 of the calling CTA (`red`: 2 x kRowThreads / 32
// floats of shared memory).  NAMED_BAR: the CTA has more threads than the stage, which then synchronises on named
// barrier 1 over its kRowThreads threads instead of __syncthreads().
template <bool NAMED_BAR>
__device__ __forceinline__ void vamp_row_stage(const RowState& st_in, const float* __restrict__ S, int b, int B, int n,
                                               int n_var, int R, float obs, float damping, int final_retry,
                                               const VampCtl* __restrict__ ctl, const RoundCtl& rc,
                                               float (*red)[kRowThreads / 32]) {
  RowState st = st_in;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (ctl) {
    if (!ctl->active) return;
    obs = (float)ctl->obs;
    if (!ctl->have_prev) st.gamma2_prev = nullptr;
  }
  const float g1w = st.gamma1_work[b];
  const float a1_raw = fmul(g1w, fdiv(st.var_rowsum[b], (float)n_var));  // gamma1 * var.mean(dim=1)
  float a1 = a1_raw;
  const bool a1_bad = !alpha_valid(a1_raw);
  if (a1_bad && final_retry) a1 = clip_alpha(a1_raw);
  const float eta1 = fdiv(g1w, a1);
  const float g2n = fmaxf(nan_to_num(fsub(eta1, g1w), 1e-12f, 1e12f, 1e-12f), 1e-12f);
  float g2 = g2n;
  const bool damp = (st.gamma2_prev != nullptr) && damping < 1.f;
  if (damp) g2 = log_damp(st.gamma2_prev[b], g2n, (float)(1.0 - (double)damping), damping);
  // gamma-only parts of linear_mmse_exact: sum_r 1/denom and sum_r s^2/denom, denom = obs*s^2 + gamma2
  float inv_sum = 0.f, tr_sum = 0.f;
  for (int r = threadIdx.x; r < R; r += kRowThreads) {
    const float s = S[r];
    const float s2 = fmul(s, s);
    const float den = fadd(fmul(obs, s2), g2);
    inv_sum += fdiv(1.f, den);
    tr_sum += fdiv(s2, den);
  }
  inv_sum = warp_sum(inv_sum);
  tr_sum = warp_sum(tr_sum);
  if (lane == 0) {
    red[0][wid] = inv_sum;
    red[1][wid] = tr_sum;
  }
  if constexpr (NAMED_BAR) {
    asm volatile("bar.sync 1, %0;\n" ::"n"(kRowThreads) : "memory");
  } else {
    __syncthreads();
  }
  if (threadIdx.x != 0) return;
  inv_sum = 0.f;
  tr_sum = 0.f;
  for (int w = 0; w < kRowThreads / 32; ++w) {
    inv_sum += red[0][w];
    tr_sum += red[1][w];
  }
  const float c0 = (float)(1.0 - (double)R / (double)n);
  const float a2_raw = fadd(c0, fmul(fdiv(g2, (float)n), inv_sum));
  const float a2 = clip_alpha(a2_raw);
  const float eta2 = fdiv(g2, a2);
  const float g1n = fmaxf(nan_to_num(fsub(eta2, g2), 1e-12f, 1e12f, 1e-12f), 1e-12f);
  const float g1c = st.gamma1[b];
  const float g1next = damping >= 1.f ? g1n : log_damp(g1c, g1n, (float)(1.0 - (double)damping), damping);
  st.alpha1[b] = a1;
  st.eta1[b] = eta1;
  st.gamma2_new[b] = g2n;
  st.gamma2[b] = g2;
  st.alpha2[b] = a2;
  st.eta2[b] = eta2;
  st.gamma1_new[b] = g1n;
  st.gamma1_next[b] = g1next;
  st.trace[b] = tr_sum;
  if (a1_bad) {
    atomicAdd(&st.flags[0], 1);
    if (!isfinite(a1_raw)) atomicAdd(&st.flags[1], 1);
  }
  if (!precision_valid(g2n)) atomicAdd(&st.flags[2], 1);
  if (!precision_valid(g2)) atomicAdd(&st.flags[3], 1);
  if (!alpha_valid(a2_raw)) atomicAdd(&st.flags[4], 1);
  if (rc.counter) {
    __threadfence();  // this row's flags and outputs before its arrival
    if (atomicAdd(rc.counter, 1u) == (unsigned)(B - 1)) {
      __threadfence();
      ctl_round_serial(rc.ctl, st.flags, st.gamma1_work, st.var_rowsum, B, rc.n_var, rc.factor, final_retry);
      *rc.counter = 0u;
    }
  }
}

}  // namespace mpq
