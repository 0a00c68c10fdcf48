// Device-resident control of the VAMP iteration: the decisions the reference takes on the host between kernel
// launches (gamma retries, skipped iterations, the EM update of the observation precision) are taken by small
// kernels from a control block in device memory, so a whole row block (and a chain of row blocks, whose only
// coupling is the observation precision) is enqueued without a host round trip.
//
// Reference: mpq/solver.py:553-699 (retry loop :553-596, invalid gamma2 :598-612, EM :629-640, iteration tail
// :645-666) and its E8P12 twin :961-1122; mpq/linear.py:59-82 (em_update_obs_precision_rankspace);
// mpq/utils.py:36-45 (log_damp_positive_scalar).  The host version of the same loop (one launch sequence per
// iteration with host reads of the flags) is in mpq_b200/solver.py.
//
// The control block (VampCtl, 64 bytes) lives in device memory.  Kernels that only act when the iteration is live
// read `skip`; the denoiser and row-stage launches of retry rounds read `active`.
#include "common.cuh"

namespace mpq {



constexpr float kAlphaEpsC = 1e-7f;
constexpr float kOneMinusAlphaEpsC = 0.99999988079071044921875f;

// Start of an iteration by one CTA (k_ctl_begin's work, also done at the end of the previous commit).
__device__ inline void ctl_begin_body(VampCtl* ctl, const float* __restrict__ gamma1, float* __restrict__ g1w, int B,
                                      int* __restrict__ flags) {
  const bool stopped = ctl->stopped != 0;
  if (!stopped)
    for (int b = threadIdx.x; b < B; b += blockDim.x) g1w[b] = gamma1[b];
  __syncthreads();  // every thread has read `stopped` before thread 0 changes the block
  if (threadIdx.x == 0) {
    for (int i = 0; i < 8; ++i) flags[i] = 0;
    ctl->active = stopped ? 0 : 1;
    ctl->skip = stopped ? 1 : 0;
  }
}

// Start of an iteration: gamma1_work = gamma1, flags cleared, the retry round opened unless the loop stopped.
__global__ void k_ctl_begin(VampCtl* ctl, const float* __restrict__ gamma1, float* __restrict__ g1w, int B,
                            int* __restrict__ flags) {
  const bool stopped = ctl->stopped != 0;
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < B; b += gridDim.x * blockDim.x)
    if (!stopped) g1w[b] = gamma1[b];
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    for (int i = 0; i < 8; ++i) flags[i] = 0;
    ctl->active = stopped ? 0 : 1;
    ctl->skip = stopped ? 1 : 0;
  }
}

// End of retry round `final_round` (mpq/solver.py:575-596): all alpha1 valid -> close the round; last round ->
// record a non-finite alpha1 and close; otherwise count the invalid rows and rescale their work precision
// (divide where alpha1 <= eps, multiply where alpha1 >= 1 - eps) for the next round.  When the round closes, the
// invalid-gamma2 test (:598-604, :614-616) decides whether the iteration continues.  One CTA.
__global__ void k_ctl_round(VampCtl* ctl, int* __restrict__ flags, float* __restrict__ g1w,
                            const float* __restrict__ var_rowsum, int B, int n_var, float factor, int final_round) {
  __shared__ int s_retry;
  if (threadIdx.x == 0) {
    s_retry = 0;
    if (ctl->active) {
      const int f0 = flags[0];
      if (f0 == 0 || final_round) {
        if (f0 != 0 && flags[1] > 0) ctl->fail = 1;
        ctl->active = 0;
        if (flags[2] > 0 || flags[3] > 0) {
          ctl->gamma2_invalid_count += 1;
          ctl->skip = 1;
        } else {
          ctl->alpha2_clip_count += flags[4];
        }
      } else {
        ctl->alpha1_retry_count += f0;
        for (int i = 0; i < 8; ++i) flags[i] = 0;
        s_retry = 1;
      }
    }
  }
  __syncthreads();
  if (!s_retry) return;
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    float g = g1w[b];
    const float a = fmul(g, fdiv(var_rowsum[b], (float)n_var));
    if (a <= kAlphaEpsC) g = fdiv(g, factor);
    if (a >= kOneMinusAlphaEpsC) g = fmul(g, factor);
    g1w[b] = fmaxf(g, 1e-12f);
  }
}

// End of a live iteration (mpq/solver.py:629-666): gamma1 <- damped gamma1_new, gamma2_prev <- gamma2, and the EM
// update of the observation precision from mean_b(resid_rowsum + trace) (mpq/linear.py:74-82): beta_new = R / mean,
// log-damped against the previous value, clamped to [min, max]; obs_hist[it] records the value (NaN when the
// iteration was skipped).  One CTA, fixed-order mean.
__global__ void __launch_bounds__(1024) k_ctl_commit(VampCtl* ctl, float* __restrict__ gamma1,
                                                     const float* __restrict__ g1next, float* __restrict__ g2p,
                                                     const float* __restrict__ g2, const float* __restrict__ resid,
                                                     const float* __restrict__ trace, int B, int R, int em_active,
                                                     double em_damping, double em_min, double em_max,
                                                     double* __restrict__ obs_hist, const float* __restrict__ a1,
                                                     const float* __restrict__ a2, double* __restrict__ a1_hist,
                                                     double* __restrict__ a2_hist, int it,
                                                     float* __restrict__ g1w_next, int* __restrict__ flags_next) {
  __shared__ float red[32];
  if (ctl->skip) {
    if (threadIdx.x == 0) {
      const double nan = __longlong_as_double(0x7ff8000000000000ll);
      if (obs_hist) obs_hist[it] = nan;
      if (a1_hist) a1_hist[it] = nan;
      if (a2_hist) a2_hist[it] = nan;
    }
    if (g1w_next) ctl_begin_body(ctl, gamma1, g1w_next, B, flags_next);
    return;
  }
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    gamma1[b] = g1next[b];
    g2p[b] = g2[b];
  }
  // the iteration's mean alpha1 (accepted, clipped) and alpha2 (clipped), mpq/solver.py:1064-1065
  if (a1_hist && a2_hist) {
    float s1 = 0.f, s2 = 0.f;
    for (int b = threadIdx.x; b < B; b += blockDim.x) {
      s1 += a1[b];
      s2 += a2[b];
    }
    const float t1 = block_sum(s1, red);
    const float t2 = block_sum(s2, red);
    if (threadIdx.x == 0) {
      a1_hist[it] = B > 0 ? (double)(t1 / (float)B) : 0.0;
      a2_hist[it] = B > 0 ? (double)(t2 / (float)B) : 0.0;
    }
  }
  float acc = 0.f;
  if (em_active)
    for (int b = threadIdx.x; b < B; b += blockDim.x) acc += fadd(resid[b], trace[b]);
  const float t = block_sum(acc, red);
  if (threadIdx.x == 0) {
    double obs = ctl->obs;
    if (em_active && R > 0) {
      const float mean = fmaxf(B > 0 ? t / (float)B : 0.f, 1e-12f);
      const double beta_new = (double)R / (double)mean;
      double beta;
      if (em_damping >= 1.0) {
        beta = beta_new;
      } else if (em_damping <= 0.0) {
        beta = obs;
      } else {
        const double prev = fmax(obs, 1e-12), nw = fmax(beta_new, 1e-12);
        beta = exp((1.0 - em_damping) * log(prev) + em_damping * log(nw));
      }
      obs = fmin(fmax(beta, em_min), em_max);
      ctl->obs = obs;
    }
    ctl->have_prev = 1;
    ctl->committed += 1;
    if (obs_hist) obs_hist[it] = obs;
  }
  if (g1w_next) {
    __syncthreads();  // gamma1 of every row and the control block updated
    ctl_begin_body(ctl, gamma1, g1w_next, B, flags_next);
  }
}

// Best-iterate test of the scalar solver (mpq/solver.py:668-699), phase 0 (one CTA): cur = mean_b err_cur[b] in a
// fixed order; improve when cur + max(1e-10, |best| 1e-8) < best.  On improvement best_mean / best_obs / best_iter
// take the current values (decision 1); otherwise obs is restored from best_obs and the loop stops (decision 0).
// Skipped iterations leave everything unchanged (decision -1).
__global__ void __launch_bounds__(1024) k_ctl_best(VampCtl* ctl, const float* __restrict__ err_cur, int B,
                                                   double* __restrict__ best_mean, double* __restrict__ best_obs,
                                                   int it, int* __restrict__ decision) {
  __shared__ float red[32];
  if (ctl->skip) {
    if (threadIdx.x == 0) decision[0] = -1;
    return;
  }
  float acc = 0.f;
  for (int b = threadIdx.x; b < B; b += blockDim.x) acc += err_cur[b];
  const float t = block_sum(acc, red);
  if (threadIdx.x == 0) {
    const double cur = B > 0 ? (double)(t / (float)B) : 0.0;
    const double best = *best_mean;
    const double tol = fmax(1e-10, fabs(best) * 1e-8);
    if (cur + tol < best) {
      *best_mean = cur;
      *best_obs = ctl->obs;
      ctl->best_iter = it;
      decision[0] = 1;
    } else {
      ctl->obs = *best_obs;
      ctl->stopped = 1;
      ctl->stop_iter = it;
      decision[0] = 0;
    }
  }
}

// Phase 1 of the best-iterate test: row copies selected by decision[0] (1: cur -> best, 0: best -> live state).
__global__ void k_ctl_best_copy(const int* __restrict__ decision, int B, int n, int64_t ld,
                                uint8_t* __restrict__ best_q, const uint8_t* __restrict__ cur_q,
                                float* __restrict__ best_x, const float* __restrict__ cur_x,
                                float* __restrict__ best_err, const float* __restrict__ err_cur,
                                float* __restrict__ best_r1, float* __restrict__ r1, float* __restrict__ best_g1,
                                float* __restrict__ gamma1) {
  const int d = decision[0];
  if (d < 0) return;
  const int64_t total = (int64_t)B * n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / n), j = (int)(i % n);
    const int64_t o = b * ld + j;
    if (d == 1) {
      best_q[o] = cur_q[o];
      best_x[o] = cur_x[o];
      best_r1[o] = r1[o];
    } else {
      r1[o] = best_r1[o];
    }
  }
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < B; b += (int64_t)gridDim.x * blockDim.x) {
    if (d == 1) {
      best_err[b] = err_cur[b];
      best_g1[b] = gamma1[b];
    } else {
      gamma1[b] = best_g1[b];
    }
  }
}

}  // namespace mpq

using namespace mpq;

MPQ_API int mpq_vamp_ctl_size(void) { return (int)sizeof(VampCtl); }

// Opens iteration: gamma1_work = gamma1 (B), flags (8) cleared, ctl.active = !stopped, ctl.skip = stopped.
MPQ_API int mpq_vamp_ctl_begin(void* ctl, const float* gamma1, float* gamma1_work, int B, int* flags, void* stream) {
  MPQ_CHECK_ARG(ctl && flags, "mpq_vamp_ctl_begin: null pointer");
  MPQ_CHECK_ARG(B == 0 || (gamma1 && gamma1_work), "mpq_vamp_ctl_begin: null pointer");
  const int blocks = B > 0 ? (B + 255) / 256 : 1;
  k_ctl_begin<<<blocks, 256, 0, (cudaStream_t)stream>>>(static_cast<VampCtl*>(ctl), gamma1, gamma1_work, B, flags);
  return launch_status("mpq_vamp_ctl_begin");
}

MPQ_API int mpq_vamp_ctl_round(void* ctl, int* flags, float* gamma1_work, const float* var_rowsum, int B, int n_var,
                               float factor, int final_round, void* stream) {
  MPQ_CHECK_ARG(ctl && flags, "mpq_vamp_ctl_round: null pointer");
  MPQ_CHECK_ARG(B == 0 || (gamma1_work && var_rowsum), "mpq_vamp_ctl_round: null pointer");
  MPQ_CHECK_ARG(n_var >= 1, "mpq_vamp_ctl_round: n_var must be >= 1");
  k_ctl_round<<<1, 256, 0, (cudaStream_t)stream>>>(static_cast<VampCtl*>(ctl), flags, gamma1_work, var_rowsum, B, n_var,
                                                   factor, final_round);
  return launch_status("mpq_vamp_ctl_round");
}

MPQ_API int mpq_vamp_ctl_commit(void* ctl, float* gamma1, const float* gamma1_next, float* gamma2_prev,
                                const float* gamma2, const float* resid_rowsum, const float* trace, int B, int R,
                                int em_active, double em_damping, double em_min, double em_max, double* obs_hist,
                                const float* alpha1, const float* alpha2, double* alpha1_hist, double* alpha2_hist,
                                int it, float* gamma1_work_next, int* flags_next, void* stream) {
  MPQ_CHECK_ARG(ctl, "mpq_vamp_ctl_commit: null pointer");
  MPQ_CHECK_ARG(B == 0 || (gamma1 && gamma1_next && gamma2_prev && gamma2 && resid_rowsum && trace),
                "mpq_vamp_ctl_commit: null pointer");
  MPQ_CHECK_ARG((gamma1_work_next == nullptr) == (flags_next == nullptr),
                "mpq_vamp_ctl_commit: the next iteration's gamma1_work and flags go together");
  MPQ_CHECK_ARG((alpha1_hist == nullptr) == (alpha2_hist == nullptr) &&
                    (alpha1_hist == nullptr || B == 0 || (alpha1 && alpha2)),
                "mpq_vamp_ctl_commit: alpha histories need both rows and both outputs");
  k_ctl_commit<<<1, 1024, 0, (cudaStream_t)stream>>>(static_cast<VampCtl*>(ctl), gamma1, gamma1_next, gamma2_prev,
                                                     gamma2, resid_rowsum, trace, B, R, em_active, em_damping, em_min,
                                                     em_max, obs_hist, alpha1, alpha2, alpha1_hist, alpha2_hist, it,
                                                     gamma1_work_next, flags_next);
  return launch_status("mpq_vamp_ctl_commit");
}

MPQ_API int mpq_vamp_ctl_best(void* ctl, const float* err_cur, int B, int n, double* best_mean, double* best_obs,
                              uint8_t* best_q, const uint8_t* cur_q, float* best_x, const float* cur_x, float* best_err,
                              float* best_r1, float* r1, float* best_g1, float* gamma1, int64_t ld, int it,
                              int* decision, void* stream) {
  MPQ_CHECK_ARG(ctl && best_mean && best_obs && decision, "mpq_vamp_ctl_best: null pointer");
  MPQ_CHECK_ARG(B == 0 || (err_cur && best_q && cur_q && best_x && cur_x && best_err && best_r1 && r1 && best_g1 &&
                           gamma1), "mpq_vamp_ctl_best: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  k_ctl_best<<<1, 1024, 0, s>>>(static_cast<VampCtl*>(ctl), err_cur, B, best_mean, best_obs, it, decision);
  int st = launch_status("mpq_vamp_ctl_best");
  if (st) return st;
  const int64_t total = (int64_t)B * n;
  int64_t g = (total + 255) / 256;
  if (g > 148 * 8) g = 148 * 8;
  if (g < 1) g = 1;
  k_ctl_best_copy<<<(int)g, 256, 0, s>>>(decision, B, n, ld, best_q, cur_q, best_x, cur_x, best_err, err_cur, best_r1,
                                         r1, best_g1, gamma1);
  return launch_status("mpq_vamp_ctl_best (copies)");
}
