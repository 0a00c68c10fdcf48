// Shared helpers for the MPQ B200 kernels (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <math.h>

#define MPQ_API extern "C" __attribute__((visibility("default")))
#define MPQ_IPC_HANDLE_BYTES 64

// Status codes returned by every C-ABI entry point (0 = success; >0 = cudaError_t).
enum MpqStatus {
  MPQ_OK = 0,
  MPQ_ERR_ARG = 10001,        // invalid argument (shape, null pointer, unsupported size)
  MPQ_ERR_UNSUPPORTED = 10002,
};

namespace mpq {

void set_last_error(const char* fmt, ...);

// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the current device (once per device and kernel;
// thread-safe).  Returns MPQ_OK or the cudaError_t of the failing call, with the message in mpq_last_error().
int smem_opt_in(const void* kernel, size_t bytes, const char* what);

// Device-resident control block of one VAMP iteration loop (see vamp_ctl.cu).
struct VampCtl {
  double obs;               //  0: observation precision (float64, as the reference's Python float)
  int active;               //  8: a retry round is still open (denoiser / row stage run while 1)
  int skip;                 // 12: the rest of this iteration is skipped (invalid gamma2) or the loop stopped
  int have_prev;            // 16: r2_prev / gamma2_prev exist (damping of r2 and gamma2)
  int stopped;              // 20: best-iterate stop (no further iteration runs)
  int fail;                 // 24: alpha1 non-finite after the last retry (the reference raises)
  int alpha1_retry_count;   // 28
  int alpha2_clip_count;    // 32
  int gamma2_invalid_count; // 36
  int committed;            // 40: iterations committed
  int best_iter;            // 44: best-iterate index (-1: the start state)
  int stop_iter;            // 48
  int pad[3];               // 52..63
};
static_assert(sizeof(VampCtl) == 64, "VampCtl layout");

// End of a retry round of the device-controlled VAMP iteration (mpq/solver.py:575-596), by one thread: all alpha1
// valid -> close the round; last round -> record a non-finite alpha1 and close; otherwise count the invalid rows and
// rescale their work precision (divide where alpha1 <= eps, multiply where alpha1 >= 1 - eps) for the next round.
// When the round closes, the invalid-gamma2 test (:598-604) decides whether the iteration continues.  `flags` is read
// through volatile loads: the row CTAs set it with atomics before the caller observed their arrival.
__device__ inline void ctl_round_serial(VampCtl* ctl, int* flags, float* g1w, const float* var_rowsum, int B,
                                        int n_var, float factor, int final_round) {
  if (!ctl->active) return;
  volatile int* vf = flags;
  const int f0 = vf[0];
  if (f0 == 0 || final_round) {
    if (f0 != 0 && vf[1] > 0) ctl->fail = 1;
    ctl->active = 0;
    if (vf[2] > 0 || vf[3] > 0) {
      ctl->gamma2_invalid_count += 1;
      ctl->skip = 1;
    } else {
      ctl->alpha2_clip_count += vf[4];
    }
    return;
  }
  ctl->alpha1_retry_count += f0;
  for (int i = 0; i < 8; ++i) vf[i] = 0;
  const volatile float* vv = var_rowsum;
  for (int b = 0; b < B; ++b) {
    float g = g1w[b];
    const float a = __fmul_rn(g, __fdiv_rn(vv[b], (float)n_var));
    if (a <= 1e-7f) g = __fdiv_rn(g, factor);
    if (a >= 0.99999988079071044921875f) g = __fmul_rn(g, factor);
    g1w[b] = fmaxf(g, 1e-12f);
  }
}

inline int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("%s: %s", what, cudaGetErrorString(e));
    return (int)e;
  }
  return MPQ_OK;
}

#define MPQ_CHECK_ARG(cond, ...)          \
  do {                                    \
    if (!(cond)) {                        \
      ::mpq::set_last_error(__VA_ARGS__); \
      return MPQ_ERR_ARG;                 \
    }                                     \
  } while (0)

// ---- exact float32 arithmetic (no FMA contraction): mirrors the reference op order ----
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

// torch.nan_to_num(x, nan, posinf, neginf)
__device__ __forceinline__ float nan_to_num(float x, float nan_v, float pinf, float ninf) {
  if (isnan(x)) return nan_v;
  if (isinf(x)) return x > 0.f ? pinf : ninf;
  return x;
}

// mpq/utils.py log_damp_positive: exp((1-d) ln max(p,1e-12) + d ln max(n,1e-12)) in float32 steps, with
// correctly rounded log/exp (double evaluation, one rounding), as torch's CPU float32 kernels return.
__device__ __forceinline__ float log_damp(float prev, float nw, float one_minus_d, float d) {
  prev = fmaxf(prev, 1e-12f);
  nw = fmaxf(nw, 1e-12f);
  const float lp = (float)log((double)prev), ln = (float)log((double)nw);
  return (float)exp((double)fadd(fmul(one_minus_d, lp), fmul(d, ln)));
}

// Deterministic block-wide sum (fixed tree order). `red` must hold blockDim.x/32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = 0.f;
  if (wid == 0) {
    t = lane < nw ? red[lane] : 0.f;
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  }
  return t;  // valid in warp 0
}

// Row-scaled fp16 split (the FP32-faithful operand format of the fp16 tensor-core products): for a row whose largest
// magnitude is mx (< 2^e), s = 2^(15 - e) and inv = 2^(e - 15); every element x of the row is stored as
// hi = fp16_rn(x s), lo = fp16_rn(x s - hi)  (x s and x s - hi are exact in fp32).
__device__ __forceinline__ void split_f16_scale(float mx, float& s, float& inv) {
  int e = 0;
  if (mx > 0.f && isfinite(mx)) frexpf(mx, &e);  // mx < 2^e
  s = ldexpf(1.f, 15 - e);
  inv = ldexpf(1.f, e - 15);
}

__device__ __forceinline__ void split_f16_store(float x, float s, unsigned short* hi, unsigned short* lo) {
  const float y = x * s;
  const __half h = __float2half_rn(y);
  *reinterpret_cast<__half*>(hi) = h;
  *reinterpret_cast<__half*>(lo) = __float2half_rn(y - __half2float(h));
}

// Deterministic block-wide maximum (valid in warp 0); `red` must hold blockDim.x/32 floats.
__device__ __forceinline__ float block_max(float v, float* red) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = 0.f;
  if (wid == 0) {
    t = lane < nw ? red[lane] : 0.f;
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
  }
  return t;
}

__device__ __forceinline__ float warp_sum(float v) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace mpq
