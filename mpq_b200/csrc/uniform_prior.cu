// Grouped-scalar (uniform grid) posterior denoiser and hard decisions.
//
// Reference: mpq/priors/uniform.py:99-213 (discrete_uniform_mmse, eager path),
//            mpq/priors/triton_vamp.py:24-102 (the CUDA kernel it replaces),
//            mpq/priors/uniform.py:287-309 (nearest_atom_idx / dequant_from_q),
//            mpq/solver.py:833-850 (_uniform_hard_decision).
//
// One CTA per row: the per-row variance sum (alpha1 = gamma * mean(var)) is reduced in a
// fixed order, so repeated calls are bit-identical.  Scores use the reference's float32
// operation order without FMA contraction, so MAP indices are bit-exact against the CPU
// oracle; ties resolve to the lowest atom index (strict '>'), as torch.argmax does.
// Group parameters are addressed as p[row * ld_p + (col >> gshift)] so either the
// group-expanded (gshift = 0) or the per-group (gshift = log2 group) layout is accepted.
#include "common.cuh"

namespace mpq {

struct UniformArgs {
  const float* r1; int64_t ld_r1;
  const float* center; int64_t ld_c;
  const float* scale; const float* zero; int64_t ld_p; int gshift;
  const float* gamma;  // (B) per-row precision
  int n; int maxq; float prior_tau; int has_prior;
};

// score of atom q:  -0.5*g*(a-r)^2  -  0.5*(a-c)^2 / (tau*max(s,1e-12))^2
__device__ __forceinline__ float uni_score(float atom, float r, float c, float ng, float st2, int has_prior) {
  float d = fsub(atom, r);
  float sc = fmul(ng, fmul(d, d));
  if (has_prior) {
    float e = fsub(atom, c);
    sc = fsub(sc, fdiv(fmul(0.5f, fmul(e, e)), st2));
  }
  return sc;
}

template <int MAXQ>
__global__ void __launch_bounds__(256) k_uniform_mmse(UniformArgs a, float* __restrict__ mean_out, int64_t ld_out,
                                                      float* __restrict__ var_out, float* __restrict__ map_value_out,
                                                      uint8_t* __restrict__ map_idx_out, float* __restrict__ var_rowsum) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  const int maxq = MAXQ > 0 ? MAXQ : a.maxq;
  const float ng = fmul(-0.5f, a.gamma[b]);
  float vacc = 0.f;
  for (int j = threadIdx.x; j < a.n; j += blockDim.x) {
    const float r = a.r1[b * a.ld_r1 + j];
    const float c = a.center[b * a.ld_c + j];
    const float s = a.scale[b * a.ld_p + (j >> a.gshift)];
    const float z = a.zero[b * a.ld_p + (j >> a.gshift)];
    const float st = fmul(a.prior_tau, fmaxf(s, 1e-12f));
    const float st2 = fmul(st, st);
    float m = -INFINITY;
    int best = 0;
    if constexpr (MAXQ > 0) {
      float sc[MAXQ + 1];
      #pragma unroll
      for (int q = 0; q <= MAXQ; ++q) {
        const float atom = fmul(s, fsub((float)q, z));
        sc[q] = uni_score(atom, r, c, ng, st2, a.has_prior);
        if (sc[q] > m) { m = sc[q]; best = q; }
      }
      float Z = 0.f, S1 = 0.f, S2 = 0.f;
      #pragma unroll
      for (int q = 0; q <= MAXQ; ++q) {
        const float atom = fmul(s, fsub((float)q, z));
        const float w = expf(sc[q] - m);
        Z += w; S1 += w * atom; S2 += w * atom * atom;
      }
      const float mean = S1 / Z;
      const float var = fmaxf(S2 / Z - mean * mean, 0.f);
      mean_out[b * ld_out + j] = mean;
      if (var_out) var_out[b * ld_out + j] = var;
      vacc += var;
    } else {
      for (int q = 0; q <= maxq; ++q) {
        const float atom = fmul(s, fsub((float)q, z));
        const float v = uni_score(atom, r, c, ng, st2, a.has_prior);
        if (v > m) { m = v; best = q; }
      }
      float Z = 0.f, S1 = 0.f, S2 = 0.f;
      for (int q = 0; q <= maxq; ++q) {
        const float atom = fmul(s, fsub((float)q, z));
        const float w = expf(uni_score(atom, r, c, ng, st2, a.has_prior) - m);
        Z += w; S1 += w * atom; S2 += w * atom * atom;
      }
      const float mean = S1 / Z;
      const float var = fmaxf(S2 / Z - mean * mean, 0.f);
      mean_out[b * ld_out + j] = mean;
      if (var_out) var_out[b * ld_out + j] = var;
      vacc += var;
    }
    if (map_value_out) map_value_out[b * ld_out + j] = fmul(s, fsub((float)best, z));
    if (map_idx_out) map_idx_out[b * ld_out + j] = (uint8_t)best;
  }
  const float t = block_sum(vacc, red);
  if (threadIdx.x == 0 && var_rowsum) var_rowsum[b] = t;
}

// nearest_atom_idx(x) then dequant: q = clamp(rint(x / max(s,1e-12) + z), 0, maxq); x = s*(q - z)
__device__ __forceinline__ int nearest_code(float x, float s, float z, int maxq) {
  float q = rintf(fadd(fdiv(x, fmaxf(s, 1e-12f)), z));
  q = fminf(fmaxf(q, 0.f), (float)maxq);
  return (int)q;
}

// MAP hard decision (mpq/solver.py:513-541 `_current_hard_state` with final_decision='map'):
// the MAP atom is re-rounded through nearest_atom_idx exactly as the reference does.
template <int MAXQ>
__global__ void __launch_bounds__(256) k_uniform_map_decision(UniformArgs a, uint8_t* __restrict__ q_out,
                                                              float* __restrict__ x_out, int64_t ld_out) {
  const int b = blockIdx.x;
  const int maxq = MAXQ > 0 ? MAXQ : a.maxq;
  const float ng = fmul(-0.5f, a.gamma[b]);
  for (int j = threadIdx.x; j < a.n; j += blockDim.x) {
    const float r = a.r1[b * a.ld_r1 + j];
    const float c = a.center[b * a.ld_c + j];
    const float s = a.scale[b * a.ld_p + (j >> a.gshift)];
    const float z = a.zero[b * a.ld_p + (j >> a.gshift)];
    const float st = fmul(a.prior_tau, fmaxf(s, 1e-12f));
    const float st2 = fmul(st, st);
    float m = -INFINITY;
    int best = 0;
    #pragma unroll 16
    for (int q = 0; q <= maxq; ++q) {
      const float atom = fmul(s, fsub((float)q, z));
      const float v = uni_score(atom, r, c, ng, st2, a.has_prior);
      if (v > m) { m = v; best = q; }
    }
    const float mapv = fmul(s, fsub((float)best, z));
    const int q = nearest_code(mapv, s, z, maxq);
    if (q_out) q_out[b * ld_out + j] = (uint8_t)q;
    if (x_out) x_out[b * ld_out + j] = fmul(s, fsub((float)q, z));
  }
}

__global__ void k_nearest_dequant(const float* __restrict__ x, int64_t ld_x, const float* __restrict__ scale,
                                  const float* __restrict__ zero, int64_t ld_p, int gshift, int B, int n, int maxq,
                                  uint8_t* __restrict__ q_out, float* __restrict__ x_out, int64_t ld_out) {
  const int64_t total = (int64_t)B * n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / n), j = (int)(i % n);
    const float s = scale[b * ld_p + (j >> gshift)];
    const float z = zero[b * ld_p + (j >> gshift)];
    const int q = nearest_code(x[b * ld_x + j], s, z, maxq);
    if (q_out) q_out[b * ld_out + j] = (uint8_t)q;
    if (x_out) x_out[b * ld_out + j] = fmul(s, fsub((float)q, z));
  }
}

static int uniform_check(const UniformArgs& a, int B) {
  MPQ_CHECK_ARG(B >= 0 && a.n >= 0, "uniform prior: negative shape");
  if (B == 0 || a.n == 0) return MPQ_OK;  // empty tensors may carry null pointers
  MPQ_CHECK_ARG(a.r1 && a.center && a.scale && a.zero && a.gamma, "uniform prior: null input pointer");
  MPQ_CHECK_ARG(a.maxq >= 1 && a.maxq <= 255, "uniform prior: maxq must be in [1, 255], got %d", a.maxq);
  MPQ_CHECK_ARG(a.gshift >= 0 && a.gshift < 31, "uniform prior: bad gshift %d", a.gshift);
  return MPQ_OK;
}

}  // namespace mpq

using namespace mpq;

MPQ_API int mpq_uniform_mmse(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* scale,
                             const float* zero, int64_t ld_p, int gshift, const float* gamma, int B, int n, int maxq,
                             float prior_tau, float* mean_out, int64_t ld_out, float* var_out, float* map_value_out,
                             uint8_t* map_idx_out, float* var_rowsum, void* stream) {
  UniformArgs a{r1, ld_r1, center, ld_c, scale, zero, ld_p, gshift, gamma, n, maxq, prior_tau, prior_tau > 0.f};
  int st = uniform_check(a, B);
  if (st) return st;
  if (B == 0 || n == 0) return MPQ_OK;
  MPQ_CHECK_ARG(mean_out && var_rowsum, "mpq_uniform_mmse: mean_out and var_rowsum are required");
  cudaStream_t s = (cudaStream_t)stream;
  switch (maxq) {
    case 1: k_uniform_mmse<1><<<B, 256, 0, s>>>(a, mean_out, ld_out, var_out, map_value_out, map_idx_out, var_rowsum); break;
    case 3: k_uniform_mmse<3><<<B, 256, 0, s>>>(a, mean_out, ld_out, var_out, map_value_out, map_idx_out, var_rowsum); break;
    case 7: k_uniform_mmse<7><<<B, 256, 0, s>>>(a, mean_out, ld_out, var_out, map_value_out, map_idx_out, var_rowsum); break;
    case 15: k_uniform_mmse<15><<<B, 256, 0, s>>>(a, mean_out, ld_out, var_out, map_value_out, map_idx_out, var_rowsum); break;
    default: k_uniform_mmse<0><<<B, 256, 0, s>>>(a, mean_out, ld_out, var_out, map_value_out, map_idx_out, var_rowsum); break;
  }
  return launch_status("mpq_uniform_mmse");
}

MPQ_API int mpq_uniform_map_decision(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c,
                                     const float* scale, const float* zero, int64_t ld_p, int gshift,
                                     const float* gamma, int B, int n, int maxq, float prior_tau, uint8_t* q_out,
                                     float* x_out, int64_t ld_out, void* stream) {
  UniformArgs a{r1, ld_r1, center, ld_c, scale, zero, ld_p, gshift, gamma, n, maxq, prior_tau, prior_tau > 0.f};
  int st = uniform_check(a, B);
  if (st) return st;
  if (B == 0 || n == 0) return MPQ_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (maxq == 15) k_uniform_map_decision<15><<<B, 256, 0, s>>>(a, q_out, x_out, ld_out);
  else k_uniform_map_decision<0><<<B, 256, 0, s>>>(a, q_out, x_out, ld_out);
  return launch_status("mpq_uniform_map_decision");
}

MPQ_API int mpq_uniform_nearest(const float* x, int64_t ld_x, const float* scale, const float* zero, int64_t ld_p,
                                int gshift, int B, int n, int maxq, uint8_t* q_out, float* x_out, int64_t ld_out,
                                void* stream) {
  MPQ_CHECK_ARG(x && scale && zero, "mpq_uniform_nearest: null input");
  MPQ_CHECK_ARG(maxq >= 1 && maxq <= 255, "mpq_uniform_nearest: maxq must be in [1, 255]");
  if ((int64_t)B * n == 0) return MPQ_OK;
  int64_t total = (int64_t)B * n;
  int grid = (int)((total + 255) / 256);
  if (grid > 148 * 32) grid = 148 * 32;
  k_nearest_dequant<<<grid, 256, 0, (cudaStream_t)stream>>>(x, ld_x, scale, zero, ld_p, gshift, B, n, maxq, q_out,
                                                            x_out, ld_out);
  return launch_status("mpq_uniform_nearest");
}

// ---------------------------------------------------------------------------------------------
// Group parameters and RTN.
//
// mpq_group_minmax restates the asymmetric per-row min-max grid of GPTQ's quantizer (GPTQModel
// Quantizer.find_params @ ed96f2e is not vendored with the reference):
//   xmin = min(row_min, 0), xmax = max(row_max, 0); all-zero rows use [-1, 1];
//   scale = (xmax - xmin) / maxq; zero = round(-xmin / scale).
// mpq_uniform_rtn follows mpq/adapters/gptqmodel.py:928-931 (note: round(W / s) + z, which
// differs from nearest_atom_idx's round(W / s + z) at exact ties):
//   q = clamp(round(W / s) + z, 0, maxq); x = s * (q - z).
// ---------------------------------------------------------------------------------------------
namespace mpq {

__global__ void k_group_minmax(const float* __restrict__ W, int64_t ldw, int rows, int cols, int group, int maxq,
                               float* __restrict__ scale, float* __restrict__ zero, int64_t ldp) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int ngroups = (cols + group - 1) / group;
  if (warp >= rows * ngroups) return;
  const int r = warp / ngroups, g = warp % ngroups;
  const int c0 = g * group, c1 = min(cols, c0 + group);
  float mn = INFINITY, mx = -INFINITY;
  for (int c = c0 + lane; c < c1; c += 32) {
    const float v = W[r * ldw + c];
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if (lane == 0) {
    float xmin = fminf(mn, 0.f), xmax = fmaxf(mx, 0.f);
    if (xmin == 0.f && xmax == 0.f) { xmin = -1.f; xmax = 1.f; }
    const float s = fdiv(fsub(xmax, xmin), (float)maxq);
    scale[r * ldp + g] = s;
    zero[r * ldp + g] = rintf(fdiv(-xmin, s));
  }
}

__global__ void k_uniform_rtn(const float* __restrict__ W, int64_t ldw, const float* __restrict__ scale,
                              const float* __restrict__ zero, int64_t ld_p, int gshift, int B, int n, int maxq,
                              uint8_t* __restrict__ q_out, float* __restrict__ x_out, int64_t ld_out) {
  const int64_t total = (int64_t)B * n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / n), j = (int)(i % n);
    const float s = scale[b * ld_p + (j >> gshift)];
    const float z = zero[b * ld_p + (j >> gshift)];
    float q = fadd(rintf(fdiv(W[b * ldw + j], s)), z);
    q = fminf(fmaxf(q, 0.f), (float)maxq);
    if (q_out) q_out[b * ld_out + j] = (uint8_t)q;
    if (x_out) x_out[b * ld_out + j] = fmul(s, fsub(q, z));
  }
}

}  // namespace mpq

MPQ_API int mpq_group_minmax(const float* W, int64_t ldw, int rows, int cols, int group, int maxq, float* scale,
                             float* zero, int64_t ldp, void* stream) {
  MPQ_CHECK_ARG(W && scale && zero, "mpq_group_minmax: null pointer");
  MPQ_CHECK_ARG(group >= 1 && maxq >= 1, "mpq_group_minmax: bad group/maxq");
  const int64_t warps = (int64_t)rows * ((cols + group - 1) / group);
  if (warps == 0) return MPQ_OK;
  k_group_minmax<<<(int)((warps * 32 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(W, ldw, rows, cols, group, maxq,
                                                                                    scale, zero, ldp);
  return launch_status("mpq_group_minmax");
}

MPQ_API int mpq_uniform_rtn(const float* W, int64_t ldw, const float* scale, const float* zero, int64_t ld_p,
                            int gshift, int B, int n, int maxq, uint8_t* q_out, float* x_out, int64_t ld_out,
                            void* stream) {
  MPQ_CHECK_ARG(W && scale && zero, "mpq_uniform_rtn: null pointer");
  MPQ_CHECK_ARG(maxq >= 1 && maxq <= 255, "mpq_uniform_rtn: bad maxq");
  const int64_t total = (int64_t)B * n;
  if (total == 0) return MPQ_OK;
  int grid = (int)((total + 255) / 256);
  if (grid > 148 * 32) grid = 148 * 32;
  k_uniform_rtn<<<grid, 256, 0, (cudaStream_t)stream>>>(W, ldw, scale, zero, ld_p, gshift, B, n, maxq, q_out, x_out,
                                                        ld_out);
  return launch_status("mpq_uniform_rtn");
}
