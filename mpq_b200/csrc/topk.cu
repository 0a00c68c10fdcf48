// Top-k candidate recipes of the polish ("topk_block_cd"): the k most probable grid atoms per coordinate, and the
// per-row choice among a block's candidates inside the block CD engine.
//
// Reference: mpq/priors/uniform.py:253-284 (uniform_map_topk), mpq/polish/block_cd.py:657-685
// (UniformTopKProvider), :93-101 and :768-860 (E8P12TopKProvider, _topk_metric_select_impl).
#include "common.cuh"

namespace mpq {

constexpr int kMaxTopK = 64;

// Per coordinate: score(q) = (-0.5 g) (atom_q - r)^2 [- 0.5 (atom_q - W)^2 / (tau max(s, 1e-12))^2],
// atom_q = s (q - z); the k best atoms in descending score (ties: lower q first).
__global__ void k_uniform_topk(const float* __restrict__ r1, int64_t ld_r1, const float* __restrict__ center,
                               int64_t ld_c, const float* __restrict__ scale, const float* __restrict__ zero,
                               int64_t ld_p, int gshift, const float* __restrict__ gamma, int B, int n, int maxq,
                               float prior_tau, int k, int* __restrict__ out_q, float* __restrict__ out_v,
                               float* __restrict__ out_s) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * n) return;
  const int b = (int)(i / n), j = (int)(i % n);
  const float r = r1[b * ld_r1 + j];
  const float s = scale[b * ld_p + (j >> gshift)];
  const float z = zero[b * ld_p + (j >> gshift)];
  const float ng = fmul(-0.5f, gamma[b]);
  const bool prior = prior_tau > 0.f && center;
  const float c = prior ? center[b * ld_c + j] : 0.f;
  float tau2 = 1.f;
  if (prior) {
    const float st = fmul(prior_tau, fmaxf(s, 1e-12f));
    tau2 = fmul(st, st);
  }
  float bs[kMaxTopK];
  int bq[kMaxTopK];
  int cnt = 0;
  for (int q = 0; q <= maxq; ++q) {
    const float atom = fmul(s, fsub((float)q, z));
    const float d = fsub(atom, r);
    float sc = fmul(ng, fmul(d, d));
    if (prior) {
      const float dc = fsub(atom, c);
      sc = fsub(sc, fdiv(fmul(0.5f, fmul(dc, dc)), tau2));
    }
    // insert into the sorted list (strictly better only: earlier q wins ties)
    int pos = cnt < k ? cnt : k;
    while (pos > 0 && sc > bs[pos - 1]) --pos;
    if (pos < k) {
      for (int t = (cnt < k ? cnt : k - 1); t > pos; --t) {
        bs[t] = bs[t - 1];
        bq[t] = bq[t - 1];
      }
      bs[pos] = sc;
      bq[pos] = q;
      if (cnt < k) ++cnt;
    }
  }
  for (int t = 0; t < k; ++t) {
    const int q = bq[t];
    out_q[i * k + t] = q;
    out_v[i * k + t] = fmul(s, fsub((float)q, z));
    if (out_s) out_s[i * k + t] = bs[t];
  }
}

// The same selection for grids of L <= 32 levels, L lanes per coordinate: lane q scores level q, its output
// position is its rank  #{q' : s[q'] > s[q] or (s[q'] == s[q] and q' < q)}  (NaN scores rank last, so the ranks
// are a permutation), and the L lanes of a coordinate write its k outputs as one contiguous segment.
template <int L>
__global__ void k_uniform_topk_lanes(const float* __restrict__ r1, int64_t ld_r1, const float* __restrict__ center,
                                     int64_t ld_c, const float* __restrict__ scale, const float* __restrict__ zero,
                                     int64_t ld_p, int gshift, const float* __restrict__ gamma, int B, int n,
                                     float prior_tau, int k, int* __restrict__ out_q, float* __restrict__ out_v,
                                     float* __restrict__ out_s) {
  const int64_t gt = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t i = gt / L;
  const int q = (int)(gt % L);
  const bool valid = i < (int64_t)B * n;  // every lane takes part in the shuffles
  const int64_t ii = valid ? i : 0;
  const int b = (int)(ii / n), j = (int)(ii % n);
  const float r = r1[b * ld_r1 + j];
  const float s = scale[b * ld_p + (j >> gshift)];
  const float z = zero[b * ld_p + (j >> gshift)];
  const float ng = fmul(-0.5f, gamma[b]);
  const bool prior = prior_tau > 0.f && center;
  const float atom = fmul(s, fsub((float)q, z));
  const float d = fsub(atom, r);
  float sc = fmul(ng, fmul(d, d));
  if (prior) {
    const float st = fmul(prior_tau, fmaxf(s, 1e-12f));
    const float dc = fsub(atom, center[b * ld_c + j]);
    sc = fsub(sc, fdiv(fmul(0.5f, fmul(dc, dc)), fmul(st, st)));
  }
  const float key = sc != sc ? -INFINITY : sc;
  int rank = 0;
  #pragma unroll
  for (int p = 0; p < L; ++p) {
    const float kp = __shfl_sync(0xffffffffu, key, p, L);
    rank += (kp > key || (kp == key && p < q)) ? 1 : 0;
  }
  if (valid && rank < k) {
    out_q[i * k + rank] = q;
    out_v[i * k + rank] = atom;
    if (out_s) out_s[i * k + rank] = sc;
  }
}

// Per row: the candidate (of k, each bs floats) nearest to the row's target.  chol != null: metric distance
// |tL|^2 + |cL|^2 - 2 (tL).(cL) clamped at 0 (products and sums in index order); otherwise sum_j (c_j - t_j)^2.
// First minimum wins.  Writes the chosen values and, when cand_idx is given, its index.
__global__ void k_topk_pick(const float* __restrict__ target, int64_t ld_t, const float* __restrict__ cand,
                            int64_t ld_cand, const int* __restrict__ cand_idx, int64_t ld_ci, int B, int k, int bs,
                            const float* __restrict__ chol, float* __restrict__ out_v, int64_t ld_o,
                            int* __restrict__ out_idx) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  float t[8], tm[8];
  for (int j = 0; j < bs; ++j) t[j] = target[b * ld_t + j];
  float tn = 0.f;
  if (chol) {
    for (int j = 0; j < bs; ++j) {
      float acc = 0.f;
      for (int i = 0; i < bs; ++i) acc = fadd(acc, fmul(t[i], chol[i * bs + j]));
      tm[j] = acc;
    }
    for (int j = 0; j < bs; ++j) tn = fadd(tn, fmul(tm[j], tm[j]));
  }
  const float* cb = cand + b * ld_cand;
  float best = INFINITY;
  int bi = 0;
  for (int c = 0; c < k; ++c) {
    const float* cv = cb + c * bs;
    float dist;
    if (chol) {
      float cn = 0.f, cross = 0.f;
      for (int j = 0; j < bs; ++j) {
        float cm = 0.f;
        for (int i = 0; i < bs; ++i) cm = fadd(cm, fmul(cv[i], chol[i * bs + j]));
        cn = fadd(cn, fmul(cm, cm));
        cross = fadd(cross, fmul(cm, tm[j]));
      }
      dist = fmaxf(fsub(fadd(tn, cn), fmul(2.f, cross)), 0.f);
    } else {
      dist = 0.f;
      for (int j = 0; j < bs; ++j) {
        const float d = fsub(cv[j], t[j]);
        dist = fadd(dist, fmul(d, d));
      }
    }
    if (dist < best) {
      best = dist;
      bi = c;
    }
  }
  for (int j = 0; j < bs; ++j) out_v[b * ld_o + j] = cb[bi * bs + j];
  if (out_idx && cand_idx) out_idx[b] = cand_idx[b * ld_ci + bi];
}

}  // namespace mpq

using namespace mpq;

// k best atoms per coordinate (k <= 16): out_q / out_v / out_s are B x n x k (out_s may be NULL).
MPQ_API int mpq_uniform_topk(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* scale,
                             const float* zero, int64_t ld_p, int gshift, const float* gamma, int B, int n, int maxq,
                             float prior_tau, int k, int* out_q, float* out_v, float* out_s, void* stream) {
  MPQ_CHECK_ARG(B >= 0 && n >= 0, "mpq_uniform_topk: bad shape");
  MPQ_CHECK_ARG(maxq >= 1 && maxq <= 255, "mpq_uniform_topk: maxq must be in [1, 255]");
  MPQ_CHECK_ARG(k >= 1 && k <= kMaxTopK && k <= maxq + 1, "mpq_uniform_topk: k must be in [1, min(64, maxq + 1)]");
  if (B == 0 || n == 0) return MPQ_OK;
  MPQ_CHECK_ARG(r1 && scale && zero && gamma && out_q && out_v, "mpq_uniform_topk: null pointer");
  const int64_t total = (int64_t)B * n;
  const unsigned grid = (unsigned)((total + 255) / 256);
  cudaStream_t st = (cudaStream_t)stream;
#define MPQ_TOPK_LANES(L_)                                                                                    \
  k_uniform_topk_lanes<L_><<<(unsigned)((total * L_ + 255) / 256), 256, 0, st>>>(                             \
      r1, ld_r1, center, ld_c, scale, zero, ld_p, gshift, gamma, B, n, prior_tau, k, out_q, out_v, out_s)
  switch (maxq) {
    case 1: MPQ_TOPK_LANES(2); break;
    case 3: MPQ_TOPK_LANES(4); break;
    case 7: MPQ_TOPK_LANES(8); break;
    case 15: MPQ_TOPK_LANES(16); break;
    case 31: MPQ_TOPK_LANES(32); break;
    default:
      k_uniform_topk<<<grid, 256, 0, st>>>(r1, ld_r1, center, ld_c, scale, zero, ld_p, gshift, gamma, B, n, maxq,
                                           prior_tau, k, out_q, out_v, out_s);
  }
#undef MPQ_TOPK_LANES
  return launch_status("mpq_uniform_topk");
}

// Per-row nearest candidate (bs <= 8): see k_topk_pick.
MPQ_API int mpq_topk_pick(const float* target, int64_t ld_t, const float* cand, int64_t ld_cand, const int* cand_idx,
                          int64_t ld_ci, int B, int k, int bs, const float* chol, float* out_v, int64_t ld_o,
                          int* out_idx, void* stream) {
  MPQ_CHECK_ARG(B >= 0 && k >= 1 && bs >= 1 && bs <= 8, "mpq_topk_pick: bad shape (bs <= 8)");
  if (B == 0) return MPQ_OK;
  MPQ_CHECK_ARG(target && cand && out_v, "mpq_topk_pick: null pointer");
  k_topk_pick<<<(B + 127) / 128, 128, 0, (cudaStream_t)stream>>>(target, ld_t, cand, ld_cand, cand_idx, ld_ci, B, k,
                                                               bs, chol, out_v, ld_o, out_idx);
  return launch_status("mpq_topk_pick");
}
