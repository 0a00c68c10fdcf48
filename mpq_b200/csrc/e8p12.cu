// E8P12 factorized posterior (MMSE) and MAP search over the 2^16-entry E8P12 codebook.
//
// Reference: mpq/priors/e8p12.py:169-308 (_branch_factorized_stats_impl), :367-449
// (_branch_factorized_map), :541-631 (vamp_vector_map_e8p12), :815-968 (vamp_vector_discrete_mmse_e8p12);
// the QUIP# nearest-codeword call cb.quantize (mpq/adapters/quip_sharp.py:235) is the MAP at unit
// precision without prior.
//
// Every codeword is  offset(branch) + sign_pattern * abs_pattern  with 2 branches (+-1/4) x 256 abs
// patterns x the sign patterns of the abs pattern's parity.  Per 8-vector item (one thread):
//   pass 1  (exact)   for each of the 512 (branch, abs) components, the best parity-valid sign and
//                     its log-score  -0.5 g (|y|^2 + |b|^2) + sum|a_k| - 2 [parity mismatch] min|a_k|,
//                     a_k = (g y_k)|b_k|; argmax (first maximum) -> MAP codeword.  Float32 operations in
//                     the oracle's order, no FMA contraction: indices are bit-exact.
//   pass 2  (MMSE)    the component log-partition (tanh / logaddexp / log1mexp algebra of the
//                     reference) and its sign means, accumulated as an online softmax (running maximum,
//                     as the reference's logsumexp).  The reference clamps tanh at 1 - 1e-7, so for large
//                     |a| with a parity mismatch its log-partition exceeds the component's MAP score by up
//                     to ~2 min|a|; the running maximum keeps that finite.  Components whose upper bound
//                     const + sum|a_k| + 8 ln 2 lies more than 30 below the running maximum are skipped
//                     (weight < e^-30 of the largest; the bound holds for the clamped formula too).
// One CTA per row; per-row variance sums are reduced in a fixed order.
#include "common.cuh"

namespace mpq {

struct E8Tab {
  const float* base_abs;    // 256 x 8
  const float* base_sqnorm; // 256
  const int* base_parity;   // 256
  const int* idx_lut;       // 2 x 256 x 256
  const float* grid;        // 65536 x 8
};

struct E8Args {
  const float* r1; int64_t ld_r1;       // B x n (n = 8 * nb)
  const float* center; int64_t ld_c;    // prior centre (W) or null
  const float* pscale; int64_t ld_s;    // per-block prior scale (B x nb) or null (= absmax of the centre block)
  const float* gamma;                   // (B) channel precision gamma1
  float prior_tau;                      // <= 0: no prior
  float fixed_gamma;                    // > 0: use this precision for every item (nearest-codeword mode)
  int B; int nb;
};

constexpr float kLn2 = 0.69314718055994530942f;
constexpr float kPrune = 30.f;

// Folded message and precision of one item (mpq/priors/e8p12.py:844-857).
__device__ __forceinline__ void fold_item(const E8Args& a, int b, int k, float y[8], float& g, float& g1) {
  const float* rp = a.r1 + b * a.ld_r1 + k * 8;
  #pragma unroll
  for (int i = 0; i < 8; ++i) y[i] = rp[i];
  g1 = a.fixed_gamma > 0.f ? a.fixed_gamma : a.gamma[b];
  g = g1;
  if (a.prior_tau > 0.f && a.center) {
    const float* cp = a.center + b * a.ld_c + k * 8;
    float c[8];
    float sc = 0.f;
    #pragma unroll
    for (int i = 0; i < 8; ++i) {
      c[i] = cp[i];
      sc = fmaxf(sc, fabsf(c[i]));
    }
    if (a.pscale) sc = a.pscale[b * a.ld_s + k];
    sc = fmaxf(sc, 1e-12f);
    const float t = fmul(fmaxf(a.prior_tau, 1e-12f), sc);
    const float pp = fdiv(1.f, fmul(t, t));
    const float gw = fadd(g1, pp);
    #pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = fdiv(fadd(fmul(g1, y[i]), fmul(pp, c[i])), gw);
    g = gw;
  }
}

// Pass 1 over one component: exact MAP log-score and the parity-fixed sign id.
__device__ __forceinline__ float comp_map(const float gy[8], const float* ab, float ng, float ynorm, float sqn,
                                          int bpar, int& sid, float& sum_abs_out) {
  float sum_abs = 0.f, mn = INFINITY;
  int neg = 0, par = 0, minpos = 0;
  #pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float av = fmul(gy[i], ab[i]);
    const float aa = fabsf(av);
    sum_abs = fadd(sum_abs, aa);
    if (av < 0.f) { neg |= 1 << i; par ^= 1; }
    if (aa < mn) { mn = aa; minpos = i; }
  }
  const bool mismatch = par != bpar;
  sid = mismatch ? (neg ^ (1 << minpos)) : neg;
  const float lin = mismatch ? fsub(sum_abs, fmul(2.f, mn)) : fsub(sum_abs, 0.f);
  sum_abs_out = sum_abs;
  return fadd(fmul(ng, fadd(ynorm, sqn)), lin);
}

__device__ __forceinline__ float log1mexp_f(float x) {  // log(1 - exp(x)), x <= 0, float32 steps as the reference
  return x < -kLn2 ? (float)log1p(-(double)(float)exp((double)x)) : (float)log(-(double)(float)expm1((double)x));
}

template <bool MMSE>
__global__ void __launch_bounds__(128) k_e8p12(E8Args a, E8Tab tab, float* __restrict__ x1_out, int64_t ld_x,
                                               float* __restrict__ var_out, int64_t ld_v, int* __restrict__ idx_out,
                                               int64_t ld_i, float* __restrict__ map_out, int64_t ld_m,
                                               float* __restrict__ var_rowsum) {
  __shared__ float s_abs[256 * 8];
  __shared__ float s_sqn[256];
  __shared__ int s_par[256];
  __shared__ float red[32];
  for (int i = threadIdx.x; i < 256 * 8; i += blockDim.x) s_abs[i] = tab.base_abs[i];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) {
    s_sqn[i] = tab.base_sqnorm[i];
    s_par[i] = tab.base_parity[i];
  }
  __syncthreads();
  const int b = blockIdx.x;
  float vacc = 0.f;
  for (int k = threadIdx.x; k < a.nb; k += blockDim.x) {
    float y[8], g, g1;
    fold_item(a, b, k, y, g, g1);
    const float ng = fmul(-0.5f, g);
    // ---- pass 1: exact MAP ----
    float best = -INFINITY;
    int best_comp = 0, best_sid = 0;
    float yb[2][8], ynorm[2];
    #pragma unroll
    for (int br = 0; br < 2; ++br) {
      const float off = br ? -0.25f : 0.25f;
      float yn = 0.f;
      #pragma unroll
      for (int i = 0; i < 8; ++i) {
        yb[br][i] = fsub(y[i], off);
        yn = fadd(yn, fmul(yb[br][i], yb[br][i]));
      }
      ynorm[br] = yn;
      float gy[8];
      #pragma unroll
      for (int i = 0; i < 8; ++i) gy[i] = fmul(g, yb[br][i]);
      for (int ai = 0; ai < 256; ++ai) {
        int sid;
        float sa;
        const float sc = comp_map(gy, s_abs + ai * 8, ng, yn, s_sqn[ai], s_par[ai], sid, sa);
        if (sc > best) { best = sc; best_comp = br * 256 + ai; best_sid = sid; }
      }
    }
    const int map_idx = tab.idx_lut[(best_comp >> 8) * 65536 + (best_comp & 255) * 256 + best_sid];
    if (idx_out) idx_out[b * ld_i + k] = map_idx;
    const float* mv = tab.grid + (int64_t)map_idx * 8;
    if (map_out) {
      #pragma unroll
      for (int i = 0; i < 8; ++i) map_out[b * ld_m + k * 8 + i] = mv[i];
    }
    if constexpr (MMSE) {
      // ---- pass 2: factorized posterior mean / second moment ----
      float W = 0.f, SEC = 0.f, MU[8];
      float mx = best;  // running maximum of the component log-weights (starts at the MAP lower bound)
      #pragma unroll
      for (int i = 0; i < 8; ++i) MU[i] = 0.f;
      #pragma unroll 1
      for (int br = 0; br < 2; ++br) {
        const float off = br ? -0.25f : 0.25f;
        #pragma unroll 1
        for (int ai = 0; ai < 256; ++ai) {
          const float* ab = s_abs + ai * 8;
          float av[8], sum_abs = 0.f;
          #pragma unroll
          for (int i = 0; i < 8; ++i) {
            av[i] = (g * yb[br][i]) * ab[i];
            sum_abs += fabsf(av[i]);
          }
          const float cst = ng * (ynorm[br] + s_sqn[ai]);
          if (cst + sum_abs + 8.f * kLn2 < mx - kPrune) continue;
          // Transcendentals are evaluated in double and rounded once (correctly rounded float32 results):
          // the reference's clamped-tanh algebra amplifies last-bit differences of tanh near +-1.
          float logC = 0.f, lpt = 0.f, t[8];
          int negp = 0;
          #pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float aa = fabsf(av[i]);
            logC += aa + (float)log1p((double)(float)exp(-2.0 * (double)aa));
            float ti = (float)tanh((double)av[i]);
            ti = fminf(fmaxf(ti, -0.99999988079071044921875f), 0.99999988079071044921875f);
            t[i] = ti;
            lpt += (float)log((double)fmaxf(fabsf(ti), 1e-7f));
            negp ^= (ti < 0.f) ? 1 : 0;
          }
          const float pabs = (float)exp((double)lpt);
          const float prod = negp ? -pabs : pabs;
          const float lae = (float)log1p((double)(float)exp((double)lpt));  // logaddexp(0, lpt), lpt <= 0
          const float l1me = log1mexp_f(lpt);
          const float lop = negp ? l1me : lae;   // log(1 + prod)
          const float lom = negp ? lae : l1me;   // log(1 - prod)
          const bool even = s_par[ai] == 0;
          const float logZ = logC + (even ? lop : lom) - kLn2;
          const float lc = cst + logZ;
          if (lc > mx) {  // rescale the accumulators to the new maximum
            const float sc = expf(mx - lc);
            W *= sc;
            SEC *= sc;
            #pragma unroll
            for (int i = 0; i < 8; ++i) MU[i] *= sc;
            mx = lc;
          }
          const float w = (float)exp((double)(lc - mx));
          float de = 1.f + prod, dodd = 1.f - prod;
          if (!(fabsf(de) > 1e-12f)) de = 1.f;
          if (!(fabsf(dodd) > 1e-12f)) dodd = 1.f;
          float pre[8];
          float acc = 1.f;
          #pragma unroll
          for (int i = 0; i < 8; ++i) { pre[i] = acc; acc *= t[i]; }
          float suf = 1.f, mcs = 0.f, mc[8];
          #pragma unroll
          for (int i = 7; i >= 0; --i) {
            const float ex = pre[i] * suf;
            float sm = even ? (t[i] + ex) / de : (t[i] - ex) / dodd;
            if (!isfinite(sm)) sm = 0.f;
            mc[i] = sm * ab[i];
            mcs += mc[i];
            suf *= t[i];
          }
          W += w;
          #pragma unroll
          for (int i = 0; i < 8; ++i) MU[i] += w * (mc[i] + off);
          SEC += w * (s_sqn[ai] + 8.f * off * off + 2.f * off * mcs);
        }
      }
      float mu[8], var;
      if (g >= 1e3f) {  // high-precision snap to the MAP codeword (mpq/priors/e8p12.py:923-926)
        #pragma unroll
        for (int i = 0; i < 8; ++i) mu[i] = mv[i];
        var = 0.f;
      } else {
        float nrm = 0.f;
        #pragma unroll
        for (int i = 0; i < 8; ++i) {
          mu[i] = MU[i] / W;
          nrm += mu[i] * mu[i];
        }
        var = fmaxf((SEC / W - nrm) / 8.f, 0.f);
      }
      #pragma unroll
      for (int i = 0; i < 8; ++i) x1_out[b * ld_x + k * 8 + i] = mu[i];
      if (var_out) var_out[b * ld_v + k] = var;
      vacc += var;
    }
  }
  if constexpr (MMSE) {
    const float tsum = block_sum(vacc, red);
    if (threadIdx.x == 0 && var_rowsum) var_rowsum[b] = tsum;
  }
}

}  // namespace mpq

using namespace mpq;

static int e8_check(const float* r1, int B, int nb, const float* base_abs, const float* base_sqnorm,
                    const int* base_parity, const int* idx_lut, const float* grid) {
  MPQ_CHECK_ARG(r1 && base_abs && base_sqnorm && base_parity && idx_lut && grid, "e8p12: null pointer");
  MPQ_CHECK_ARG(B >= 0 && nb >= 0 && B <= 2147483647, "e8p12: bad shape");
  return MPQ_OK;
}

// Factorized posterior (MMSE): x1 (B x 8nb), optional var (B x nb), MAP idx (B x nb) and values, and the
// per-row variance sum (alpha1 = gamma1 * var_rowsum / nb).
MPQ_API int mpq_e8p12_mmse(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* pscale,
                           int64_t ld_s, const float* gamma, float prior_tau, int B, int nb, const float* base_abs,
                           const float* base_sqnorm, const int* base_parity, const int* idx_lut, const float* grid,
                           float* x1_out, int64_t ld_x, float* var_out, int64_t ld_v, int* idx_out, int64_t ld_i,
                           float* map_out, int64_t ld_m, float* var_rowsum, void* stream) {
  int st = e8_check(r1, B, nb, base_abs, base_sqnorm, base_parity, idx_lut, grid);
  if (st) return st;
  MPQ_CHECK_ARG(gamma && x1_out && var_rowsum, "mpq_e8p12_mmse: gamma, x1_out and var_rowsum are required");
  if (B == 0 || nb == 0) return MPQ_OK;
  E8Args a{r1, ld_r1, center, ld_c, pscale, ld_s, gamma, prior_tau, 0.f, B, nb};
  E8Tab t{base_abs, base_sqnorm, base_parity, idx_lut, grid};
  k_e8p12<true><<<B, 128, 0, (cudaStream_t)stream>>>(a, t, x1_out, ld_x, var_out, ld_v, idx_out, ld_i, map_out, ld_m,
                                                    var_rowsum);
  return launch_status("mpq_e8p12_mmse");
}

// MAP codeword under the folded message (fixed_gamma > 0 replaces gamma for every row, e.g. 1 with no
// prior = nearest codeword / RTN).
MPQ_API int mpq_e8p12_map(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* pscale,
                          int64_t ld_s, const float* gamma, float fixed_gamma, float prior_tau, int B, int nb,
                          const float* base_abs, const float* base_sqnorm, const int* base_parity, const int* idx_lut,
                          const float* grid, int* idx_out, int64_t ld_i, float* map_out, int64_t ld_m, void* stream) {
  int st = e8_check(r1, B, nb, base_abs, base_sqnorm, base_parity, idx_lut, grid);
  if (st) return st;
  MPQ_CHECK_ARG(gamma || fixed_gamma > 0.f, "mpq_e8p12_map: gamma or fixed_gamma required");
  if (B == 0 || nb == 0) return MPQ_OK;
  E8Args a{r1, ld_r1, center, ld_c, pscale, ld_s, gamma, prior_tau, fixed_gamma, B, nb};
  E8Tab t{base_abs, base_sqnorm, base_parity, idx_lut, grid};
  k_e8p12<false><<<B, 128, 0, (cudaStream_t)stream>>>(a, t, nullptr, 0, nullptr, 0, idx_out, ld_i, map_out, ld_m,
                                                     nullptr);
  return launch_status("mpq_e8p12_map");
}
