// E8P12 factorized posterior (MMSE) and MAP search over the 2^16-entry E8P12 codebook.
//
// Reference: mpq/priors/e8p12.py:169-308 (_branch_factorized_stats_impl), :367-449
// (_branch_factorized_map), :541-631 (vamp_vector_map_e8p12), :815-968 (vamp_vector_discrete_mmse_e8p12);
// the QUIP# nearest-codeword call cb.quantize (mpq/adapters/quip_sharp.py:235) is the MAP at unit
// precision without prior.
//
// Every codeword is  offset(branch) + sign_pattern * abs_pattern  with 2 branches (+-1/4) x 256 abs
// patterns x the sign patterns of the abs pattern's parity.  The abs patterns' coordinates only take the
// magnitudes 1/2, 3/2 and 5/2, so for one item and branch every per-coordinate quantity of the reference's
// factorized formulas (a_k = (g y_k) |b_k|, logaddexp(a_k, -a_k), the clamped tanh and its log) takes one
// of 8 x 3 values.  Each item is handled by one warp, which first evaluates those 2 x 24 entries once
// (the same float32 operations the reference applies per component, so every per-component value is
// bit-identical to the undeduplicated evaluation) and then scores the 512 (branch, abs) components with
// table look-ups:
//   pass 1  (exact)   each lane scores 16 components: the best parity-valid sign and its log-score
//                     -0.5 g (|y|^2 + |b|^2) + sum|a_k| - 2 [parity mismatch] min|a_k| (float32, the
//                     reference's order, no FMA contraction); a warp reduction on (score, component) gives
//                     the first maximum -> MAP codeword, bit-exact.
//   pass 2  (MMSE)    components whose upper bound const + logC (logZ = logC + log(1 +- prod) - ln 2 <=
//                     logC) lies more than kPrune = 20 below the MAP score are dropped (weight < e^-20 of
//                     the largest); the survivors are compacted with a warp ballot and spread over the lanes,
//                     each lane accumulating an online softmax (running maximum, as the reference's
//                     logsumexp) of the component log-partitions and sign means; the lanes' partial sums
//                     are merged in a fixed butterfly order.  The reference clamps tanh at 1 - 1e-7, so for
//                     large |a| with a parity mismatch its log-partition exceeds the component's MAP score by
//                     up to ~2 min|a|; the running maximum keeps that finite.
// Items with g >= 1e3 take the MAP codeword with zero variance (the reference's snap) and skip pass 2.
// One CTA of 8 warps per row; per-row variance sums are reduced in a fixed order.
#include <algorithm>

#include "common.cuh"
#include "vamp_rows.cuh"

namespace mpq {

struct E8Tab {
  const float* base_abs;    // 256 x 8
  const float* base_sqnorm; // 256
  const int* base_parity;   // 256
  const int* idx_lut;       // 2 x 256 x 256
  const float* grid;        // 65536 x 8
};

// Row split of the posterior launch (several CTAs per row when rows are few) and device-side launch control.
struct RowSplit {
  float* part;           // B x chunks per-chunk variance sums (chunks > 1)
  unsigned* counters;    // B arrival counters, zero between launches (chunks > 1)
  const int* active;     // optional: the launch does nothing while *active == 0
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
// Components whose log-weight bound lies more than kPrune below the MAP score are dropped: each weighs
// < e^-20 of the largest; on the 4096 x 4096 E8P12 layer solve the dropped posterior mass stays below 5e-8
// of the total (float32 resolution) in every item and iteration.
constexpr float kPrune = 20.f;

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

constexpr int kWarps = 8;  // items in flight per CTA (one warp each)

// 4-byte asynchronous global -> shared copies (cp.async, cached at L1), one commit group per call site.
__device__ __forceinline__ void async_copy4(float* dst, const float* src) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// Per-item table of the per-(branch, coordinate k, magnitude m) values, entry e = 3 k + m.  Signs are
// canonical (a value that is not < 0 has its sign bit clear), so the XOR of sign bits is the parity of
// the reference's (x < 0) tests.
struct ItemTab {
  float2 am[2][24];  // {a, T}: a = (g (y_k - off)) |b| with |b| = 1/2, 3/2, 5/2; T = |a| + log1p(exp(-2|a|))
  float4 pt[2][24];  // {T, t, lt, |b|}: t = tanh(a) clamped to +-(1 - 2^-23), lt = log(max(|t|, 1e-7))
  float tb[24][2];   // {T of branch 0, T of branch 1} per entry: the bound pass reads both branches in one load
};

// Folded message of one item with the work spread over the warp (the posterior kernel): lane l holds
// coordinate l & 7 of r1 (yv) and of the prior centre (cv), every lane the item's prior scale (sv, when given)
// and the row's precision g1.  The same float32 operations as fold_item per coordinate, so the folded y and the
// precision are bit-identical.  Every group of 8 lanes holds the item's 8 coordinates (lane l: coordinate
// l & 7); returns the lane's coordinate of the folded y.
__device__ __forceinline__ float fold_item_lanes(const E8Args& a, bool prior, float yv, float cv, float sv, float g1,
                                                 float& g) {
  float yl = yv;
  g = g1;
  if (prior) {
    // max |c| over the block (fmaxf is exact in any order; a NaN entry is skipped as in the sequential scan)
    float sc = fmaxf(0.f, fabsf(cv));
    #pragma unroll
    for (int o = 4; o > 0; o >>= 1) sc = fmaxf(sc, __shfl_xor_sync(0xffffffffu, sc, o));
    if (a.pscale) sc = sv;
    sc = fmaxf(sc, 1e-12f);
    const float t = fmul(fmaxf(a.prior_tau, 1e-12f), sc);
    const float pp = fdiv(1.f, fmul(t, t));
    const float gw = fadd(g1, pp);
    yl = fdiv(fadd(fmul(g1, yv), fmul(pp, cv)), gw);
    g = gw;
  }
  return yl;
}

__device__ __forceinline__ float canon_sign(float x) { return x < 0.f ? x : fabsf(x); }
__device__ __forceinline__ unsigned sign_bit(float x) { return __float_as_uint(x) >> 31; }

// One component's log-weight from the item table: lc = const + logC + log(1 +- prod) - ln 2 (the reference's
// clamped-tanh formula), with the per-coordinate t and |b| and the products the sign means need.
struct CompTerms {
  float lc, prod, t[8], mag[8];
  bool even;
};

__device__ __forceinline__ void comp_terms(const ItemTab& T, int br, int ai, uint2 of, float ng, float ynorm_br,
                                           float sqn, int parity, CompTerms& o) {
  const char* base = reinterpret_cast<const char*>(T.pt[br]);
  float logC = 0.f, lpt = 0.f;
  unsigned sx = 0;
  #pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const unsigned byte = __byte_perm(kk < 4 ? of.x : of.y, 0u, 0x4440u + (kk & 3));
    const float4 v = *reinterpret_cast<const float4*>(base + 2u * byte);
    logC = fadd(logC, v.x);
    o.t[kk] = v.y;
    sx ^= __float_as_uint(v.y);
    lpt = fadd(lpt, v.z);
    o.mag[kk] = v.w;
  }
  const bool negp = (sx >> 31) != 0u;
  const float cst = fmul(ng, fadd(ynorm_br, sqn));
  // Hardware exp2/log2 approximations (relative error ~2^-21): a component's log-weight lc is O(10^2-10^3) in
  // magnitude, so its own float32 rounding (~1e-5) exceeds their error.  The only ill-conditioned term,
  // 1 - |prod| for |prod| near 1, is evaluated through expm1f and belongs to parity-mismatched components whose
  // log-partition lies ~14 nats below their bound (the reference's tanh clamp).
  const float pabs = __expf(lpt);
  o.prod = negp ? -pabs : pabs;
  const float lae = __logf(1.f + pabs);  // logaddexp(0, lpt), lpt <= 0: 1 + pabs in (1, 2]
  float l1me;  // log(1 - exp(lpt)); a branch, so expm1f runs only for the lanes that need it
  if (lpt < -kLn2) l1me = __logf(1.f - pabs);
  else l1me = __logf(-expm1f(lpt));
  const float lop = negp ? l1me : lae;  // log(1 + prod)
  const float lom = negp ? lae : l1me;  // log(1 - prod)
  o.even = parity == 0;
  o.lc = fadd(cst, fsub(fadd(logC, o.even ? lop : lom), kLn2));
}

// Stages the 256 abs patterns in shared memory: s_off[ai] packs byte k = 8 (3 k + m_k), the offset of coordinate
// k's 8-byte table entry (magnitude index m_k of 1/2, 3/2, 5/2).  Returns true (for every thread) when base_abs
// holds any other magnitude, i.e. is not an E8P12 abs table.
__device__ __forceinline__ bool stage_abs_patterns(const E8Tab& tab, uint2* s_off, float* s_sqn, int* s_par,
                                                   int* s_bad) {
  if (threadIdx.x == 0) *s_bad = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += blockDim.x) {
    unsigned lo = 0, hi = 0;
    #pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float v = tab.base_abs[i * 8 + k];
      const unsigned m = v == 0.5f ? 0u : v == 1.5f ? 1u : v == 2.5f ? 2u : 3u;
      if (m == 3u) *s_bad = 1;
      const unsigned byte = 8u * (3u * k + (m & 3u));
      if (k < 4) lo |= byte << (8 * k); else hi |= byte << (8 * (k - 4));
    }
    s_off[i] = make_uint2(lo, hi);
    s_sqn[i] = tab.base_sqnorm[i];
    s_par[i] = tab.base_parity[i];
  }
  __syncthreads();
  return *s_bad != 0;
}

// Optional row stage fused behind the posterior (on = 1): the CTA that completes row b's variance sum runs the
// VAMP row stage of row b (vamp_row_stage, threads 0 .. kRowThreads - 1), so a retry round is one launch instead of
// a posterior launch and a row-stage launch.
struct RowsFuse {
  int on;
  RowState st;
  const float* S;
  int n, n_var, R;
  float damping;
  int final_retry;
  const VampCtl* ctl;
  RoundCtl rc;
};

template <bool MMSE>
__global__ void __launch_bounds__(kWarps * 32, 4)
k_e8p12(E8Args a, E8Tab tab, float* __restrict__ x1_out, int64_t ld_x, float* __restrict__ var_out, int64_t ld_v,
        int* __restrict__ idx_out, int64_t ld_i, float* __restrict__ map_out, int64_t ld_m,
        float* __restrict__ var_rowsum, RowSplit rs, RowsFuse fz) {
  // s_off[ai]: byte k of the pair = 8 * (3 k + m_k), the offset of coordinate k's float2 entry
  __shared__ uint2 s_off[256];
  __shared__ float s_sqn[256];
  __shared__ int s_par[256];
  __shared__ ItemTab s_tab[kWarps];
  __shared__ unsigned short s_list[MMSE ? kWarps : 1][512];
  __shared__ float s_ub[MMSE ? kWarps : 1][512];
  __shared__ float s_var[kWarps];
  __shared__ float s_stage[kWarps][17];
  __shared__ int s_bad;
  if (rs.active && *rs.active == 0) return;  // device-side control: this launch is not needed
  const bool bad = stage_abs_patterns(tab, s_off, s_sqn, s_par, &s_bad);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x;
  // items [k0, k1) of row b: the row is cut into gridDim.y contiguous chunks (one CTA each)
  const int k0 = (int)((int64_t)a.nb * blockIdx.y / gridDim.y), k1 = (int)((int64_t)a.nb * (blockIdx.y + 1) / gridDim.y);
  ItemTab& T = s_tab[warp];
  float vacc = 0.f;
  // The next item's r1 (lanes 0-7), prior centre (lanes 8-15) and prior scale (lane 16) are copied into the
  // warp's staging slot with asynchronous copies while the current item is scored, so their latency is hidden
  // behind the item's arithmetic without holding registers.
  const bool prior = a.prior_tau > 0.f && a.center;
  float* stage = s_stage[warp];
  if ((lane >= 8 && lane < 16 && !prior) || (lane == 16 && !(prior && a.pscale))) stage[lane] = 0.f;
  auto prefetch = [&](int kn) {
    if (kn < k1) {
      const float* src = nullptr;
      if (lane < 8) src = a.r1 + b * a.ld_r1 + kn * 8 + lane;
      else if (lane < 16 && prior) src = a.center + b * a.ld_c + kn * 8 + (lane - 8);
      else if (lane == 16 && prior && a.pscale) src = a.pscale + b * a.ld_s + kn;
      if (src) async_copy4(stage + lane, src);
    }
    async_commit();
  };
  prefetch(k0 + warp);
  for (int k = k0 + warp; k < k1; k += kWarps) {
    async_wait_all();
    __syncwarp();
    const float yv = stage[lane & 7], cv = stage[8 + (lane & 7)], sv = stage[16];
    __syncwarp();
    prefetch(k + kWarps);
    float g;
    const float yl = fold_item_lanes(a, prior, yv, cv, sv, a.fixed_gamma > 0.f ? a.fixed_gamma : a.gamma[b], g);
    if (bad) {  // base_abs is not an E8P12 abs table: poison the outputs
      if (lane == 0 && idx_out) idx_out[b * ld_i + k] = -1;
      if (lane < 8) {
        if (map_out) map_out[b * ld_m + k * 8 + lane] = __int_as_float(0x7fc00000);
        if (MMSE) x1_out[b * ld_x + k * 8 + lane] = __int_as_float(0x7fc00000);
      }
      if (MMSE && lane == 0) {
        if (var_out) var_out[b * ld_v + k] = __int_as_float(0x7fc00000);
        vacc = __int_as_float(0x7fc00000);
      }
      continue;
    }
    const float ng = fmul(-0.5f, g);
    float ynorm[2] = {0.f, 0.f};
    #pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float yi = __shfl_sync(0xffffffffu, yl, i);
      ynorm[0] = fadd(ynorm[0], fmul(fsub(yi, 0.25f), fsub(yi, 0.25f)));
      ynorm[1] = fadd(ynorm[1], fmul(fsub(yi, -0.25f), fsub(yi, -0.25f)));
    }
    // the coordinates of the lane's table entries e = lane and e = lane + 32 (coordinate (e mod 24) / 3)
    const float yk_a = __shfl_sync(0xffffffffu, yl, (lane < 24 ? lane : lane - 24) / 3);
    const float yk_b = __shfl_sync(0xffffffffu, yl, min((lane + 8) / 3, 7));
    // ---- per-item table ----
    __syncwarp();
    #pragma unroll 1
    for (int e = lane; e < 48; e += 32) {
      const int br = e / 24, r = e - br * 24, m = r % 3;
      const float yk = e < 32 ? yk_a : yk_b;
      const float off = br ? -0.25f : 0.25f;
      const float mag = 0.5f + (float)m;
      const float av = fmul(fmul(g, fsub(yk, off)), mag);
      const float aa = fabsf(av);
      float Tv = 0.f;
      if constexpr (MMSE) {
        // tanh and its log are evaluated in double and rounded once (correctly rounded float32 results): the
        // reference's clamped-tanh algebra amplifies last-bit differences of tanh near +-1.  The logaddexp
        // term is well conditioned.
        Tv = aa + log1pf(expf(-2.f * aa));
        const float ti =
            fminf(fmaxf((float)tanh((double)av), -0.99999988079071044921875f), 0.99999988079071044921875f);
        T.pt[br][r] = make_float4(Tv, canon_sign(ti), (float)log((double)fmaxf(fabsf(ti), 1e-7f)), mag);
      }
      T.am[br][r] = make_float2(canon_sign(av), Tv);
      T.tb[r][br] = Tv;
    }
    __syncwarp();
    // Lane's components c = 32 j + lane = (branch c >> 8, abs c & 255), the reference's component order.
    // The exact MAP scan runs when MAP outputs are requested, for MAP-only calls and for items that snap to
    // the MAP codeword (g >= 1e3); otherwise only the bounds const + logC are needed, and the pruning
    // reference is the largest exact log-weight among the lanes' best-bound components.
    const bool need_map = !MMSE || idx_out != nullptr || map_out != nullptr || g >= 1e3f;
    float best = -INFINITY;  // lower bound on the largest component log-weight
    const float* mv = nullptr;
    if (need_map) {
      // ---- pass 1: exact MAP (both branches of an abs pattern share its coordinate offsets; ties keep the
      // smaller component, so the lane's candidate is its first maximum in component order) ----
      int best_c = -1;
      #pragma unroll 1
      for (int j = 0; j < 8; ++j) {
        const int ai = (j << 5) | lane;
        const uint2 of = s_off[ai];
        const char* base = reinterpret_cast<const char*>(T.am[0]);
        float sum_abs[2] = {0.f, 0.f}, mn[2] = {INFINITY, INFINITY}, lcs[2] = {0.f, 0.f};
        unsigned sx[2] = {0u, 0u};
        #pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const unsigned byte = __byte_perm(kk < 4 ? of.x : of.y, 0u, 0x4440u + (kk & 3));
          const float2* e = reinterpret_cast<const float2*>(base + byte);
          #pragma unroll
          for (int br = 0; br < 2; ++br) {
            const float2 v = e[24 * br];  // the same coordinate and magnitude in branch br
            const float aa = fabsf(v.x);
            sum_abs[br] = fadd(sum_abs[br], aa);
            sx[br] ^= __float_as_uint(v.x);
            mn[br] = fminf(mn[br], aa);
            if constexpr (MMSE) lcs[br] = fadd(lcs[br], v.y);
          }
        }
        const float sq = s_sqn[ai];
        const int par = s_par[ai];
        #pragma unroll
        for (int br = 0; br < 2; ++br) {
          const bool mismatch = (int)(sx[br] >> 31) != par;
          const float lin = mismatch ? fsub(sum_abs[br], fmul(2.f, mn[br])) : sum_abs[br];
          const float cst = fmul(ng, fadd(ynorm[br], sq));
          const float sc = fadd(cst, lin);
          const int c = (j + 8 * br) * 32 + lane;
          if (sc > best || (sc == best && best_c >= 0 && c < best_c)) { best = sc; best_c = c; }
          if constexpr (MMSE) s_ub[warp][c] = fadd(cst, lcs[br]);
        }
      }
      // first maximum over the warp: valid before invalid, higher score, then smaller component
      #pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oc = __shfl_xor_sync(0xffffffffu, best_c, o);
        const bool take = oc >= 0 && (best_c < 0 || ob > best || (ob == best && oc < best_c));
        if (take) { best = ob; best_c = oc; }
      }
      int comp = 0, sid = 0;
      if (best_c >= 0) {  // the winner's parity-fixed sign pattern (first minimum of |a| flips)
        comp = best_c;
        const int br = comp >> 8, ai = comp & 255;
        const uint2 of = s_off[ai];
        const char* base = reinterpret_cast<const char*>(T.am[br]);
        float mn = INFINITY;
        int neg = 0, par = 0, minpos = 0;
        #pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const unsigned byte = __byte_perm(kk < 4 ? of.x : of.y, 0u, 0x4440u + (kk & 3));
          const float av = reinterpret_cast<const float2*>(base + byte)->x;
          const float aa = fabsf(av);
          if (av < 0.f) { neg |= 1 << kk; par ^= 1; }
          if (aa < mn) { mn = aa; minpos = kk; }
        }
        sid = par != s_par[ai] ? (neg ^ (1 << minpos)) : neg;
      }
      const int map_idx = tab.idx_lut[(comp >> 8) * 65536 + (comp & 255) * 256 + sid];
      if (lane == 0 && idx_out) idx_out[b * ld_i + k] = map_idx;
      mv = tab.grid + (int64_t)map_idx * 8;
      if (map_out && lane < 8) map_out[b * ld_m + k * 8 + lane] = mv[lane];
    } else if constexpr (MMSE) {
      // ---- pass 1: bounds only (both branches of an abs pattern share its coordinate offsets) ----
      float bub = -INFINITY;
      int bc = -1;
      #pragma unroll 1
      for (int j = 0; j < 8; ++j) {
        const int ai = (j << 5) | lane;
        const uint2 of = s_off[ai];
        const char* base = reinterpret_cast<const char*>(T.tb);  // 8-byte entries, as T.am[br]
        float l0 = 0.f, l1 = 0.f;
        #pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const unsigned byte = __byte_perm(kk < 4 ? of.x : of.y, 0u, 0x4440u + (kk & 3));
          const float2 v = *reinterpret_cast<const float2*>(base + byte);  // T of both branches
          l0 = fadd(l0, v.x);
          l1 = fadd(l1, v.y);
        }
        const float sq = s_sqn[ai];
        const float ub0 = fadd(fmul(ng, fadd(ynorm[0], sq)), l0);
        const float ub1 = fadd(fmul(ng, fadd(ynorm[1], sq)), l1);
        s_ub[warp][j * 32 + lane] = ub0;
        s_ub[warp][(j + 8) * 32 + lane] = ub1;
        if (ub0 > bub) { bub = ub0; bc = j * 32 + lane; }
        if (ub1 > bub) { bub = ub1; bc = (j + 8) * 32 + lane; }
      }
      // exact log-weight of each lane's best-bound component; the warp maximum is the pruning reference
      float lcb = -INFINITY;
      if (bc >= 0) {
        CompTerms ct;
        const int br = bc >> 8, ai = bc & 255;
        comp_terms(T, br, ai, s_off[ai], ng, br ? ynorm[1] : ynorm[0], s_sqn[ai], s_par[ai], ct);
        if (ct.lc == ct.lc) lcb = ct.lc;
      }
      #pragma unroll
      for (int o = 16; o > 0; o >>= 1) lcb = fmaxf(lcb, __shfl_xor_sync(0xffffffffu, lcb, o));
      best = lcb;
    }
    if constexpr (MMSE) {
      float mu_l = 0.f, var = 0.f;  // lane l < 8 ends with coordinate l of the posterior mean
      if (g >= 1e3f) {  // high-precision snap to the MAP codeword (mpq/priors/e8p12.py:923-926)
        mu_l = lane < 8 ? mv[lane] : 0.f;
      } else {
        // ---- pass 2: compact the surviving components (bound within kPrune of the reference) ----
        const float thr = best - kPrune;
        unsigned short* list = s_list[warp];
        int cnt = 0;
        #pragma unroll
        for (int j = 0; j < 16; ++j) {
          const bool keep = !(s_ub[warp][j * 32 + lane] < thr);
          const unsigned msk = __ballot_sync(0xffffffffu, keep);
          if (keep) list[cnt + __popc(msk & ((1u << lane) - 1u))] = (unsigned short)(j * 32 + lane);
          cnt += __popc(msk);
        }
        __syncwarp();
        float W = 0.f, WOFF = 0.f, SEC = 0.f, MU[8];
        float mx = best;  // running maximum of the component log-weights (starts at the pruning reference)
        #pragma unroll
        for (int i = 0; i < 8; ++i) MU[i] = 0.f;
        for (int li = lane; li < cnt; li += 32) {
          const int c = list[li];
          const int br = c >> 8, ai = c & 255;
          const float off = br ? -0.25f : 0.25f;
          CompTerms ct;
          comp_terms(T, br, ai, s_off[ai], ng, br ? ynorm[1] : ynorm[0], s_sqn[ai], s_par[ai], ct);
          const float lc = ct.lc, prod = ct.prod;
          const bool even = ct.even;
          const float* t = ct.t;
          const float* mag = ct.mag;
          if (lc > mx) {  // rescale the accumulators to the new maximum
            const float sc = expf(mx - lc);
            W *= sc;
            WOFF *= sc;
            SEC *= sc;
            #pragma unroll
            for (int i = 0; i < 8; ++i) MU[i] *= sc;
            mx = lc;
          }
          const float w = __expf(lc - mx);  // lc - mx in [-kPrune - margin, 0]
          float de = 1.f + prod, dodd = 1.f - prod;
          if (!(fabsf(de) > 1e-12f)) de = 1.f;
          if (!(fabsf(dodd) > 1e-12f)) dodd = 1.f;
          // sign means (t_i +- prod_{j != i} t_j) / (1 +- prod): |t| < 1 and the denominator is clamped away
          // from 0, so they are finite (the reference's nan_to_num never fires)
          const float rden = __frcp_rn(even ? de : dodd);
          const float sgn = even ? 1.f : -1.f;
          float pre[8];
          float acc = 1.f;
          #pragma unroll
          for (int i = 0; i < 8; ++i) { pre[i] = acc; acc = fmul(acc, t[i]); }
          float suf = 1.f, mcs = 0.f, mc[8];
          #pragma unroll
          for (int i = 7; i >= 0; --i) {
            const float ex = fmul(pre[i], suf);
            mc[i] = fmul(fmul(__fmaf_rn(sgn, ex, t[i]), rden), mag[i]);  // sgn * ex is exact
            mcs = fadd(mcs, mc[i]);
            suf = fmul(suf, t[i]);
          }
          W += w;
          WOFF += w * off;  // the branch offset's share of every coordinate's mean
          #pragma unroll
          for (int i = 0; i < 8; ++i) MU[i] += w * mc[i];
          SEC += w * (s_sqn[ai] + 8.f * off * off + 2.f * off * mcs);
        }
        // merge the lanes' online softmax states (fixed butterfly order)
        float M = mx;
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        const float scl = (mx == M) ? 1.f : expf(mx - M);
        W = warp_sum(W * scl);
        WOFF = warp_sum(WOFF * scl);
        SEC = warp_sum(SEC * scl);
        // The eight coordinate sums as a reduce-scatter over the same xor-16, 8, 4, 2, 1 butterfly: at each
        // stage a lane keeps half of its coordinates and adds its partner's values of them, so lane l ends with
        // the full sum of coordinate (l >> 2) & 7, bit-identical to a warp_sum of that coordinate.
        const bool h4 = (lane & 16) != 0, h3 = (lane & 8) != 0, h2 = (lane & 4) != 0;
        float v4[4], v2[2];
        #pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float lo = MU[j] * scl, hi = MU[j + 4] * scl;
          v4[j] = (h4 ? hi : lo) + __shfl_xor_sync(0xffffffffu, h4 ? lo : hi, 16);
        }
        #pragma unroll
        for (int j = 0; j < 2; ++j)
          v2[j] = (h3 ? v4[j + 2] : v4[j]) + __shfl_xor_sync(0xffffffffu, h3 ? v4[j] : v4[j + 2], 8);
        float v1 = (h2 ? v2[1] : v2[0]) + __shfl_xor_sync(0xffffffffu, h2 ? v2[0] : v2[1], 4);
        v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
        v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
        const float mown = (v1 + WOFF) / W;  // coordinate (lane >> 2) & 7 of the posterior mean
        float nrm = 0.f;
        #pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float mi = __shfl_sync(0xffffffffu, mown, 4 * i);
          nrm += mi * mi;
          mu_l = (lane == i) ? mi : mu_l;
        }
        var = fmaxf((SEC / W - nrm) / 8.f, 0.f);
      }
      if (lane < 8) x1_out[b * ld_x + k * 8 + lane] = mu_l;
      if (lane == 0) {
        if (var_out) var_out[b * ld_v + k] = var;
        vacc += var;
      }
    }
  }
  if constexpr (MMSE) {
    __shared__ int s_last;
    __shared__ float s_red[2][kRowThreads / 32];
    if (lane == 0) s_var[warp] = vacc;
    __syncthreads();
    if (threadIdx.x == 0 && var_rowsum) {
      float tsum = 0.f;
      for (int w = 0; w < kWarps; ++w) tsum += s_var[w];
      int last = 1;
      if (gridDim.y == 1) {
        var_rowsum[b] = tsum;
      } else {
        // chunk partials in a fixed order: the last chunk of the row to finish sums them (c = 0, 1, ...)
        rs.part[(int64_t)b * gridDim.y + blockIdx.y] = tsum;
        __threadfence();
        const unsigned prev = atomicAdd(&rs.counters[b], 1u);
        last = prev == gridDim.y - 1;
        if (last) {
          __threadfence();
          float t = 0.f;
          for (unsigned c = 0; c < gridDim.y; ++c) t += __ldcg(&rs.part[(int64_t)b * gridDim.y + c]);
          var_rowsum[b] = t;
          rs.counters[b] = 0u;  // ready for the next launch
        }
      }
      s_last = last;
    }
    if (fz.on) {
      __syncthreads();  // s_last and thread 0's var_rowsum[b] store, for the row stage's threads
      if (s_last && threadIdx.x < kRowThreads)
        vamp_row_stage<true>(fz.st, fz.S, b, a.B, fz.n, fz.n_var, fz.R, 0.f, fz.damping, fz.final_retry, fz.ctl,
                             fz.rc, s_red);
    }
  }
}


// ---- posterior diagnostics (mpq/priors/e8p12.py:292-306, :945-960; need_stats) ----
// Per item: logZ = logsumexp of the 512 component log-weights; entropy = -sum w log w + sum w H_sign(component)
// with H_sign = max(logZ_sign - sum_k a_k m_k, 0) (m_k the component's sign means); margin = the gap between the
// two largest of the 1024 log-scores {best, second-best parity-valid sign pattern} of the components.  All 512
// components are evaluated (no pruning): these are diagnostics, off the solve's path.  One warp per item; the
// per-coordinate table is the posterior kernel's (correctly rounded tanh and its log).
__global__ void __launch_bounds__(kWarps * 32) k_e8p12_stats(E8Args a, E8Tab tab, float* __restrict__ logz_out,
                                                             float* __restrict__ ent_out, float* __restrict__ mar_out,
                                                             int64_t ld) {
  __shared__ uint2 s_off[256];
  __shared__ float s_sqn[256];
  __shared__ int s_par[256];
  __shared__ ItemTab s_tab[kWarps];
  __shared__ int s_bad;
  const bool bad = stage_abs_patterns(tab, s_off, s_sqn, s_par, &s_bad);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t it = (int64_t)blockIdx.x * kWarps + warp;
  if (it >= (int64_t)a.B * a.nb) return;
  const int b = (int)(it / a.nb), k = (int)(it % a.nb);
  if (bad) {
    if (lane == 0) {
      logz_out[b * ld + k] = __int_as_float(0x7fc00000);
      ent_out[b * ld + k] = __int_as_float(0x7fc00000);
      mar_out[b * ld + k] = __int_as_float(0x7fc00000);
    }
    return;
  }
  float y[8], g, g1;
  fold_item(a, b, k, y, g, g1);
  const float ng = fmul(-0.5f, g);
  float ynorm[2];
  #pragma unroll
  for (int br = 0; br < 2; ++br) {
    const float off = br ? -0.25f : 0.25f;
    float yn = 0.f;
    #pragma unroll
    for (int i = 0; i < 8; ++i) yn = fadd(yn, fmul(fsub(y[i], off), fsub(y[i], off)));
    ynorm[br] = yn;
  }
  ItemTab& T = s_tab[warp];
  for (int e = lane; e < 48; e += 32) {
    const int br = e / 24, r = e - br * 24, kk = r / 3, m = r - kk * 3;
    float yk = y[0];
    #pragma unroll
    for (int i = 1; i < 8; ++i) yk = (kk == i) ? y[i] : yk;
    const float off = br ? -0.25f : 0.25f;
    const float mag = 0.5f + (float)m;
    const float av = fmul(fmul(g, fsub(yk, off)), mag);
    const float aa = fabsf(av);
    const float Tv = aa + log1pf(expf(-2.f * aa));
    const float ti = fminf(fmaxf((float)tanh((double)av), -0.99999988079071044921875f), 0.99999988079071044921875f);
    T.pt[br][r] = make_float4(Tv, canon_sign(ti), (float)log((double)fmaxf(fabsf(ti), 1e-7f)), mag);
    T.am[br][r] = make_float2(canon_sign(av), Tv);
  }
  __syncwarp();
  float mx = -INFINITY, S = 0.f, SL = 0.f, SE = 0.f;  // online softmax: sum w, sum w (lc - mx), sum w H_sign
  float t1 = -INFINITY, t2 = -INFINITY;             // the lane's two largest log-scores
  for (int j = 0; j < 16; ++j) {
    const int c = j * 32 + lane, br = c >> 8, ai = c & 255;
    const uint2 of = s_off[ai];
    const char* bp = reinterpret_cast<const char*>(T.pt[br]);
    const char* ba = reinterpret_cast<const char*>(T.am[br]);
    float logC = 0.f, lpt = 0.f, t[8], av[8];
    unsigned sx = 0;
    int nneg = 0;
    #pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const unsigned byte = __byte_perm(kk < 4 ? of.x : of.y, 0u, 0x4440u + (kk & 3));
      const float4 v = *reinterpret_cast<const float4*>(bp + 2u * byte);
      logC = fadd(logC, v.x);
      t[kk] = v.y;
      sx ^= __float_as_uint(v.y);
      lpt = fadd(lpt, v.z);
      av[kk] = reinterpret_cast<const float2*>(ba + byte)->x;
      nneg += av[kk] < 0.f ? 1 : 0;
    }
    const bool negp = (sx >> 31) != 0u, even = s_par[ai] == 0;
    const float pabs = expf(lpt);
    const float prod = negp ? -pabs : pabs;
    const float lae = log1pf(pabs);
    const float l1me = lpt < -kLn2 ? log1pf(-pabs) : logf(-expm1f(lpt));
    const float lzs = fsub(fadd(logC, even ? (negp ? l1me : lae) : (negp ? lae : l1me)), kLn2);
    const float cst = fmul(ng, fadd(br ? ynorm[1] : ynorm[0], s_sqn[ai]));
    const float lc = fadd(cst, lzs);
    // sign means and the component's sign entropy
    float de = fadd(1.f, prod), dodd = fsub(1.f, prod);
    if (!(fabsf(de) > 1e-12f)) de = 1.f;
    if (!(fabsf(dodd) > 1e-12f)) dodd = 1.f;
    float pre[8], acc = 1.f;
    #pragma unroll
    for (int i = 0; i < 8; ++i) { pre[i] = acc; acc = fmul(acc, t[i]); }
    float suf = 1.f, am[8];
    #pragma unroll
    for (int i = 7; i >= 0; --i) {
      const float ex = fmul(pre[i], suf);
      float smv = even ? fdiv(fadd(t[i], ex), de) : fdiv(fsub(t[i], ex), dodd);
      if (!isfinite(smv)) smv = 0.f;
      am[i] = fmul(av[i], smv);
      suf = fmul(suf, t[i]);
    }
    float asum = 0.f;
    #pragma unroll
    for (int i = 0; i < 8; ++i) asum = fadd(asum, am[i]);
    const float hs = isfinite(lzs) ? fmaxf(fsub(lzs, asum), 0.f) : 0.f;
    // best and second-best parity-valid sign patterns of the component
    float sum_abs = 0.f, m1 = INFINITY, m2 = INFINITY;
    int p1 = 0;
    #pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float x = fabsf(av[i]);
      sum_abs = fadd(sum_abs, x);
      if (x < m1) { m1 = x; p1 = i; }
    }
    #pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i != p1) m2 = fminf(m2, fabsf(av[i]));
    const bool mismatch = (nneg & 1) != s_par[ai];
    const float bl = mismatch ? fsub(sum_abs, fmul(2.f, m1)) : sum_abs;
    const float sl = mismatch ? fsub(sum_abs, fmul(2.f, m2)) : fsub(sum_abs, fmul(2.f, fadd(m1, m2)));
    const float sc1 = fadd(cst, bl), sc2 = fadd(cst, sl);
    if (sc1 > t1) { t2 = t1; t1 = sc1; } else if (sc1 > t2) { t2 = sc1; }
    if (sc2 > t1) { t2 = t1; t1 = sc2; } else if (sc2 > t2) { t2 = sc2; }
    if (lc == lc && lc > -INFINITY) {
      if (lc > mx) {
        const float sc = (mx == -INFINITY) ? 0.f : expf(mx - lc);
        SL = sc * (SL + S * (mx == -INFINITY ? 0.f : (mx - lc)));
        S *= sc;
        SE *= sc;
        mx = lc;
      }
      const float w = expf(lc - mx);
      S += w;
      SL += w * (lc - mx);
      SE += w * hs;
    }
  }
  // merge the lanes (fixed butterfly order)
  float M = mx;
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  if (mx > -INFINITY) {
    const float sc = expf(mx - M);
    SL = sc * (SL + S * (mx - M));
    S *= sc;
    SE *= sc;
  } else {
    S = SL = SE = 0.f;
  }
  S = warp_sum(S);
  SL = warp_sum(SL);
  SE = warp_sum(SE);
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float o1 = __shfl_xor_sync(0xffffffffu, t1, o), o2 = __shfl_xor_sync(0xffffffffu, t2, o);
    const float n1 = fmaxf(t1, o1);
    const float n2 = fmaxf(fminf(t1, o1), fmaxf(t2, o2));
    t1 = n1;
    t2 = n2;
  }
  if (lane == 0) {
    const float ls = logf(S);
    logz_out[b * ld + k] = M + ls;
    ent_out[b * ld + k] = ls - SL / S + SE / S;
    mar_out[b * ld + k] = t1 - t2;
  }
}

// ---- top-k candidates (mpq/priors/e8p12.py:367-449 with need_stats, :453-538) ----
// Per item and (branch, abs pattern): the best parity-valid sign pattern (flip the first minimum of |a| on a parity
// mismatch) and the second best (mismatch: flip the second minimum instead; match: flip both minima), scored
// const + linear as the MAP pass.  The 1024 candidates sit in the reference's flat order f = 2 (256 br + ai) + s;
// the k largest scores are selected by k rounds of a warp argmax (ties: smaller f first).
constexpr int kTopkWarps = 8;

__global__ void __launch_bounds__(kTopkWarps * 32)
k_e8p12_topk(E8Args a, E8Tab tab, int k, int* __restrict__ idx_out, float* __restrict__ score_out,
             float* __restrict__ val_out) {
  __shared__ uint2 s_off[256];
  __shared__ float s_sqn[256];
  __shared__ int s_par[256];
  __shared__ float s_a[kTopkWarps][48];              // a = (g (y_k - off)) |b| per (branch, 3 k + m)
  // candidate f = 2 (256 br + ai) + s lives in slot e = f >> 5 of lane (f + e) & 31, at [e * 32 + lane]: the
  // best / second-best of an abs pattern and its two branches sit in different lanes (so the top candidates,
  // which cluster by abs pattern, are spread over lanes), a lane's slots run in ascending f, and the 32 lanes of
  // one scoring store hit 32 different banks
  __shared__ float s_sc[kTopkWarps][1024];
  __shared__ unsigned char s_sid[kTopkWarps][1024];  // its sign pattern (bit k: coordinate k negative)
  __shared__ int s_bad;
  const bool bad = stage_abs_patterns(tab, s_off, s_sqn, s_par, &s_bad);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sa = s_a[warp];
  float* ssc = s_sc[warp];
  unsigned char* ssid = s_sid[warp];
  const int64_t items = (int64_t)a.B * a.nb;
  for (int64_t it = (int64_t)blockIdx.x * kTopkWarps + warp; it < items; it += (int64_t)gridDim.x * kTopkWarps) {
    const int b = (int)(it / a.nb), kb = (int)(it - (int64_t)b * a.nb);
    int* io = idx_out + it * k;
    float* so = score_out ? score_out + it * k : nullptr;
    float* vo = val_out ? val_out + it * k * 8 : nullptr;
    if (bad) {
      for (int t = lane; t < k; t += 32) {
        io[t] = -1;
        if (so) so[t] = __int_as_float(0x7fc00000);
      }
      if (vo)
        for (int t = lane; t < 8 * k; t += 32) vo[t] = __int_as_float(0x7fc00000);
      continue;
    }
    float y[8], g, g1;
    fold_item(a, b, kb, y, g, g1);
    const float ng = fmul(-0.5f, g);
    float ynorm[2];
    #pragma unroll
    for (int br = 0; br < 2; ++br) {
      const float off = br ? -0.25f : 0.25f;
      float yn = 0.f;
      #pragma unroll
      for (int i = 0; i < 8; ++i) yn = fadd(yn, fmul(fsub(y[i], off), fsub(y[i], off)));
      ynorm[br] = yn;
    }
    __syncwarp();
    for (int e = lane; e < 48; e += 32) {
      const int br = e / 24, r = e - br * 24, kk = r / 3, m = r - kk * 3;
      float yk = y[0];
      #pragma unroll
      for (int i = 1; i < 8; ++i) yk = (kk == i) ? y[i] : yk;
      const float off = br ? -0.25f : 0.25f;
      sa[e] = canon_sign(fmul(fmul(g, fsub(yk, off)), 0.5f + (float)m));
    }
    __syncwarp();
    #pragma unroll 1
    for (int j = 0; j < 8; ++j) {
      const int ai = (j << 5) | lane;
      const uint2 of = s_off[ai];
      float sum_abs[2] = {0.f, 0.f}, mn[2] = {INFINITY, INFINITY}, mn2[2] = {INFINITY, INFINITY};
      int p1[2] = {0, 0}, p2[2] = {0, 0};
      unsigned neg[2] = {0u, 0u};
      #pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const unsigned ent = __byte_perm(kk < 4 ? of.x : of.y, 0u, 0x4440u + (kk & 3)) >> 3;
        #pragma unroll
        for (int br = 0; br < 2; ++br) {
          const float av = sa[24 * br + ent];
          const float aa = fabsf(av);
          sum_abs[br] = fadd(sum_abs[br], aa);
          neg[br] |= sign_bit(av) << kk;
          if (aa < mn[br]) {  // first minimum, then the first minimum of the others
            mn2[br] = mn[br]; p2[br] = p1[br];
            mn[br] = aa; p1[br] = kk;
          } else if (aa < mn2[br]) {
            mn2[br] = aa; p2[br] = kk;
          }
        }
      }
      const float sq = s_sqn[ai];
      const int par = s_par[ai];
      #pragma unroll
      for (int br = 0; br < 2; ++br) {
        const bool mismatch = (int)(__popc(neg[br]) & 1) != par;
        const float cst = fmul(ng, fadd(ynorm[br], sq));
        const float lin1 = mismatch ? fsub(sum_abs[br], fmul(2.f, mn[br])) : sum_abs[br];
        const float lin2 = mismatch ? fsub(sum_abs[br], fmul(2.f, mn2[br]))
                                    : fsub(sum_abs[br], fmul(2.f, fadd(mn[br], mn2[br])));
        const unsigned b1 = 1u << p1[br], b2 = 1u << p2[br];
        const int f0 = 2 * (256 * br + ai);  // s = 0; s = 1 is f0 + 1, in the same slot and the next lane
        const int slot = (f0 >> 5) * 32, own = (f0 + (f0 >> 5)) & 31;
        ssc[slot + own] = fadd(cst, lin1);
        ssid[slot + own] = (unsigned char)(mismatch ? neg[br] ^ b1 : neg[br]);
        ssc[slot + ((own + 1) & 31)] = fadd(cst, lin2);
        ssid[slot + ((own + 1) & 31)] = (unsigned char)(mismatch ? neg[br] ^ b2 : neg[br] ^ b1 ^ b2);
      }
    }
    // k rounds of a warp argmax.  Each lane keeps the two best of its own 32 entries (ascending e = ascending f,
    // so a strict comparison keeps the first of equal scores); a lane rescans its entries only when it wins a
    // round with no valid second entry.  Round t's winner is parked in lane t % 32 and written out every 32
    // rounds (the index-table and codeword loads of 32 winners run in parallel).
    auto top2 = [&](unsigned taken_mask, float& b1, int& e1, float& b2, int& e2) {
      b1 = -INFINITY; e1 = -1; b2 = -INFINITY; e2 = -1;
      #pragma unroll 4
      for (int e = 0; e < 32; ++e) {
        if ((taken_mask >> e) & 1u) continue;
        const float v = ssc[e * 32 + lane];
        if (e1 < 0 || v > b1) {
          b2 = b1; e2 = e1; b1 = v; e1 = e;
        } else if (e2 < 0 || v > b2) {
          b2 = v; e2 = e;
        }
      }
    };
    unsigned taken = 0u;
    float b1, b2;
    int e1, e2;
    top2(0u, b1, e1, b2, e2);
    bool second_valid = true;
    int park_f = -1;
    float park_sc = 0.f;
    #pragma unroll 1
    for (int t = 0; t < k; ++t) {
      float wb = b1;
      int wf = e1 < 0 ? -1 : e1 * 32 + ((lane - e1) & 31);
      #pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, wb, o);
        const int of2 = __shfl_xor_sync(0xffffffffu, wf, o);
        if (of2 >= 0 && (wf < 0 || ob > wb || (ob == wb && of2 < wf))) { wb = ob; wf = of2; }
      }
      if (lane == (t & 31)) { park_f = wf; park_sc = wb; }
      if (wf >= 0 && lane == ((wf + (wf >> 5)) & 31)) {  // the winner's lane drops the entry
        taken |= 1u << e1;
        if (second_valid && e2 >= 0) {
          b1 = b2; e1 = e2; b2 = -INFINITY; e2 = -1;
          second_valid = false;
        } else {
          top2(taken, b1, e1, b2, e2);
          second_valid = true;
        }
      }
      if ((t & 31) == 31 || t == k - 1) {  // write the parked winners of rounds (t & ~31) .. t
        const int tt = (t & ~31) + lane;
        if (tt <= t) {
          int cidx = -1;
          if (park_f >= 0) {
            const int pbr = park_f >> 9, pai = (park_f >> 1) & 255;
            cidx = tab.idx_lut[pbr * 65536 + pai * 256 + ssid[(park_f >> 5) * 32 + ((park_f + (park_f >> 5)) & 31)]];
          }
          io[tt] = cidx;
          if (so) so[tt] = park_sc;
          if (vo) {
            float4 v0 = make_float4(__int_as_float(0x7fc00000), __int_as_float(0x7fc00000),
                                    __int_as_float(0x7fc00000), __int_as_float(0x7fc00000));
            float4 v1 = v0;
            if (cidx >= 0) {
              v0 = __ldg(reinterpret_cast<const float4*>(tab.grid + (int64_t)cidx * 8));
              v1 = __ldg(reinterpret_cast<const float4*>(tab.grid + (int64_t)cidx * 8 + 4));
            }
            reinterpret_cast<float4*>(vo + (int64_t)tt * 8)[0] = v0;
            reinterpret_cast<float4*>(vo + (int64_t)tt * 8)[1] = v1;
          }
        }
      }
    }
    __syncwarp();
  }
}

}  // namespace mpq

using namespace mpq;

static int e8_check(const float* r1, int B, int nb, const float* base_abs, const float* base_sqnorm,
                    const int* base_parity, const int* idx_lut, const float* grid) {
  MPQ_CHECK_ARG(B >= 0 && nb >= 0, "e8p12: bad shape");
  if (B == 0 || nb == 0) return MPQ_OK;  // empty tensors may carry null pointers
  MPQ_CHECK_ARG(r1 && base_abs && base_sqnorm && base_parity && idx_lut && grid, "e8p12: null pointer");
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
  if (B == 0 || nb == 0) return MPQ_OK;
  MPQ_CHECK_ARG(gamma && x1_out && var_rowsum, "mpq_e8p12_mmse: gamma, x1_out and var_rowsum are required");
  E8Args a{r1, ld_r1, center, ld_c, pscale, ld_s, gamma, prior_tau, 0.f, B, nb};
  E8Tab t{base_abs, base_sqnorm, base_parity, idx_lut, grid};
  k_e8p12<true><<<dim3(B, 1), kWarps * 32, 0, (cudaStream_t)stream>>>(a, t, x1_out, ld_x, var_out, ld_v, idx_out, ld_i,
                                                                      map_out, ld_m, var_rowsum, RowSplit{}, RowsFuse{});
  return launch_status("mpq_e8p12_mmse");
}

// mpq_e8p12_mmse with each row cut into `chunks` contiguous item ranges (one CTA each, so a few rows still fill the
// GPU) and optional device-side launch control.  work: caller-owned B * (chunks + 1) 32-bit words, zeroed before the
// first call (the chunk partials and the per-row arrival counters, which every launch leaves at zero); the row's
// variance sum adds the chunk partials in chunk order (deterministic).  active: optional device int, the launch
// does nothing while it is 0.
MPQ_API int mpq_e8p12_mmse_rows(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* pscale,
                                int64_t ld_s, const float* gamma, float prior_tau, int B, int nb, const float* base_abs,
                                const float* base_sqnorm, const int* base_parity, const int* idx_lut, const float* grid,
                                float* x1_out, int64_t ld_x, float* var_rowsum, int chunks, void* work,
                                const int* active, void* stream) {
  int st = e8_check(r1, B, nb, base_abs, base_sqnorm, base_parity, idx_lut, grid);
  if (st) return st;
  if (B == 0 || nb == 0) return MPQ_OK;
  MPQ_CHECK_ARG(gamma && x1_out && var_rowsum, "mpq_e8p12_mmse_rows: gamma, x1_out and var_rowsum are required");
  MPQ_CHECK_ARG(chunks >= 1 && chunks <= nb && chunks <= 1024, "mpq_e8p12_mmse_rows: chunks must be in [1, min(nb, 1024)]");
  MPQ_CHECK_ARG(chunks == 1 || work, "mpq_e8p12_mmse_rows: work buffer required for chunks > 1");
  E8Args a{r1, ld_r1, center, ld_c, pscale, ld_s, gamma, prior_tau, 0.f, B, nb};
  E8Tab t{base_abs, base_sqnorm, base_parity, idx_lut, grid};
  RowSplit rs{static_cast<float*>(work), work ? reinterpret_cast<unsigned*>(static_cast<float*>(work) + (int64_t)B * chunks)
                                              : nullptr, active};
  k_e8p12<true><<<dim3(B, chunks), kWarps * 32, 0, (cudaStream_t)stream>>>(a, t, x1_out, ld_x, nullptr, 0, nullptr, 0,
                                                                           nullptr, 0, var_rowsum, rs, RowsFuse{});
  return launch_status("mpq_e8p12_mmse_rows");
}

// mpq_e8p12_mmse_rows with the retry round's row stage fused behind it (mpq_vamp_rows_round_ctl's arguments after
// `active`): the CTA that completes a row's variance sum runs that row's stage, and the last row to finish takes the
// round's decision.  One launch per retry round instead of two, with the same arithmetic.
MPQ_API int mpq_e8p12_mmse_rows_round_ctl(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c,
                                          const float* pscale, int64_t ld_s, const float* gamma, float prior_tau, int B,
                                          int nb, const float* base_abs, const float* base_sqnorm,
                                          const int* base_parity, const int* idx_lut, const float* grid, float* x1_out,
                                          int64_t ld_x, float* var_rowsum, int chunks, void* work, const int* active,
                                          float* gamma1, float* alpha1, float* eta1, float* gamma2_new, float* gamma2,
                                          const float* gamma2_prev, float* alpha2, float* eta2, float* gamma1_new,
                                          float* gamma1_next, float* trace, int* flags, const float* S, int n, int R,
                                          float damping, int final_retry, void* ctl, float factor, unsigned* counter,
                                          void* stream) {
  int st = e8_check(r1, B, nb, base_abs, base_sqnorm, base_parity, idx_lut, grid);
  if (st) return st;
  if (B == 0 || nb == 0) return MPQ_OK;
  MPQ_CHECK_ARG(gamma && x1_out && var_rowsum, "mpq_e8p12_mmse_rows_round_ctl: gamma, x1_out and var_rowsum are required");
  MPQ_CHECK_ARG(chunks >= 1 && chunks <= nb && chunks <= 1024,
                "mpq_e8p12_mmse_rows_round_ctl: chunks must be in [1, min(nb, 1024)]");
  MPQ_CHECK_ARG(chunks == 1 || work, "mpq_e8p12_mmse_rows_round_ctl: work buffer required for chunks > 1");
  MPQ_CHECK_ARG(gamma1 && alpha1 && eta1 && gamma2_new && gamma2 && gamma2_prev && alpha2 && eta2 && gamma1_new &&
                    gamma1_next && trace && flags && S && ctl && counter,
                "mpq_e8p12_mmse_rows_round_ctl: null pointer");
  E8Args a{r1, ld_r1, center, ld_c, pscale, ld_s, gamma, prior_tau, 0.f, B, nb};
  E8Tab t{base_abs, base_sqnorm, base_parity, idx_lut, grid};
  RowSplit rs{static_cast<float*>(work), work ? reinterpret_cast<unsigned*>(static_cast<float*>(work) + (int64_t)B * chunks)
                                              : nullptr, active};
  // gamma1_work of the row stage is the posterior's own precision vector
  RowState rst{var_rowsum, gamma1, const_cast<float*>(gamma), alpha1, eta1, gamma2_new, gamma2,
               damping < 1.f ? gamma2_prev : nullptr, alpha2, eta2, gamma1_new, gamma1_next, trace, flags};
  RowsFuse fz{1, rst, S, n, nb, R, damping, final_retry, static_cast<const VampCtl*>(ctl),
              RoundCtl{static_cast<VampCtl*>(ctl), counter, factor, nb}};
  k_e8p12<true><<<dim3(B, chunks), kWarps * 32, 0, (cudaStream_t)stream>>>(a, t, x1_out, ld_x, nullptr, 0, nullptr, 0,
                                                                           nullptr, 0, var_rowsum, rs, fz);
  return launch_status("mpq_e8p12_mmse_rows_round_ctl");
}

// Posterior diagnostics per item (B x nb outputs with leading dimension ld): log-partition, entropy, margin.
MPQ_API int mpq_e8p12_stats(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* pscale,
                            int64_t ld_s, const float* gamma, float prior_tau, int B, int nb, const float* base_abs,
                            const float* base_sqnorm, const int* base_parity, const int* idx_lut, const float* grid,
                            float* logz_out, float* entropy_out, float* margin_out, int64_t ld, void* stream) {
  int st = e8_check(r1, B, nb, base_abs, base_sqnorm, base_parity, idx_lut, grid);
  if (st) return st;
  if (B == 0 || nb == 0) return MPQ_OK;
  MPQ_CHECK_ARG(gamma && logz_out && entropy_out && margin_out, "mpq_e8p12_stats: gamma and the outputs are required");
  MPQ_CHECK_ARG(ld >= nb, "mpq_e8p12_stats: ld < nb");
  E8Args a{r1, ld_r1, center, ld_c, pscale, ld_s, gamma, prior_tau, 0.f, B, nb};
  E8Tab t{base_abs, base_sqnorm, base_parity, idx_lut, grid};
  const int64_t items = (int64_t)B * nb;
  k_e8p12_stats<<<(unsigned)((items + kWarps - 1) / kWarps), kWarps * 32, 0, (cudaStream_t)stream>>>(
      a, t, logz_out, entropy_out, margin_out, ld);
  return launch_status("mpq_e8p12_stats");
}

// MAP codeword under the folded message (fixed_gamma > 0 replaces gamma for every row, e.g. 1 with no
// prior = nearest codeword / RTN).
MPQ_API int mpq_e8p12_map(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* pscale,
                          int64_t ld_s, const float* gamma, float fixed_gamma, float prior_tau, int B, int nb,
                          const float* base_abs, const float* base_sqnorm, const int* base_parity, const int* idx_lut,
                          const float* grid, int* idx_out, int64_t ld_i, float* map_out, int64_t ld_m, void* stream) {
  int st = e8_check(r1, B, nb, base_abs, base_sqnorm, base_parity, idx_lut, grid);
  if (st) return st;
  if (B == 0 || nb == 0) return MPQ_OK;
  MPQ_CHECK_ARG(gamma || fixed_gamma > 0.f, "mpq_e8p12_map: gamma or fixed_gamma required");
  E8Args a{r1, ld_r1, center, ld_c, pscale, ld_s, gamma, prior_tau, fixed_gamma, B, nb};
  E8Tab t{base_abs, base_sqnorm, base_parity, idx_lut, grid};
  // MAP only: no per-row reduction, so rows split freely into chunks of 64 items (enough CTAs for small row counts)
  const int chunks = std::max(1, std::min(nb / 64, (1776 + B - 1) / B));
  k_e8p12<false><<<dim3(B, chunks), kWarps * 32, 0, (cudaStream_t)stream>>>(a, t, nullptr, 0, nullptr, 0, idx_out, ld_i,
                                                                            map_out, ld_m, nullptr, RowSplit{}, RowsFuse{});
  return launch_status("mpq_e8p12_map");
}

// Top-k candidates per block (1 <= k <= 1024): idx_out (B x nb x k codebook indices, -1 where the index table has
// no entry), optional score_out (B x nb x k log-scores, descending) and val_out (B x nb x k x 8 codewords).
MPQ_API int mpq_e8p12_topk(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* pscale,
                           int64_t ld_s, const float* gamma, float prior_tau, int B, int nb, const float* base_abs,
                           const float* base_sqnorm, const int* base_parity, const int* idx_lut, const float* grid,
                           int k, int* idx_out, float* score_out, float* val_out, void* stream) {
  MPQ_CHECK_ARG(k >= 1 && k <= 1024, "mpq_e8p12_topk: k must be in [1, 1024]");
  int st = e8_check(r1, B, nb, base_abs, base_sqnorm, base_parity, idx_lut, grid);
  if (st) return st;
  if (B == 0 || nb == 0) return MPQ_OK;
  MPQ_CHECK_ARG(gamma && idx_out, "mpq_e8p12_topk: gamma and idx_out are required");
  MPQ_CHECK_ARG(((uintptr_t)grid & 15) == 0 && ((uintptr_t)val_out & 15) == 0,
                "mpq_e8p12_topk: grid and val_out must be 16-byte aligned");
  E8Args a{r1, ld_r1, center, ld_c, pscale, ld_s, gamma, prior_tau, 0.f, B, nb};
  E8Tab t{base_abs, base_sqnorm, base_parity, idx_lut, grid};
  const int64_t items = (int64_t)B * nb;
  const int64_t blocks = std::min<int64_t>((items + kTopkWarps - 1) / kTopkWarps, 148 * 32);
  k_e8p12_topk<<<(unsigned)blocks, kTopkWarps * 32, 0, (cudaStream_t)stream>>>(a, t, k, idx_out, score_out, val_out);
  return launch_status("mpq_e8p12_topk");
}
