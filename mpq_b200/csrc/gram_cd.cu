// Gram-metric block coordinate descent over E8P12 8-blocks (the E8P12 polish).
//
// Reference: mpq/polish/block_cd.py:332-625 (block_coordinate_descent_rankspace) with the E8P12
// provider's full-grid search (_cd_gram_step_impl :212-246, E8P12Provider._metric_map_assign :702-739),
// per-block metadata :383-404 (Vs_blk Vs_blk^T, stabilize_cholesky mpq/linear.py:121-141,
// cholesky_inverse) and the greedy block order _batched_greedy_gain :286-306.
//
// Search.  For target t and Cholesky factor L of the block gram, the reference scores every codeword c
// by  |tL|^2 + |cL|^2 - 2 (tL).(cL)  and takes the first minimum.  Here the same float32 score (products
// and sums in index order, no FMA contraction) decides, but codewords are skipped when a lower bound
// proves they cannot reach the running minimum:  score(c) >= lam_min(L L^T) |c - t|^2, and the Euclidean
// distance of every codeword of a (branch, abs) component is  sum_k (|y_k| - |b_k|)^2 + 4 sum_{k flipped}
// |y_k||b_k|  (y = t - offset) in closed form.  The bound carries a relative safety factor and an
// absolute margin far above the float32 rounding of the score, so the result equals the exhaustive
// first-minimum search.
//
// Blocks are visited in the greedy order in chunks of up to 16 blocks (128 columns): one warp per row
// runs the chunk's sequential block decisions with the chunk's cross-block grams in shared memory, and
// the accepted steps are applied to the rank-space residual by one tensor-core GEMM per chunk.
#include "common.cuh"

namespace mpq {

constexpr int kChunkBlocks = 16;
constexpr int kChunkCols = kChunkBlocks * 8;
// The chunk kernel reads only the strict upper block triangle of Hsub (rows of block p, columns of the later blocks):
// block row p is kept as 8 rows of width 128 - 8 (p + 1), starting at hs_tri_off(p).
constexpr int kHsTri = 8 * 8 * (kChunkBlocks * (kChunkBlocks - 1) / 2);
__host__ __device__ constexpr int hs_tri_off(int p) { return 960 * p - 32 * p * (p - 1); }
static_assert(hs_tri_off(kChunkBlocks) == kHsTri, "triangle layout");

// ---------------------------------------------------------------------------------------------
// per-block metadata
// ---------------------------------------------------------------------------------------------

// Cholesky of an 8x8 SPD matrix (float32, lower), column-by-column as LAPACK's unblocked potf2.
__device__ bool chol8(const float A[64], float L[64]) {
  for (int i = 0; i < 64; ++i) L[i] = 0.f;
  for (int j = 0; j < 8; ++j) {
    float s = A[j * 8 + j];
    for (int k = 0; k < j; ++k) s -= L[j * 8 + k] * L[j * 8 + k];
    if (!(s > 0.f) || !isfinite(s)) return false;
    const float d = sqrtf(s);
    L[j * 8 + j] = d;
    for (int i = j + 1; i < 8; ++i) {
      float t = A[i * 8 + j];
      for (int k = 0; k < j; ++k) t -= L[i * 8 + k] * L[j * 8 + k];
      L[i * 8 + j] = t / d;
    }
  }
  return true;
}

// Symmetric 8x8 eigenvalue bounds by cyclic Jacobi in double.
__device__ void eig8_bounds(const double S[64], double& lo, double& hi) {
  double A[64];
  for (int i = 0; i < 64; ++i) A[i] = S[i];
  for (int sweep = 0; sweep < 30; ++sweep) {
    double off = 0.0;
    for (int p = 0; p < 8; ++p)
      for (int q = p + 1; q < 8; ++q) off += A[p * 8 + q] * A[p * 8 + q];
    if (off < 1e-30) break;
    for (int p = 0; p < 8; ++p)
      for (int q = p + 1; q < 8; ++q) {
        const double apq = A[p * 8 + q];
        if (fabs(apq) < 1e-300) continue;
        const double theta = (A[q * 8 + q] - A[p * 8 + p]) / (2.0 * apq);
        const double t = (theta >= 0 ? 1.0 : -1.0) / (fabs(theta) + sqrt(theta * theta + 1.0));
        const double c = 1.0 / sqrt(t * t + 1.0), s = t * c;
        for (int k = 0; k < 8; ++k) {
          const double akp = A[k * 8 + p], akq = A[k * 8 + q];
          A[k * 8 + p] = c * akp - s * akq;
          A[k * 8 + q] = s * akp + c * akq;
        }
        for (int k = 0; k < 8; ++k) {
          const double apk = A[p * 8 + k], aqk = A[q * 8 + k];
          A[p * 8 + k] = c * apk - s * aqk;
          A[q * 8 + k] = s * apk + c * aqk;
        }
      }
  }
  double off = 0.0;
  for (int p = 0; p < 8; ++p)
    for (int q = 0; q < 8; ++q)
      if (p != q) off += A[p * 8 + q] * A[p * 8 + q];
  const double r = sqrt(off);  // Gershgorin-style slack for the residual off-diagonal mass
  lo = 1e300;
  hi = -1e300;
  for (int i = 0; i < 8; ++i) {
    lo = fmin(lo, A[i * 8 + i]);
    hi = fmax(hi, A[i * 8 + i]);
  }
  lo -= r;
  hi += r;
}

// One warp per block: gram = Vs_blk Vs_blk^T, L = stabilize_cholesky(gram), ginv = (L L^T)^-1 and
// eigenvalue bounds of L L^T.  meta layout per block: [gram 64 | L 64 | ginv 64 | lam_lo, lam_hi, ok, pad]
constexpr int kMeta = 196;

__global__ void k_gram_meta(const float* __restrict__ Vs, int64_t ld, int R, int nb, float* __restrict__ meta,
                            int* __restrict__ fail_count) {
  const int blk = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (blk >= nb) return;
  float g[64];
  for (int i = 0; i < 8; ++i)
    for (int j = i; j < 8; ++j) {
      const float* a = Vs + (int64_t)(blk * 8 + i) * ld;
      const float* b = Vs + (int64_t)(blk * 8 + j) * ld;
      float acc = 0.f;
      for (int r = lane; r < R; r += 32) acc += a[r] * b[r];
      acc = warp_sum(acc);
      g[i * 8 + j] = acc;
      g[j * 8 + i] = acc;
    }
  if (lane != 0) return;
  float* m = meta + (int64_t)blk * kMeta;
  for (int i = 0; i < 64; ++i) m[i] = g[i];
  // stabilize_cholesky: add 2^k * floor * I cumulatively until the factorization succeeds
  float dmax = 0.f;
  for (int i = 0; i < 8; ++i) dmax = fmaxf(dmax, fabsf(g[i * 9]));
  const float floor_ = dmax * 1e-6f + 1e-6f;
  float A[64], L[64];
  for (int i = 0; i < 64; ++i) A[i] = g[i];
  bool ok = false;
  for (int k = 0; k < 7 && !ok; ++k) {
    ok = chol8(A, L);
    if (!ok && k < 6)
      for (int i = 0; i < 8; ++i) A[i * 9] += (float)(1 << k) * floor_;
  }
  if (!ok) {
    atomicAdd(fail_count, 1);
    for (int i = 0; i < 64; ++i) L[i] = (i % 9 == 0) ? 1.f : 0.f;
  }
  for (int i = 0; i < 64; ++i) m[64 + i] = L[i];
  // (L L^T)^-1 = Linv^T Linv  in double
  double Li[64];
  for (int i = 0; i < 64; ++i) Li[i] = 0.0;
  for (int j = 0; j < 8; ++j) {
    Li[j * 8 + j] = 1.0 / (double)L[j * 8 + j];
    for (int i = j + 1; i < 8; ++i) {
      double s = 0.0;
      for (int k = j; k < i; ++k) s += (double)L[i * 8 + k] * Li[k * 8 + j];
      Li[i * 8 + j] = -s / (double)L[i * 8 + i];
    }
  }
  double S[64];
  for (int i = 0; i < 8; ++i)
    for (int j = 0; j < 8; ++j) {
      double s = 0.0, q = 0.0;
      for (int k = 0; k < 8; ++k) {
        s += Li[k * 8 + i] * Li[k * 8 + j];
        q += (double)L[i * 8 + k] * (double)L[j * 8 + k];
      }
      m[128 + i * 8 + j] = (float)s;
      S[i * 8 + j] = q;
    }
  double lo, hi;
  eig8_bounds(S, lo, hi);
  m[192] = (float)fmax(lo * (1.0 - 1e-6), 0.0);
  m[193] = (float)(hi * (1.0 + 1e-6));
  m[194] = ok ? 1.f : 0.f;
  m[195] = 0.f;
}

// gain[k] = mean_b sum_j rhs[b,8k+j] (rhs_bk Ginv_k)_j  (mpq/polish/block_cd.py:298-303); one CTA per block.
__global__ void __launch_bounds__(256) k_gram_gain(const float* __restrict__ rhs, int64_t ld, int B,
                                                   const float* __restrict__ meta, float* __restrict__ gain) {
  __shared__ float red[32];
  __shared__ float gi[64];
  const int k = blockIdx.x;
  for (int i = threadIdx.x; i < 64; i += blockDim.x) gi[i] = meta[(int64_t)k * kMeta + 128 + i];
  __syncthreads();
  float acc = 0.f;
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    float r[8];
    #pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = rhs[b * ld + k * 8 + j];
    float s = 0.f;
    #pragma unroll
    for (int j = 0; j < 8; ++j) {
      float d = 0.f;
      #pragma unroll
      for (int i = 0; i < 8; ++i) d += r[i] * gi[i * 8 + j];
      s += r[j] * d;
    }
    acc += s;
  }
  const float t = block_sum(acc, red);
  if (threadIdx.x == 0) gain[k] = t / (float)(B > 0 ? B : 1);
}

// Chunk operands for the blocks order[c0 : c0 + Kb]:  VsJ (128 x R) = rows of Vs for the chunk's columns,
// VsJT (R x 128) its transpose, Hsub (128 x 128) = Hf[cols, cols] with Hf = Vs Vs^T.
// Pre-split rows of Vs (its row-scaled fp16 split: hi, lo, 1/scale) gathered like VsJ: the split of a row depends on
// that row only, so the gathered split equals the split of the gathered rows.
struct SplitRows {
  const unsigned short* hi; const unsigned short* lo; int64_t ld; const float* inv;  // Vs's split (n rows)
  unsigned short* hiJ; unsigned short* loJ; int64_t ldJ; float* invJ;                // chunk rows (128)
  unsigned short* hiT; unsigned short* loT; int64_t ldT; float* invT;                // VsJT's own split (R rows)
};

__global__ void __launch_bounds__(256) k_gram_gather(const float* __restrict__ Vs, int64_t ldv, int R,
                                                     const float* __restrict__ Hf, int64_t ldh,
                                                     const int* __restrict__ order, int c0, int Kb,
                                                     float* __restrict__ VsJ, float* __restrict__ VsJT,
                                                     float* __restrict__ Hsub, SplitRows sp) {
  // CTA (x, y): rows r0 .. r0 + 31 of VsJT and the chunk columns k0 = 32 y, 32 (y + gridDim.y), ...; with the
  // split of VsJT requested the grid has one column of CTAs, so each CTA holds its rows' 128 columns (tileT) and
  // splits them as k_split_f16 splits the rows of VsJT[:, :8 Kb] (the zero columns beyond do not change a row's
  // maximum).
  __shared__ float tile[32][33];
  __shared__ float tileT[32][kChunkCols + 1];
  const int r0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int k0 = blockIdx.y * 32; k0 < kChunkCols; k0 += gridDim.y * 32) {
    for (int kk = ty; kk < 32; kk += 8) {
      const int k = k0 + kk, r = r0 + tx;
      float v = 0.f;
      const int64_t row = k < Kb * 8 ? (int64_t)(order[c0 + k / 8] * 8 + (k & 7)) : -1;
      if (row >= 0 && r < R) v = Vs[row * ldv + r];
      tile[kk][tx] = v;
      if (VsJ && r < R) VsJ[(int64_t)k * R + r] = v;
      if (sp.hiJ && row >= 0 && r < R) {
        sp.hiJ[(int64_t)k * sp.ldJ + r] = sp.hi[row * sp.ld + r];
        sp.loJ[(int64_t)k * sp.ldJ + r] = sp.lo[row * sp.ld + r];
        if (r == 0) sp.invJ[k] = sp.inv[row];
      }
    }
    __syncthreads();
    for (int rr = ty; rr < 32; rr += 8) {
      const int r = r0 + rr, k = k0 + tx;
      if (r < R) VsJT[(int64_t)r * kChunkCols + k] = tile[tx][rr];
      if (sp.hiT) tileT[rr][k] = tile[tx][rr];
    }
    __syncthreads();
    // Hsub rows k0 .. k0 + 31 spread over the CTAs of the grid's first row (one row of 128 entries per warp step)
    for (int i = blockIdx.x * 256 + threadIdx.x; i < 32 * kChunkCols; i += gridDim.x * 256) {
      const int k = k0 + i / kChunkCols, l = i % kChunkCols;
      float v = 0.f;
      if (k < Kb * 8 && l < Kb * 8)
        v = Hf[(int64_t)(order[c0 + k / 8] * 8 + (k & 7)) * ldh + order[c0 + l / 8] * 8 + (l & 7)];
      Hsub[k * kChunkCols + l] = v;
    }
  }
  if (sp.hiT) {
    for (int rr = ty; rr < 32; rr += 8) {  // one warp per row of VsJT
      const int r = r0 + rr;
      if (r >= R) continue;
      float mx = 0.f;
      for (int k = tx; k < Kb * 8; k += 32) mx = fmaxf(mx, fabsf(tileT[rr][k]));
      #pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float sc, inv;
      split_f16_scale(mx, sc, inv);
      for (int k = tx; k < Kb * 8; k += 32)
        split_f16_store(tileT[rr][k], sc, sp.hiT + (int64_t)r * sp.ldT + k, sp.loT + (int64_t)r * sp.ldT + k);
      if (tx == 0) sp.invT[r] = inv;
    }
  }
}

// ---------------------------------------------------------------------------------------------
// exact pruned gram search (warp-cooperative)
// ---------------------------------------------------------------------------------------------

struct E8Small {
  const float* base_abs;   // 256 x 8 (shared memory)
  const int* base_parity;  // 256 (shared memory)
  const float* grid;       // 65536 x 8 (global)
  const uint8_t* sign_id;  // 65536: sign bits of (grid[c] - offset(c)) (global)
};

// exact float32 score of codeword c:  (tn + |gL|^2) - 2 (tl . gL), index-ordered sums, no FMA
__device__ __forceinline__ float exact_score(const float* __restrict__ grid, int c, const float* L, const float tl[8],
                                             float tn) {
  float gv[8];
  const float4* gp = reinterpret_cast<const float4*>(grid + (int64_t)c * 8);
  const float4 g0 = __ldg(gp), g1 = __ldg(gp + 1);
  gv[0] = g0.x; gv[1] = g0.y; gv[2] = g0.z; gv[3] = g0.w;
  gv[4] = g1.x; gv[5] = g1.y; gv[6] = g1.z; gv[7] = g1.w;
  float gn = 0.f, cr = 0.f;
  #pragma unroll
  for (int j = 0; j < 8; ++j) {
    float gl = 0.f;
    #pragma unroll
    for (int k = j; k < 8; ++k) gl = fadd(gl, fmul(gv[k], L[k * 8 + j]));  // L lower: k >= j
    gn = fadd(gn, fmul(gl, gl));
    cr = fadd(cr, fmul(tl[j], gl));
  }
  return fsub(fadd(tn, gn), fmul(2.f, cr));
}

__device__ __forceinline__ bool better(float s, int c, float bs, int bc) { return s < bs || (s == bs && c < bc); }

__device__ __forceinline__ void warp_argmin(float& s, int& c) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const int oc = __shfl_xor_sync(0xffffffffu, c, o);
    if (better(os, oc, s, c)) { s = os; c = oc; }
  }
}

// Returns the first-minimum codeword index (identical in every lane) and the number of exact evaluations.
__device__ int gram_search_warp(const E8Small& e8, const float t[8], const float* L, float lam_lo, float lam_hi,
                                int* n_exact) {
  const int lane = threadIdx.x & 31;
  float tl[8], tn = 0.f;
  {
    // tl = t L (L lower): lane l computes coordinate l & 7 in the same order (k = j .. 7), then broadcast
    const int j = lane & 7;
    float s = 0.f;
    #pragma unroll
    for (int k = 0; k < 8; ++k)
      if (k >= j) s = fadd(s, fmul(t[k], L[k * 8 + j]));
    #pragma unroll
    for (int q = 0; q < 8; ++q) tl[q] = __shfl_sync(0xffffffffu, s, q);
  }
  #pragma unroll
  for (int j = 0; j < 8; ++j) tn = fadd(tn, fmul(tl[j], tl[j]));
  // closed-form Euclidean data per component: base distance, per-coordinate flip weights, sign pattern
  // lane owns abs = lane + 32*i, i = 0..7, for both branches
  float dmin[16];
  #pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int a = lane + 32 * i;
    const float* ab = e8.base_abs + a * 8;
    #pragma unroll
    for (int br = 0; br < 2; ++br) {
      const float off = br ? -0.25f : 0.25f;
      float base = 0.f, mn = INFINITY;
      int par = 0;
      #pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float y = t[k] - off;
        const float ay = fabsf(y);
        const float d = ay - ab[k];
        base += d * d;
        const float w = ay * ab[k];
        mn = fminf(mn, w);
        par ^= (y < 0.f) ? 1 : 0;
      }
      dmin[i * 2 + br] = base + ((par != e8.base_parity[a]) ? 4.f * mn : 0.f);
    }
  }
  // initial incumbent: the Euclidean-nearest codeword
  float bd = INFINITY;
  int bcomp = 0;
  #pragma unroll
  for (int q = 0; q < 16; ++q) {
    const int comp = (lane + 32 * (q >> 1)) * 2 + (q & 1);
    if (dmin[q] < bd || (dmin[q] == bd && comp < bcomp)) { bd = dmin[q]; bcomp = comp; }
  }
  {
    float s = bd;
    int c = bcomp;
    warp_argmin(s, c);
    bcomp = c;
  }
  int count = 0;
  float best = INFINITY;
  int best_c = 0x7fffffff;
  // Safety margin on the bound: relative 1e-5 (float32 rounding of the distances) and an absolute term
  // 1e-5 * (|tL|^2 + lam_hi * 16) well above the rounding of the float32 score.
  const float marg = 1e-5f * (tn + lam_hi * 20.f) + 1e-30f;
  const float lam = lam_lo * (1.f - 1e-5f);
  auto eval_comp = [&](int comp) {
    const int a = comp >> 1, br = comp & 1;
    const float off = br ? -0.25f : 0.25f;
    const float* ab = e8.base_abs + a * 8;
    float w[8], base = 0.f;
    int sgn = 0;
    #pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float y = t[k] - off;
      const float ay = fabsf(y);
      const float d = ay - ab[k];
      base += d * d;
      w[k] = 4.f * ay * ab[k];
      if (y < 0.f) sgn |= 1 << k;
    }
    // the 128 codewords (a<<8)|s with parity(s) = br; their sign pattern relative to the offset comes
    // from the codebook's sign table, and the coordinates whose sign differs from y's cost 4|y_k||b_k|.
    // Bounds first (lane: raw sign bytes s = 2 m + bit0, m = 4 lane + u, bit0 giving parity br); then one round
    // in which every lane scores its smallest-bound codeword exactly; then the warp's best so far prunes the
    // rest.  Whatever the order, every codeword whose bound is within the margin of the final best is scored
    // exactly, so the result is the first minimum of the exact scores.
    float dEu[4];
    int u1 = 0;
    #pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int m = lane * 4 + u;  // 0..127
      const int hi7 = m << 1;
      const int s = hi7 | ((__popc(hi7) & 1) ^ br);
      const int real = __ldg(e8.sign_id + ((a << 8) | s));
      const int diff = real ^ sgn;
      float dE = base;
      #pragma unroll
      for (int k = 0; k < 8; ++k)
        if (diff & (1 << k)) dE += w[k];
      dEu[u] = dE;
      if (dE < dEu[u1]) u1 = u;
    }
    auto code_of = [&](int u) {
      const int hi7 = (lane * 4 + u) << 1;
      return (a << 8) | hi7 | ((__popc(hi7) & 1) ^ br);
    };
    if (!(lam * dEu[u1] > best + marg)) {
      const int c = code_of(u1);
      const float sc = exact_score(e8.grid, c, L, tl, tn);
      ++count;
      if (better(sc, c, best, best_c)) { best = sc; best_c = c; }
    }
    warp_argmin(best, best_c);
    #pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (u == u1 || lam * dEu[u] > best + marg) continue;
      const int c = code_of(u);
      const float sc = exact_score(e8.grid, c, L, tl, tn);
      ++count;
      if (better(sc, c, best, best_c)) { best = sc; best_c = c; }
    }
    warp_argmin(best, best_c);
  };
  eval_comp(bcomp);
  #pragma unroll
  for (int q = 0; q < 16; ++q) {
    const int comp = (lane + 32 * (q >> 1)) * 2 + (q & 1);
    unsigned mask = __ballot_sync(0xffffffffu, comp != bcomp && lam * dmin[q] <= best + marg);
    while (mask) {
      const int src = __ffs(mask) - 1;
      mask &= mask - 1;
      const int cc = (src + 32 * (q >> 1)) * 2 + (q & 1);
      if (lam * __shfl_sync(0xffffffffu, dmin[q], src) <= best + marg) eval_comp(cc);
    }
  }
  if (n_exact) *n_exact = count;
  return best_c;
}

// The fused path's gather (mpq_gram_gather_split with the split of VsJT requested): CTA x copies the fp16 split
// row k = x of the chunk (16-byte vectors), transposes and splits rows r = 32 x .. 32 x + 31 of VsJT[:, :8 Kb]
// (128 chunk columns held in shared memory; VsJT itself is written only when asked for), and gathers its share of
// Hsub.  The same values as k_gram_gather, with fewer and wider memory operations.
// Sweep mode (nb_sweep > 0): CTA row y gathers chunk y of the sweep (blocks order[16 y ..], Kb = min(16, nb - 16 y))
// into its own slice of each output (chunk-major: 128 rows of hiJ / loJ / invJ, R rows of hiT / loT / invT, one
// 128 x 128 Hsub), with exactly the per-chunk launch's arithmetic.
__global__ void __launch_bounds__(256) k_gram_gather_fused(const float* __restrict__ Vs, int64_t ldv, int R,
                                                           const float* __restrict__ Hf, int64_t ldh,
                                                           const int* __restrict__ order, int c0, int Kb,
                                                           float* __restrict__ VsJT, float* __restrict__ Hsub,
                                                           SplitRows sp, int nb_sweep) {
  __shared__ float tileT[32][kChunkCols + 1];
  __shared__ int s_row[kChunkCols];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  if (nb_sweep > 0) {
    const int ch = blockIdx.y;
    c0 = ch * kChunkBlocks;
    Kb = min(kChunkBlocks, nb_sweep - c0);
    sp.hiJ += (int64_t)ch * kChunkCols * sp.ldJ;
    sp.loJ += (int64_t)ch * kChunkCols * sp.ldJ;
    sp.invJ += (int64_t)ch * kChunkCols;
    sp.hiT += (int64_t)ch * R * sp.ldT;
    sp.loT += (int64_t)ch * R * sp.ldT;
    sp.invT += (int64_t)ch * R;
    Hsub += (int64_t)ch * kChunkCols * kChunkCols;
  }
  const int kc = Kb * 8;
  for (int k = threadIdx.x; k < kChunkCols; k += blockDim.x) s_row[k] = k < kc ? order[c0 + k / 8] * 8 + (k & 7) : -1;
  __syncthreads();
  // (1) split rows of the chunk: row k = blockIdx.x, blockIdx.x + gridDim.x, ... (R halves = R / 8 vectors)
  if ((R & 7) == 0 && ((sp.ld | sp.ldJ) & 7) == 0) {
    for (int k = blockIdx.x; k < kc; k += gridDim.x) {
      const int64_t row = s_row[k];
      const int4* shi = reinterpret_cast<const int4*>(sp.hi + row * sp.ld);
      const int4* slo = reinterpret_cast<const int4*>(sp.lo + row * sp.ld);
      int4* dhi = reinterpret_cast<int4*>(sp.hiJ + (int64_t)k * sp.ldJ);
      int4* dlo = reinterpret_cast<int4*>(sp.loJ + (int64_t)k * sp.ldJ);
      for (int v = threadIdx.x; v < R / 8; v += blockDim.x) {
        dhi[v] = shi[v];
        dlo[v] = slo[v];
      }
      if (threadIdx.x == 0) sp.invJ[k] = sp.inv[row];
    }
  } else {
    for (int k = blockIdx.x; k < kc; k += gridDim.x) {
      const int64_t row = s_row[k];
      for (int r = threadIdx.x; r < R; r += blockDim.x) {
        sp.hiJ[(int64_t)k * sp.ldJ + r] = sp.hi[row * sp.ld + r];
        sp.loJ[(int64_t)k * sp.ldJ + r] = sp.lo[row * sp.ld + r];
      }
      if (threadIdx.x == 0) sp.invJ[k] = sp.inv[row];
    }
  }
  // (2) rows r0 .. r0 + 31 of VsJT (warp ty reads chunk columns k = ty, ty + 8, ...; lane = r)
  for (int r0 = blockIdx.x * 32; r0 < R; r0 += gridDim.x * 32) {
    const int r = r0 + tx;
    for (int k = ty; k < kChunkCols; k += 8) {
      const int64_t row = s_row[k];
      tileT[tx][k] = (row >= 0 && r < R) ? Vs[row * ldv + r] : 0.f;
    }
    __syncthreads();
    for (int rr = ty; rr < 32; rr += 8) {  // one warp per row of VsJT
      const int rw = r0 + rr;
      if (rw >= R) continue;
      float mx = 0.f;
      for (int k = tx; k < kc; k += 32) mx = fmaxf(mx, fabsf(tileT[rr][k]));
      #pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float sc, inv;
      split_f16_scale(mx, sc, inv);
      for (int k = tx; k < kc; k += 32)
        split_f16_store(tileT[rr][k], sc, sp.hiT + (int64_t)rw * sp.ldT + k, sp.loT + (int64_t)rw * sp.ldT + k);
      if (tx == 0) sp.invT[rw] = inv;
      if (VsJT)
        for (int k = tx; k < kChunkCols; k += 32) VsJT[(int64_t)rw * kChunkCols + k] = tileT[rr][k];
    }
    __syncthreads();
  }
  // (3) Hsub (128 x 128), spread over the grid
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < kChunkCols * kChunkCols; i += gridDim.x * blockDim.x) {
    const int k = i / kChunkCols, l = i % kChunkCols;
    Hsub[i] = (k < kc && l < kc) ? Hf[(int64_t)s_row[k] * ldh + s_row[l]] : 0.f;
  }
}

// ---------------------------------------------------------------------------------------------
// chunk of greedy block decisions (one warp per row)
// ---------------------------------------------------------------------------------------------

struct GramChunkArgs {
  float* x; int64_t ldx;           // B x n  (current decisions)
  const float* rhs; int64_t ldr;   // B x 128: residual_u @ Vs_J^T at chunk start
  const float* Hsub;               // 128 x 128 cross-block grams of the chunk
  const float* meta;               // nb x kMeta
  const int* order; int c0; int Kb;
  const float* base_abs; const int* base_parity; const float* grid; const uint8_t* sign_id;
  float* res;                      // B residual norms
  int* idx; int64_t ldi;           // B x nb codeword indices
  float* delta;                    // B x 128 accepted steps
  int* accepted;                   // accepted-update counter
  long long* evals;                // exact score evaluations (diagnostic)
  int B; float accept_tol;
  // top-k candidate mode: per (row, block) kc codewords (values B x nb x kc x 8, indices B x nb x kc)
  const float* cand; const int* cand_idx; int kc; int nb;
  // rhs_splits > 0: rhs holds the split-K partial planes of the rhs product (plane s at rhs + s * rhs_plane,
  // leading dimension ldr), added in plane order as the split-K reduction adds them
  int rhs_splits; int64_t rhs_plane;
  // optional: the row-scaled fp16 split of delta[:, :8 Kb] (as mpq_split_f16), for the residual update product
  unsigned short* dhi; unsigned short* dlo; int64_t ldd; float* dinv;
};

// Top-k candidate choice of one block (mpq/polish/block_cd.py:137-172 _topk_gram_step_impl): metric distance
// |tL|^2 + |cL|^2 - 2 (tL).(cL) clamped at 0 (index-ordered sums), first minimum over the candidates.
__device__ __forceinline__ int topk_pick_warp(const float t[8], const float* L, const float* cv, int kc) {
  const int lane = threadIdx.x & 31;
  float tm[8], tn = 0.f;
  #pragma unroll
  for (int j = 0; j < 8; ++j) {
    float acc = 0.f;
    #pragma unroll
    for (int i = 0; i < 8; ++i) acc = fadd(acc, fmul(t[i], L[i * 8 + j]));
    tm[j] = acc;
  }
  #pragma unroll
  for (int j = 0; j < 8; ++j) tn = fadd(tn, fmul(tm[j], tm[j]));
  float key = INFINITY;
  int ci = 0x7fffffff;
  for (int c = lane; c < kc; c += 32) {
    const float4 v0 = __ldg(reinterpret_cast<const float4*>(cv + c * 8));
    const float4 v1 = __ldg(reinterpret_cast<const float4*>(cv + c * 8 + 4));
    const float cvv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    float cn = 0.f, cross = 0.f;
    #pragma unroll
    for (int j = 0; j < 8; ++j) {
      float cm = 0.f;
      #pragma unroll
      for (int i = 0; i < 8; ++i) cm = fadd(cm, fmul(cvv[i], L[i * 8 + j]));
      cn = fadd(cn, fmul(cm, cm));
      cross = fadd(cross, fmul(cm, tm[j]));
    }
    float dist = fmaxf(fsub(fadd(tn, cn), fmul(2.f, cross)), 0.f);
    if (dist != dist) dist = INFINITY;
    if (ci == 0x7fffffff || dist < key) { key = dist; ci = c; }
  }
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ok = __shfl_xor_sync(0xffffffffu, key, o);
    const int oc = __shfl_xor_sync(0xffffffffu, ci, o);
    if (oc != 0x7fffffff && (ci == 0x7fffffff || ok < key || (ok == key && oc < ci))) { key = ok; ci = oc; }
  }
  return ci;
}

// topk_pick_warp for kc <= 32 with each lane's candidate already in registers (v0, v1; valid = lane < kc).
__device__ __forceinline__ int topk_pick_reg(const float t[8], const float* L, float4 v0, float4 v1, bool valid) {
  float tm[8], tn = 0.f;
  #pragma unroll
  for (int j = 0; j < 8; ++j) {
    float acc = 0.f;
    #pragma unroll
    for (int i = 0; i < 8; ++i) acc = fadd(acc, fmul(t[i], L[i * 8 + j]));
    tm[j] = acc;
  }
  #pragma unroll
  for (int j = 0; j < 8; ++j) tn = fadd(tn, fmul(tm[j], tm[j]));
  const float cvv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
  float cn = 0.f, cross = 0.f;
  #pragma unroll
  for (int j = 0; j < 8; ++j) {
    float cm = 0.f;
    #pragma unroll
    for (int i = 0; i < 8; ++i) cm = fadd(cm, fmul(cvv[i], L[i * 8 + j]));
    cn = fadd(cn, fmul(cm, cm));
    cross = fadd(cross, fmul(cm, tm[j]));
  }
  float key = fmaxf(fsub(fadd(tn, cn), fmul(2.f, cross)), 0.f);
  if (key != key) key = INFINITY;
  int ci = valid ? (int)(threadIdx.x & 31) : 0x7fffffff;
  if (!valid) key = INFINITY;
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ok = __shfl_xor_sync(0xffffffffu, key, o);
    const int oc = __shfl_xor_sync(0xffffffffu, ci, o);
    if (oc != 0x7fffffff && (ci == 0x7fffffff || ok < key || (ok == key && oc < ci))) { key = ok; ci = oc; }
  }
  return ci;
}

template <bool TOPK>
__global__ void __launch_bounds__(256) k_gram_chunk(GramChunkArgs a) {
  extern __shared__ float sm[];
  float* Hs = sm;                                    // strict upper block triangle of the 128 x 128 Hsub
  float* s_abs = Hs + kHsTri;                        // 256 x 8
  int* s_par = reinterpret_cast<int*>(s_abs + 2048); // 256
  float* s_meta = reinterpret_cast<float*>(s_par + 256);  // 16 x kMeta
  float* s_rhs = s_meta + kChunkBlocks * kMeta;      // 8 warps x 128
  for (int i = threadIdx.x; i < kChunkCols * kChunkCols; i += blockDim.x) {
    const int k = i / kChunkCols, l = i % kChunkCols, p = k >> 3, c0 = (p + 1) * 8;
    if (l >= c0) Hs[hs_tri_off(p) + (k & 7) * (kChunkCols - c0) + (l - c0)] = a.Hsub[i];
  }
  if constexpr (!TOPK) {
    for (int i = threadIdx.x; i < 2048; i += blockDim.x) s_abs[i] = a.base_abs[i];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) s_par[i] = a.base_parity[i];
  }
  for (int i = threadIdx.x; i < a.Kb * kMeta; i += blockDim.x)
    s_meta[i] = a.meta[(int64_t)a.order[a.c0 + i / kMeta] * kMeta + i % kMeta];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x * 8 + warp;
  if (b >= a.B) return;
  float* rh = s_rhs + warp * kChunkCols;
  for (int i = lane; i < kChunkCols; i += 32) {
    float v = 0.f;
    if (i < a.Kb * 8) {
      const int64_t o = (int64_t)b * a.ldr + i;
      v = a.rhs[o];
      for (int sp = 1; sp < a.rhs_splits; ++sp) v += a.rhs[sp * a.rhs_plane + o];
    }
    rh[i] = v;
  }
  __syncwarp();
  E8Small e8{s_abs, s_par, a.grid, a.sign_id};
  float res = a.res[b];
  int acc_n = 0;
  long long evals = 0;
  // top-k with kc <= 32: each lane holds its candidate of the current block and loads the next block's ahead
  const bool reg_cand = TOPK && a.kc <= 32;
  float4 cv0 = make_float4(0.f, 0.f, 0.f, 0.f), cv1 = cv0;
  auto load_cand = [&](int p, float4& v0, float4& v1) {
    const float* cp = a.cand + (((int64_t)b * a.nb + a.order[a.c0 + p]) * a.kc + lane) * 8;
    v0 = __ldg(reinterpret_cast<const float4*>(cp));
    v1 = __ldg(reinterpret_cast<const float4*>(cp + 4));
  };
  if (reg_cand && lane < a.kc) load_cand(0, cv0, cv1);
  // Per-block 8 x 8 algebra is spread over the lanes (lane l: coordinate l & 7, each sum in the sequential order)
  // and broadcast.  The next block's current decision is loaded a block ahead (a decision only writes its own
  // block).
  const int jl = lane & 7;
  float xb_next = a.Kb > 0 ? a.x[b * a.ldx + a.order[a.c0] * 8 + jl] : 0.f;
  for (int p = 0; p < a.Kb; ++p) {
    const int blk = a.order[a.c0 + p];
    const float* m = s_meta + p * kMeta;
    const float* G = m;
    const float* L = m + 64;
    const float* Gi = m + 128;
    const float xb_l = xb_next;
    if (p + 1 < a.Kb) xb_next = a.x[b * a.ldx + a.order[a.c0 + p + 1] * 8 + jl];
    float xb[8], r[8], t[8];
    #pragma unroll
    for (int j = 0; j < 8; ++j) {
      xb[j] = __shfl_sync(0xffffffffu, xb_l, j);
      r[j] = rh[p * 8 + j];
    }
    // target = x_blk + rhs @ ginv
    {
      float s = 0.f;
      #pragma unroll
      for (int i = 0; i < 8; ++i) s = fadd(s, fmul(r[i], Gi[i * 8 + jl]));
      const float tj = fadd(xb_l, s);
      #pragma unroll
      for (int j = 0; j < 8; ++j) t[j] = __shfl_sync(0xffffffffu, tj, j);
    }
    int c;
    const float* gv;
    if constexpr (TOPK) {
      const int64_t item = (int64_t)b * a.nb + blk;
      const float* cv = a.cand + item * a.kc * 8;
      int pick;
      if (reg_cand) {
        float4 nv0 = make_float4(0.f, 0.f, 0.f, 0.f), nv1 = nv0;
        if (p + 1 < a.Kb && lane < a.kc) load_cand(p + 1, nv0, nv1);
        pick = topk_pick_reg(t, L, cv0, cv1, lane < a.kc);
        cv0 = nv0;
        cv1 = nv1;
      } else {
        pick = topk_pick_warp(t, L, cv, a.kc);
      }
      gv = cv + pick * 8;
      c = a.cand_idx ? a.cand_idx[item * a.kc + pick] : pick;
      evals += a.kc;
    } else {
      int ne = 0;
      c = gram_search_warp(e8, t, L, m[192], m[193], &ne);
      evals += ne;
      gv = a.grid + (int64_t)c * 8;
    }
    float d[8], cross = 0.f, dn = 0.f;
    #pragma unroll
    for (int j = 0; j < 8; ++j) {
      d[j] = fsub(__ldg(gv + j), xb[j]);
      cross = fadd(cross, fmul(r[j], d[j]));
    }
    {
      // (d G)_j on lane j & 7, then dn = sum_j (d G)_j d_j in order
      float s = 0.f;
      #pragma unroll
      for (int i = 0; i < 8; ++i) s = fadd(s, fmul(d[i], G[i * 8 + jl]));
      #pragma unroll
      for (int j = 0; j < 8; ++j) dn = fadd(dn, fmul(__shfl_sync(0xffffffffu, s, j), d[j]));
    }
    dn = fmaxf(dn, 0.f);
    const float cand = fmaxf(fsub(fadd(res, dn), fmul(2.f, cross)), 0.f);
    const bool acc = fadd(cand, 1e-12f) < fmul(res, 1.f + a.accept_tol);
    if (acc) {
      res = cand;
      ++acc_n;
      if (lane < 8) a.x[b * a.ldx + blk * 8 + lane] = __ldg(gv + lane);
      if (lane == 0) a.idx[b * a.ldi + blk] = c;
      // later blocks of the chunk see this step: rhs_q -= d @ Hsub[p-block, q-block]
      const int cb = (p + 1) * 8, wp = kChunkCols - cb;
      const float* hp = Hs + hs_tri_off(p);  // hp[i * wp + col - cb] = Hsub[p * 8 + i][col] for col >= cb
      for (int col = lane; col < a.Kb * 8; col += 32) {
        if (col >= cb) {
          float s = 0.f;
          #pragma unroll
          for (int i = 0; i < 8; ++i) s = fadd(s, fmul(d[i], hp[i * wp + (col - cb)]));
          rh[col] = fsub(rh[col], s);
        }
      }
    }
    if (lane < 8) a.delta[(int64_t)b * kChunkCols + p * 8 + lane] = acc ? d[lane] : 0.f;
    __syncwarp();
  }
  for (int i = a.Kb * 8 + lane; i < kChunkCols; i += 32) a.delta[(int64_t)b * kChunkCols + i] = 0.f;
  if (a.dhi) {
    __syncwarp();  // the warp's delta stores above are visible to its lanes
    const float* dr = a.delta + (int64_t)b * kChunkCols;
    float mx = 0.f;
    for (int i = lane; i < a.Kb * 8; i += 32) mx = fmaxf(mx, fabsf(dr[i]));
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sc, inv;
    split_f16_scale(mx, sc, inv);
    for (int i = lane; i < a.Kb * 8; i += 32)
      split_f16_store(dr[i], sc, a.dhi + (int64_t)b * a.ldd + i, a.dlo + (int64_t)b * a.ldd + i);
    if (lane == 0) a.dinv[b] = inv;
  }
  if (lane == 0) {
    a.res[b] = res;
    if (acc_n) atomicAdd(a.accepted, acc_n);
    if (a.evals) atomicAdd((unsigned long long*)a.evals, (unsigned long long)evals);
  }
}

// Standalone search for a batch of targets that share one block factor (the provider entry point).
__global__ void k_gram_search(const float* __restrict__ targets, int N, const float* __restrict__ L,
                              float lam_lo, float lam_hi, const float* __restrict__ base_abs,
                              const int* __restrict__ base_parity, const float* __restrict__ grid,
                              const uint8_t* __restrict__ sign_id, int* __restrict__ out_idx) {
  __shared__ float s_abs[2048];
  __shared__ int s_par[256];
  __shared__ float s_L[64];
  for (int i = threadIdx.x; i < 2048; i += blockDim.x) s_abs[i] = base_abs[i];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) s_par[i] = base_parity[i];
  for (int i = threadIdx.x; i < 64; i += blockDim.x) s_L[i] = L[i];
  __syncthreads();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (w >= N) return;
  float t[8];
  #pragma unroll
  for (int j = 0; j < 8; ++j) t[j] = targets[(int64_t)w * 8 + j];
  E8Small e8{s_abs, s_par, grid, sign_id};
  const int c = gram_search_warp(e8, t, s_L, lam_lo, lam_hi, nullptr);
  if ((threadIdx.x & 31) == 0) out_idx[w] = c;
}

}  // namespace mpq

using namespace mpq;

MPQ_API int mpq_gram_meta(const float* Vs, int64_t ld, int R, int nb, float* meta, int* fail_count, void* stream) {
  MPQ_CHECK_ARG(Vs && meta && fail_count, "mpq_gram_meta: null pointer");
  if (nb == 0) return MPQ_OK;
  k_gram_meta<<<(nb * 32 + 127) / 128, 128, 0, (cudaStream_t)stream>>>(Vs, ld, R, nb, meta, fail_count);
  return launch_status("mpq_gram_meta");
}

MPQ_API int mpq_gram_gain(const float* rhs, int64_t ld, int B, int nb, const float* meta, float* gain, void* stream) {
  MPQ_CHECK_ARG(rhs && meta && gain, "mpq_gram_gain: null pointer");
  if (nb == 0) return MPQ_OK;
  k_gram_gain<<<nb, 256, 0, (cudaStream_t)stream>>>(rhs, ld, B, meta, gain);
  return launch_status("mpq_gram_gain");
}

MPQ_API int mpq_gram_gather(const float* Vs, int64_t ldv, int R, const float* Hf, int64_t ldh, const int* order,
                            int c0, int Kb, float* VsJ, float* VsJT, float* Hsub, void* stream) {
  MPQ_CHECK_ARG(Vs && Hf && order && VsJ && VsJT && Hsub, "mpq_gram_gather: null pointer");
  MPQ_CHECK_ARG(Kb >= 1 && Kb <= kChunkBlocks, "mpq_gram_gather: Kb must be in [1, %d]", kChunkBlocks);
  dim3 grid((R + 31) / 32, kChunkCols / 32);
  k_gram_gather<<<grid, 256, 0, (cudaStream_t)stream>>>(Vs, ldv, R, Hf, ldh, order, c0, Kb, VsJ, VsJT, Hsub,
                                                        SplitRows{});
  return launch_status("mpq_gram_gather");
}

// mpq_gram_gather with the chunk's rows of Vs taken from Vs's row-scaled fp16 split (vs_hi / vs_lo, leading
// dimension ld16, vs_inv) into j_hi / j_lo (ldj16) / j_inv instead of fp32 VsJ: the product with them needs no
// split of its own.  With t_hi (optional; t_lo, ldt16 >= 8 Kb, t_inv) the split of VsJT[:, :8 Kb] is written
// too, equal to mpq_split_f16 of that matrix.
MPQ_API int mpq_gram_gather_split(const float* Vs, int64_t ldv, int R, const float* Hf, int64_t ldh, const int* order,
                                  int c0, int Kb, const void* vs_hi, const void* vs_lo, int64_t ld16,
                                  const float* vs_inv, void* j_hi, void* j_lo, int64_t ldj16, float* j_inv,
                                  float* VsJT, float* Hsub, void* t_hi, void* t_lo, int64_t ldt16, float* t_inv,
                                  void* stream) {
  MPQ_CHECK_ARG(Vs && Hf && order && vs_hi && vs_lo && vs_inv && j_hi && j_lo && j_inv && (VsJT || t_hi) && Hsub,
                "mpq_gram_gather_split: null pointer");
  MPQ_CHECK_ARG(Kb >= 1 && Kb <= kChunkBlocks, "mpq_gram_gather_split: Kb must be in [1, %d]", kChunkBlocks);
  MPQ_CHECK_ARG(ld16 >= R && ldj16 >= R, "mpq_gram_gather_split: fp16 leading dimensions below R");
  MPQ_CHECK_ARG(!t_hi || (t_lo && t_inv && ldt16 >= 8 * Kb), "mpq_gram_gather_split: bad VsJT split buffers");
  dim3 grid((R + 31) / 32, t_hi ? 1 : kChunkCols / 32);
  SplitRows sp{static_cast<const unsigned short*>(vs_hi), static_cast<const unsigned short*>(vs_lo), ld16, vs_inv,
               static_cast<unsigned short*>(j_hi), static_cast<unsigned short*>(j_lo), ldj16, j_inv,
               static_cast<unsigned short*>(t_hi), static_cast<unsigned short*>(t_lo), ldt16, t_inv};
  if (t_hi) {
    const int nblk = (R + 31) / 32 > 8 * Kb ? (R + 31) / 32 : 8 * Kb;
    k_gram_gather_fused<<<nblk, 256, 0, (cudaStream_t)stream>>>(Vs, ldv, R, Hf, ldh, order, c0, Kb, VsJT, Hsub, sp,
                                                                0);
  } else {
    k_gram_gather<<<grid, 256, 0, (cudaStream_t)stream>>>(Vs, ldv, R, Hf, ldh, order, c0, Kb, nullptr, VsJT, Hsub, sp);
  }
  return launch_status("mpq_gram_gather_split");
}

// Every chunk of one sweep gathered in one launch (the block order is fixed for the whole sweep, and the gathered
// values depend only on Vs, Hf and the order): chunk c = 0 .. ceil(nb / 16) - 1 gets what mpq_gram_gather_split
// with t_hi would write for c0 = 16 c, at j_hi / j_lo + 128 c ldj16, j_inv + 128 c, Hsub + 16384 c,
// t_hi / t_lo + R c ldt16 (ldt16 >= 128) and t_inv + R c.
MPQ_API int mpq_gram_gather_sweep(const float* Vs, int64_t ldv, int R, const float* Hf, int64_t ldh, const int* order,
                                  int nb, const void* vs_hi, const void* vs_lo, int64_t ld16, const float* vs_inv,
                                  void* j_hi, void* j_lo, int64_t ldj16, float* j_inv, float* Hsub, void* t_hi,
                                  void* t_lo, int64_t ldt16, float* t_inv, void* stream) {
  MPQ_CHECK_ARG(R >= 0 && nb >= 0, "mpq_gram_gather_sweep: negative size");
  if (R == 0 || nb == 0) return MPQ_OK;
  MPQ_CHECK_ARG(Vs && Hf && order && vs_hi && vs_lo && vs_inv && j_hi && j_lo && j_inv && Hsub && t_hi && t_lo && t_inv,
                "mpq_gram_gather_sweep: null pointer");
  MPQ_CHECK_ARG(ld16 >= R && ldj16 >= R, "mpq_gram_gather_sweep: fp16 leading dimensions below R");
  MPQ_CHECK_ARG(ldt16 >= kChunkCols, "mpq_gram_gather_sweep: ldt16 must be at least %d", kChunkCols);
  const int nchunks = (nb + kChunkBlocks - 1) / kChunkBlocks;
  MPQ_CHECK_ARG(nchunks <= 65535, "mpq_gram_gather_sweep: too many chunks");
  SplitRows sp{static_cast<const unsigned short*>(vs_hi), static_cast<const unsigned short*>(vs_lo), ld16, vs_inv,
               static_cast<unsigned short*>(j_hi), static_cast<unsigned short*>(j_lo), ldj16, j_inv,
               static_cast<unsigned short*>(t_hi), static_cast<unsigned short*>(t_lo), ldt16, t_inv};
  const int nblk = (R + 31) / 32 > kChunkCols ? (R + 31) / 32 : kChunkCols;
  k_gram_gather_fused<<<dim3(nblk, nchunks), 256, 0, (cudaStream_t)stream>>>(Vs, ldv, R, Hf, ldh, order, 0,
                                                                             kChunkBlocks, nullptr, Hsub, sp, nb);
  return launch_status("mpq_gram_gather_sweep");
}

MPQ_API int mpq_gram_chunk(float* x, int64_t ldx, const float* rhs, int64_t ldr, const float* Hsub, const float* meta,
                           const int* order, int c0, int Kb, const float* base_abs, const int* base_parity,
                           const float* grid, const uint8_t* sign_id, float* res, int* idx, int64_t ldi, float* delta,
                           int* accepted, long long* evals, int B, float accept_tol, void* stream) {
  MPQ_CHECK_ARG(x && rhs && Hsub && meta && order && base_abs && base_parity && grid && sign_id && res && idx && delta &&
                    accepted,
                "mpq_gram_chunk: null pointer");
  MPQ_CHECK_ARG(Kb >= 1 && Kb <= kChunkBlocks, "mpq_gram_chunk: Kb must be in [1, %d]", kChunkBlocks);
  MPQ_CHECK_ARG(((uintptr_t)grid & 15) == 0, "mpq_gram_chunk: grid must be 16-byte aligned");
  if (B == 0) return MPQ_OK;
  GramChunkArgs a{x, ldx, rhs, ldr, Hsub, meta, order, c0, Kb, base_abs, base_parity, grid, sign_id, res, idx, ldi,
                  delta, accepted, evals, B, accept_tol, nullptr, nullptr, 0, 0};
  const size_t smem = (size_t)(kHsTri + 2048 + 256 + kChunkBlocks * kMeta + 8 * kChunkCols) * 4;
  {
    const int ast = smem_opt_in((const void*)k_gram_chunk<false>, smem, "mpq_gram_chunk");
    if (ast) return ast;
  }
  k_gram_chunk<false><<<(B + 7) / 8, 256, smem, (cudaStream_t)stream>>>(a);
  return launch_status("mpq_gram_chunk");
}

// mpq_gram_chunk reading the rhs product as `splits` split-K partial planes (plane s at rhs + s * plane, leading
// dimension ldr, added in plane order as the split-K reduction adds them) and writing the row-scaled fp16 split of
// delta[:, :8 Kb] (d_hi / d_lo, leading dimension ldd >= 8 Kb, multiple of 8; d_inv), equal to mpq_split_f16 of it:
// the chunk's two products then need neither a reduction nor a split launch of their own.
MPQ_API int mpq_gram_chunk_planes(float* x, int64_t ldx, const float* rhs, int64_t ldr, int splits, int64_t plane,
                                  const float* Hsub, const float* meta, const int* order, int c0, int Kb,
                                  const float* base_abs, const int* base_parity, const float* grid,
                                  const uint8_t* sign_id, float* res, int* idx, int64_t ldi, float* delta, void* d_hi,
                                  void* d_lo, int64_t ldd, float* d_inv, int* accepted, long long* evals, int B,
                                  float accept_tol, void* stream) {
  MPQ_CHECK_ARG(Kb >= 1 && Kb <= kChunkBlocks, "mpq_gram_chunk_planes: Kb must be in [1, %d]", kChunkBlocks);
  MPQ_CHECK_ARG(splits >= 1 && ldr >= 8 * Kb && plane >= (int64_t)B * ldr, "mpq_gram_chunk_planes: bad plane layout");
  if (B == 0) return MPQ_OK;
  MPQ_CHECK_ARG(x && rhs && Hsub && meta && order && base_abs && base_parity && grid && sign_id && res && idx && delta &&
                    accepted && d_hi && d_lo && d_inv,
                "mpq_gram_chunk_planes: null pointer");
  MPQ_CHECK_ARG(ldd >= 8 * Kb, "mpq_gram_chunk_planes: ldd below 8 Kb");
  MPQ_CHECK_ARG(((uintptr_t)grid & 15) == 0, "mpq_gram_chunk_planes: grid must be 16-byte aligned");
  GramChunkArgs a{x, ldx, rhs, ldr, Hsub, meta, order, c0, Kb, base_abs, base_parity, grid, sign_id, res, idx, ldi,
                  delta, accepted, evals, B, accept_tol, nullptr, nullptr, 0, 0, splits, plane,
                  static_cast<unsigned short*>(d_hi), static_cast<unsigned short*>(d_lo), ldd, d_inv};
  const size_t smem = (size_t)(kHsTri + 2048 + 256 + kChunkBlocks * kMeta + 8 * kChunkCols) * 4;
  {
    const int ast = smem_opt_in((const void*)k_gram_chunk<false>, smem, "mpq_gram_chunk_planes");
    if (ast) return ast;
  }
  k_gram_chunk<false><<<(B + 7) / 8, 256, smem, (cudaStream_t)stream>>>(a);
  return launch_status("mpq_gram_chunk_planes");
}

MPQ_API int mpq_gram_chunk_topk(float* x, int64_t ldx, const float* rhs, int64_t ldr, const float* Hsub,
                                const float* meta, const int* order, int c0, int Kb, const float* cand,
                                const int* cand_idx, int kc, int nb, float* res, int* idx, int64_t ldi, float* delta,
                                int* accepted, long long* evals, int B, float accept_tol, void* stream) {
  MPQ_CHECK_ARG(Kb >= 1 && Kb <= kChunkBlocks, "mpq_gram_chunk_topk: Kb must be in [1, %d]", kChunkBlocks);
  MPQ_CHECK_ARG(kc >= 1 && nb >= 1, "mpq_gram_chunk_topk: bad candidate shape");
  if (B == 0) return MPQ_OK;
  MPQ_CHECK_ARG(x && rhs && Hsub && meta && order && cand && res && idx && delta && accepted,
                "mpq_gram_chunk_topk: null pointer");
  MPQ_CHECK_ARG(((uintptr_t)cand & 15) == 0, "mpq_gram_chunk_topk: candidates must be 16-byte aligned");
  GramChunkArgs a{x, ldx, rhs, ldr, Hsub, meta, order, c0, Kb, nullptr, nullptr, nullptr, nullptr, res, idx, ldi,
                  delta, accepted, evals, B, accept_tol, cand, cand_idx, kc, nb};
  const size_t smem = (size_t)(kHsTri + 2048 + 256 + kChunkBlocks * kMeta + 8 * kChunkCols) * 4;
  {
    const int ast = smem_opt_in((const void*)k_gram_chunk<true>, smem, "mpq_gram_chunk_topk");
    if (ast) return ast;
  }
  k_gram_chunk<true><<<(B + 7) / 8, 256, smem, (cudaStream_t)stream>>>(a);
  return launch_status("mpq_gram_chunk_topk");
}

MPQ_API int mpq_gram_search(const float* targets, int N, const float* L, float lam_lo, float lam_hi,
                            const float* base_abs, const int* base_parity, const float* grid, const uint8_t* sign_id,
                            int* out_idx, void* stream) {
  MPQ_CHECK_ARG(targets && L && base_abs && base_parity && grid && sign_id && out_idx, "mpq_gram_search: null pointer");
  MPQ_CHECK_ARG(((uintptr_t)grid & 15) == 0, "mpq_gram_search: grid must be 16-byte aligned");
  if (N == 0) return MPQ_OK;
  k_gram_search<<<(N * 32 + 255) / 256, 256, 0, (cudaStream_t)stream>>>(targets, N, L, lam_lo, lam_hi, base_abs,
                                                                        base_parity, grid, sign_id, out_idx);
  return launch_status("mpq_gram_search");
}
