// Per-block steps of the generic rank-space block coordinate descent (any candidate provider).
//
// Reference: mpq/polish/block_cd.py:520-547 (the eager block step: target, provider proposal, accept test,
// residual update) with _cd_accept_step_impl :28-48.  The residual products rhs = residual Vs_blk^T and
// residual -= delta Vs_blk run as GEMMs between these kernels; blocks have bs <= 8 coordinates.
#include "common.cuh"

namespace mpq {

// target = x_blk + rhs Ginv (Ginv bs x bs, row-major) or x_blk + rhs * diag_inv[start .. start+bs)
__global__ void k_cd_target(const float* __restrict__ x, int64_t ldx, const float* __restrict__ rhs, int64_t ldr, int B,
                            int bs, const float* __restrict__ ginv, const float* __restrict__ diag_inv,
                            float* __restrict__ target, int64_t ldt) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  float r[8];
  for (int i = 0; i < bs; ++i) r[i] = rhs[b * ldr + i];
  for (int j = 0; j < bs; ++j) {
    float step;
    if (ginv) {
      step = 0.f;
      for (int i = 0; i < bs; ++i) step = fadd(step, fmul(r[i], ginv[i * bs + j]));
    } else {
      step = fmul(r[j], diag_inv[j]);
    }
    target[b * ldt + j] = fadd(x[b * ldx + j], step);
  }
}

// Accept test of one block's proposal per row (mpq/polish/block_cd.py:28-48, :535-547):
//   delta = cand - x_blk; cross = rhs.delta; dn = max(delta gram delta^T, 0); err = max(res + dn - 2 cross, 0);
//   accept = err + 1e-12 < res (1 + tol).  Accepted rows take the candidate, its index and err; delta_out is
//   delta for accepted rows and 0 otherwise (the residual update operand).
__global__ void k_cd_accept(float* __restrict__ x, int64_t ldx, const float* __restrict__ cand, int64_t ldc,
                            const float* __restrict__ rhs, int64_t ldr, const float* __restrict__ gram,
                            float* __restrict__ res_norm, int B, int bs, float accept_tol, float* __restrict__ delta_out,
                            int64_t ldd, const int* __restrict__ cand_idx, int* __restrict__ idx, int64_t ldi,
                            int* __restrict__ accepted) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  bool acc = false;
  if (b < B) {
    float d[8], cross = 0.f;
    for (int i = 0; i < bs; ++i) {
      d[i] = fsub(cand[b * ldc + i], x[b * ldx + i]);
      cross = fadd(cross, fmul(rhs[b * ldr + i], d[i]));
    }
    float dn = 0.f;
    for (int j = 0; j < bs; ++j) {
      float dg = 0.f;
      for (int i = 0; i < bs; ++i) dg = fadd(dg, fmul(d[i], gram[i * bs + j]));
      dn = fadd(dn, fmul(dg, d[j]));
    }
    dn = fmaxf(dn, 0.f);
    const float res = res_norm[b];
    const float err = fmaxf(fsub(fadd(res, dn), fmul(2.f, cross)), 0.f);
    acc = fadd(err, 1e-12f) < fmul(res, 1.f + accept_tol);
    for (int i = 0; i < bs; ++i) {
      if (acc) x[b * ldx + i] = cand[b * ldc + i];
      delta_out[b * ldd + i] = acc ? d[i] : 0.f;
    }
    if (acc) {
      res_norm[b] = err;
      if (idx && cand_idx) idx[b * ldi] = cand_idx[b];
    }
  }
  const unsigned m = __ballot_sync(0xffffffffu, acc);
  if ((threadIdx.x & 31) == 0 && m) atomicAdd(accepted, __popc(m));
}

}  // namespace mpq

using namespace mpq;

MPQ_API int mpq_cd_target(const float* x, int64_t ldx, const float* rhs, int64_t ldr, int B, int bs, const float* ginv,
                          const float* diag_inv, float* target, int64_t ldt, void* stream) {
  MPQ_CHECK_ARG(x && rhs && target && (ginv || diag_inv), "mpq_cd_target: null pointer");
  MPQ_CHECK_ARG(B >= 0 && bs >= 1 && bs <= 8, "mpq_cd_target: bad shape (bs must be 1..8)");
  if (B == 0) return MPQ_OK;
  k_cd_target<<<(B + 127) / 128, 128, 0, (cudaStream_t)stream>>>(x, ldx, rhs, ldr, B, bs, ginv, diag_inv, target, ldt);
  return launch_status("mpq_cd_target");
}

MPQ_API int mpq_cd_accept(float* x, int64_t ldx, const float* cand, int64_t ldc, const float* rhs, int64_t ldr,
                          const float* gram, float* res_norm, int B, int bs, float accept_tol, float* delta, int64_t ldd,
                          const int* cand_idx, int* idx, int64_t ldi, int* accepted, void* stream) {
  MPQ_CHECK_ARG(x && cand && rhs && gram && res_norm && delta && accepted, "mpq_cd_accept: null pointer");
  MPQ_CHECK_ARG(B >= 0 && bs >= 1 && bs <= 8, "mpq_cd_accept: bad shape (bs must be 1..8)");
  if (B == 0) return MPQ_OK;
  k_cd_accept<<<(B + 127) / 128, 128, 0, (cudaStream_t)stream>>>(x, ldx, cand, ldc, rhs, ldr, gram, res_norm, B, bs,
                                                                accept_tol, delta, ldd, cand_idx, idx, ldi, accepted);
  return launch_status("mpq_cd_accept");
}
