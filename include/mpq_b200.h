/*
 * mpq_b200.h — C ABI of libmpq_b200.so, the sm_100a kernels of MPQ's per-layer quantization solve.
 *
 * Conventions (all entry points):
 *   - plain device pointers and sizes; row-major float32 matrices with an explicit leading
 *     dimension (elements); `stream` is a cudaStream_t (NULL = legacy default stream);
 *   - work is enqueued on `stream` and the call returns without synchronizing;
 *   - return 0 on success, 10001 for an invalid argument, or a cudaError_t from the launch;
 *     mpq_last_error() gives a message for the calling thread's last failure;
 *   - grouped quantizer parameters (scale, zero) are addressed p[row * ld_p + (col >> gshift)]:
 *     gshift = 0 for group-expanded (B x n) tensors, log2(group) for per-group (B x n/group).
 *
 * The reference (poseidonchan/MPQ) is a Python package; the functions below replace the device
 * work behind its Python plugin points.  Each declaration names the reference code it replaces
 * (path:line within the reference project).
 */
#ifndef MPQ_B200_H
#define MPQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- library ---- */
const char* mpq_last_error(void);
int mpq_abi_version(void);

/* ---- grouped-scalar prior (K1) ----
 * Exact discrete posterior over the maxq+1 grid atoms with a Gaussian prior centred on W:
 * outputs the posterior mean (and optionally var, MAP value, MAP index), plus the per-row
 * variance sum (alpha1 = gamma * var_rowsum / n).  prior_tau <= 0 disables the prior.
 * Replaces mpq/priors/uniform.py:99-213 (discrete_uniform_mmse) and
 * mpq/priors/triton_vamp.py:24-102,446-517 (_uniform_mmse_kernel / uniform_mmse_triton). */
int mpq_uniform_mmse(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* scale,
                     const float* zero, int64_t ld_p, int gshift, const float* gamma, int B, int n, int maxq,
                     float prior_tau, float* mean_out, int64_t ld_out, float* var_out, float* map_value_out,
                     uint8_t* map_idx_out, float* var_rowsum, void* stream);

/* MAP hard decision: argmax atom re-rounded through nearest_atom_idx, codes (u8) and dequantized values.
 * Replaces mpq/solver.py:513-541 (_current_hard_state) + :833-850 (_uniform_hard_decision, 'map'). */
int mpq_uniform_map_decision(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* scale,
                             const float* zero, int64_t ld_p, int gshift, const float* gamma, int B, int n, int maxq,
                             float prior_tau, uint8_t* q_out, float* x_out, int64_t ld_out, void* stream);

/* q = clamp(rint(x / max(s,1e-12) + z), 0, maxq); x_out = s (q - z).
 * Replaces mpq/priors/uniform.py:287-309 (nearest_atom_idx, dequant_from_q). */
int mpq_uniform_nearest(const float* x, int64_t ld_x, const float* scale, const float* zero, int64_t ld_p, int gshift,
                        int B, int n, int maxq, uint8_t* q_out, float* x_out, int64_t ld_out, void* stream);

/* Per-(row, group) asymmetric min-max grid (scale, zero); the restated GPTQ quantizer called at
 * mpq/adapters/gptqmodel.py:899-909 (GPTQModel Quantizer.find_params, not vendored). */
int mpq_group_minmax(const float* W, int64_t ldw, int rows, int cols, int group, int maxq, float* scale, float* zero,
                     int64_t ldp, void* stream);

/* RTN init q = clamp(rint(W / s) + z, 0, maxq); x = s (q - z).  Replaces mpq/adapters/gptqmodel.py:928-931,968-969. */
int mpq_uniform_rtn(const float* W, int64_t ldw, const float* scale, const float* zero, int64_t ld_p, int gshift,
                    int B, int n, int maxq, uint8_t* q_out, float* x_out, int64_t ld_out, void* stream);

/* ---- VAMP message algebra (mpq/solver.py:553-699, mpq/linear.py:10-94) ---- */

/* Per-row scalar stage of one iteration: alpha1 = gamma1_work * var_rowsum / n_var (n_var = n for the scalar
 * grid, n/8 for E8P12 blocks), gamma2 (damped), the
 * gamma-only terms of linear_mmse_exact (alpha2, eta2, gamma1_new, damped gamma1) and the EM
 * trace term.  flags[0..4] count invalid alpha1 / non-finite alpha1 / invalid gamma2_new /
 * invalid gamma2 / clipped alpha2 rows.  final_retry != 0 clips alpha1 instead of failing.
 * Replaces mpq/solver.py:559-653 (scalar parts), mpq/linear.py:44-54,74-75. */
int mpq_vamp_rows(const float* var_rowsum, float* gamma1, float* gamma1_work, float* alpha1, float* eta1,
                  float* gamma2_new, float* gamma2, const float* gamma2_prev, float* alpha2, float* eta2,
                  float* gamma1_new, float* gamma1_next, float* trace, int* flags, const float* S, int B, int n,
                  int R, float obs, float damping, int final_retry, void* stream);

/* gamma retry of rows with alpha1 = gamma1_work * var_rowsum / n_var outside (1e-7, 1-1e-7).
 * Replaces mpq/solver.py:593-596 (and :998-1001). */
int mpq_gamma_retry(float* gamma1_work, const float* var_rowsum, int B, int n_var, float factor, void* stream);

/* r2 = damp(r2_prev, (eta1 x1 - gamma1w r1) / gamma2_new); r2_prev NULL = undamped.  mpq/solver.py:605-612. */
int mpq_vamp_r2(const float* x1, const float* r1, const float* r2_prev, float* r2, const float* eta1,
                const float* gamma1_work, const float* gamma2_new, int B, int n, int64_t ld, float damping,
                void* stream);

/* Linear-module epilogue over P = r2 V: u = (Y_u - P s) obs s / denom and rowsum(residual_after^2).
 * Replaces mpq/linear.py:46-55 and the residual term of mpq/linear.py:76. */
int mpq_linear_epilogue(const float* P, const float* Y_u, const float* S, const float* gamma2, float obs, int B, int R,
                        int64_t ld, float* u, float* resid_rowsum, void* stream);

/* r1 = damp(r1, (eta2 (r2 + D) - gamma2 r2) / gamma1_new) with D = u V^T.  mpq/linear.py:51-52, mpq/solver.py:645-653. */
int mpq_vamp_r1(const float* D, const float* r2, float* r1, const float* eta2, const float* gamma2,
                const float* gamma1_new, int B, int n, int64_t ld, float damping, void* stream);

/* out[b] = sum_r (Y[b,r] - C[b,r])^2.  Replaces mpq/linear.py:85-94 (vamp_rankspace_error) after C = x Vs. */
int mpq_row_sqerr(const float* Y, const float* C, int B, int R, int64_t ldy, int64_t ldc, float* out, void* stream);

/* C <- Y - C and rowsum(C^2).  Replaces mpq/polish/triton_scalar_cd.py:195-197 (residual_u, residual_norm). */
int mpq_residual(const float* Y, float* C, int B, int R, int64_t ld, float* rowsum, void* stream);

/* out = mean_b (a[b] + c[b]) (c may be NULL), fixed-order reduction.  mpq/linear.py:77, mpq/solver.py:679. */
int mpq_mean_rows(const float* a, const float* c, int B, float* out, void* stream);

/* Row-wise polish merge where err_after + 1e-12 < err_before.  Replaces mpq/solver.py:749-754. */
int mpq_polish_merge(const float* err_after, float* err_final, const float* err_before, const float* x_src,
                     float* x_dst, const uint8_t* q_src, uint8_t* q_dst, int B, int n, int64_t ld,
                     int* improved_count, void* stream);

/* gamma1 = gamma_start * 0.25 / max(mean_j (W - x)^2, 1e-12).  Replaces mpq/solver.py:86-87,481. */
int mpq_gamma_init(const float* W, const float* x, int B, int n, int64_t ld, float gamma_start, float* gamma1,
                   void* stream);

/* out[b] = sum_j A[b,j] C[b,j].  The raw-Hessian audit of mpq/adapters/gptqmodel.py:1048-1056. */
int mpq_row_dot(const float* A, int64_t lda, const float* C, int64_t ldc, int B, int n, float* out, void* stream);

/* D = A - C (same leading dimension).  mpq/adapters/gptqmodel.py:932, :1049. */
int mpq_sub(const float* A, const float* C, float* D, int B, int n, int64_t ld, void* stream);

/* ---- device-resident VAMP control (mpq/solver.py:553-699 and :961-1122 without host round trips) ----
 * The host decisions of the reference's loop -- gamma retries (:553-596), skipped iterations on invalid gamma2
 * (:598-616), the EM update of the observation precision (mpq/linear.py:59-82, log-damped as
 * mpq/utils.py:36-45) and the scalar best-iterate test (:668-699) -- are taken by small kernels reading and writing
 * a 64-byte control block in device memory (mpq_vamp_ctl_size() bytes, zeroed, then obs (float64 at offset 0) set
 * to the starting precision).  Layout: double obs; int active, skip, have_prev, stopped, fail, alpha1_retry_count,
 * alpha2_clip_count, gamma2_invalid_count, committed, best_iter, stop_iter; 3 ints padding.  The *_ctl variants of
 * the iteration kernels do nothing on a skipped iteration and read obs from the block. */
int mpq_vamp_ctl_size(void);
/* Opens an iteration: gamma1_work = gamma1, flags[0..7] = 0, active = !stopped, skip = stopped. */
int mpq_vamp_ctl_begin(void* ctl, const float* gamma1, float* gamma1_work, int B, int* flags, void* stream);
/* Closes retry round `final_round` (0 or 1 for the last): counts retries and rescales gamma1_work of invalid rows, or
 * closes the round and applies the invalid-gamma2 skip / alpha2 clip counts. */
int mpq_vamp_ctl_round(void* ctl, int* flags, float* gamma1_work, const float* var_rowsum, int B, int n_var,
                       float factor, int final_round, void* stream);
/* Commits a live iteration: gamma1 <- gamma1_next, gamma2_prev <- gamma2, EM update of obs from
 * mean(resid_rowsum + trace); obs_hist[it] (optional) records obs, alpha1_hist[it] / alpha2_hist[it] (optional,
 * together) the row means of alpha1 and alpha2 (the reference's alpha1_mean / alpha2_mean terms,
 * mpq/solver.py:1064-1065); NaN for a skipped iteration. */
int mpq_vamp_ctl_commit(void* ctl, float* gamma1, const float* gamma1_next, float* gamma2_prev, const float* gamma2,
                        const float* resid_rowsum, const float* trace, int B, int R, int em_active, double em_damping,
                        double em_min, double em_max, double* obs_hist, const float* alpha1, const float* alpha2,
                        double* alpha1_hist, double* alpha2_hist, int it, float* gamma1_work_next, int* flags_next,
                        void* stream);
/* gamma1_work_next / flags_next (optional, together): the commit also opens the next iteration (mpq_vamp_ctl_begin's
 * work), saving a launch per iteration. */
/* Best-iterate test and state copies of the scalar loop (mpq/solver.py:668-699); decision[0] = 1 improved, 0 stopped
 * (r1, gamma1, obs restored), -1 skipped. */
int mpq_vamp_ctl_best(void* ctl, const float* err_cur, int B, int n, double* best_mean, double* best_obs,
                      uint8_t* best_q, const uint8_t* cur_q, float* best_x, const float* cur_x, float* best_err,
                      float* best_r1, float* r1, float* best_g1, float* gamma1, int64_t ld, int it, int* decision,
                      void* stream);
int mpq_vamp_rows_ctl(const float* var_rowsum, float* gamma1, float* gamma1_work, float* alpha1, float* eta1,
                      float* gamma2_new, float* gamma2, const float* gamma2_prev, float* alpha2, float* eta2,
                      float* gamma1_new, float* gamma1_next, float* trace, int* flags, const float* S, int B, int n,
                      int n_var, int R, float damping, int final_retry, const void* ctl, void* stream);
/* mpq_vamp_rows_ctl and the end of the retry round (mpq_vamp_ctl_round) in one launch: the last row CTA to finish
 * takes the round's decision.  counter: caller-owned device word, zero before the first launch and left at zero. */
int mpq_vamp_rows_round_ctl(const float* var_rowsum, float* gamma1, float* gamma1_work, float* alpha1, float* eta1,
                            float* gamma2_new, float* gamma2, const float* gamma2_prev, float* alpha2, float* eta2,
                            float* gamma1_new, float* gamma1_next, float* trace, int* flags, const float* S, int B,
                            int n, int n_var, int R, float damping, int final_retry, void* ctl, float factor,
                            unsigned* counter, void* stream);
int mpq_vamp_r2_ctl(const float* x1, const float* r1, const float* r2_prev, float* r2, const float* eta1,
                    const float* gamma1_work, const float* gamma2_new, int B, int n, int64_t ld, float damping,
                    const void* ctl, void* stream);
int mpq_linear_epilogue_ctl(const float* P, const float* Y_u, const float* S, const float* gamma2, int B, int R,
                            int64_t ld, float* u, float* resid_rowsum, const void* ctl, void* stream);
/* r2_keep (optional) receives r2 (the next iteration's r2_prev). */
int mpq_vamp_r1_ctl(const float* D, const float* r2, float* r1, const float* eta2, const float* gamma2,
                    const float* gamma1_new, int B, int n, int64_t ld, float damping, float* r2_keep, const void* ctl,
                    void* stream);

/* Fused forms of the loop above (same arithmetic): the rank-space products come as split-K partial planes that the
 * consumer adds in plane order (mpq_gemm_f16x3_parts), and the producers of a product's A operand write it in the
 * row-scaled fp16 split of mpq_split_f16 (mpq/solver.py:605-653, mpq/linear.py:46-55). */
int mpq_vamp_r2_split_ctl(const float* x1, const float* r1, const float* r2_prev, float* r2, const float* eta1,
                          const float* gamma1_work, const float* gamma2_new, int B, int n, int64_t ld, float damping,
                          void* hi, void* lo, int64_t ldo, float* inv_scale, const void* ctl, void* stream);
int mpq_linear_epilogue_parts_ctl(const float* parts, int splits, const float* Y_u, int64_t ldy, const float* S,
                                  const float* gamma2, int B, int R, float* u, void* hi, void* lo, int64_t ldo,
                                  float* inv_scale, float* resid_rowsum, const void* ctl, void* stream);
int mpq_vamp_r1_parts_ctl(const float* parts, int splits, const float* r2, float* r1, const float* eta2,
                          const float* gamma2, const float* gamma1_new, int B, int n, int64_t ld, float damping,
                          float* r2_keep, const void* ctl, void* stream);

/* ---- dense products (K7/K8, scalar-CD block updates) ----
 * C = alpha A op(B) + beta C with A: M x K row-major; layout 0: B is N x K ("NT"), layout 1: B is K x N ("NN").
 * Replaces the torch matmuls of mpq/linear.py:48,51,94, mpq/solver.py:485 and
 * mpq/polish/triton_scalar_cd.py:195-196,286-288. */
int mpq_gemm_f32(int layout, int M, int N, int K, float alpha, const float* A, int64_t lda, const float* B,
                 int64_t ldb, float beta, float* C, int64_t ldc, void* stream);

/* ---- scalar greedy CD (K2): mpq/polish/triton_scalar_cd.py:164-307 ---- */
/* diag = max(rowsum(Vs^2), 1e-12), diag_inv = 1/diag.  :198-199 */
int mpq_cd_diag(const float* Vs, int n, int R, int64_t ld, float* diag, float* diag_inv, void* stream);
/* gain[j] = sum_b rhs[b,j]^2 diag_inv[j] / B.  :242 */
int mpq_cd_gain(const float* rhs, int B, int n, int64_t ld, const float* diag_inv, float* gain, void* stream);
/* order = argsort(key, descending), ties by ascending index; n <= 16384.  :243 */
int mpq_argsort_desc(const float* key, int n, int* order, void* stream);
/* HJT[j,k] = H[order[c0+k], j] (n x 128, leading dimension 128), Hsub[k,l] = H[order[c0+k], order[c0+l]]
 * (128 x 128); the block's rows of the raw Hessian in the layouts of the update GEMM and of mpq_cd_block. */
int mpq_cd_gather(const float* H, int64_t ldh, int n, const int* order, int c0, int K, float* HJT, float* Hsub,
                  void* stream);
/* Sequential greedy decisions of the columns order[c0 : c0+K] (K <= 128) for every row; writes x, the
 * residual norms, the accepted steps delta (B x 128) and the accepted count.  Replaces the column loop
 * of the persistent Triton sweep :59-107 for one block of columns. */
int mpq_cd_block(float* x, int64_t ldx, const float* rhs, int64_t ldr, const float* scale, const float* zero,
                 int64_t ld_p, int gshift, const float* diag, const float* diag_inv, const int* order, int c0, int K,
                 const float* Hsub, float* res, float* delta, int* accepted, int B, int maxq, float accept_tol,
                 void* stream);
/* mpq_cd_block with the top-k provider's candidates: each column's step goes to the nearest (first minimum of
 * the squared distance to the target) of its kc <= 32 candidate values cand[b, col, :] (row stride ld_cand);
 * an accepted step writes the candidate's grid level cand_q[b, col, c] to qout.  With H = Vs Vs^T this is the
 * generic block CD of mpq/polish/block_cd.py:548-580 with UniformTopKProvider :657-685, block size 1. */
int mpq_cd_block_topk(float* x, int64_t ldx, const float* rhs, int64_t ldr, const float* cand, const int32_t* cand_q,
                      int64_t ld_cand, int kc, int32_t* qout, int64_t ldq, const float* diag, const float* diag_inv,
                      const int* order, int c0, int K, const float* Hsub, float* res, float* delta, int* accepted,
                      int B, float accept_tol, void* stream);

/* ---- tensor-core products (tcgen05 + TMEM + TMA, sm_100a) ----
 * C = alpha * sum_{r < nreg} A[r] B[r]^T + beta C, TF32 operands with FP32 accumulation; A[r]: M x K row-major,
 * B[r]: N x K row-major (host arrays of device pointers); nreg = 3 with (A_hi,B_hi),(A_hi,B_lo),(A_lo,B_hi) is the
 * FP32-faithful 3xTF32 product.  16-byte aligned operands, lda/ldb multiples of 4.  `status` (device int) records a
 * pipeline-wait timeout.  Replaces the FP32 torch matmuls of mpq/linear.py:48,51,94, mpq/solver.py:485 and
 * mpq/polish/triton_scalar_cd.py:195-196,286-288. */
int mpq_gemm_tc(int nreg, int M, int N, int K, float alpha, const float* const* A, int64_t lda, const float* const* B,
                int64_t ldb, float beta, float* C, int64_t ldc, int* status, void* stream);
/* FP32-faithful product on the fp16 tensor cores (kind::f16, twice the TF32 rate): C = alpha (sum over (hi,hi), (hi,lo),
 * (lo,hi) of diag(sa) A B^T diag(sb)) + beta C from the row-scaled fp16 splits of mpq_split_f16 (16-bit row-major,
 * lda/ldb multiples of 8, 16-byte aligned).  Same products as mpq_gemm_tc (mpq/linear.py:48,51,94, mpq/solver.py:485). */
int mpq_gemm_f16x3(int M, int N, int K, float alpha, const void* a_hi, const void* a_lo, int64_t lda, const float* sa,
                   const void* b_hi, const void* b_lo, int64_t ldb, const float* sb, float beta, float* C, int64_t ldc,
                   int* status, void* stream);
/* mpq_gemm_f16x3 with split-K for small-M products (a 128-row VAMP block against the n x n basis, mpq/linear.py:48,51
 * at the block sizes of mpq/adapters/quip_sharp.py:28): the k-blocks of each output tile are cut into `splits`
 * ranges run by different CTAs; their partials go to ws (caller-owned, splits * M * N floats) and are summed in a
 * fixed order (deterministic).  1 <= splits <= 3 * ceil(K / 64). */
/* The partial products of mpq_gemm_f16x3_splitk without the reduction: plane s of ws (M x N, leading dimension N)
 * holds the s-th k-range's sum (row scales applied); consumers add planes 0, 1, ... in order. */
int mpq_gemm_f16x3_parts(int M, int N, int K, const void* a_hi, const void* a_lo, int64_t lda, const float* sa,
                         const void* b_hi, const void* b_lo, int64_t ldb, const float* sb, int splits, float* ws,
                         int64_t ws_floats, int* status, void* stream);
int mpq_gemm_f16x3_splitk(int M, int N, int K, float alpha, const void* a_hi, const void* a_lo, int64_t lda,
                          const float* sa, const void* b_hi, const void* b_lo, int64_t ldb, const float* sb, float beta,
                          float* C, int64_t ldc, int splits, float* ws, int64_t ws_floats, int* status, void* stream);
/* Row-scaled fp16 split: s = 2^(15 - E) with max|x_row| < 2^E, hi = fp16(x s), lo = fp16(x s - hi), inv_scale = 1 / s. */
int mpq_split_f16(const float* x, int64_t ldx, int rows, int cols, void* hi, void* lo, int64_t ldo, float* inv_scale,
                  void* stream);
/* hi = TF32 round-to-nearest of x, lo = x - hi (the operand split of the 3xTF32 product). */
int mpq_split_tf32(const float* x, int64_t ldx, float* hi, float* lo, int64_t ldo, int rows, int cols, void* stream);
/* ---- calibration Hessian (K11) ----
 * Symmetric product C = alpha sum_{r < nreg} A[r] B[r]^T + beta C (n x n) where A[r], B[r] (n x K row-major, lda) are
 * halves of one matrix (3xTF32: (hi,hi),(hi,lo),(lo,hi)); only tiles with entries col <= row are computed and each
 * entry is also stored at its mirror, so C is exactly symmetric; beta reads the lower triangle.  With the
 * operand X^T this is the H += X^T X accumulation of the Hessian hooks the MPQ drivers consume (GPTQModel
 * GPTQ.add_batch and QUIP# utils.register_H_hook, un-vendored; finalised at mpq/quip_generic.py:906-918). */
int mpq_syrk_tc(int nreg, int n, int K, float alpha, const float* const* A, const float* const* B, int64_t lda,
                float beta, float* C, int64_t ldc, int* status, void* stream);
/* Transposing split of token-major activations X (T x n; dtype 0 = f32, 1 = bf16): hi[j,t] = tf32(X[t,j]),
 * lo[j,t] = X[t,j] - hi[j,t] (lo may be NULL: bf16 values are exact in TF32). */
int mpq_split_tf32_t(const void* x, int dtype, int64_t ldx, int tokens, int n, float* hi, float* lo, int64_t ldo,
                     void* stream);
/* Symmetric product of a bf16 operand C = alpha A A^T + beta C (A: n x K row-major bf16, lda a multiple of 8) with
 * kind::f16 tensor-core MMAs (exact bf16 products, FP32 accumulation); mirror = 0 updates the lower triangle only
 * (intermediate accumulation steps), 1 also stores every entry at its mirror.  The Hessian hooks' X^T X for bf16
 * activations (see mpq_syrk_tc). */
int mpq_syrk_bf16(int n, int K, float alpha, const void* A, int64_t lda, float beta, float* C, int64_t ldc, int mirror,
                  int* status, void* stream);
/* The whole-K forms of mpq_syrk_bf16 / mpq_syrk_tc in one launch (the same H += X^T X accumulation): the tensor core
 * accumulates `chunk` columns of K at a time (a multiple of 64 for bf16, of 32 for fp32) and each chunk is added,
 * round to nearest, into a running sum held in tensor memory; C is read (beta != 0, lower triangle) and written once
 * per tile, every entry also at its mirror (exactly symmetric). */
int mpq_syrk_bf16_acc(int n, int K, float alpha, const void* A, int64_t lda, float beta, float* C, int64_t ldc,
                      int chunk, int* status, void* stream);
int mpq_syrk_tc_acc(int nreg, int n, int K, float alpha, const float* const* A, const float* const* B, int64_t lda,
                    float beta, float* C, int64_t ldc, int chunk, int* status, void* stream);
/* out[j,t] = X[t,j] for bf16 activations X (T x n): the K-major operand of mpq_syrk_bf16. */
int mpq_transpose_bf16(const void* x, int64_t ldx, int tokens, int n, void* out, int64_t ldo, void* stream);
/* out[j] = beta out[j] + alpha sum_t X[t,j] (the QUIP# hook's running sum of inputs, mpq/quip_generic.py:906-918). */
int mpq_col_sum(const void* x, int dtype, int64_t ldx, int tokens, int n, float alpha, float beta, float* out,
                void* stream);

/* Allocation-free 3xTF32 product C = alpha A B^T + beta C (A: M x K, B: N x K, row-major fp32).  No counterpart in
 * the reference: it serves callers that cannot allocate device memory where they need the product (memory-capped
 * pools, FFI hosts holding only the buffers handed to them, paths where a cudaMalloc would synchronise).  The
 * TF32 operand split and the status word live in a 16 MiB file-scope device array held by every GPU that loads
 * the library until exit; 2 (M + N) round_up(K, 4) <= 4,194,240 floats, larger products return MPQ_ERR_ARG.
 * Calls share the array: executions that overlap on the GPU race.  The first call on a device looks up the
 * array's address; make it before any stream capture.  status: optional caller-owned device int (NULL: unreported). */
int mpq_gemm_tf32x3_noalloc(int M, int N, int K, float alpha, const float* A, int64_t lda, const float* B, int64_t ldb,
                            float beta, float* C, int64_t ldc, int* status, void* stream);

/* ---- E8P12 (K3, K4, K6): mpq/priors/e8p12.py ----
 * Tables (from the codebook grid, as mpq/priors/e8p12.py:83-151 derives them): base_abs 256x8, base_sqnorm 256,
 * base_parity 256, idx_lut 2x256x256 (branch, abs, sign id) -> index, grid 65536x8, sign_id 65536 (u8).
 * Items are the nb = n/8 consecutive 8-blocks of each of B rows; the prior (tau > 0, centre W) is folded
 * per block with scale = absmax of the centre block unless pscale (B x nb) is given. */
/* Factorized posterior mean x1 (B x n), per-block variance, MAP index / values and the per-row variance sum.
 * Replaces mpq/priors/e8p12.py:815-968 (vamp_vector_discrete_mmse_e8p12, _branch_factorized_stats :169-308). */
/* Posterior diagnostics per 8-block (need_stats / return_{logZ,margin,entropy}_blocks): log-partition over the
 * 512 (branch, abs) components, entropy -sum w log w + sum w H_sign and the gap between the two largest
 * best / second-best sign-pattern log-scores; outputs B x nb with leading dimension ld.  Replaces
 * mpq/priors/e8p12.py:292-306 and :945-960 (all components evaluated, no pruning). */
int mpq_e8p12_stats(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* pscale,
                    int64_t ld_s, const float* gamma, float prior_tau, int B, int nb, const float* base_abs,
                    const float* base_sqnorm, const int* base_parity, const int* idx_lut, const float* grid,
                    float* logz_out, float* entropy_out, float* margin_out, int64_t ld, void* stream);
int mpq_e8p12_mmse(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* pscale,
                   int64_t ld_s, const float* gamma, float prior_tau, int B, int nb, const float* base_abs,
                   const float* base_sqnorm, const int* base_parity, const int* idx_lut, const float* grid,
                   float* x1_out, int64_t ld_x, float* var_out, int64_t ld_v, int* idx_out, int64_t ld_i,
                   float* map_out, int64_t ld_m, float* var_rowsum, void* stream);
/* The posterior mean and per-row variance sum of mpq_e8p12_mmse with each row cut into `chunks` item ranges (one CTA
 * each), so a 128-row block (mpq/adapters/quip_sharp.py:28, 555-586) still fills the GPU.  work: caller-owned
 * B (chunks + 1) 32-bit words, zeroed once before the first call (chunk partials + arrival counters, left at zero);
 * partials are added in chunk order.  active: optional device int; while it is 0 the launch does nothing (the gamma
 * retries of mpq/solver.py:553-596 decided on the device). */
int mpq_e8p12_mmse_rows(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* pscale,
                        int64_t ld_s, const float* gamma, float prior_tau, int B, int nb, const float* base_abs,
                        const float* base_sqnorm, const int* base_parity, const int* idx_lut, const float* grid,
                        float* x1_out, int64_t ld_x, float* var_rowsum, int chunks, void* work, const int* active,
                        void* stream);
/* mpq_e8p12_mmse_rows with the retry round's row stage fused behind it: the CTA that completes a row's variance sum
 * runs that row's alpha1 / gamma2 / alpha2 / gamma1 algebra (mpq/solver.py:559-631, as mpq_vamp_rows_round_ctl with
 * gamma1_work = gamma and n_var = nb), and the last row to finish takes the retry round's decision
 * (mpq/solver.py:575-604).  One launch per retry round instead of two; the same arithmetic. */
int mpq_e8p12_mmse_rows_round_ctl(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* pscale,
                                  int64_t ld_s, const float* gamma, float prior_tau, int B, int nb,
                                  const float* base_abs, const float* base_sqnorm, const int* base_parity,
                                  const int* idx_lut, const float* grid, float* x1_out, int64_t ld_x, float* var_rowsum,
                                  int chunks, void* work, const int* active, float* gamma1, float* alpha1, float* eta1,
                                  float* gamma2_new, float* gamma2, const float* gamma2_prev, float* alpha2, float* eta2,
                                  float* gamma1_new, float* gamma1_next, float* trace, int* flags, const float* S, int n,
                                  int R, float damping, int final_retry, void* ctl, float factor, unsigned* counter,
                                  void* stream);
/* MAP codeword (bit-exact first maximum); fixed_gamma > 0 with prior_tau <= 0 is the nearest codeword (RTN).
 * Replaces mpq/priors/e8p12.py:541-631 (vamp_vector_map_e8p12, _branch_factorized_map :367-449) and the
 * nearest-codeword cb.quantize of mpq/adapters/quip_sharp.py:212-241. */
int mpq_e8p12_map(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* pscale,
                  int64_t ld_s, const float* gamma, float fixed_gamma, float prior_tau, int B, int nb,
                  const float* base_abs, const float* base_sqnorm, const int* base_parity, const int* idx_lut,
                  const float* grid, int* idx_out, int64_t ld_i, float* map_out, int64_t ld_m, void* stream);

/* ---- top-k polish candidates ----
 * Per block, the k (1..1024) highest-scoring of 1024 candidates: for each (branch, abs pattern) the best and the
 * second-best parity-valid sign pattern under the folded message (mpq/priors/e8p12.py:367-449 need_stats and
 * :453-538 vamp_vector_map_topk_e8p12); scores descending, ties by the reference's flat candidate order.
 * idx_out B x nb x k; score_out and val_out (B x nb x k x 8 codewords) may be NULL.
 * Replaces mpq/solver.py:227-260 (build_e8p12_vamp_topk_candidates). */
int mpq_e8p12_topk(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* pscale,
                   int64_t ld_s, const float* gamma, float prior_tau, int B, int nb, const float* base_abs,
                   const float* base_sqnorm, const int* base_parity, const int* idx_lut, const float* grid, int k,
                   int32_t* idx_out, float* score_out, float* val_out, void* stream);

/* k (1..min(64, maxq+1)) best grid atoms per coordinate by the score -g/2 (atom - r1)^2 [- (atom - W)^2 / (2 tau^2
 * max(s, 1e-12)^2)], descending, ties to the lower level: out_q / out_v / out_s (out_s may be NULL) are B x n x k.
 * Replaces mpq/priors/uniform.py:253-284 (uniform_map_topk) behind mpq/solver.py:201-224. */
int mpq_uniform_topk(const float* r1, int64_t ld_r1, const float* center, int64_t ld_c, const float* scale,
                     const float* zero, int64_t ld_p, int gshift, const float* gamma, int B, int n, int maxq,
                     float prior_tau, int k, int32_t* out_q, float* out_v, float* out_s, void* stream);

/* Per row, the candidate (k candidates of bs <= 8 values, row stride ld_cand) nearest to the row's target: with
 * chol (bs x bs) the metric distance max(|t L|^2 + |c L|^2 - 2 (t L).(c L), 0), else the squared distance; first
 * minimum wins.  Writes the values (out_v) and, with cand_idx, the chosen index (out_idx).
 * Replaces the selection of mpq/polish/block_cd.py:657-685 (UniformTopKProvider) and :93-101, :768-860
 * (E8P12TopKProvider, _topk_metric_select_impl). */
int mpq_topk_pick(const float* target, int64_t ld_t, const float* cand, int64_t ld_cand, const int32_t* cand_idx,
                  int64_t ld_ci, int B, int k, int bs, const float* chol, float* out_v, int64_t ld_o,
                  int32_t* out_idx, void* stream);

/* ---- gram-metric block CD (K5, K10): mpq/polish/block_cd.py:332-625 ----
 * meta per block (196 floats): gram Vs_blk Vs_blk^T | L = stabilize_cholesky(gram) | (L L^T)^-1 | eigenvalue
 * bounds of L L^T.  Replaces mpq/polish/block_cd.py:383-404 and mpq/linear.py:121-141. */
int mpq_gram_meta(const float* Vs, int64_t ld, int R, int nb, float* meta, int* fail_count, void* stream);
/* greedy block gain mean_b rhs_bk Ginv_k rhs_bk^T.  Replaces mpq/polish/block_cd.py:286-306. */
int mpq_gram_gain(const float* rhs, int64_t ld, int B, int nb, const float* meta, float* gain, void* stream);
/* chunk operands for blocks order[c0:c0+Kb] (Kb <= 16): VsJ 128 x R, VsJT R x 128, Hsub 128 x 128 of Hf = Vs Vs^T. */
int mpq_gram_gather(const float* Vs, int64_t ldv, int R, const float* Hf, int64_t ldh, const int* order, int c0,
                    int Kb, float* VsJ, float* VsJT, float* Hsub, void* stream);
/* mpq_gram_gather with the chunk's rows of Vs gathered from Vs's row-scaled fp16 split (vs_hi / vs_lo with leading
 * dimension ld16, vs_inv = 1 / row scale) into j_hi / j_lo / j_inv: the split of a row depends on that row alone,
 * so the product with the gathered split equals the product with the split of the gathered rows.  With t_hi
 * (optional; t_lo, leading dimension ldt16 >= 8 Kb, t_inv) it also writes the split of VsJT[:, :8 Kb], equal to
 * mpq_split_f16 of that matrix, and VsJT itself only when it is not NULL. */
int mpq_gram_gather_split(const float* Vs, int64_t ldv, int R, const float* Hf, int64_t ldh, const int* order, int c0,
                          int Kb, const void* vs_hi, const void* vs_lo, int64_t ld16, const float* vs_inv,
                          void* j_hi, void* j_lo, int64_t ldj16, float* j_inv, float* VsJT, float* Hsub,
                          void* t_hi, void* t_lo, int64_t ldt16, float* t_inv, void* stream);
/* Every chunk of one sweep in one launch: the block order is fixed for the sweep (mpq/polish/block_cd.py:286-306,
 * sorted once per sweep) and the gathered operands depend only on Vs, Hf and that order.  Chunk c = 0 .. ceil(nb/16)-1
 * receives what mpq_gram_gather_split with t_hi writes for c0 = 16 c, in chunk-major slices: j_hi / j_lo + 128 c ldj16,
 * j_inv + 128 c, Hsub + 16384 c, t_hi / t_lo + R c ldt16 (ldt16 >= 128), t_inv + R c.  Replaces the per-chunk
 * gathers of the greedy block loop, mpq/polish/block_cd.py:534-547. */
int mpq_gram_gather_sweep(const float* Vs, int64_t ldv, int R, const float* Hf, int64_t ldh, const int* order, int nb,
                          const void* vs_hi, const void* vs_lo, int64_t ld16, const float* vs_inv, void* j_hi,
                          void* j_lo, int64_t ldj16, float* j_inv, float* Hsub, void* t_hi, void* t_lo, int64_t ldt16,
                          float* t_inv, void* stream);
/* Sequential block decisions of one chunk per row: target = x + rhs Ginv, exact first-minimum gram search,
 * accept test, x / idx / residual-norm updates, accepted steps delta (B x 128).  Replaces the block loop of
 * mpq/polish/block_cd.py:534-547 with _cd_gram_step_impl :212-246. */
int mpq_gram_chunk(float* x, int64_t ldx, const float* rhs, int64_t ldr, const float* Hsub, const float* meta,
                   const int* order, int c0, int Kb, const float* base_abs, const int* base_parity, const float* grid,
                   const uint8_t* sign_id, float* res, int* idx, int64_t ldi, float* delta, int* accepted,
                   long long* evals, int B, float accept_tol, void* stream);
/* mpq_gram_chunk reading the rhs product as `splits` split-K partial planes (plane s at rhs + s * plane, leading
 * dimension ldr, added in plane order as the split-K reduction does) and also writing the row-scaled fp16 split of
 * delta[:, :8 Kb] (d_hi / d_lo, leading dimension ldd; d_inv) exactly as mpq_split_f16 would: the chunk's products
 * need no reduction or split launch of their own (same block loop, mpq/polish/block_cd.py:332-625). */
int mpq_gram_chunk_planes(float* x, int64_t ldx, const float* rhs, int64_t ldr, int splits, int64_t plane,
                          const float* Hsub, const float* meta, const int* order, int c0, int Kb,
                          const float* base_abs, const int* base_parity, const float* grid, const uint8_t* sign_id,
                          float* res, int* idx, int64_t ldi, float* delta, void* d_hi, void* d_lo, int64_t ldd,
                          float* d_inv, int* accepted, long long* evals, int B, float accept_tol, void* stream);
/* mpq_gram_chunk over each block's kc precomputed candidates (cand B x nb x kc x 8, 16-byte aligned; cand_idx
 * B x nb x kc codebook indices): first minimum of the metric distance.  Replaces the top-k block step
 * mpq/polish/block_cd.py:137-172 (_topk_gram_step_impl) with E8P12TopKProvider :768-860. */
int mpq_gram_chunk_topk(float* x, int64_t ldx, const float* rhs, int64_t ldr, const float* Hsub, const float* meta,
                        const int* order, int c0, int Kb, const float* cand, const int32_t* cand_idx, int kc, int nb,
                        float* res, int* idx, int64_t ldi, float* delta, int* accepted, long long* evals, int B,
                        float accept_tol, void* stream);
/* Standalone exact gram-metric search for N targets sharing one factor L (first minimum of
 * |tL|^2 + |cL|^2 - 2 (tL).(cL) over the grid).  Replaces E8P12Provider._metric_map_assign
 * (mpq/polish/block_cd.py:702-739) and the Triton search mpq/polish/triton_e8p12_cd.py:83-180. */
int mpq_gram_search(const float* targets, int N, const float* L, float lam_lo, float lam_hi, const float* base_abs,
                    const int* base_parity, const float* grid, const uint8_t* sign_id, int* out_idx, void* stream);

/* ---- generic rank-space block CD steps (any candidate provider): mpq/polish/block_cd.py:520-547 ----
 * target = x_blk + rhs Ginv (bs x bs) or x_blk + rhs * diag_inv (bs <= 8).  Replaces :521-526. */
int mpq_cd_target(const float* x, int64_t ldx, const float* rhs, int64_t ldr, int B, int bs, const float* ginv,
                  const float* diag_inv, float* target, int64_t ldt, void* stream);
/* Accept test of a proposal per row, x / residual norm / index updates, masked delta for the residual update and
 * the accepted count.  Replaces _cd_accept_step_impl (mpq/polish/block_cd.py:28-48) and :538-547. */
int mpq_cd_accept(float* x, int64_t ldx, const float* cand, int64_t ldc, const float* rhs, int64_t ldr,
                  const float* gram, float* res_norm, int B, int bs, float accept_tol, float* delta, int64_t ldd,
                  const int* cand_idx, int* idx, int64_t ldi, int* accepted, void* stream);

/* ---- export (GPTQ format) ----
 * Little-endian bit-stream packing of b-bit codes (b in 2, 3, 4, 8) along one axis into int32 words: code (p, o) at
 * src[p sp + o so], output word (w, o) holds stream bits [32 w, 32 w + 32) of line o; (code - offset) is masked to
 * b bits (offset 1 gives the v1 qzeros).  The qweight/qzeros of GPTQModel's packer, applied to the codes of
 * mpq/adapters/gptqmodel.py:650-1163 (patches/gptqmodel.patch:370-395; the packer itself is not vendored). */
int mpq_pack_bits(const uint8_t* src, int64_t sp, int64_t so, int n_pack, int n_other, int bits, int offset,
                  int32_t* out, int64_t ld_out, void* stream);

/* ---- rotation ----
 * Block Walsh-Hadamard of the last dim, blocks of `had` (power of two <= 16384), normalized by sqrt(had);
 * mode 0: y = H(x * signs) (right rotation), mode 1: y = H(x) * signs (inverse).  signs may be NULL.
 * Replaces mpq/rotation.py:404-441 (apply_block_hadamard, apply_right_block_hadamard[_inverse]). */
int mpq_block_hadamard(const float* x, int64_t ldx, float* y, int64_t ldy, int rows, int n, int had,
                       const float* signs, int mode, void* stream);

/* ---- peer memory between the processes of one node ----
 * Multi-GPU layer solves compute each layer's eigendecomposition (mpq/adapters/quip_sharp.py:33-67) on one rank;
 * the ranks solving the layer's other row shards copy it from that rank's memory over NVLink instead of repeating
 * it.  The reference has no multi-GPU path; these replace nothing in it.
 * mpq_peer_alloc: cudaMalloc on the current device and export the CUDA IPC handle (64 bytes into out_handle).
 * mpq_peer_open / mpq_peer_close: map / unmap another process's exported buffer in this device's context.
 * mpq_peer_free: free an mpq_peer_alloc buffer after every peer closed it.
 * mpq_copy_bytes: asynchronous copy on `stream`; either side may be a peer mapping. */
int mpq_peer_alloc(size_t bytes, void** out_ptr, void* out_handle, void* stream);
int mpq_peer_open(const void* handle, void** out_ptr, void* stream);
int mpq_peer_close(void* ptr, void* stream);
int mpq_peer_free(void* ptr, void* stream);
int mpq_copy_bytes(void* dst, const void* src, size_t bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* MPQ_B200_H */
