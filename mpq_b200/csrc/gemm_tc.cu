// tcgen05 tensor-core GEMM for sm_100a (TF32 operands, FP32 accumulation in TMEM).
//
//   C[M, N] = alpha * sum_r A_r[M, K] * B_r[N, K]^T + beta * C        (r = 0 .. nreg-1, nreg <= 3)
//
// With (A_hi, B_hi), (A_hi, B_lo), (A_lo, B_hi) this is the 3xTF32 split product, which keeps the
// rank-space VAMP products at FP32 accuracy (plain TF32 flips ~6% of the VAMP codes); with one
// region it is a plain TF32 GEMM.  The regions are concatenated along K, so one accumulator and
// one pipeline serve both.
//
// Structure (one 128 x BN output tile per CTA, 192 threads):
//   warp 0      TMA producer: 2-D tiled loads (128B swizzle) of A and B k-blocks into a STAGES-deep
//               shared-memory ring, completion signalled on per-stage mbarriers (expect_tx);
//   warp 1      allocates BN TMEM columns, issues tcgen05.mma (M=128, N=BN, K=8) from one thread,
//               frees ring slots with tcgen05.commit, and finally commits the accumulator;
//   warps 2..5  epilogue: tcgen05.ld 32x32b of the accumulator (one row per thread) -> global.
// Every mbarrier wait is bounded (globaltimer); on timeout the kernel records an error code in
// `status`, drains its own in-flight copies / MMAs (bounded), frees TMEM and exits.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <algorithm>
#include <cuda_fp16.h>
#include "common.cuh"

namespace mpq {
namespace tc {

constexpr int BM = 128;
// A k-block is one 128-byte swizzle row per operand row: 32 fp32 or 64 16-bit elements.
constexpr int kThreads = 192;
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s per wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false when the deadline passes first.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitNs) return false;
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// UMMA shared-memory descriptor, K-major operand in the 128B-swizzled canonical layout:
// rows of 128 B, 8-row swizzle atoms 1024 B apart (SBO), version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)(16 >> 4) << 16;    // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // SBO: 8 rows x 128 B
  d |= (uint64_t)1 << 46;            // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;            // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::tf32, D = F32, A = B = TF32, both K-major, M = 128, N = bn.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Instruction descriptor: kind::f16 with BF16 A and B (both the same type), D = F32, both K-major, M = 128, N = bn.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Instruction descriptor: kind::f16 with F16 A and B, D = F32, both K-major, M = 128, N = bn.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

struct Maps {
  CUtensorMap a[3];
  CUtensorMap b[3];
};

// 32-bit operands: kind::tf32 (K = 8 per MMA); 16-bit operands: kind::f16 (K = 16 per MMA).  Either way a k-block is
// one 128-byte swizzle row per operand row (32 fp32 or 64 16-bit elements) and 4 MMAs of 32 bytes.
// sym: 0 general product; 1 symmetric (tiles with col <= row, entries stored with their mirrors); 2 symmetric,
// lower triangle only (intermediate accumulation steps).
// One 32-column chunk of a thread's accumulator row -> C (alpha, beta, split row scales, symmetric modes).
__device__ __forceinline__ void store_chunk(uint32_t (&v)[32], int row, int n0, int c0, int M, int N, float alpha,
                                            float beta, float* __restrict__ C, int64_t ldc, int sym,
                                            const float* __restrict__ sa, const float* __restrict__ sb) {
  if (sa) {  // power-of-two row scales of the fp16 split: exact unless the result over/underflows
    const float ra = sa[row < M ? row : 0];
    #pragma unroll
    for (int t = 0; t < 32; ++t) {
      const int col = n0 + c0 + t;
      v[t] = __float_as_uint(__uint_as_float(v[t]) * (ra * (col < N ? sb[col] : 0.f)));
    }
  }
  if (sym) {
    // lower entries (col <= row) and their mirrors: the result is exactly symmetric.  Chunks entirely below
    // the diagonal use 16-byte row stores per thread; the mirror stores of a warp (32 consecutive rows, one
    // column) are contiguous.
    const int cb = n0 + c0;
    float* crow = C + (int64_t)row * ldc + cb;
    if (row < M && cb + 31 < row && cb + 32 <= N && ((reinterpret_cast<uintptr_t>(crow) & 15) == 0)) {
      #pragma unroll
      for (int t = 0; t < 32; t += 4) {
        float4 o;
        o.x = alpha * __uint_as_float(v[t]);
        o.y = alpha * __uint_as_float(v[t + 1]);
        o.z = alpha * __uint_as_float(v[t + 2]);
        o.w = alpha * __uint_as_float(v[t + 3]);
        float4* dst = reinterpret_cast<float4*>(crow + t);
        if (beta != 0.f) {
          const float4 c = *dst;
          o.x += beta * c.x; o.y += beta * c.y; o.z += beta * c.z; o.w += beta * c.w;
        }
        *dst = o;
        if (sym == 1) {
          C[(int64_t)(cb + t) * ldc + row] = o.x;
          C[(int64_t)(cb + t + 1) * ldc + row] = o.y;
          C[(int64_t)(cb + t + 2) * ldc + row] = o.z;
          C[(int64_t)(cb + t + 3) * ldc + row] = o.w;
        }
      }
    } else if (row < M) {
      #pragma unroll
      for (int t = 0; t < 32; ++t) {
        const int col = cb + t;
        if (col < N && col <= row) {
          float o = alpha * __uint_as_float(v[t]);
          if (beta != 0.f) o += beta * C[(int64_t)row * ldc + col];
          C[(int64_t)row * ldc + col] = o;
          if (col != row && sym == 1) C[(int64_t)col * ldc + row] = o;
        }
      }
    }
  } else if (row < M) {
    float* crow = C + (int64_t)row * ldc + n0 + c0;
    const int ncol = min(32, N - (n0 + c0));
    if (ncol == 32 && ((reinterpret_cast<uintptr_t>(crow) & 15) == 0)) {
      #pragma unroll
      for (int t = 0; t < 32; t += 4) {
        float4 o;
        o.x = alpha * __uint_as_float(v[t]);
        o.y = alpha * __uint_as_float(v[t + 1]);
        o.z = alpha * __uint_as_float(v[t + 2]);
        o.w = alpha * __uint_as_float(v[t + 3]);
        float4* dst = reinterpret_cast<float4*>(crow + t);
        if (beta != 0.f) {
          const float4 c = *dst;
          o.x += beta * c.x; o.y += beta * c.y; o.z += beta * c.z; o.w += beta * c.w;
        }
        *dst = o;
      }
    } else {
      #pragma unroll
      for (int t = 0; t < 32; ++t) {
        if (t < ncol) {
          float o = alpha * __uint_as_float(v[t]);
          if (beta != 0.f) o += beta * crow[t];
          crow[t] = o;
        }
      }
    }
  }
}

// KIND 0: fp32 operands, kind::tf32; 1: bf16, kind::f16; 2: fp16, kind::f16.  sa / sb (optional, with KIND 2): per-row
// scales of A's rows and of B's rows applied to the accumulator (the row-scaled fp16 split).
template <int BN, int STAGES, int KIND>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ Maps maps, int nreg, int M, int N, int K, float alpha, float beta,
              float* __restrict__ C, int64_t ldc, int* __restrict__ status, int sym, const float* __restrict__ sa,
              const float* __restrict__ sb) {
  constexpr bool BF16 = KIND != 0;  // 16-bit operands
  constexpr uint32_t kStageA = BM * 128;
  constexpr uint32_t kStageB = BN * 128;
  constexpr int kBKE = BF16 ? 64 : 32;  // elements per k-block
  constexpr uint32_t kIdesc = KIND == 2 ? idesc_f16(BM, BN) : (KIND == 1 ? idesc_bf16(BM, BN) : idesc_tf32(BM, BN));
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte aligned ring (swizzle atoms need 1024 B alignment)
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = base;
  unsigned char* sB = base + STAGES * kStageA;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * kStageB);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_bar = empty + STAGES;
  uint64_t* drain_bar = acc_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  // symmetric product (A_r and B_r are the same operand): only tiles holding entries col <= row run
  if (sym && n0 > m0 + BM - 1) return;
  const int kb_per_reg = (K + kBKE - 1) / kBKE;
  const int total_kb = kb_per_reg * nreg;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_bar, 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < total_kb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
        if (*abort_flag || !mbar_wait(&empty[s], ph ^ 1u)) {
          *abort_flag = 1;
          break;
        }
        const int r = kb / kb_per_reg;
        const int k0 = (kb % kb_per_reg) * kBKE;
        mbar_expect_tx(&full[s], kStageA + kStageB);
        tma_load_2d(sA + s * kStageA, &maps.a[r], &full[s], k0, m0);
        tma_load_2d(sB + s * kStageB, &maps.b[r], &full[s], k0, n0);
        issued = kb + 1;
      }
      if (*abort_flag) {
        // drain: wait (bounded) for every copy this thread issued into the ring
        for (int kb = issued - STAGES < 0 ? 0 : issued - STAGES; kb < issued; ++kb)
          mbar_wait(&full[kb % STAGES], (uint32_t)(kb / STAGES) & 1u);
        atomicCAS(status, 0, 2);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = true;
      for (int kb = 0; kb < total_kb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
        if (*abort_flag || !mbar_wait(&full[s], ph)) {
          ok = false;
          *abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a_addr = smem_u32(sA + s * kStageA);
        const uint32_t b_addr = smem_u32(sB + s * kStageB);
        #pragma unroll
        for (int j = 0; j < 4; ++j) {  // 4 MMAs of 32 bytes per 128-byte k-block row (K = 8 tf32 / 16 bf16)
          const uint64_t da = smem_desc_k_sw128(a_addr + j * 32);
          const uint64_t db = smem_desc_k_sw128(b_addr + j * 32);
          const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
          if constexpr (BF16) {  // 16-bit operands (bf16 or fp16, as the instruction descriptor says)
            asm volatile(
                "{\n\t.reg .pred p;\n\t"
                "setp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
                "l"(da), "l"(db), "r"(kIdesc), "r"(acc)
                : "memory");
          } else {
            asm volatile(
                "{\n\t.reg .pred p;\n\t"
                "setp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
                "l"(da), "l"(db), "r"(kIdesc), "r"(acc)
                : "memory");
          }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&empty[s]))
                     : "memory");
      }
      // accumulator ready (or, after an abort, all issued MMAs retired) -> epilogue / teardown
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_u32(acc_bar))
                   : "memory");
      if (!ok) atomicCAS(status, 0, 3);
    }
  } else {
    // epilogue warps 2..5 -> TMEM lane quadrant (warp % 4)
    const int quad = warp & 3;
    const int row = m0 + quad * 32 + lane;
    const bool ready = mbar_wait(acc_bar, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!ready) {
      *abort_flag = 1;
      atomicCAS(status, 0, 4);
    } else if (!*abort_flag) {
      #pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c0;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
            "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
              "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
              "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        store_chunk(v, row, n0, c0, M, N, alpha, beta, C, ldc, sym, sa, sb);
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BN) : "memory");
  }
}

// ---- persistent form: one CTA per SM walks a tile list; two TMEM accumulators (2 x BN = 512 columns) let the
// epilogue of one tile overlap the MMAs of the next.  Roles as above; acc_full[b] is committed by the MMA thread when
// buffer b holds a finished tile, acc_empty[b] collects one arrival per epilogue warp when it has been drained.
// Symmetric products enumerate only the tiles holding entries col <= row.
//
// Chunked accumulation (ckb > 0, no split-K): the tensor core's FP32 accumulator does not round to nearest, so a
// long K extent is cut into chunks of ckb k-blocks.  Each chunk is accumulated in TMEM columns [0, BN) and the
// epilogue warps add it, round to nearest, into a running sum held in TMEM columns [BN, 2 BN); the tile is written
// to C once, after its last chunk.  The MMAs of chunk q + 1 wait only for the epilogue to have read chunk q.

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Tile t -> (m-block, n-block): row-major over the n-blocks of each m-block; with sym only n-blocks whose first
// column is <= the m-block's last row.
template <int BN>
__device__ __forceinline__ void tile_coords(int t, int mt, int nt, int sym, int& mb, int& nb) {
  if (!sym) {
    mb = t / nt;
    nb = t - mb * nt;
    return;
  }
  mb = 0;
  for (;; ++mb) {
    const int cnt = min((mb * BM + BM - 1) / BN + 1, nt);
    if (t < cnt || mb == mt - 1) break;
    t -= cnt;
  }
  nb = t;
}

// k-block range [kb0, kb1) of split s of `splits` over total_kb k-blocks (near-equal contiguous pieces).
__device__ __forceinline__ void split_range(int s, int splits, int total_kb, int& kb0, int& kb1) {
  kb0 = (int)((int64_t)total_kb * s / splits);
  kb1 = (int)((int64_t)total_kb * (s + 1) / splits);
}

// Split-K reduction in a fixed order: C = alpha * sum_{s < splits} ws[s] + beta * C  (ws: splits x M x N).
__global__ void k_splitk_reduce(const float* __restrict__ ws, int splits, int M, int N, float alpha, float beta,
                                float* __restrict__ C, int64_t ldc) {
  const int64_t total = (int64_t)M * N;
  const int64_t plane = total;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    float acc = ws[i];
    for (int s = 1; s < splits; ++s) acc += ws[(int64_t)s * plane + i];
    const int r = (int)(i / N), c = (int)(i % N);
    float* cp = C + (int64_t)r * ldc + c;
    *cp = beta != 0.f ? alpha * acc + beta * *cp : alpha * acc;
  }
}

template <int BN, int STAGES, int KIND>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc_pt(const __grid_constant__ Maps maps, int nreg, int M, int N, int K, float alpha, float beta,
                 float* __restrict__ C, int64_t ldc, int* __restrict__ status, int sym, const float* __restrict__ sa,
                 const float* __restrict__ sb, int mt, int nt, int ntiles, int splits, float* __restrict__ ws,
                 int ckb) {
  constexpr bool B16 = KIND != 0;
  constexpr uint32_t kStageA = BM * 128;
  constexpr uint32_t kStageB = BN * 128;
  constexpr int kBKE = B16 ? 64 : 32;
  constexpr uint32_t kIdesc = KIND == 2 ? idesc_f16(BM, BN) : (KIND == 1 ? idesc_bf16(BM, BN) : idesc_tf32(BM, BN));
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = base;
  unsigned char* sB = base + STAGES * kStageA;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * kStageB);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* drain_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb_per_reg = (K + kBKE - 1) / kBKE;
  const int total_kb = kb_per_reg * nreg;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)(2 * BN))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        int mb, nb, kb0, kb1;
        tile_coords<BN>(t / splits, mt, nt, sym, mb, nb);
        split_range(t % splits, splits, total_kb, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++g) {
          const int s = g % STAGES;
          const uint32_t ph = (uint32_t)(g / STAGES) & 1u;
          if (*abort_flag || !mbar_wait(&empty[s], ph ^ 1u)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          const int r = kb / kb_per_reg;
          const int k0 = (kb % kb_per_reg) * kBKE;
          mbar_expect_tx(&full[s], kStageA + kStageB);
          tma_load_2d(sA + s * kStageA, &maps.a[r], &full[s], k0, mb * BM);
          tma_load_2d(sB + s * kStageB, &maps.b[r], &full[s], k0, nb * BN);
        }
      }
      if (!ok) {
        // drain: wait (bounded) for the copies this thread issued into the ring
        for (int q = g - STAGES < 0 ? 0 : g - STAGES; q < g; ++q) mbar_wait(&full[q % STAGES], (uint32_t)(q / STAGES) & 1u);
        atomicCAS(status, 0, 2);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      // k-blocks [kb0, kb1) into the accumulator at dacc (the first MMA overwrites it); false on a timed-out wait
      auto issue = [&](int kb0, int kb1, uint32_t dacc) -> bool {
        for (int kb = kb0; kb < kb1; ++kb, ++g) {
          const int s = g % STAGES;
          const uint32_t ph = (uint32_t)(g / STAGES) & 1u;
          if (*abort_flag || !mbar_wait(&full[s], ph)) {
            *abort_flag = 1;
            return false;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_addr = smem_u32(sA + s * kStageA);
          const uint32_t b_addr = smem_u32(sB + s * kStageB);
          #pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint64_t da = smem_desc_k_sw128(a_addr + j * 32);
            const uint64_t db = smem_desc_k_sw128(b_addr + j * 32);
            const uint32_t acc = (kb > kb0 || j > 0) ? 1u : 0u;
            if constexpr (B16) {
              asm volatile(
                  "{\n\t.reg .pred p;\n\t"
                  "setp.ne.b32 p, %4, 0;\n\t"
                  "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(dacc),
                  "l"(da), "l"(db), "r"(kIdesc), "r"(acc)
                  : "memory");
            } else {
              asm volatile(
                  "{\n\t.reg .pred p;\n\t"
                  "setp.ne.b32 p, %4, 0;\n\t"
                  "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(dacc),
                  "l"(da), "l"(db), "r"(kIdesc), "r"(acc)
                  : "memory");
            }
          }
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                           smem_u32(&empty[s]))
                       : "memory");
        }
        return true;
      };
      if (ckb > 0) {
        // chunked accumulation: every chunk of every tile goes to the accumulator in columns [0, BN)
        int u = 0;
        for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
          for (int cs = 0; cs < total_kb; cs += ckb, ++u) {
            if (*abort_flag || !mbar_wait(&acc_empty[0], ((uint32_t)u & 1u) ^ 1u)) {
              *abort_flag = 1;
              ok = false;
              break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (!(ok = issue(cs, min(cs + ckb, total_kb), tmem))) break;
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(&acc_full[0]))
                         : "memory");
          }
        }
      } else {
        int i = 0;
        for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++i) {
          const int b = i & 1;
          const uint32_t use = (uint32_t)(i >> 1);
          if (*abort_flag || !mbar_wait(&acc_empty[b], (use & 1u) ^ 1u)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          int kb0, kb1;
          split_range(t % splits, splits, total_kb, kb0, kb1);
          if (!(ok = issue(kb0, kb1, tmem + (uint32_t)(b * BN)))) break;
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                           smem_u32(&acc_full[b]))
                       : "memory");
        }
      }
      // every MMA this thread issued has retired before teardown (bounded)
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_u32(drain_bar))
                   : "memory");
      mbar_wait(drain_bar, 0);
      if (!ok) atomicCAS(status, 0, 3);
    }
  } else if (ckb > 0) {
    // chunked epilogue: fold each chunk into the running sum (TMEM columns [BN, 2 BN)), then write the tile
    const int quad = warp & 3;
    const uint32_t lanes = (uint32_t)(quad * 32) << 16;
    const int nq = (total_kb + ckb - 1) / ckb;
    int u = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      for (int q = 0; q < nq; ++q, ++u) {
        if (*abort_flag) { ok = false; break; }
        if (!mbar_wait(&acc_full[0], (uint32_t)u & 1u)) {
          *abort_flag = 1;
          atomicCAS(status, 0, 4);
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        #pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t v[32];
          tmem_ld32(tmem + lanes + (uint32_t)c0, v);
          if (q > 0) {
            uint32_t r[32];
            tmem_ld32(tmem + lanes + (uint32_t)(BN + c0), r);
            #pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(r[e]) + __uint_as_float(v[e]));
          }
          tmem_st32(tmem + lanes + (uint32_t)(BN + c0), v);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[0]);  // the accumulator may take the next chunk
      }
      if (!ok) break;
      int mb, nb;
      tile_coords<BN>(t, mt, nt, sym, mb, nb);
      const int row = mb * BM + quad * 32 + lane;
      #pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + lanes + (uint32_t)(BN + c0), v);
        store_chunk(v, row, nb * BN, c0, M, N, alpha, beta, C, ldc, sym, sa, sb);
      }
    }
  } else {
    // epilogue warps 2..5 -> TMEM lane quadrant (warp % 4)
    const int quad = warp & 3;
    int i = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
      const int b = i & 1;
      const uint32_t use = (uint32_t)(i >> 1);
      if (*abort_flag) break;
      if (!mbar_wait(&acc_full[b], use & 1u)) {
        *abort_flag = 1;
        atomicCAS(status, 0, 4);
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      int mb, nb;
      tile_coords<BN>(t / splits, mt, nt, sym, mb, nb);
      const int row = mb * BM + quad * 32 + lane;
      // split-K: the unit's partial sum (row scales applied, no alpha / beta) goes to its own M x N slice of ws
      float* dst = splits > 1 ? ws + (int64_t)(t % splits) * M * N : C;
      const int64_t ldd = splits > 1 ? (int64_t)N : ldc;
      const float al = splits > 1 ? 1.f : alpha, be = splits > 1 ? 0.f : beta;
      #pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * BN + c0), v);
        store_chunk(v, row, nb * BN, c0, M, N, al, be, dst, ldd, sym, sa, sb);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)(2 * BN)) : "memory");
  }
}

// ---- host: tensor maps through the driver entry point (no libcuda link dependency) ----
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int get_encoder() {
  if (g_encode) return MPQ_OK;
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
    set_last_error("cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorString(e));
    return MPQ_ERR_UNSUPPORTED;
  }
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return MPQ_OK;
}

// rows x K row-major fp32 (leading dimension ld), box = box_rows x 32, 128B swizzle
// kind: 0 fp32, 1 bf16, 2 fp16
static int make_map(CUtensorMap* m, const void* p, int rows, int K, int64_t ld, int box_rows, int kind = 0) {
  const int esz = kind ? 2 : 4;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * esz};
  cuuint32_t box[2] = {(cuuint32_t)(128 / esz), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, kind == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                     : (kind == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32), 2,
                        const_cast<void*>(p), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed (%d) rows=%d K=%d ld=%lld", (int)r, rows, K, (long long)ld);
    return MPQ_ERR_ARG;
  }
  return MPQ_OK;
}

template <int BN, int STAGES, int KIND = 0>
static int launch(const Maps& maps, int nreg, int M, int N, int K, float alpha, float beta, float* C, int64_t ldc,
                  int* status, cudaStream_t stream, int sym = 0, const float* sa = nullptr, const float* sb = nullptr) {
  const size_t smem = 1024 + (size_t)STAGES * (BM + BN) * 128 + 256;
  const int ast = smem_opt_in((const void*)k_gemm_tc<BN, STAGES, KIND>, smem, "mpq_gemm_tc");
  if (ast) return ast;
  dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
  k_gemm_tc<BN, STAGES, KIND><<<grid, kThreads, smem, stream>>>(maps, nreg, M, N, K, alpha, beta, C, ldc, status, sym,
                                                                 sa, sb);
  return launch_status("mpq_gemm_tc");
}

static int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// Persistent launch: one CTA per SM (the ring and two TMEM accumulators need the whole SM) over the tile list.
template <int BN, int STAGES, int KIND>
static int launch_pt(const Maps& maps, int nreg, int M, int N, int K, float alpha, float beta, float* C, int64_t ldc,
                     int* status, cudaStream_t stream, int sym = 0, const float* sa = nullptr, const float* sb = nullptr,
                     int splits = 1, float* ws = nullptr, bool reduce = true, int ckb = 0) {
  const size_t smem = 1024 + (size_t)STAGES * (BM + BN) * 128 + 256;
  const int ast = smem_opt_in((const void*)k_gemm_tc_pt<BN, STAGES, KIND>, smem, "mpq_gemm_tc (persistent)");
  if (ast) return ast;
  const int mt = (M + BM - 1) / BM, nt = (N + BN - 1) / BN;
  int64_t ntiles = 0;
  if (sym) {
    for (int mb = 0; mb < mt; ++mb) ntiles += std::min((mb * BM + BM - 1) / BN + 1, nt);
  } else {
    ntiles = (int64_t)mt * nt;
  }
  if (ntiles == 0) return MPQ_OK;
  if (splits < 1 || !ws) splits = 1;
  if (ckb > 0) splits = 1;  // chunked accumulation keeps each tile's whole K extent in one CTA
  const int64_t units = ntiles * splits;
  const int grid = (int)std::min<int64_t>(units, num_sms());
  k_gemm_tc_pt<BN, STAGES, KIND><<<grid, kThreads, smem, stream>>>(maps, nreg, M, N, K, alpha, beta, C, ldc, status,
                                                                    sym, sa, sb, mt, nt, (int)units, splits, ws, ckb);
  int st = launch_status("mpq_gemm_tc (persistent)");
  if (st || splits == 1 || !reduce) return st;
  const int64_t total = (int64_t)M * N;
  const int rgrid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 8);
  k_splitk_reduce<<<rgrid, 256, 0, stream>>>(ws, splits, M, N, alpha, beta, C, ldc);
  return launch_status("mpq_gemm_tc (split-K reduction)");
}

}  // namespace tc
}  // namespace mpq

using namespace mpq;

// C = alpha * sum_{r < nreg} A_r B_r^T + beta * C.  A_r: M x K row-major (lda), B_r: N x K row-major (ldb).
// Requirements (TMA): 16-byte aligned base pointers, lda/ldb multiples of 4 elements.  `status` (device int,
// required) receives a non-zero code if a pipeline wait timed out (2: producer, 3: MMA, 4: epilogue).
MPQ_API int mpq_gemm_tc(int nreg, int M, int N, int K, float alpha, const float* const* A, int64_t lda,
                        const float* const* B, int64_t ldb, float beta, float* C, int64_t ldc, int* status,
                        void* stream) {
  MPQ_CHECK_ARG(nreg >= 1 && nreg <= 3, "mpq_gemm_tc: nreg must be 1..3");
  MPQ_CHECK_ARG(M >= 0 && N >= 0 && K >= 1, "mpq_gemm_tc: bad shape");
  if (M == 0 || N == 0) return MPQ_OK;  // empty tensors may carry null pointers
  MPQ_CHECK_ARG(A && B && C, "mpq_gemm_tc: null pointer");
  MPQ_CHECK_ARG(lda % 4 == 0 && ldb % 4 == 0 && lda >= K && ldb >= K, "mpq_gemm_tc: lda/ldb must be multiples of 4 and >= K");
  int st = tc::get_encoder();
  if (st) return st;
  tc::Maps maps;
  memset(&maps, 0, sizeof(maps));
  for (int r = 0; r < nreg; ++r) {
    MPQ_CHECK_ARG(A[r] && B[r], "mpq_gemm_tc: null operand %d", r);
    MPQ_CHECK_ARG(((uintptr_t)A[r] & 15) == 0 && ((uintptr_t)B[r] & 15) == 0, "mpq_gemm_tc: operands must be 16-byte aligned");
    st = tc::make_map(&maps.a[r], A[r], M, K, lda, tc::BM);
    if (st) return st;
    st = tc::make_map(&maps.b[r], B[r], N, K, ldb, 256);
    if (st) return st;
  }
  MPQ_CHECK_ARG(status, "mpq_gemm_tc: status word required");
  return tc::launch<256, 4>(maps, nreg, M, N, K, alpha, beta, C, ldc, status, (cudaStream_t)stream);
}

// Symmetric product C = alpha * sum_{r < nreg} A_r B_r^T + beta * C for B_r holding the same matrix as A_r
// (B_r = A_r, or the other half of the same 3xTF32 split), n x n result: only the tiles holding entries
// col <= row are computed and every computed entry is also stored at its mirror position, so C is exactly
// symmetric.  beta reads only the lower triangle of C (C must be symmetric on entry when beta != 0).
MPQ_API int mpq_syrk_tc(int nreg, int n, int K, float alpha, const float* const* A, const float* const* B, int64_t lda,
                        float beta, float* C, int64_t ldc, int* status, void* stream) {
  MPQ_CHECK_ARG(nreg >= 1 && nreg <= 3, "mpq_syrk_tc: nreg must be 1..3");
  MPQ_CHECK_ARG(A && B && C && status, "mpq_syrk_tc: null pointer");
  MPQ_CHECK_ARG(n >= 0 && K >= 1, "mpq_syrk_tc: bad shape");
  MPQ_CHECK_ARG(lda % 4 == 0 && lda >= K && ldc >= n, "mpq_syrk_tc: lda must be a multiple of 4 and >= K, ldc >= n");
  if (n == 0) return MPQ_OK;
  int st = tc::get_encoder();
  if (st) return st;
  tc::Maps maps;
  memset(&maps, 0, sizeof(maps));
  for (int r = 0; r < nreg; ++r) {
    MPQ_CHECK_ARG(A[r] && B[r], "mpq_syrk_tc: null operand %d", r);
    MPQ_CHECK_ARG(((uintptr_t)A[r] & 15) == 0 && ((uintptr_t)B[r] & 15) == 0, "mpq_syrk_tc: operands must be 16-byte aligned");
    st = tc::make_map(&maps.a[r], A[r], n, K, lda, tc::BM);
    if (st) return st;
    st = tc::make_map(&maps.b[r], B[r], n, K, lda, 256);
    if (st) return st;
  }
  return tc::launch<256, 4>(maps, nreg, n, n, K, alpha, beta, C, ldc, status, (cudaStream_t)stream, 1);
}

// Symmetric product of a bf16 operand, C = alpha A A^T + beta C (A: n x K row-major bf16, lda a multiple of 8):
// kind::f16 MMAs (bf16 x bf16 products are exact in FP32).  mirror != 0 stores every entry at its mirror too;
// mirror == 0 updates the lower triangle only (intermediate steps of an accumulation).
MPQ_API int mpq_syrk_bf16(int n, int K, float alpha, const void* A, int64_t lda, float beta, float* C, int64_t ldc,
                          int mirror, int* status, void* stream) {
  MPQ_CHECK_ARG(A && C && status, "mpq_syrk_bf16: null pointer");
  MPQ_CHECK_ARG(n >= 0 && K >= 1, "mpq_syrk_bf16: bad shape");
  MPQ_CHECK_ARG(lda % 8 == 0 && lda >= K && ldc >= n, "mpq_syrk_bf16: lda must be a multiple of 8 and >= K, ldc >= n");
  MPQ_CHECK_ARG(((uintptr_t)A & 15) == 0, "mpq_syrk_bf16: A must be 16-byte aligned");
  if (n == 0) return MPQ_OK;
  int st = tc::get_encoder();
  if (st) return st;
  tc::Maps maps;
  memset(&maps, 0, sizeof(maps));
  st = tc::make_map(&maps.a[0], A, n, K, lda, tc::BM, 1);
  if (st) return st;
  st = tc::make_map(&maps.b[0], A, n, K, lda, 256, 1);
  if (st) return st;
  return tc::launch_pt<256, 4, 1>(maps, 1, n, n, K, alpha, beta, C, ldc, status, (cudaStream_t)stream, mirror ? 1 : 2);
}

// Whole-K symmetric accumulation of a bf16 operand in one launch, C = alpha A A^T + beta C, exactly symmetric: the
// K extent is accumulated by the tensor core in chunks of `chunk` columns (a multiple of 64) that are added, round
// to nearest, into a running sum kept in TMEM; C is read (beta != 0, lower triangle) and written once per tile.
MPQ_API int mpq_syrk_bf16_acc(int n, int K, float alpha, const void* A, int64_t lda, float beta, float* C,
                              int64_t ldc, int chunk, int* status, void* stream) {
  MPQ_CHECK_ARG(n >= 0 && K >= 1, "mpq_syrk_bf16_acc: bad shape");
  MPQ_CHECK_ARG(chunk >= 64 && chunk % 64 == 0, "mpq_syrk_bf16_acc: chunk must be a positive multiple of 64");
  if (n == 0) return MPQ_OK;
  MPQ_CHECK_ARG(A && C && status, "mpq_syrk_bf16_acc: null pointer");
  MPQ_CHECK_ARG(lda % 8 == 0 && lda >= K && ldc >= n, "mpq_syrk_bf16_acc: lda must be a multiple of 8 and >= K, ldc >= n");
  MPQ_CHECK_ARG(((uintptr_t)A & 15) == 0, "mpq_syrk_bf16_acc: A must be 16-byte aligned");
  int st = tc::get_encoder();
  if (st) return st;
  tc::Maps maps;
  memset(&maps, 0, sizeof(maps));
  st = tc::make_map(&maps.a[0], A, n, K, lda, tc::BM, 1);
  if (st) return st;
  st = tc::make_map(&maps.b[0], A, n, K, lda, 256, 1);
  if (st) return st;
  return tc::launch_pt<256, 4, 1>(maps, 1, n, n, K, alpha, beta, C, ldc, status, (cudaStream_t)stream, 1, nullptr,
                                  nullptr, 1, nullptr, true, chunk / 64);
}

// Whole-K symmetric accumulation of fp32 operands (the 3xTF32 split, as mpq_syrk_tc) in one launch: the regions'
// K extents are concatenated and accumulated in chunks of `chunk` columns (a multiple of 32) added, round to
// nearest, into a running sum in TMEM; C is read and written once per tile, exactly symmetric.
MPQ_API int mpq_syrk_tc_acc(int nreg, int n, int K, float alpha, const float* const* A, const float* const* B,
                            int64_t lda, float beta, float* C, int64_t ldc, int chunk, int* status, void* stream) {
  MPQ_CHECK_ARG(nreg >= 1 && nreg <= 3, "mpq_syrk_tc_acc: nreg must be 1..3");
  MPQ_CHECK_ARG(n >= 0 && K >= 1, "mpq_syrk_tc_acc: bad shape");
  MPQ_CHECK_ARG(chunk >= 32 && chunk % 32 == 0, "mpq_syrk_tc_acc: chunk must be a positive multiple of 32");
  if (n == 0) return MPQ_OK;
  MPQ_CHECK_ARG(A && B && C && status, "mpq_syrk_tc_acc: null pointer");
  MPQ_CHECK_ARG(lda % 4 == 0 && lda >= K && ldc >= n, "mpq_syrk_tc_acc: lda must be a multiple of 4 and >= K, ldc >= n");
  int st = tc::get_encoder();
  if (st) return st;
  tc::Maps maps;
  memset(&maps, 0, sizeof(maps));
  for (int r = 0; r < nreg; ++r) {
    MPQ_CHECK_ARG(A[r] && B[r], "mpq_syrk_tc_acc: null operand %d", r);
    MPQ_CHECK_ARG(((uintptr_t)A[r] & 15) == 0 && ((uintptr_t)B[r] & 15) == 0,
                  "mpq_syrk_tc_acc: operands must be 16-byte aligned");
    st = tc::make_map(&maps.a[r], A[r], n, K, lda, tc::BM);
    if (st) return st;
    st = tc::make_map(&maps.b[r], B[r], n, K, lda, 256);
    if (st) return st;
  }
  return tc::launch_pt<256, 4, 0>(maps, nreg, n, n, K, alpha, beta, C, ldc, status, (cudaStream_t)stream, 1, nullptr,
                                  nullptr, 1, nullptr, true, chunk / 32);
}

// FP32-faithful product on the fp16 tensor cores: C = alpha sum_{(a,b) in (hi,hi),(hi,lo),(lo,hi)} diag(sa) A_a B_b^T diag(sb)
// + beta C, from the row-scaled fp16 split of mpq_split_f16 (A: M x K, B: N x K, 16-bit row-major, lda/ldb multiples
// of 8; sa / sb the splits' per-row scales).  fp16 MMAs run at twice the TF32 rate; the split keeps 22 significant
// bits per element as the 3xTF32 split does.
MPQ_API int mpq_gemm_f16x3(int M, int N, int K, float alpha, const void* a_hi, const void* a_lo, int64_t lda,
                           const float* sa, const void* b_hi, const void* b_lo, int64_t ldb, const float* sb, float beta,
                           float* C, int64_t ldc, int* status, void* stream) {
  MPQ_CHECK_ARG(M >= 0 && N >= 0 && K >= 1, "mpq_gemm_f16x3: bad shape");
  if (M == 0 || N == 0) return MPQ_OK;  // empty tensors may carry null pointers
  MPQ_CHECK_ARG(a_hi && a_lo && b_hi && b_lo && sa && sb && C && status, "mpq_gemm_f16x3: null pointer");
  MPQ_CHECK_ARG(lda % 8 == 0 && ldb % 8 == 0 && lda >= K && ldb >= K, "mpq_gemm_f16x3: lda/ldb must be multiples of 8 and >= K");
  const void* ptrs[4] = {a_hi, a_lo, b_hi, b_lo};
  for (int i = 0; i < 4; ++i)
    MPQ_CHECK_ARG(((uintptr_t)ptrs[i] & 15) == 0, "mpq_gemm_f16x3: operands must be 16-byte aligned");
  int st = tc::get_encoder();
  if (st) return st;
  tc::Maps maps;
  memset(&maps, 0, sizeof(maps));
  const void* As[3] = {a_hi, a_hi, a_lo};
  const void* Bs[3] = {b_hi, b_lo, b_hi};
  for (int r = 0; r < 3; ++r) {
    st = tc::make_map(&maps.a[r], As[r], M, K, lda, tc::BM, 2);
    if (st) return st;
    st = tc::make_map(&maps.b[r], Bs[r], N, K, ldb, 256, 2);
    if (st) return st;
  }
  return tc::launch_pt<256, 4, 2>(maps, 3, M, N, K, alpha, beta, C, ldc, status, (cudaStream_t)stream, 0, sa, sb);
}

// mpq_gemm_f16x3 with split-K: the 3 x round_up(K, 64) / 64 k-blocks of each 128 x 256 output tile are cut into
// `splits` contiguous ranges processed by different CTAs, so small-M products (a 128-row VAMP block against a
// 4096-wide basis: 16 tiles) still occupy every SM.  Each range's partial (row scales applied) is stored to its own
// M x N slice of `ws` (caller-owned, splits * M * N floats), then C = alpha * sum_s ws[s] + beta * C is summed in a
// fixed order (deterministic).  splits = 1 is mpq_gemm_f16x3.
MPQ_API int mpq_gemm_f16x3_splitk(int M, int N, int K, float alpha, const void* a_hi, const void* a_lo, int64_t lda,
                                  const float* sa, const void* b_hi, const void* b_lo, int64_t ldb, const float* sb,
                                  float beta, float* C, int64_t ldc, int splits, float* ws, int64_t ws_floats,
                                  int* status, void* stream) {
  MPQ_CHECK_ARG(M >= 0 && N >= 0 && K >= 1, "mpq_gemm_f16x3_splitk: bad shape");
  MPQ_CHECK_ARG(splits >= 1 && splits <= 1024, "mpq_gemm_f16x3_splitk: splits must be in [1, 1024]");
  if (M == 0 || N == 0) return MPQ_OK;
  const int total_kb = 3 * ((K + 63) / 64);
  MPQ_CHECK_ARG(splits <= total_kb, "mpq_gemm_f16x3_splitk: %d splits for %d k-blocks", splits, total_kb);
  MPQ_CHECK_ARG(splits == 1 || (ws && ws_floats >= (int64_t)splits * M * N),
                "mpq_gemm_f16x3_splitk: workspace of %lld floats < splits * M * N", (long long)ws_floats);
  MPQ_CHECK_ARG(a_hi && a_lo && b_hi && b_lo && sa && sb && C && status, "mpq_gemm_f16x3_splitk: null pointer");
  MPQ_CHECK_ARG(lda % 8 == 0 && ldb % 8 == 0 && lda >= K && ldb >= K,
                "mpq_gemm_f16x3_splitk: lda/ldb must be multiples of 8 and >= K");
  const void* ptrs[4] = {a_hi, a_lo, b_hi, b_lo};
  for (int i = 0; i < 4; ++i)
    MPQ_CHECK_ARG(((uintptr_t)ptrs[i] & 15) == 0, "mpq_gemm_f16x3_splitk: operands must be 16-byte aligned");
  int st = tc::get_encoder();
  if (st) return st;
  tc::Maps maps;
  memset(&maps, 0, sizeof(maps));
  const void* As[3] = {a_hi, a_hi, a_lo};
  const void* Bs[3] = {b_hi, b_lo, b_hi};
  for (int r = 0; r < 3; ++r) {
    st = tc::make_map(&maps.a[r], As[r], M, K, lda, tc::BM, 2);
    if (st) return st;
    st = tc::make_map(&maps.b[r], Bs[r], N, K, ldb, 256, 2);
    if (st) return st;
  }
  return tc::launch_pt<256, 4, 2>(maps, 3, M, N, K, alpha, beta, C, ldc, status, (cudaStream_t)stream, 0, sa, sb,
                                  splits, splits > 1 ? ws : nullptr);
}

// The split-K partial products of mpq_gemm_f16x3_splitk without the reduction: plane s (M x N, leading dimension N) of
// ws holds the sum over the s-th k-range (row scales applied); a consumer adds the planes in order 0, 1, ...
// (which reproduces the reduction's result bit for bit).  splits = 1 writes the whole product to plane 0.
MPQ_API int mpq_gemm_f16x3_parts(int M, int N, int K, const void* a_hi, const void* a_lo, int64_t lda, const float* sa,
                                 const void* b_hi, const void* b_lo, int64_t ldb, const float* sb, int splits,
                                 float* ws, int64_t ws_floats, int* status, void* stream) {
  MPQ_CHECK_ARG(M >= 0 && N >= 0 && K >= 1, "mpq_gemm_f16x3_parts: bad shape");
  MPQ_CHECK_ARG(splits >= 1 && splits <= 1024, "mpq_gemm_f16x3_parts: splits must be in [1, 1024]");
  if (M == 0 || N == 0) return MPQ_OK;
  const int total_kb = 3 * ((K + 63) / 64);
  MPQ_CHECK_ARG(splits <= total_kb, "mpq_gemm_f16x3_parts: %d splits for %d k-blocks", splits, total_kb);
  MPQ_CHECK_ARG(ws && ws_floats >= (int64_t)splits * M * N, "mpq_gemm_f16x3_parts: workspace of %lld floats < splits * M * N",
                (long long)ws_floats);
  MPQ_CHECK_ARG(a_hi && a_lo && b_hi && b_lo && sa && sb && status, "mpq_gemm_f16x3_parts: null pointer");
  MPQ_CHECK_ARG(lda % 8 == 0 && ldb % 8 == 0 && lda >= K && ldb >= K,
                "mpq_gemm_f16x3_parts: lda/ldb must be multiples of 8 and >= K");
  const void* ptrs[4] = {a_hi, a_lo, b_hi, b_lo};
  for (int i = 0; i < 4; ++i)
    MPQ_CHECK_ARG(((uintptr_t)ptrs[i] & 15) == 0, "mpq_gemm_f16x3_parts: operands must be 16-byte aligned");
  int st = tc::get_encoder();
  if (st) return st;
  tc::Maps maps;
  memset(&maps, 0, sizeof(maps));
  const void* As[3] = {a_hi, a_hi, a_lo};
  const void* Bs[3] = {b_hi, b_lo, b_hi};
  // N <= 128 (a polish chunk's 128 columns): 128-wide tiles, so no MMA or B load is spent on padding (every output
  // element's k-order, and so its value, is the same as with 256-wide tiles)
  const int bn = N <= 128 ? 128 : 256;
  for (int r = 0; r < 3; ++r) {
    st = tc::make_map(&maps.a[r], As[r], M, K, lda, tc::BM, 2);
    if (st) return st;
    st = tc::make_map(&maps.b[r], Bs[r], N, K, ldb, bn, 2);
    if (st) return st;
  }
  if (bn == 128)
    return tc::launch_pt<128, 4, 2>(maps, 3, M, N, K, 1.f, 0.f, ws, N, status, (cudaStream_t)stream, 0, sa, sb, splits,
                                    splits > 1 ? ws : nullptr, false);
  return tc::launch_pt<256, 4, 2>(maps, 3, M, N, K, 1.f, 0.f, ws, N, status, (cudaStream_t)stream, 0, sa, sb, splits,
                                  splits > 1 ? ws : nullptr, false);
}

namespace mpq {
// Row-scaled fp16 split, one warp per row: s = 2^(15 - E) with max|x_row| < 2^E, y = x s (exact),
// hi = fp16_rn(y), lo = fp16_rn(y - hi) (y - hi exact in fp32); inv_scale[row] = 1 / s.
__global__ void k_split_f16(const float* __restrict__ x, int64_t ldx, int rows, int cols, __half* __restrict__ hi,
                            __half* __restrict__ lo, int64_t ldo, float* __restrict__ inv_scale) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float* xr = x + (int64_t)warp * ldx;
  float mx = 0.f;
  for (int c = lane; c < cols; c += 32) mx = fmaxf(mx, fabsf(xr[c]));
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float s, inv;
  split_f16_scale(mx, s, inv);
  for (int c = lane; c < cols; c += 32)
    split_f16_store(xr[c], s, reinterpret_cast<unsigned short*>(hi + (int64_t)warp * ldo + c),
                    reinterpret_cast<unsigned short*>(lo + (int64_t)warp * ldo + c));
  if (lane == 0) inv_scale[warp] = inv;
}

// The same split with one CTA per row, 16-byte loads and 8-byte stores of four halves (rows whose length, leading
// dimensions and base addresses allow it): a few hundred rows fill the GPU instead of a few dozen warps.  The row
// maximum is order independent, so every output equals k_split_f16's.
__global__ void __launch_bounds__(256) k_split_f16_v4(const float* __restrict__ x, int64_t ldx, int cols,
                                                      __half* __restrict__ hi, __half* __restrict__ lo, int64_t ldo,
                                                      float* __restrict__ inv_scale) {
  __shared__ float red[8];
  const int row = blockIdx.x, nv = cols >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + (int64_t)row * ldx);
  float mx = 0.f;
  for (int v = threadIdx.x; v < nv; v += blockDim.x) {
    const float4 q = xr[v];
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(q.x), fabsf(q.y)), fmaxf(fabsf(q.z), fabsf(q.w))));
  }
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = red[0];
  #pragma unroll
  for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
  float s, inv;
  split_f16_scale(mx, s, inv);
  uint2* hr = reinterpret_cast<uint2*>(hi + (int64_t)row * ldo);
  uint2* lr = reinterpret_cast<uint2*>(lo + (int64_t)row * ldo);
  for (int v = threadIdx.x; v < nv; v += blockDim.x) {
    const float4 q = xr[v];
    const float e[4] = {q.x, q.y, q.z, q.w};
    unsigned short h[4], l[4];
    #pragma unroll
    for (int i = 0; i < 4; ++i) split_f16_store(e[i], s, &h[i], &l[i]);
    hr[v] = make_uint2(h[0] | ((unsigned)h[1] << 16), h[2] | ((unsigned)h[3] << 16));
    lr[v] = make_uint2(l[0] | ((unsigned)l[1] << 16), l[2] | ((unsigned)l[3] << 16));
  }
  if (threadIdx.x == 0) inv_scale[row] = inv;
}
}  // namespace mpq

MPQ_API int mpq_split_f16(const float* x, int64_t ldx, int rows, int cols, void* hi, void* lo, int64_t ldo,
                          float* inv_scale, void* stream) {
  MPQ_CHECK_ARG(rows >= 0 && cols >= 0 && ldo >= cols && ldx >= cols, "mpq_split_f16: bad shape");
  if (rows == 0 || cols == 0) return MPQ_OK;
  MPQ_CHECK_ARG(x && hi && lo && inv_scale, "mpq_split_f16: null pointer");
  const bool v4 = (cols & 3) == 0 && (ldx & 3) == 0 && (ldo & 3) == 0 && ((uintptr_t)x & 15) == 0 &&
                  ((uintptr_t)hi & 7) == 0 && ((uintptr_t)lo & 7) == 0;
  if (v4) {
    k_split_f16_v4<<<rows, 256, 0, (cudaStream_t)stream>>>(x, ldx, cols, (__half*)hi, (__half*)lo, ldo, inv_scale);
    return launch_status("mpq_split_f16");
  }
  const int warps_per_block = 8;
  k_split_f16<<<(rows + warps_per_block - 1) / warps_per_block, 32 * warps_per_block, 0, (cudaStream_t)stream>>>(
      x, ldx, rows, cols, (__half*)hi, (__half*)lo, ldo, inv_scale);
  return launch_status("mpq_split_f16");
}

// hi = tf32 round-to-nearest of x (low 13 mantissa bits cleared), lo = x - hi (exact in fp32).
namespace mpq {
__global__ void k_split_tf32(const float* __restrict__ x, int64_t ldx, float* __restrict__ hi, float* __restrict__ lo,
                             int64_t ldo, int rows, int cols) {
  const int64_t total = (int64_t)rows * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i % cols);
    const float v = x[r * ldx + c];
    uint32_t h;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
    const float hv = __uint_as_float(h);
    hi[r * ldo + c] = hv;
    lo[r * ldo + c] = fsub(v, hv);
  }
}
}  // namespace mpq

MPQ_API int mpq_split_tf32(const float* x, int64_t ldx, float* hi, float* lo, int64_t ldo, int rows, int cols,
                           void* stream) {
  const int64_t total = (int64_t)rows * cols;
  if (total <= 0) return MPQ_OK;  // empty tensors may carry null pointers
  MPQ_CHECK_ARG(x && hi && lo, "mpq_split_tf32: null pointer");
  int64_t g = (total + 255) / 256;
  if (g > 148 * 16) g = 148 * 16;
  k_split_tf32<<<(int)g, 256, 0, (cudaStream_t)stream>>>(x, ldx, hi, lo, ldo, rows, cols);
  return launch_status("mpq_split_tf32");
}

// ---------------------------------------------------------------------------------------------------------
// Allocation-free 3xTF32 product.
//
// Some callers cannot allocate device memory at the point where they need this product: code that runs
// while a caching allocator is forbidden from growing (inside a memory-capped pool or an allocator hook),
// host runtimes that bind only a fixed set of device buffers handed to them (an FFI caller that receives
// raw pointers and no allocator), and latency-critical paths where a cudaMalloc would synchronise the
// device.  mpq_gemm_tc needs the hi/lo TF32 halves of both operands in caller-provided buffers; this
// variant keeps them, and its pipeline status word, in one file-scope device array instead.
//
// The array (kNoAllocBytes = 16 MiB) exists on every GPU that loads the library, from module load until
// process exit.  Its first 256 bytes hold the status word, the rest the four split operands, each
// row-major with a leading dimension of round_up(K, 4) floats: 2 * (M + N) * round_up(K, 4) floats must
// fit in (kNoAllocBytes - 256) / 4 = 4,194,240; larger products are rejected with MPQ_ERR_ARG.
// Every call on a device shares the array and it keeps the previous call's contents: the status word is
// cleared at the start of each call and the split operands are rewritten before they are read.  Calls
// whose executions overlap on the GPU (different streams, or different host threads without ordering)
// race on the array.
// ---------------------------------------------------------------------------------------------------------
#include <mutex>

namespace mpq {
namespace noalloc {

constexpr size_t kNoAllocBytes = 16u << 20;
constexpr size_t kStatusBytes = 256;
constexpr int64_t kMaxOperandFloats = (int64_t)((kNoAllocBytes - kStatusBytes) / 4);
constexpr int kMaxDevices = 64;

// Device-side scratch.  In host code this name is only a handle for cudaGetSymbolAddress, never an address.
static __device__ __align__(256) unsigned char g_scratch[kNoAllocBytes];

static std::mutex g_mu;
static unsigned char* g_base[kMaxDevices] = {};  // device address of g_scratch per device

// Set-up, once per device, with that device current: look up the array's device address.
static int scratch_base(unsigned char** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_error("mpq_gemm_tf32x3_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return (int)e;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_last_error("mpq_gemm_tf32x3_noalloc: device %d out of range", dev);
    return MPQ_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_base[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess || !p) {
      set_last_error("mpq_gemm_tf32x3_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return e != cudaSuccess ? (int)e : MPQ_ERR_UNSUPPORTED;
    }
    g_base[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_base[dev];
  return MPQ_OK;
}

}  // namespace noalloc
}  // namespace mpq

// C = alpha * A B^T + beta * C in 3xTF32 (A: M x K, B: N x K, row-major fp32), with no device allocation.
// `status` (optional, device int owned by the caller) is cleared and receives a non-zero code if a pipeline
// wait timed out; when it is NULL the status word inside the array is used and the code is not reported.
// The first call on each device performs the set-up above; make it before any stream capture.
MPQ_API int mpq_gemm_tf32x3_noalloc(int M, int N, int K, float alpha, const float* A, int64_t lda, const float* B,
                                    int64_t ldb, float beta, float* C, int64_t ldc, int* status, void* stream) {
  MPQ_CHECK_ARG(M >= 0 && N >= 0 && K >= 1, "mpq_gemm_tf32x3_noalloc: bad shape");
  MPQ_CHECK_ARG(lda >= K && ldb >= K && ldc >= N, "mpq_gemm_tf32x3_noalloc: leading dimensions too small");
  const int64_t kp = ((int64_t)K + 3) / 4 * 4;
  const int64_t need = 2 * ((int64_t)M + N) * kp;
  MPQ_CHECK_ARG(need <= noalloc::kMaxOperandFloats,
                "mpq_gemm_tf32x3_noalloc: 2*(M+N)*round_up(K,4) = %lld floats exceeds the %lld-float scratch",
                (long long)need, (long long)noalloc::kMaxOperandFloats);
  if (M == 0 || N == 0) return MPQ_OK;  // empty tensors may carry null pointers
  MPQ_CHECK_ARG(A && B && C, "mpq_gemm_tf32x3_noalloc: null pointer");
  unsigned char* base = nullptr;
  int st = noalloc::scratch_base(&base);
  if (st) return st;
  st = tc::get_encoder();
  if (st) return st;
  cudaStream_t s = (cudaStream_t)stream;
  if (!status) status = reinterpret_cast<int*>(base);
  float* a_hi = reinterpret_cast<float*>(base + noalloc::kStatusBytes);
  float* a_lo = a_hi + (int64_t)M * kp;
  float* b_hi = a_lo + (int64_t)M * kp;
  float* b_lo = b_hi + (int64_t)N * kp;
  cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int), s);
  if (e != cudaSuccess) {
    set_last_error("mpq_gemm_tf32x3_noalloc: clearing the status word: %s", cudaGetErrorString(e));
    return (int)e;
  }
  st = mpq_split_tf32(A, lda, a_hi, a_lo, kp, M, K, stream);
  if (st) return st;
  st = mpq_split_tf32(B, ldb, b_hi, b_lo, kp, N, K, stream);
  if (st) return st;
  tc::Maps maps;
  memset(&maps, 0, sizeof(maps));
  const float* As[3] = {a_hi, a_hi, a_lo};
  const float* Bs[3] = {b_hi, b_lo, b_hi};
  for (int r = 0; r < 3; ++r) {
    st = tc::make_map(&maps.a[r], As[r], M, K, kp, tc::BM);
    if (st) return st;
    st = tc::make_map(&maps.b[r], Bs[r], N, K, kp, 256);
    if (st) return st;
  }
  return tc::launch<256, 4>(maps, 3, M, N, K, alpha, beta, C, ldc, status, s);
}
