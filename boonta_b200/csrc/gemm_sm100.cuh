// K2 (tensor-core path): tcgen05 GEMM for sm_100a with TMA-staged bf16 operands and the
// fp32 accumulator in tensor memory, with the learner's epilogues fused.
//
//   D[M, N] (fp32, TMEM) = sum_k A[m, k] * B[n, k]       A, B bf16 in shared memory
//
// One CTA computes one 128 x BN output tile over a range of K (split-K over gridDim.z):
//   warp 0      TMA producer: one elected lane loads 64-wide K blocks of A and B into a
//               ring of shared-memory stages (128-byte swizzle), arming "full" mbarriers;
//   warp 1      allocates BN TMEM columns; one elected lane issues tcgen05.mma
//               (kind::f16, M = 128, N = BN, K = 16; four per K block) and frees a stage
//               with tcgen05.commit on its "empty" mbarrier;
//   warps 2-9   epilogue: after the final commit, each warp reads its 32-lane quarter of
//               the accumulator (two warps per quarter, each on half of the columns) with
//               tcgen05.ld (32 columns at a time) and applies the fused epilogue (bias +
//               activation + bf16/fp32 stores, activation derivative, or transposed
//               split-K partial stores).
// Operands may be K-major (rows of K contiguous) or MN-major (the M/N index contiguous),
// selected per operand by template flags, so the forward (A K-major, B MN-major), dX
// (both K-major) and dW^T (both MN-major) contractions all read the row-major activation
// and weight buffers directly, with no transposed copies.
//
// Every mbarrier wait is bounded (ptx.cuh): a wait that gives up records an error code in
// `err`, the CTA skips the rest of its work, waits (bounded) for its own copies in flight,
// frees its TMEM and returns.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "ptx.cuh"

namespace bt {
namespace umma {

constexpr int BM = 128;
constexpr int BK = 64;  // one 128-byte swizzle span of bf16
constexpr int kEpiWarps = 8;  // two warps per TMEM lane quarter, each on half the columns
constexpr int kThreads = 64 + 32 * kEpiWarps;
// K blocks (64 rows each) accumulated in tensor memory before the epilogue warps add the partial
// sum into fp32 registers (two-level accumulation of the split-K kernel).
constexpr int kChunk = 32;
constexpr int kErrTimeoutFull = 11, kErrTimeoutEmpty = 12, kErrTimeoutAcc = 13,
              kErrTimeoutEpiIn = 14;
// Store epilogues (kTma): each epilogue warp owns 4 KB of shared memory that holds, one
// after the other, the 32 x 32 fp32 input sub-tile (dX), the fp32 output sub-tile (128-byte
// swizzle) and the two 32 x 32 bf16 output sub-tiles (2 KB each, 64-byte swizzle), written in
// the swizzled order the tensor maps expect and sent out by TMA stores.
constexpr int kEpiWarpBytes = 4096;
// Dynamic shared memory per CTA on sm_100 (227 KB).
constexpr int kMaxSmem = 227 * 1024;

// Shared-memory budget: a ring of stages of A (and, in the split mode, A_lo) and B (B_lo)
// tiles, each stage 1024-byte aligned. The ring is sized so that two to three CTAs fit on
// an SM (about 72 KB each): one CTA's epilogue then overlaps the others' main loops, which
// matters for the learner's short-K GEMMs (K = 87..512); for long K the co-resident CTAs
// keep enough TMA loads in flight.
// kDeep: a long-K GEMM (the dW contractions over the minibatch rows, about one CTA per
// SM) gets a deep ring of up to 200 KB instead, to keep enough TMA loads in flight.
template <int BN, bool X3, bool kDeep = false>
struct Cfg {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = (kABytes + kBBytes) * (X3 ? 2 : 1);
  static constexpr int kFit = ((kDeep ? 200 : 72) * 1024) / kStageBytes;
  static constexpr int kStages = kFit < 2 ? 2 : (kFit > 6 ? 6 : kFit);
  static constexpr int kSmem = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

// ---- PTX wrappers ------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// Tiled bulk store shared -> global (coordinates {x = column, y = row}); the engine clips
// the box at the tensor's bounds. Completion is tracked per thread through bulk groups.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0,
                                             int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(smem_u32(src))
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// The source shared memory of every committed store may be overwritten.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Every committed store has been performed.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), descriptor version 1.
// K-major: 8-row x 128-byte atoms stacked along M/N, SBO = 1024 B between atoms.
// MN-major: 8 K-rows x 128 bytes (64 M/N elements) per atom; SBO = 1024 B between K
// groups; LBO = 8192 B between 64-wide M/N blocks (each block holds the 64 K rows of the
// stage).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // version
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

template <bool kMN>
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int kstep) {
  if (kMN) return smem_desc(base + kstep * 2048, 8192, 1024);
  return smem_desc(base + kstep * 32, 16, 1024);
}

// Instruction descriptor: D fp32, A/B bf16, majors, N >> 3 at bit 17, M >> 4 at bit 24.
template <int BN, bool A_MN, bool B_MN>
__device__ __forceinline__ constexpr uint32_t instr_desc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((A_MN ? 1u : 0u) << 15) |
         ((B_MN ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

struct GemmShape {
  int M, N, K;
  int kblocks_per_split;
  const int* m_count;  // nullable: live rows bound M (forward / dX)
  const int* k_count;  // nullable: live rows bound K (dW)
  int* err;
};

// Tensor maps of the operands; a_lo / b_lo are the low bf16 halves of split fp32 operands
// (X3 mode: x = hi + lo, the product taken as hi*hi + hi*lo + lo*hi).
struct Operands {
  CUtensorMap a, b, a_lo, b_lo;
};

template <int BN, bool A_MN, bool B_MN, bool X3, class Epi>
__global__ void __launch_bounds__(kThreads, 1)
    umma_gemm_kernel(const __grid_constant__ Operands ops, GemmShape sh,
                     const __grid_constant__ Epi epi) {
  using C = Cfg<BN, X3, Epi::kDeep>;
  static_assert(!Epi::kTma, "store epilogues run in the persistent kernel");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  __shared__ int s_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();  // the operands and live counts come from earlier kernels
  int M = sh.M, K = sh.K;
  if (sh.m_count) M = min(M, *sh.m_count);
  if (sh.k_count) K = min(K, *sh.k_count);
  const int m0 = blockIdx.x * BM;
  const int n0 = blockIdx.y * BN;
  if (m0 >= M) return;  // whole CTA leaves before any barrier or TMEM use
  const int kb0 = blockIdx.z * sh.kblocks_per_split;
  const int kb1 = min(ceil_div(K, BK), kb0 + sh.kblocks_per_split);
  const int nk = max(0, kb1 - kb0);
  // Two-level accumulation: the tensor cores' fp32 accumulation loses low bits as a chain of
  // products grows (measured on B200: the relative error of a 16,384-long chain of positive
  // products is ~7e-5, growing with the chain), so every kChunk K blocks (2,048 rows) the TMEM
  // accumulator is read into fp32 registers by the epilogue warps and added there with
  // round-to-nearest, while the MMAs start the next chunk in the other of two TMEM buffers.
  const int nchunks = max(1, ceil_div(nk, kChunk));
  const uint32_t tcols = nchunks > 1 ? 2 * BN : BN;

  if (threadIdx.x == 0) {
    s_fail = 0;
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, tcols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  // stage layout: A | B | (A_lo | B_lo)
  auto load_a = [&](uint8_t* dst, const CUtensorMap* map, int k0, uint64_t* bar) {
    if (A_MN) {
      tma_load_2d(dst, map, m0, k0, bar);
      tma_load_2d(dst + 8192, map, m0 + 64, k0, bar);
    } else {
      tma_load_2d(dst, map, k0, m0, bar);
    }
  };
  auto load_b = [&](uint8_t* dst, const CUtensorMap* map, int k0, uint64_t* bar) {
    if (B_MN) {
#pragma unroll
      for (int j = 0; j < BN / 64; ++j) tma_load_2d(dst + j * 8192, map, n0 + 64 * j, k0, bar);
    } else {
      tma_load_2d(dst, map, k0, n0, bar);
    }
  };

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % C::kStages;
        if (i >= C::kStages) {
          if (!mbar_wait_bounded(&empty[s], ((i / C::kStages) - 1) & 1)) {
            atomicExch(&s_fail, kErrTimeoutEmpty);
            break;
          }
        }
        if (*(volatile int*)&s_fail) break;
        uint8_t* sa = smem + s * C::kStageBytes;
        uint8_t* sb = sa + C::kABytes;
        mbar_arrive_expect_tx(&full[s], C::kStageBytes);
        const int k0 = (kb0 + i) * BK;
        load_a(sa, &ops.a, k0, &full[s]);
        load_b(sb, &ops.b, k0, &full[s]);
        if (X3) {
          load_a(sb + C::kBBytes, &ops.a_lo, k0, &full[s]);
          load_b(sb + C::kBBytes + C::kABytes, &ops.b_lo, k0, &full[s]);
        }
        issued = i + 1;
      }
      // Let every copy this CTA issued land before the CTA may leave.
      for (int i = max(0, issued - C::kStages); i < issued; ++i) {
        const int s = i % C::kStages;
        if (!mbar_wait_bounded(&full[s], (i / C::kStages) & 1)) atomicExch(&s_fail, kErrTimeoutFull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc<BN, A_MN, B_MN>();
      for (int i = 0; i < nk; ++i) {
        const int c = i / kChunk, b = c & 1;
        const bool fresh = i % kChunk == 0;  // first K block of a chunk: overwrite the buffer
        if (fresh && c >= 2) {
          // the epilogue warps have read this buffer's previous chunk
          if (!mbar_wait_bounded(&acc_empty[b], ((c >> 1) - 1) & 1)) {
            atomicExch(&s_fail, kErrTimeoutAcc);
            break;
          }
          fence_after_sync();
        }
        const int s = i % C::kStages;
        if (!mbar_wait_bounded(&full[s], (i / C::kStages) & 1)) {
          atomicExch(&s_fail, kErrTimeoutFull);
          break;
        }
        fence_after_sync();
        const uint32_t sa = smem_u32(smem + s * C::kStageBytes);
        const uint32_t sb = sa + C::kABytes;
        const uint32_t sa_lo = sb + C::kBBytes;
        const uint32_t sb_lo = sa_lo + C::kABytes;
        const uint32_t acc = tmem + (uint32_t)(b * BN);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint64_t ah = operand_desc<A_MN>(sa, k), bh = operand_desc<B_MN>(sb, k);
          const uint32_t keep = (!fresh || k > 0) ? 1u : 0u;
          if (X3) {
            // small cross terms first, then the leading product
            mma_bf16(acc, operand_desc<A_MN>(sa_lo, k), bh, idesc, keep);
            mma_bf16(acc, ah, operand_desc<B_MN>(sb_lo, k), idesc, 1u);
            mma_bf16(acc, ah, bh, idesc, 1u);
          } else {
            mma_bf16(acc, ah, bh, idesc, keep);
          }
        }
        mma_commit(&empty[s]);
        if (i % kChunk == kChunk - 1 || i == nk - 1) mma_commit(&acc_full[b]);
      }
      if (nk == 0) mma_commit(&acc_full[0]);  // nothing to accumulate: release the epilogue
    }
  } else if constexpr (Epi::kRowWise) {
    // Row-wise epilogue (BN = 64, K within one accumulation chunk): the four warps of column
    // half 0 (warps 2..5, one per TMEM lane quarter) read their rows whole, thread = row; the
    // other four only release the buffer.
    static_assert(BN == 64, "row-wise epilogues take 64-column tiles");
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const bool ok = mbar_wait_bounded(&acc_full[0], 0);
    if (!ok && lane == 0) atomicExch(&s_fail, kErrTimeoutAcc);
    fence_after_sync();
    float v[BN];
#pragma unroll
    for (int j = 0; j < BN; ++j) v[j] = 0.f;
    if (ok && half == 0 && nk > 0) {
      float a[32], b[32];
      tmem_ld32(tmem + ((uint32_t)(q * 32) << 16), a);
      tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + 32u, b);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        v[j] = a[j];
        v[32 + j] = b[j];
      }
    }
    fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(&acc_empty[0]);
    if (half == 0) epi.apply_row(m0 + q * 32 + lane, M, v, smem, q * 32 + lane);
    if constexpr (Epi::kCoop) {
      // then all eight epilogue warps work on the tile's rows together
      asm volatile("bar.sync 2, 256;" ::: "memory");
      epi.coop(smem, m0, M, warp - 2, lane);
    }
  } else {
    // Epilogue warps 2..9: TMEM lane quarter = warp % 4 (the hardware's access rule), column
    // half = (warp - 2) / 4. After the final commit the stage ring is idle, so each warp
    // stages 32 x 32 chunks through its own piece of it to turn the row-per-thread
    // accumulator layout into row-contiguous (coalesced) stores.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    float* scr = reinterpret_cast<float*>(smem) + (warp - 2) * (32 * 33);
    const int row = m0 + q * 32 + lane;
    constexpr int kHalf = BN / 2 >= 32 ? BN / 2 : 32;
    constexpr int kGroups = kHalf / 32;
    // this thread's row of its column half, summed over the chunks in fp32
    float run[kGroups][32];
#pragma unroll
    for (int g = 0; g < kGroups; ++g)
#pragma unroll
      for (int j = 0; j < 32; ++j) run[g][j] = 0.f;
    bool ok = true;
    for (int c = 0; c < nchunks && ok; ++c) {
      const int b = c & 1;
      ok = mbar_wait_bounded(&acc_full[b], (c >> 1) & 1);
      if (!ok) {
        if (lane == 0) atomicExch(&s_fail, kErrTimeoutAcc);
        break;
      }
      fence_after_sync();
      if (nk > 0) {
#pragma unroll
        for (int g = 0; g < kGroups; ++g) {
          const int col = half * kHalf + 32 * g;
          if (col >= BN || n0 + col >= sh.N) continue;
          float v[32];
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN + col), v);
#pragma unroll
          for (int j = 0; j < 32; ++j) run[g][j] += v[j];
        }
      }
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
    // (run stays zero without K blocks; after a failed wait the results are invalid anyway)
#pragma unroll
    for (int g = 0; g < kGroups; ++g) {
      const int c = half * kHalf + 32 * g;
      if (c >= BN || n0 + c >= sh.N) break;
      float(&v)[32] = run[g];
      if constexpr (Epi::kStaged) {
#pragma unroll
        for (int j = 0; j < 32; ++j) scr[lane * 33 + j] = v[j];
        __syncwarp();
        float col_v[32];
#pragma unroll
        for (int r = 0; r < 32; ++r) col_v[r] = scr[r * 33 + lane];
        __syncwarp();
        const int col = n0 + c + lane;
        const int row0 = m0 + q * 32;
        if (col < sh.N) epi.apply_col(row0, min(32, M - row0), col, col_v, blockIdx.z);
      } else {
        if (row < M) epi.apply(row, n0 + c, v, blockIdx.z);
      }
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    fence_after_sync();
    tmem_dealloc(tmem, tcols);
  }
  if (threadIdx.x == 0 && s_fail && sh.err) atomicExch(sh.err, s_fail);
}

// Swizzled staging of one thread's row of a 32 x 32 sub-tile (thread = row `lane`). The
// orders are the TMA engine's: 128-byte swizzle for fp32 rows (16-byte chunk j of row r at
// chunk j ^ (r % 8)), 64-byte swizzle for bf16 rows (chunk j at j ^ ((r / 2) % 4)); both keep
// the warp's 16-byte shared stores free of bank conflicts.
__device__ __forceinline__ void stage_row_f32(uint8_t* tile, int lane, const float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<float4*>(tile + lane * 128 + ((j ^ (lane & 7)) << 4)) =
        make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}
__device__ __forceinline__ float4 load_row_f32(const uint8_t* tile, int lane, int j) {
  return *reinterpret_cast<const float4*>(tile + lane * 128 + ((j ^ (lane & 7)) << 4));
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&p);
}
// bf16 of v (hi) and, when `lo` is set, of the remainders v - hi.
__device__ __forceinline__ void stage_row_bf16(uint8_t* hi, uint8_t* lo, int lane,
                                               const float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = v[8 * j + 2 * i], b = v[8 * j + 2 * i + 1];
      h[i] = pack_bf16(a, b);
      if (lo) {
        const __nv_bfloat162 hp = *reinterpret_cast<__nv_bfloat162*>(&h[i]);
        l[i] = pack_bf16(a - __low2float(hp), b - __high2float(hp));
      }
    }
    const int off = lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4);
    *reinterpret_cast<uint4*>(hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
    if (lo) *reinterpret_cast<uint4*>(lo + off) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

// ---- persistent kernel with store epilogues ------------------------------------------------
// One CTA per SM walks the output tiles t = blockIdx.x, blockIdx.x + gridDim.x, ... (N tile
// fastest, so the CTAs running at the same time share the A row block through L2). The
// accumulator is double-buffered in TMEM (2 x BN columns): the MMA warp fills buffer i % 2
// while the epilogue warps drain the other, so a tile's epilogue overlaps the next tile's
// main loop. The stage ring runs on across tiles; the epilogue has its own 32 KB of shared
// memory (4 KB per warp, kEpiWarpBytes), and the ring takes what is left. Barriers: full/empty per stage (TMA -> MMA ->
// TMA), acc_full per buffer (MMA commit -> epilogue), acc_empty per buffer (the eight
// epilogue warps -> MMA, after their last tcgen05.ld of the buffer), and one input barrier
// per epilogue warp for the dX pre-activation tile. Every wait is bounded; a role that
// gives up records the error and leaves its loop, and the others then run out of work or
// out of time.
template <int BN, bool X3>
struct PCfg {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = (kABytes + kBBytes) * (X3 ? 2 : 1);
  static constexpr int kEpiBytes = kEpiWarps * kEpiWarpBytes;
  static constexpr int kFit = (kMaxSmem - kEpiBytes - 1024 /*align*/ - 256) / kStageBytes;
  static constexpr int kStages = kFit > 8 ? 8 : kFit;
  static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int kSmem = kStages * kStageBytes + kEpiBytes + 1024 /*align*/ + 256;
  static_assert(kStages >= 2, "stage ring too small");
  static_assert(kTmemCols <= 512, "TMEM has 512 columns");
};

template <int BN, bool A_MN, bool B_MN, bool X3, class Epi>
__global__ void __launch_bounds__(kThreads, 1)
    umma_persistent_kernel(const __grid_constant__ Operands ops, GemmShape sh,
                           const __grid_constant__ Epi epi) {
  using C = PCfg<BN, X3>;
  static_assert(Epi::kTma, "persistent kernel runs store epilogues");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* epi_smem = smem + C::kStages * C::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_smem + C::kEpiBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint64_t* epi_in = acc_empty + 2;         // [kEpiWarps]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_in + kEpiWarps);
  __shared__ int s_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  if (threadIdx.x == 0) {
    s_fail = 0;
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    for (int w = 0; w < kEpiWarps; ++w) mbar_init(&epi_in[w], 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::kTmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  auto failed = [&]() { return *(volatile int*)&s_fail != 0; };
  // The prologue above overlaps the previous kernel's tail; everything below reads its
  // outputs. A CTA without tiles runs no loop and frees its TMEM at the end.
  pdl_wait();
  int M = sh.M;
  if (sh.m_count) M = min(M, *sh.m_count);
  const int ntn = ceil_div(sh.N, BN);
  const int tiles = ceil_div(M, BM) * ntn;
  const int nk = ceil_div(sh.K, BK);

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;  // K blocks issued so far (across tiles)
      for (int t = blockIdx.x; t < tiles && !failed(); t += gridDim.x) {
        const int m0 = (t / ntn) * BM, n0 = (t % ntn) * BN;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % C::kStages;
          if (g >= C::kStages && !mbar_wait_bounded(&empty[s], ((g / C::kStages) - 1) & 1)) {
            atomicExch(&s_fail, kErrTimeoutEmpty);
            break;
          }
          uint8_t* sa = smem + s * C::kStageBytes;
          uint8_t* sb = sa + C::kABytes;
          mbar_arrive_expect_tx(&full[s], C::kStageBytes);
          const int k0 = kb * BK;
#pragma unroll
          for (int part = 0; part < (X3 ? 2 : 1); ++part) {
            uint8_t* pa = part ? sb + C::kBBytes : sa;
            uint8_t* pb = part ? sb + C::kBBytes + C::kABytes : sb;
            const CUtensorMap* ma = part ? &ops.a_lo : &ops.a;
            const CUtensorMap* mb = part ? &ops.b_lo : &ops.b;
            if (A_MN) {
              tma_load_2d(pa, ma, m0, k0, &full[s]);
              tma_load_2d(pa + 8192, ma, m0 + 64, k0, &full[s]);
            } else {
              tma_load_2d(pa, ma, k0, m0, &full[s]);
            }
            if (B_MN) {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j) tma_load_2d(pb + j * 8192, mb, n0 + 64 * j, k0, &full[s]);
            } else {
              tma_load_2d(pb, mb, k0, n0, &full[s]);
            }
          }
        }
      }
      // Let every copy this CTA issued land before the CTA may leave.
      for (int i = max(0, g - C::kStages); i < g; ++i) {
        const int s = i % C::kStages;
        if (!mbar_wait_bounded(&full[s], (i / C::kStages) & 1)) atomicExch(&s_fail, kErrTimeoutFull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc<BN, A_MN, B_MN>();
      int g = 0, i = 0;
      for (int t = blockIdx.x; t < tiles && !failed(); t += gridDim.x, ++i) {
        const int b = i & 1;
        if (i >= 2 && !mbar_wait_bounded(&acc_empty[b], ((i >> 1) - 1) & 1)) {
          atomicExch(&s_fail, kErrTimeoutAcc);
          break;
        }
        fence_after_sync();
        const uint32_t acc = tmem + (uint32_t)(b * BN);
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % C::kStages;
          if (!mbar_wait_bounded(&full[s], (g / C::kStages) & 1)) {
            atomicExch(&s_fail, kErrTimeoutFull);
            ok = false;
            break;
          }
          fence_after_sync();
          const uint32_t sa = smem_u32(smem + s * C::kStageBytes);
          const uint32_t sb = sa + C::kABytes;
          const uint32_t sa_lo = sb + C::kBBytes;
          const uint32_t sb_lo = sa_lo + C::kABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ah = operand_desc<A_MN>(sa, k), bh = operand_desc<B_MN>(sb, k);
            const uint32_t accumulate = (kb > 0 || k > 0) ? 1u : 0u;
            if (X3) {
              mma_bf16(acc, operand_desc<A_MN>(sa_lo, k), bh, idesc, accumulate);
              mma_bf16(acc, ah, operand_desc<B_MN>(sb_lo, k), idesc, 1u);
              mma_bf16(acc, ah, bh, idesc, 1u);
            } else {
              mma_bf16(acc, ah, bh, idesc, accumulate);
            }
          }
          mma_commit(&empty[s]);
        }
        if (!ok) break;
        mma_commit(&acc_full[b]);
      }
    }
  } else {
    // Epilogue warps 2..9: lane quarter q = warp % 4 (rows q*32 .. q*32+31, thread = row),
    // column half = (warp - 2) / 4, 32 columns at a time; outputs staged swizzled in the
    // warp's 8 KB and sent out by TMA stores. Rows at or past the live row count are
    // written as zeros.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    uint8_t* wbuf = epi_smem + (warp - 2) * kEpiWarpBytes;
    uint64_t* ibar = &epi_in[warp - 2];
    const bool load_in = Epi::kIn && epi.uses_in();
    constexpr int kHalf = BN / 2 >= 32 ? BN / 2 : 32;
    const int c_begin = half * kHalf, c_end = min(BN, (half + 1) * kHalf);
    int loads = 0;        // input tiles loaded by this warp (parity of ibar)
    bool pending = false;  // stores committed from this warp's staging buffer
    int i = 0;
    for (int t = blockIdx.x; t < tiles && !failed(); t += gridDim.x, ++i) {
      const int b = i & 1;
      const int m0 = (t / ntn) * BM, n0 = (t % ntn) * BN;
      const bool ok = mbar_wait_bounded(&acc_full[b], (i >> 1) & 1);
      if (!ok) {
        if (lane == 0) atomicExch(&s_fail, kErrTimeoutAcc);
        break;
      }
      fence_after_sync();
      const int row0 = m0 + q * 32;
      const bool live = row0 + lane < M;
      bool released = false;
      bool broke = false;
      for (int c = c_begin; c < c_end; c += 32) {
        const int col0 = n0 + c;
        const bool last = c + 32 >= c_end || col0 + 32 >= sh.N;
        if (col0 >= sh.N) break;
        if (pending) {  // earlier stores have read the staging buffer
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
          pending = false;
        }
        if (load_in && lane == 0) {
          mbar_arrive_expect_tx(ibar, epi.in_bytes());
          tma_load_2d(wbuf, &epi.in_map, col0, row0, ibar);
        }
        float v[32];
        tmem_ld32(tmem + (uint32_t)(b * BN) + ((uint32_t)(q * 32) << 16) + (uint32_t)c, v);
        if (last) {
          // the accumulator buffer is free for the MMA warp once every warp has read it
          fence_before_sync();
          if (lane == 0) mbar_arrive(&acc_empty[b]);
          released = true;
        }
        if (load_in) {
          const bool got = mbar_wait_bounded(ibar, loads & 1);
          ++loads;
          if (!got) {
            if (lane == 0) atomicExch(&s_fail, kErrTimeoutEpiIn);
            mbar_wait_bounded(ibar, (loads - 1) & 1);  // let the copy land before leaving
            broke = true;
            break;
          }
        }
        epi.prep(v, wbuf, lane, col0, live, sh.N);
        __syncwarp();  // the input tile is consumed before the buffer is overwritten
        if (epi.has_f32) {
          stage_row_f32(wbuf, lane, v);
          fence_proxy_async_smem();  // generic-proxy smem writes before the async proxy reads
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&epi.f32_map, wbuf, col0, row0);
            bulk_commit();
          }
          if (epi.has_hi) {
            if (lane == 0) bulk_wait_read_all();
            __syncwarp();
          }
        }
        if (epi.has_hi) {
          epi.post(v);
          stage_row_bf16(wbuf, epi.has_lo ? wbuf + 2048 : nullptr, lane, v);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&epi.hi_map, wbuf, col0, row0);
            if (epi.has_lo) tma_store_2d(&epi.lo_map, wbuf + 2048, col0, row0);
            bulk_commit();
          }
        }
        pending = true;
      }
      if (!released) {
        fence_before_sync();
        if (lane == 0) mbar_arrive(&acc_empty[b]);
      }
      if (broke) break;
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    fence_after_sync();
    tmem_dealloc(tmem, C::kTmemCols);
  }
  if (threadIdx.x == 0 && s_fail && sh.err) atomicExch(sh.err, s_fail);
}

__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
  hi = __float2bfloat16_rn(x);
  lo = __float2bfloat16_rn(x - __bfloat162float(hi));
}

// ---- epilogues -----------------------------------------------------------------------------
// Staged epilogues (kStaged) see one element at a time with consecutive lanes on
// consecutive columns; unstaged ones see a thread's 32 consecutive columns of one row.

// Forward: z = acc + bias; stores z (fp32, when has_f32) and h = act(z) as bf16 (split into
// hi/lo halves when has_lo) through TMA. Maps: f32_map over z (fp32, box 32 x 32, 128-byte
// swizzle), hi_map / lo_map over the bf16 outputs (box 32 x 32, 64-byte swizzle).
struct EpiFwd {
  static constexpr bool kStaged = false;
  static constexpr bool kDeep = false;
  static constexpr bool kTma = true;
  static constexpr bool kIn = false;
  CUtensorMap in_map;  // unused
  CUtensorMap f32_map, hi_map, lo_map;
  const float* bias;
  int act;
  bool has_f32, has_hi, has_lo;
  __device__ __forceinline__ bool uses_in() const { return false; }
  __device__ __forceinline__ uint32_t in_bytes() const { return 0; }
  // v = acc + bias (zero for rows past the live count): the fp32 output z
  __device__ __forceinline__ void prep(float (&v)[32], const uint8_t*, int, int col0, bool live,
                                       int N) const {
    if (col0 + 32 <= N) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 b = __ldg(reinterpret_cast<const float4*>(bias + col0) + j);
        v[4 * j] += b.x;
        v[4 * j + 1] += b.y;
        v[4 * j + 2] += b.z;
        v[4 * j + 3] += b.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += col0 + j < N ? __ldg(bias + col0 + j) : 0.f;
    }
    if (!live) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = 0.f;
    }
  }
  // the bf16 output h = act(z)
  __device__ __forceinline__ void post(float (&v)[32]) const {
    with_act(act, [&](auto tag) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = act_fwd<decltype(tag)::value>(v[j]);
    });
  }
};

// dX of a layer: g = acc * act'(pre) of the previous layer, from its pre-activation alone
// (loaded as a TMA tile through in_map: fp32, box 32 x 32, 128-byte swizzle) or, for a ReLU
// previous layer with in_bf16, from its bf16 output h (box 32 x 32, 64-byte swizzle: relu'(y) =
// [h > 0]); stores g as fp32 (LayerNorm previous layer, has_f32) or bf16 (hi/lo halves when
// has_lo).
struct EpiDx {
  static constexpr bool kStaged = false;
  static constexpr bool kDeep = false;
  static constexpr bool kTma = true;
  static constexpr bool kIn = true;
  CUtensorMap in_map;
  CUtensorMap f32_map, hi_map, lo_map;
  int act;
  bool has_f32, has_hi, has_lo;
  bool in_bf16 = false;
  __device__ __forceinline__ bool uses_in() const { return act != BT_ACT_NONE; }
  __device__ __forceinline__ uint32_t in_bytes() const { return in_bf16 ? 32 * 32 * 2 : 32 * 32 * 4; }
  // g = acc * act'(pre) with pre from the input tile (zero for rows past the live count)
  __device__ __forceinline__ void prep(float (&v)[32], const uint8_t* in, int lane, int,
                                       bool live, int) const {
    if (in_bf16) {
      // the row's four 16-byte chunks of 8 bf16 outputs, 64-byte swizzle (stage_row_bf16)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 w = *reinterpret_cast<const uint4*>(in + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4));
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const __nv_bfloat162 hp = *reinterpret_cast<const __nv_bfloat162*>(&ws[i]);
          v[8 * j + 2 * i] *= act_dz_from_out<BT_ACT_RELU>(__low2float(hp));
          v[8 * j + 2 * i + 1] *= act_dz_from_out<BT_ACT_RELU>(__high2float(hp));
        }
      }
    } else {
      with_act(act, [&](auto tag) {
        constexpr int A = decltype(tag)::value;
        if constexpr (A != BT_ACT_NONE) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 p = load_row_f32(in, lane, j);
            v[4 * j] *= act_dz<A>(p.x);
            v[4 * j + 1] *= act_dz<A>(p.y);
            v[4 * j + 2] *= act_dz<A>(p.z);
            v[4 * j + 3] *= act_dz<A>(p.w);
          }
        }
      });
    }
    if (!live) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = 0.f;
    }
  }
  __device__ __forceinline__ void post(float (&)[32]) const {}
};

// dW^T tile: acc[m = output feature][n = input feature (bias row last)] stored transposed
// into out[split][n][m] (the [K_in + 1, N_out] kernel+bias layout); coalesced across the
// warp's rows.
struct EpiDwT {
  static constexpr bool kRowWise = false;
  static constexpr bool kStaged = false;
  static constexpr bool kDeep = true;
  static constexpr bool kTma = false;
  float* out;
  int ld;  // N_out
  size_t split_stride;
  int N;  // K_in + 1
  __device__ __forceinline__ void apply(int row, int col0, const float (&v)[32], int split) const {
    float* o = out + (size_t)split * split_stride;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = col0 + j;
      if (n >= N) break;
      o[(size_t)n * ld + row] = v[j];
    }
  }
};

// Plain fp32 store of the tile (diagnostics and tests).
struct EpiStore {
  static constexpr bool kRowWise = false;
  static constexpr bool kStaged = true;
  static constexpr bool kDeep = false;
  static constexpr bool kTma = false;
  float* out;
  int ld;
  __device__ __forceinline__ void apply_col(int row0, int nrows, int col, const float (&v)[32],
                                            int) const {
#pragma unroll
    for (int r = 0; r < 32; ++r)
      if (r < nrows) out[(size_t)(row0 + r) * ld + col] = v[r];
  }
};

// dW tile in the parameter layout: acc[m = input feature (the bias row last)][n = output
// feature] stored as split-K partial out[split][m][n] (the [K_in + 1, N_out] kernel+bias
// layout), staged so that a warp writes 32 consecutive outputs of a row at a time.
struct EpiDw {
  static constexpr bool kRowWise = false;
  static constexpr bool kStaged = true;
  static constexpr bool kDeep = true;
  static constexpr bool kTma = false;
  float* out;
  int ld;  // N_out
  size_t split_stride;
  __device__ __forceinline__ void apply_col(int row0, int nrows, int col, const float (&v)[32],
                                            int split) const {
    float* o = out + (size_t)split * split_stride;
#pragma unroll
    for (int r = 0; r < 32; ++r)
      if (r < nrows) o[(size_t)(row0 + r) * ld + col] = v[r];
  }
};

// 2-D bf16 tensor map with 128-byte swizzle: `inner` elements contiguous (row stride
// `row_bytes`), `outer` rows; box {box_inner, box_outer}.
int encode_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
               uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer);

// Epilogue tile map: 32 x 32 box over a row-major [outer, inner] fp32 (128-byte swizzle) or
// bf16 (64-byte swizzle) tensor with row stride `row_bytes`.
int encode_tile_map(CUtensorMap* map, const void* base, bool f32, uint64_t inner,
                    uint64_t outer, uint64_t row_bytes, int swizzle_bytes);

template <int BN, bool A_MN, bool B_MN, bool X3, class Epi>
int launch_gemm(const Operands& ops, const GemmShape& sh, const Epi& epi, int splits,
                cudaStream_t stream) {
  if (sh.M <= 0 || sh.N <= 0) return BT_OK;
  static bool configured = false;  // per template instance (attribute is per function)
  if constexpr (Epi::kTma) {
    using C = PCfg<BN, X3>;
    auto kernel = umma_persistent_kernel<BN, A_MN, B_MN, X3, Epi>;
    if (!configured) {
      BT_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
      configured = true;
    }
    const int tiles = ceil_div(sh.M, BM) * ceil_div(sh.N, BN);
    BT_CUDA(launch_pdl(kernel, dim3(min(tiles, kNumSMs)), dim3(kThreads), C::kSmem, stream, ops,
                       sh, epi));
  } else {
    using C = Cfg<BN, X3, Epi::kDeep>;
    auto kernel = umma_gemm_kernel<BN, A_MN, B_MN, X3, Epi>;
    if (!configured) {
      BT_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
      configured = true;
    }
    dim3 grid(ceil_div(sh.M, BM), ceil_div(sh.N, BN), max(1, splits));
    BT_CUDA(launch_pdl(kernel, grid, dim3(kThreads), C::kSmem, stream, ops, sh, epi));
  }
  return BT_OK;
}

}  // namespace umma
}  // namespace bt
