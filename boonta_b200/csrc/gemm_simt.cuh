// K2 (fp32 path): CUDA-core GEMM C[M, N] = sum_k A(m, k) B(k, n) with fused operand
// gathers and epilogues, used for fp32-exact layers and every narrow layer.
//
// Tile 128 x 128 x 8, 256 threads, 8 x 8 outputs per thread (as 2 x 2 blocks of 4 x 4 so
// that shared-memory reads are conflict-free float4s), double-buffered shared memory.
// The operand "loaders" let one kernel serve every contraction of the learner step:
//   ARows     A(m, k) = src[row(m) * ld + k]           activations, or obs rows gathered
//                                                     through the minibatch indices
//   ACols     A(m, k) = src[row(k) * ld + m]           transposed activations (dW GEMMs)
//   BRows     B(k, n) = src[k * ld + n]                kernel [K+1, N] (bias row last)
//   BCols     B(k, n) = src[n * ld + k]                kernel^T (dX GEMMs)
// A "ones" column (forward) or row (dW) at index K_in makes the bias part of the GEMM:
// z = [x, 1] [W; b] and [dW; db] = [x, 1]^T dz.
// Split-K (gridDim.z) writes fp32 partials that a fixed-order reduction sums, so every
// result is deterministic.
#pragma once

#include "common.cuh"

namespace bt {

constexpr int kBM = 128, kBN = 128, kBK = 8, kGemmThreads = 256;

// ---- A loaders ------------------------------------------------------------------------
struct ARows {  // k contiguous
  static constexpr bool kMContig = false;
  const float* src;
  const int* idx;  // nullable row gather
  int ld;
  int kin;  // k == kin -> 1.0 (bias column); k > kin -> 0
  __device__ __forceinline__ float load(int m, int k, int M, int /*K*/) const {
    if (m >= M) return 0.f;
    if (k < kin) {
      const int r = idx ? idx[m] : m;
      return src[(size_t)r * ld + k];
    }
    return k == kin ? 1.f : 0.f;
  }
};

struct ACols {  // m contiguous: A(m, k) = src[row(k) * ld + m]
  static constexpr bool kMContig = true;
  const float* src;
  const int* idx;
  int ld;
  int kin;  // m == kin -> 1.0 (bias row); m > kin -> 0
  __device__ __forceinline__ float load(int m, int k, int /*M*/, int K) const {
    if (k >= K) return 0.f;
    if (m < kin) {
      const int r = idx ? idx[k] : k;
      return src[(size_t)r * ld + m];
    }
    return m == kin ? 1.f : 0.f;
  }
};

// ---- B loaders --------------------------------------------------------------------------
struct BRows {  // n contiguous
  static constexpr bool kNContig = true;
  const float* src;
  int ld;
  int K;  // rows of B
  __device__ __forceinline__ float load(int k, int n, int N) const {
    if (n >= N || k >= K) return 0.f;
    return src[(size_t)k * ld + n];
  }
};

struct BCols {  // B(k, n) = src[n * ld + k]
  static constexpr bool kNContig = false;
  const float* src;
  int ld;
  int K;
  __device__ __forceinline__ float load(int k, int n, int N) const {
    if (n >= N || k >= K) return 0.f;
    return src[(size_t)n * ld + k];
  }
};

// ---- epilogues ---------------------------------------------------------------------------
struct EpiForward {  // z (nullable) and h = act(z)
  float* z;
  float* h;
  int ld;
  int act;
  __device__ __forceinline__ void store(int m, int n, float v, int /*split*/) const {
    if (z) z[(size_t)m * ld + n] = v;
    if (h) h[(size_t)m * ld + n] = act_forward(v, act);
  }
};

struct EpiActGrad {  // out = v * act'(pre, post); act NONE stores v
  float* out;
  const float* pre;
  const float* post;
  int ld;
  int act;
  __device__ __forceinline__ void store(int m, int n, float v, int /*split*/) const {
    const size_t i = (size_t)m * ld + n;
    if (act != BT_ACT_NONE) v *= act_grad(pre ? pre[i] : 0.f, post ? post[i] : 0.f, act);
    out[i] = v;
  }
};

struct EpiPartial {  // split-K partial sums [split][M][N]
  float* out;
  int ld;
  size_t split_stride;
  __device__ __forceinline__ void store(int m, int n, float v, int split) const {
    out[(size_t)split * split_stride + (size_t)m * ld + n] = v;
  }
};

// M, N: output extent; K: reduction extent. `m_count`/`k_count` (nullable) shrink M or K
// at run time to the live rows of a padded minibatch (times `count_scale`, the pixels per
// row of a convolution).
template <class AL, class BL, class EP>
__global__ void __launch_bounds__(kGemmThreads)
    gemm_simt_kernel(AL a, BL b, EP ep, int M, int N, int K, int k_per_split,
                     const int* m_count, const int* k_count, int count_scale) {
  __shared__ __align__(16) float As[2][kBK][kBM + 4];
  __shared__ __align__(16) float Bs[2][kBK][kBN + 4];

  if (m_count) M = min(M, *m_count * count_scale);
  if (k_count) K = min(K, *k_count * count_scale);
  const int m0 = blockIdx.x * kBM;
  const int n0 = blockIdx.y * kBN;
  if (m0 >= M) return;
  const int split = blockIdx.z;
  const int kb = split * k_per_split;
  const int ke = min(K, kb + k_per_split);

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  float ra[4], rb[4];
  auto load_tiles = [&](int k0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (AL::kMContig) {
        const int kk = tid >> 5, mm = ((tid & 31) << 2) + j;
        ra[j] = (k0 + kk < ke) ? a.load(m0 + mm, k0 + kk, M, ke) : 0.f;
      } else {
        const int mm = tid >> 1, kk = ((tid & 1) << 2) + j;
        ra[j] = (k0 + kk < ke) ? a.load(m0 + mm, k0 + kk, M, ke) : 0.f;
      }
      if (BL::kNContig) {
        const int kk = tid >> 5, nn = ((tid & 31) << 2) + j;
        rb[j] = (k0 + kk < ke) ? b.load(k0 + kk, n0 + nn, N) : 0.f;
      } else {
        const int nn = tid >> 1, kk = ((tid & 1) << 2) + j;
        rb[j] = (k0 + kk < ke) ? b.load(k0 + kk, n0 + nn, N) : 0.f;
      }
    }
  };
  auto store_tiles = [&](int buf) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (AL::kMContig) {
        As[buf][tid >> 5][((tid & 31) << 2) + j] = ra[j];
      } else {
        As[buf][((tid & 1) << 2) + j][tid >> 1] = ra[j];
      }
      if (BL::kNContig) {
        Bs[buf][tid >> 5][((tid & 31) << 2) + j] = rb[j];
      } else {
        Bs[buf][((tid & 1) << 2) + j][tid >> 1] = rb[j];
      }
    }
  };

  int buf = 0;
  if (kb < ke) {
    load_tiles(kb);
    store_tiles(0);
  }
  __syncthreads();
  for (int k0 = kb; k0 < ke; k0 += kBK) {
    const bool more = k0 + kBK < ke;
    if (more) load_tiles(k0 + kBK);
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (more) {
      store_tiles(buf ^ 1);
      __syncthreads();
      buf ^= 1;
    }
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (n < N) ep.store(m, n, acc[i][j], split);
    }
  }
}

// Small-output variant for the recurrent per-step products (M = environments of a
// minibatch, N and K a few hundred): BM x 32 tiles, K in steps of 32 with the next step's
// operands loaded into registers while the current one is multiplied (one shared-memory
// buffer per step, two barriers), 128 threads each computing (BM / 16) x 4 outputs, so a
// 256 x 256 product still spreads over 64-128 CTAs. Same loader / epilogue interface, no
// split-K, live rows through m_count.
template <int BM, class AL, class BL, class EP>
__global__ void __launch_bounds__(128)
    gemm_simt_small_kernel(AL a, BL b, EP ep, int M, int N, int K, const int* m_count) {
  constexpr int BN = 32, BK = 32, RM = BM / 16;
  constexpr int NA = BM * BK / 128, NB = BN * BK / 128;  // elements per thread per step
  __shared__ float As[BK][BM + 1];
  __shared__ float Bs[BK][BN + 1];
  if (m_count) M = min(M, *m_count);
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  if (m0 >= M) return;
  const int tid = threadIdx.x;
  const int tm = tid >> 3, tn = tid & 7;  // rows tm*RM .. +RM-1, columns tn*4 .. +3
  float acc[RM][4];
#pragma unroll
  for (int i = 0; i < RM; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  float ra[NA], rb[NB];
  auto load = [&](int k0) {  // consecutive threads on consecutive k (or n when contiguous)
#pragma unroll
    for (int u = 0; u < NA; ++u) {
      const int e = tid + 128 * u, mm = e / BK, kk = e % BK;
      ra[u] = (k0 + kk < K) ? a.load(m0 + mm, k0 + kk, M, K) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < NB; ++u) {
      const int e = tid + 128 * u;
      const int kk = BL::kNContig ? e / BN : e % BK, nn = BL::kNContig ? e % BN : e / BK;
      rb[u] = (k0 + kk < K) ? b.load(k0 + kk, n0 + nn, N) : 0.f;
    }
  };
  load(0);
  for (int k0 = 0; k0 < K; k0 += BK) {
#pragma unroll
    for (int u = 0; u < NA; ++u) {
      const int e = tid + 128 * u;
      As[e % BK][e / BK] = ra[u];
    }
#pragma unroll
    for (int u = 0; u < NB; ++u) {
      const int e = tid + 128 * u;
      if (BL::kNContig) {
        Bs[e / BN][e % BN] = rb[u];
      } else {
        Bs[e % BK][e / BK] = rb[u];
      }
    }
    __syncthreads();
    if (k0 + BK < K) load(k0 + BK);  // in flight during the products below
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float av[RM], bv[4];
#pragma unroll
      for (int i = 0; i < RM; ++i) av[i] = As[kk][tm * RM + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tn * 4 + j];
#pragma unroll
      for (int i = 0; i < RM; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < RM; ++i) {
    const int m = m0 + tm * RM + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tn * 4 + j;
      if (n < N) ep.store(m, n, acc[i][j], 0);
    }
  }
}

template <int BM, class AL, class BL, class EP>
int launch_gemm_simt_small(const AL& a, const BL& b, const EP& ep, int M, int N, int K,
                           cudaStream_t stream, const int* m_count = nullptr) {
  if (M <= 0 || N <= 0) return BT_OK;
  dim3 grid(ceil_div(M, BM), ceil_div(N, 32));
  gemm_simt_small_kernel<BM, AL, BL, EP><<<grid, 128, 0, stream>>>(a, b, ep, M, N, K, m_count);
  BT_LAUNCH_CHECK("gemm_simt_small_kernel");
  return BT_OK;
}

template <class AL, class BL, class EP>
int launch_gemm_simt(const AL& a, const BL& b, const EP& ep, int M, int N, int K, int splits,
                     cudaStream_t stream, const int* m_count = nullptr,
                     const int* k_count = nullptr, int count_scale = 1) {
  if (M <= 0 || N <= 0) return BT_OK;
  if (splits < 1) splits = 1;
  int kps = ceil_div(K, splits);
  kps = ceil_div(kps, kBK) * kBK;
  dim3 grid(ceil_div(M, kBM), ceil_div(N, kBN), splits);
  gemm_simt_kernel<AL, BL, EP><<<grid, kGemmThreads, 0, stream>>>(a, b, ep, M, N, K, kps,
                                                                   m_count, k_count,
                                                                   count_scale);
  BT_LAUNCH_CHECK("gemm_simt_kernel");
  return BT_OK;
}

}  // namespace bt
