// K5/K6/K7/K13: fused policy/value heads, PPO loss, loss gradient, head weight gradient
// and logged statistics.
//
// For every live row of a minibatch the kernel computes
//   actor head  out = act(f_pi) [W_pi; b_pi]    (logits, or the gaussian mean)
//   critic head v   = act(f_v)  [w_v; b_v]
//   the clipped-surrogate / clipped-value / entropy loss of boonta/algorithms/ppo.py:77-121
//   and its gradient dL/d(out), dL/dv (JAX's balanced tie rule for min/max/clip,
//   ppo.py:95-114), dL/d f through the head kernels times the derivative of the tower's
//   last activation, the per-block partial sums behind the eight logged statistics
//   (ppo.py:167-179) and, when the head is small enough to keep its gradient in registers,
//   the head weight gradients [f, 1]^T dL/d(out) and [f, 1]^T dL/dv as per-block partials.
//
// Work unit: a tile of 32 rows, 256 threads (8 warps), grid-stride over the tiles.
//   1. the tile's pre-activations are loaded (float4, coalesced) and act(f) staged in
//      shared memory, row stride F + 4 (16-byte rows, conflict-free float4 access);
//   2. head outputs: warp w sums the feature slices w, w + 8, ... (4 features each) of row
//      `lane` against the head kernel columns (shared memory, [j][k], broadcast float4
//      reads) for all A + 1 outputs at once; the eight warp partials are added in order;
//   3. loss: eight threads per row, thread `sub` owning outputs j = sub, sub + 8, ...;
//      softmax / gaussian terms reduced over the eight with shuffles;
//   4. dL/d f for the tile (same float4 mapping as 1, the pre-activation re-read for the
//      activation derivative), stored as fp32 or bf16 (hi/lo);
//   5. (fused head dW) thread k accumulates sum_r f[r][k] dL/d(out)[r][j] over its tiles.
// Statistics are summed in double; all partial sums have a fixed order, so results are
// deterministic for a fixed grid.
#include "common.cuh"
#include "kernels.cuh"
#include "mma_sync.cuh"
#include "ppo_row.cuh"

namespace bt {

constexpr int kHeadThreads = 256;
constexpr int kHeadWarps = kHeadThreads / 32;
constexpr int kTileRows = 32;

// Shared-memory layout of the heads kernel, in floats (every region 16-byte aligned).
struct HeadsLayout {
  int F, Fv, A, JP;
  bool shared, mma;
  int ldf, ldv;
  int ldj;  // row stride of the head kernel in shared memory (see heads_layout)
  int ldd;  // row stride of the output gradients d
  size_t f, fv, wj, wv, bias, red, vred, d, sig, isig, lsig, total;
};

// Padded output count JP of the kernel instance that serves A actions (A + 1 outputs):
// 4, 8, 12 or 16 with the fused head weight gradient, 16, 32, 48 or 64 without.
__host__ __device__ inline int heads_inst_jp(int A, bool fuse) {
  const int n = A + 1;
  if (fuse && n <= 16) return n <= 4 ? 4 : n <= 8 ? 8 : n <= 12 ? 12 : 16;
  return n <= 16 ? 16 : n <= 32 ? 32 : n <= 48 ? 48 : 64;
}

// Wide heads (JP >= 32, no fused head dW) may run the head products on warp-level tensor
// cores (`mma`): the head kernel is then kept feature-major, wj[k][j] with row stride
// ldj = JP + 8, and the features and output gradients get row strides (F + 8, JP + 8) whose
// 16-byte fragment reads fall on distinct banks. Otherwise wj[j][k] (stride F), rows F + 4.
__host__ __device__ inline HeadsLayout heads_layout(int F, int Fv, int A, bool shared, int JP,
                                                    bool mma = false) {
  HeadsLayout L{};
  L.F = F;
  L.Fv = Fv;
  L.A = A;
  L.JP = JP;
  L.shared = shared;
  L.mma = mma;
  L.ldf = F + (mma ? 8 : 4);
  L.ldv = Fv + 4;
  L.ldj = mma ? JP + 8 : F;
  L.ldd = mma ? JP + 8 : JP;
  size_t o = 0;
  auto take = [&](size_t n) {
    const size_t at = o;
    o += (n + 3) / 4 * 4;
    return at;
  };
  L.f = take((size_t)kTileRows * L.ldf);
  L.fv = take(shared ? 0 : (size_t)kTileRows * L.ldv);
  L.wj = take(mma ? (size_t)F * L.ldj : (size_t)L.JP * F);
  L.wv = take(shared ? 0 : Fv);
  L.bias = take(L.JP);
  // phase-2 partials; after the last tile the same space holds the final reductions
  // (32 x 12 doubles of statistics and 32 x JP floats of gaussian scale gradient)
  const size_t red_a = (size_t)(mma ? 1 : kHeadWarps) * kTileRows * L.JP;
  const size_t red_b = (size_t)kTileRows * kNumStatSums * 2 + (size_t)kTileRows * L.JP;
  L.red = take(red_a > red_b ? red_a : red_b);
  L.vred = take(shared ? 0 : (size_t)kHeadWarps * kTileRows);
  L.d = take((size_t)kTileRows * L.ldd);
  L.sig = take(L.JP);
  L.isig = take(L.JP);
  L.lsig = take(L.JP);
  L.total = o;
  return L;
}

// Whether the instance serving these heads runs its products on tensor cores: wide heads
// (32 or more outputs), features in whole 16-column steps, and the layout within the 227 KB of
// shared memory.
static bool heads_use_mma(int F_pi, int F_v, int A, bool shared, bool fuse) {
  const int jp = heads_inst_jp(A, fuse);
  if (jp < 32 || F_pi % 16 != 0) return false;
  return heads_layout(F_pi, F_v, A, shared, jp, true).total * sizeof(float) <= 227 * 1024;
}

// Whether the heads kernel accumulates the head weight gradients itself: small heads with up
// to one feature per thread, or wide tensor-core heads over a shared torso with up to two
// features per thread.
bool heads_fuse_dw(int F_pi, int F_v, int A, bool shared) {
  if (A + 1 <= 16) return F_pi <= kHeadThreads && F_v <= kHeadThreads;
  return shared && F_pi <= 2 * kHeadThreads && heads_use_mma(F_pi, F_v, A, shared, true);
}

static size_t heads_smem_for(int F_pi, int F_v, int A, bool shared, bool fuse) {
  return heads_layout(F_pi, F_v, A, shared, heads_inst_jp(A, fuse),
                      heads_use_mma(F_pi, F_v, A, shared, fuse))
             .total *
         sizeof(float);
}

size_t heads_smem_bytes(int F_pi, int F_v, int A, bool shared) {
  return heads_smem_for(F_pi, F_v, A, shared, heads_fuse_dw(F_pi, F_v, A, shared));
}

// Sum / max over the eight threads of a row group (lanes differing in bits 0..2).
__device__ __forceinline__ float group8_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  return v;
}
__device__ __forceinline__ float group8_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
  return v;
}

template <int A>
__device__ __forceinline__ float4 act4(float4 z) {
  return make_float4(act_fwd<A>(z.x), act_fwd<A>(z.y), act_fwd<A>(z.z), act_fwd<A>(z.w));
}

// Chunk coordinates without integer division in the loops (a division costs several
// special-function-unit instructions, the unit the activations already keep busy): chunk
// c = tid + 256 i of a tile with q4 float4 columns per row sits at row r, column q, and the
// next chunk of the same thread is 256 further on.
struct ChunkWalk {
  int r, q, dr, dq, q4;
  __device__ __forceinline__ ChunkWalk(int q4_) : q4(q4_) {
    dr = kHeadThreads / q4;
    dq = kHeadThreads - dr * q4;
    r = threadIdx.x / q4;
    q = threadIdx.x - r * q4;
  }
  __device__ __forceinline__ void next() {
    q += dq;
    r += dr;
    if (q >= q4) {
      q -= q4;
      ++r;
    }
  }
};

// Stage act(pre) of the tile's rows [row0, row0 + 32) into f_s (rows past `live` as 0).
// Each thread handles float4 chunks c = tid + 256 i; the loads of a batch of eight chunks
// are all issued before any is used, so their latencies overlap.
constexpr int kBatch = 8;

template <int ACT>
__device__ __forceinline__ void stage_features(const float* pre, int F, int ld, int row0,
                                               int live, float* f_s) {
  const int q4 = F / 4, total = kTileRows * q4;
  ChunkWalk w(q4);
  for (int c0 = threadIdx.x; c0 < total; c0 += kBatch * kHeadThreads) {
    float4 z[kBatch];
    ChunkWalk at = w;
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int c = c0 + i * kHeadThreads;
      z[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < total && row0 + at.r < live)
        z[i] = __ldg(reinterpret_cast<const float4*>(pre + (size_t)(row0 + at.r) * F) + at.q);
      at.next();
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int c = c0 + i * kHeadThreads;
      if (c < total)
        *reinterpret_cast<float4*>(f_s + w.r * ld + 4 * w.q) = act4<ACT>(z[i]);
      w.next();
    }
  }
}

// dL/d pre of the tile: g = (sum_j d[r][j] w[j][k]) * act'(pre), for the actor tower
// (JP outputs through wj_s) or the critic tower (output jcol through wv_s). Batches of
// eight chunks as in stage_features (pre-activations loaded first).
// For tanh / relu the derivative comes from the staged act(pre) in shared memory (f_s, row
// stride ld); only silu re-reads the pre-activation.
template <int JP, int Act>
__device__ __forceinline__ void store_feature_grad(const float* pre, int F, int row0,
                                                   int live, int rows_cap, const float* d_s,
                                                   int ldd, const float* w_s, int nj, int jcol,
                                                   const float* f_s, int ld, float* df,
                                                   __nv_bfloat16* dfb, __nv_bfloat16* dfb_lo) {
  const int q4 = F / 4, total = kTileRows * q4;
  ChunkWalk w(q4);
  for (int c0 = threadIdx.x; c0 < total; c0 += kBatch * kHeadThreads) {
    float4 z[kBatch];
    if constexpr (Act == BT_ACT_SILU) {
      ChunkWalk at = w;
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        const int c = c0 + i * kHeadThreads;
        z[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c < total && row0 + at.r < live)
          z[i] = __ldg(reinterpret_cast<const float4*>(pre + (size_t)(row0 + at.r) * F) + at.q);
        at.next();
      }
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int c = c0 + i * kHeadThreads;
      const int r = w.r, q = w.q;
      w.next();
      const int row = row0 + r;
      if (c >= total || row >= rows_cap) continue;
      float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
      if (nj > 1) {
#pragma unroll 4
        for (int j = 0; j < JP; ++j) {
          const float dj = d_s[r * ldd + j];
          const float4 wv = *reinterpret_cast<const float4*>(w_s + (size_t)j * F + 4 * q);
          g.x = fmaf(dj, wv.x, g.x);
          g.y = fmaf(dj, wv.y, g.y);
          g.z = fmaf(dj, wv.z, g.z);
          g.w = fmaf(dj, wv.w, g.w);
        }
      } else {
        const float dj = d_s[r * ldd + jcol];
        const float4 wv = *reinterpret_cast<const float4*>(w_s + 4 * q);
        g = make_float4(dj * wv.x, dj * wv.y, dj * wv.z, dj * wv.w);
      }
      if constexpr (Act == BT_ACT_SILU) {
        g.x *= act_dz<Act>(z[i].x);
        g.y *= act_dz<Act>(z[i].y);
        g.z *= act_dz<Act>(z[i].z);
        g.w *= act_dz<Act>(z[i].w);
      } else if constexpr (Act != BT_ACT_NONE) {
        const float4 h = *reinterpret_cast<const float4*>(f_s + r * ld + 4 * q);
        g.x *= act_dz_from_out<Act>(h.x);
        g.y *= act_dz_from_out<Act>(h.y);
        g.z *= act_dz_from_out<Act>(h.z);
        g.w *= act_dz_from_out<Act>(h.w);
      }
      const size_t e = (size_t)row * F + 4 * q;
      if (dfb) {
        store_bf16x4(dfb, dfb_lo, e, g);
      } else {
        *reinterpret_cast<float4*>(df + e) = g;
      }
    }
  }
}

// The head kernel of the tensor-core instances is held in shared memory pre-split: one 32-bit
// word per element, bf16 hi = bf16(w) in the upper half and lo = bf16(w - hi) in the lower
// (the split of split_pair, done once per block instead of per tile and warp).
__device__ __forceinline__ uint32_t pack_split(float w) {
  const __nv_bfloat16 hi = __float2bfloat16_rn(w);
  const __nv_bfloat16 lo = __float2bfloat16_rn(w - __bfloat162float(hi));
  return ((uint32_t)__bfloat16_as_ushort(hi) << 16) | (uint32_t)__bfloat16_as_ushort(lo);
}
// The bf16x2 fragment registers (first element in the low half) of two packed words.
__device__ __forceinline__ uint32_t packed_hi(uint32_t a, uint32_t b) { return __byte_perm(a, b, 0x7632); }
__device__ __forceinline__ uint32_t packed_lo(uint32_t a, uint32_t b) { return __byte_perm(a, b, 0x5410); }

// Phase 2 on tensor cores (MMA instances): out[32][JP] = f[32][F] W[F][JP] in split bf16.
// Warp w takes m-tile w % 2 (16 rows) and the n-tiles w / 2 and w / 2 + 4 (8 outputs each).
template <int JP>
__device__ __forceinline__ void heads_outputs_mma(const float* f_s, int ldf, const uint32_t* wj_s,
                                                  int ldj, int F, float* out_s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3, mt = warp & 1, nt0 = warp >> 1;
  constexpr int NT = JP / 8;
  float acc[2][4] = {};
  const float* a0 = f_s + (mt * 16 + gid) * ldf + 2 * tig;
  const float* a1 = a0 + 8 * ldf;
  for (int ks = 0; ks < F / 16; ++ks) {
    uint32_t ah[4], al[4];
    load_a_split(a0 + 16 * ks, a1 + 16 * ks, ah, al);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int nt = nt0 + 4 * i;
      if (nt >= NT) continue;
      const uint32_t* b = wj_s + (16 * ks + 2 * tig) * ldj + nt * 8 + gid;
      const uint32_t w0 = b[0], w1 = b[ldj], w8 = b[8 * ldj], w9 = b[9 * ldj];
      const uint32_t bh[2] = {packed_hi(w0, w1), packed_hi(w8, w9)};
      const uint32_t bl[2] = {packed_lo(w0, w1), packed_lo(w8, w9)};
      mma_split(acc[i], ah, al, bh, bl);
    }
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int nt = nt0 + 4 * i;
    if (nt >= NT) continue;
    float* o = out_s + (mt * 16 + gid) * JP + nt * 8 + 2 * tig;
    o[0] = acc[i][0];
    o[1] = acc[i][1];
    o[8 * JP] = acc[i][2];
    o[8 * JP + 1] = acc[i][3];
  }
}

// Phase 4 of the actor tower on tensor cores (MMA instances): dL/d pre [32][F] =
// (d[32][JP] W^T) * act'(pre), stored as fp32 or bf16 (hi/lo). Warp w takes m-tile w % 2 and
// the feature n-tiles w / 2, w / 2 + 4, ...; the d fragments stay in registers across them.
template <int JP, int Act>
__device__ __forceinline__ void heads_feature_grad_mma(const float* pre, int F, int row0,
                                                       int live, int rows_cap, const float* d_s,
                                                       int ldd, const uint32_t* wj_s, int ldj,
                                                       const float* f_s, int ldf, float* df,
                                                       __nv_bfloat16* dfb,
                                                       __nv_bfloat16* dfb_lo) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3, mt = warp & 1;
  constexpr int KD = JP / 16;
  uint32_t dh[KD][4], dl[KD][4];
  const float* a0 = d_s + (mt * 16 + gid) * ldd + 2 * tig;
#pragma unroll
  for (int kd = 0; kd < KD; ++kd) load_a_split(a0 + 16 * kd, a0 + 8 * ldd + 16 * kd, dh[kd], dl[kd]);
  for (int nt = warp >> 1; nt < F / 8; nt += 4) {
    float acc[4] = {};
    const uint32_t* wb = wj_s + (nt * 8 + gid) * ldj + 2 * tig;
#pragma unroll
    for (int kd = 0; kd < KD; ++kd) {
      const uint2 b0 = *reinterpret_cast<const uint2*>(wb + 16 * kd);
      const uint2 b1 = *reinterpret_cast<const uint2*>(wb + 16 * kd + 8);
      const uint32_t bh[2] = {packed_hi(b0.x, b0.y), packed_hi(b1.x, b1.y)};
      const uint32_t bl[2] = {packed_lo(b0.x, b0.y), packed_lo(b1.x, b1.y)};
      mma_split(acc, dh[kd], dl[kd], bh, bl);
    }
    const int c = nt * 8 + 2 * tig;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = row0 + mt * 16 + gid + 8 * h;
      if (row >= rows_cap) continue;
      float2 g = make_float2(acc[2 * h], acc[2 * h + 1]);
      if constexpr (Act == BT_ACT_SILU) {
        float2 z = make_float2(0.f, 0.f);
        if (row < live) z = __ldg(reinterpret_cast<const float2*>(pre + (size_t)row * F + c));
        g.x *= act_dz<Act>(z.x);
        g.y *= act_dz<Act>(z.y);
      } else if constexpr (Act != BT_ACT_NONE) {
        // the derivative from the staged act(pre) (rows past the live count are zero there)
        const float2 hv =
            *reinterpret_cast<const float2*>(f_s + (mt * 16 + gid + 8 * h) * ldf + c);
        g.x *= act_dz_from_out<Act>(hv.x);
        g.y *= act_dz_from_out<Act>(hv.y);
      }
      const size_t e = (size_t)row * F + c;
      if (dfb) {
        const __nv_bfloat162 hv = __floats2bfloat162_rn(g.x, g.y);
        *reinterpret_cast<__nv_bfloat162*>(dfb + e) = hv;
        if (dfb_lo)
          *reinterpret_cast<__nv_bfloat162*>(dfb_lo + e) =
              __floats2bfloat162_rn(g.x - __low2float(hv), g.y - __high2float(hv));
      } else {
        *reinterpret_cast<float2*>(df + e) = g;
      }
    }
  }
}

// Phase 5 on tensor cores (fused MMA instances): the tile's head weight gradient
// dW[F][JP] += f^T[F][32] d[32][JP] in split bf16, accumulated in registers across tiles. Warp w
// owns the 16-feature m-tiles w, w + 8, w + 16, w + 24 (F <= 512) and every output n-tile.
template <int JP>
__device__ __forceinline__ void heads_weight_grad_mma(const float* f_s, int ldf, const float* d_s,
                                                      int ldd, int F, float (&acc)[4][JP / 8][4]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  constexpr int NT = JP / 8;
#pragma unroll
  for (int ks = 0; ks < kTileRows / 16; ++ks) {
    const int r0 = 16 * ks + 2 * tig;  // rows (the reduction index) of this lane's fragments
    uint32_t bh[NT][2], bl[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const float* d0 = d_s + r0 * ldd + nt * 8 + gid;
      split_pair(d0[0], d0[ldd], bh[nt][0], bl[nt][0]);
      split_pair(d0[8 * ldd], d0[9 * ldd], bh[nt][1], bl[nt][1]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m0 = 16 * (warp + 8 * i);
      if (m0 >= F) break;
      const float* f0 = f_s + r0 * ldf + m0 + gid;  // f^T[m][k] = f_s[k][m]
      uint32_t ah[4], al[4];
      split_pair(f0[0], f0[ldf], ah[0], al[0]);
      split_pair(f0[8], f0[ldf + 8], ah[1], al[1]);
      split_pair(f0[8 * ldf], f0[9 * ldf], ah[2], al[2]);
      split_pair(f0[8 * ldf + 8], f0[9 * ldf + 8], ah[3], al[3]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_split(acc[i][nt], ah, al, bh[nt], bl[nt]);
    }
  }
}

template <int JP, bool FUSE, int ACT, bool MMA>
__global__ void __launch_bounds__(kHeadThreads, (FUSE && MMA) ? 1 : 2)
    heads_loss_kernel(HeadsParams p) {
  constexpr int JJ = (JP + 7) / 8;  // outputs per thread in the loss phase
  static_assert(!MMA || JP % 16 == 0, "tensor-core heads: whole 16-output steps");

  extern __shared__ __align__(16) float sm[];
  const int F = p.F_pi, Fv = p.F_v, A = p.A;
  const bool shared = (p.f_v == p.f_pi);
  const HeadsLayout Lo = heads_layout(F, Fv, A, shared, JP, MMA);
  float* f_s = sm + Lo.f;
  float* fv_s = sm + Lo.fv;
  float* wj_s = sm + Lo.wj;
  uint32_t* wp_s = reinterpret_cast<uint32_t*>(wj_s);  // packed split words (MMA instances)
  float* wv_s = sm + Lo.wv;
  float* bias_s = sm + Lo.bias;
  float* red_s = sm + Lo.red;
  float* vred_s = sm + Lo.vred;
  float* d_s = sm + Lo.d;
  float* isig_s = sm + Lo.isig;
  float* lsig_s = sm + Lo.lsig;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_trigger();
  pdl_wait();  // parameters, features and targets come from earlier kernels
  const int live = live_rows(p.count, p.rows);
  // Tiles up to the next 64-row boundary: the rows past the live count get zero feature
  // gradients (the bf16 operands of the tensor-core weight-gradient GEMMs need them).
  const int tiles = ceil_div(dz_rows_end(live, p.rows), kTileRows);

  // head kernels as columns wj[j][k] (j < A actor outputs, j = A the value when the torso
  // is shared, the rest zero), biases, gaussian constants
  for (int i = tid; i < JP * F; i += kHeadThreads) {
    int j, k;
    if constexpr (MMA) {  // feature-major: wj[k][j]
      k = i / JP;
      j = i - k * JP;
    } else {
      j = i / F;
      k = i - j * F;
    }
    float w = 0.f;
    if (j < A) w = p.w_pi[(size_t)k * A + j];
    else if (j == A && shared) w = p.w_v[k];
    if constexpr (MMA) {
      wp_s[k * Lo.ldj + j] = pack_split(w);
    } else {
      wj_s[i] = w;
    }
  }
  if (!shared)
    for (int k = tid; k < Fv; k += kHeadThreads) wv_s[k] = p.w_v[k];
  for (int j = tid; j < JP; j += kHeadThreads)
    bias_s[j] = j < A ? p.w_pi[(size_t)F * A + j] : (j == A ? p.w_v[Fv] : 0.f);
  if (p.head == BT_HEAD_GAUSSIAN) {
    for (int j = tid; j < A; j += kHeadThreads) {
      const float sc = p.scale[j];
      const float sig = (fmaxf(sc, 0.f) + log1pf(expf(-fabsf(sc)))) + 1e-3f;  // softplus + 1e-3
      isig_s[j] = 1.f / sig;
      lsig_s[j] = logf(sig);
    }
  }
  __syncthreads();

  // loss-phase identity: row r of the tile, output group sub
  const int r = tid >> 3, sub = tid & 7;
  double st[kNumStatSums];
#pragma unroll
  for (int s = 0; s < kNumStatSums; ++s) st[s] = 0.0;
  float dsc[JJ];
#pragma unroll
  for (int jj = 0; jj < JJ; ++jj) dsc[jj] = 0.f;
  // fused head dW: the thread's feature tid over all outputs (CUDA cores), or its fragments of
  // the warp's m-tiles (tensor cores)
  float accw[(FUSE && !MMA) ? JP : 1];
#pragma unroll
  for (int j = 0; j < ((FUSE && !MMA) ? JP : 1); ++j) accw[j] = 0.f;
  float accm[(FUSE && MMA) ? 4 : 1][(FUSE && MMA) ? JP / 8 : 1][4];
#pragma unroll
  for (int i = 0; i < ((FUSE && MMA) ? 4 : 1); ++i)
#pragma unroll
    for (int nt = 0; nt < ((FUSE && MMA) ? JP / 8 : 1); ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) accm[i][nt][e] = 0.f;
  float accv = 0.f, accb = 0.f;

  for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int row0 = tile * kTileRows;
    // 1. features
    stage_features<ACT>(p.f_pi, F, Lo.ldf, row0, live, f_s);
    if (!shared) stage_features<ACT>(p.f_v, Fv, Lo.ldv, row0, live, fv_s);
    __syncthreads();

    // 2. head outputs: warp partials over interleaved 4-feature slices (CUDA cores), or the
    // finished outputs from the tensor cores
    if constexpr (MMA) {
      heads_outputs_mma<JP>(f_s, Lo.ldf, wp_s, Lo.ldj, F, red_s);
      if (!shared) {
        float v = 0.f;
        const float* vrow = fv_s + lane * Lo.ldv;
        for (int sl = warp; sl < Fv / 4; sl += kHeadWarps) {
          const float4 x = *reinterpret_cast<const float4*>(vrow + 4 * sl);
          const float4 w = *reinterpret_cast<const float4*>(wv_s + 4 * sl);
          v = fmaf(x.x, w.x, v);
          v = fmaf(x.y, w.y, v);
          v = fmaf(x.z, w.z, v);
          v = fmaf(x.w, w.w, v);
        }
        vred_s[warp * kTileRows + lane] = v;
      }
    } else {
      float acc[JP];
#pragma unroll
      for (int j = 0; j < JP; ++j) acc[j] = 0.f;
      const float* frow = f_s + lane * Lo.ldf;
      for (int sl = warp; sl < F / 4; sl += kHeadWarps) {
        const float4 x = *reinterpret_cast<const float4*>(frow + 4 * sl);
#pragma unroll
        for (int j = 0; j < JP; ++j) {
          const float4 w = *reinterpret_cast<const float4*>(wj_s + (size_t)j * F + 4 * sl);
          acc[j] = fmaf(x.x, w.x, acc[j]);
          acc[j] = fmaf(x.y, w.y, acc[j]);
          acc[j] = fmaf(x.z, w.z, acc[j]);
          acc[j] = fmaf(x.w, w.w, acc[j]);
        }
      }
      float* rp = red_s + (size_t)(warp * kTileRows + lane) * JP;
#pragma unroll
      for (int j = 0; j < JP; j += 4)
        *reinterpret_cast<float4*>(rp + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
      if (!shared) {
        float v = 0.f;
        const float* vrow = fv_s + lane * Lo.ldv;
        for (int sl = warp; sl < Fv / 4; sl += kHeadWarps) {
          const float4 x = *reinterpret_cast<const float4*>(vrow + 4 * sl);
          const float4 w = *reinterpret_cast<const float4*>(wv_s + 4 * sl);
          v = fmaf(x.x, w.x, v);
          v = fmaf(x.y, w.y, v);
          v = fmaf(x.z, w.z, v);
          v = fmaf(x.w, w.w, v);
        }
        vred_s[warp * kTileRows + lane] = v;
      }
    }
    __syncthreads();

    // 3. loss and output gradients, eight threads per row
    {
      const int row = row0 + r;
      const bool on = row < live;
      float o[JJ];
#pragma unroll
      for (int jj = 0; jj < JJ; ++jj) {
        const int j = sub + 8 * jj;
        float t = 0.f;
        if (j < JP) {
          t = bias_s[j];
          if constexpr (MMA) {
            t += red_s[(size_t)r * JP + j];
          } else {
            for (int w = 0; w < kHeadWarps; ++w) t += red_s[(size_t)(w * kTileRows + r) * JP + j];
          }
        }
        o[jj] = t;
      }
      float value = bias_s[A];
      if (shared) {
        if constexpr (MMA) {
          value += red_s[(size_t)r * JP + A];
        } else {
          for (int w = 0; w < kHeadWarps; ++w) value += red_s[(size_t)(w * kTileRows + r) * JP + A];
        }
      } else {
        for (int w = 0; w < kHeadWarps; ++w) value += vred_s[w * kTileRows + r];
      }
      const int flat = on ? (p.idx ? p.idx[row] : row) : 0;
      const float lp_old = on ? p.lp_old[flat] : 0.f;
      const float adv = on ? p.adv[flat] : 0.f;
      const float ret = on ? p.ret[flat] : 0.f;
      const float v_old = on ? p.v_old[flat] : 0.f;
      float lp, ent;
      float pj[JJ], lpj[JJ], zj[JJ];
#pragma unroll
      for (int jj = 0; jj < JJ; ++jj) pj[jj] = lpj[jj] = zj[jj] = 0.f;
      int action = 0;
      if (p.head == BT_HEAD_CATEGORICAL) {
        if (on) action = reinterpret_cast<const int*>(p.action)[flat];
        float mx = -INFINITY;
#pragma unroll
        for (int jj = 0; jj < JJ; ++jj)
          if (sub + 8 * jj < A) mx = fmaxf(mx, o[jj]);
        mx = group8_max(mx);
        float se = 0.f;
#pragma unroll
        for (int jj = 0; jj < JJ; ++jj)
          if (sub + 8 * jj < A) se += expf(o[jj] - mx);
        se = group8_sum(se);
        const float lse = logf(se);
        float h = 0.f, mine = 0.f;
#pragma unroll
        for (int jj = 0; jj < JJ; ++jj) {
          const int j = sub + 8 * jj;
          if (j < A) {
            lpj[jj] = (o[jj] - mx) - lse;
            pj[jj] = expf(lpj[jj]);
            h -= pj[jj] * lpj[jj];
            if (j == action) mine = lpj[jj];
          }
        }
        ent = group8_sum(h);
        lp = group8_sum(mine);  // one thread holds the action's log-prob, the rest 0
      } else {
        const float* av = reinterpret_cast<const float*>(p.action) + (size_t)flat * A;
        float acc = 0.f, e = 0.f;
#pragma unroll
        for (int jj = 0; jj < JJ; ++jj) {
          const int j = sub + 8 * jj;
          if (j < A) {
            const float a = on ? av[j] : 0.f;
            zj[jj] = (a - o[jj]) * isig_s[j];
            acc += -0.5f * zj[jj] * zj[jj] - lsig_s[j] - 0.5f * kLog2Pi;
            e += 0.5f + 0.5f * kLog2Pi + lsig_s[j];
          }
        }
        lp = group8_sum(acc);
        ent = group8_sum(e);
      }
      // Surrogate and value loss (ppo.py:90-115), JAX's balanced tie rule for min/max/clip.
      const float eps = p.clip;
      const RowLoss rl = ppo_row_loss(lp, lp_old, adv, ret, v_old, value, on, eps, p.clip_value,
                                      p.inv_mb, p.vf_coef);
      const float g_lp = rl.g_lp;
      const float g_ent = -p.ent_coef * p.inv_mb;
      const float d_value = rl.d_value;
#pragma unroll
      for (int jj = 0; jj < JJ; ++jj) {
        const int j = sub + 8 * jj;
        if (j >= JP) continue;
        float g = 0.f;
        if (j < A && on) {
          if (p.head == BT_HEAD_CATEGORICAL) {
            g = g_lp * (((j == action) ? 1.f : 0.f) - pj[jj]) +
                g_ent * (-pj[jj] * (lpj[jj] + ent));
          } else {
            g = g_lp * (zj[jj] * isig_s[j]);
            dsc[jj] += g_lp * ((zj[jj] * zj[jj] - 1.f) * isig_s[j]) + g_ent * isig_s[j];
          }
          if (p.d_out) p.d_out[(size_t)row * A + j] = g;
        }
        d_s[r * Lo.ldd + j] = (j == A) ? d_value : g;
      }
      if (sub == 0 && on) {
        if (p.d_val) p.d_val[row] = d_value;
        add_row_stats(st, rl, ent, lp, lp_old, adv, ret, value, eps);
      }
    }
    __syncthreads();

    // 4. dL/d pre for the towers
    if constexpr (MMA) {
      heads_feature_grad_mma<JP, ACT>(p.f_pi, F, row0, live, p.rows, d_s, Lo.ldd, wp_s, Lo.ldj,
                                      f_s, Lo.ldf, p.d_fpi, p.d_fpi_b, p.d_fpi_b_lo);
    } else {
      store_feature_grad<JP, ACT>(p.f_pi, F, row0, live, p.rows, d_s, Lo.ldd, wj_s, JP, 0, f_s,
                                  Lo.ldf, p.d_fpi, p.d_fpi_b, p.d_fpi_b_lo);
    }
    if (!shared)
      store_feature_grad<JP, ACT>(p.f_v, Fv, row0, live, p.rows, d_s, Lo.ldd, wv_s, 1, A, fv_s,
                                  Lo.ldv, p.d_fv, p.d_fv_b, p.d_fv_b_lo);
    // 5. head weight gradients
    if constexpr (FUSE && MMA) {
      heads_weight_grad_mma<JP>(f_s, Lo.ldf, d_s, Lo.ldd, F, accm);
    } else if constexpr (FUSE) {
      if (tid < F) {
        for (int rr = 0; rr < kTileRows; ++rr) {
          const float fk = f_s[rr * Lo.ldf + tid];
#pragma unroll
          for (int j = 0; j < JP; j += 4) {
            const float4 dd = *reinterpret_cast<const float4*>(d_s + rr * Lo.ldd + j);
            accw[j] = fmaf(fk, dd.x, accw[j]);
            accw[j + 1] = fmaf(fk, dd.y, accw[j + 1]);
            accw[j + 2] = fmaf(fk, dd.z, accw[j + 2]);
            accw[j + 3] = fmaf(fk, dd.w, accw[j + 3]);
          }
        }
      }
    }
    if constexpr (FUSE) {
      if (!shared && tid < Fv)
        for (int rr = 0; rr < kTileRows; ++rr) accv = fmaf(fv_s[rr * Lo.ldv + tid], d_s[rr * Lo.ldd + A], accv);
      if (tid < JP)
        for (int rr = 0; rr < kTileRows; ++rr) accb += d_s[rr * Lo.ldd + tid];
    }
    __syncthreads();
  }

  if constexpr (FUSE) {
    float* pp = p.dw_pi_partials + (size_t)blockIdx.x * (F + 1) * A;
    float* pv = p.dw_v_partials + (size_t)blockIdx.x * (Fv + 1);
    if constexpr (MMA) {
      const int gid = lane >> 2, tig = lane & 3;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int m0 = 16 * (warp + 8 * i);
        if (m0 >= F) break;
#pragma unroll
        for (int nt = 0; nt < JP / 8; ++nt) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int k = m0 + gid + 8 * (e >> 1), j = nt * 8 + 2 * tig + (e & 1);
            if (j < A) pp[(size_t)k * A + j] = accm[i][nt][e];
            if (shared && j == A) pv[k] = accm[i][nt][e];
          }
        }
      }
    } else if (tid < F) {
#pragma unroll
      for (int j = 0; j < JP; ++j) {
        if (j < A) pp[(size_t)tid * A + j] = accw[j];
        if (shared && j == A) pv[tid] = accw[j];
      }
    }
    if (tid < A) pp[(size_t)F * A + tid] = accb;
    if (!shared && tid < Fv) pv[tid] = accv;
    if (tid == A) pv[Fv] = accb;
  }

  // Block partial sums in a fixed order: row slots -> thread 0..11 (statistics), row slots
  // -> thread j (gaussian scale gradient).
  double* st_s = reinterpret_cast<double*>(red_s);
  float* ds_s = red_s + kTileRows * kNumStatSums * 2;
  if (sub == 0) {
#pragma unroll
    for (int s = 0; s < kNumStatSums; ++s) st_s[r * kNumStatSums + s] = st[s];
  }
  if (p.head == BT_HEAD_GAUSSIAN) {
#pragma unroll
    for (int jj = 0; jj < JJ; ++jj) {
      const int j = sub + 8 * jj;
      if (j < A) ds_s[r * JP + j] = dsc[jj];
    }
  }
  __syncthreads();
  if (tid < kNumStatSums) {
    double s = 0.0;
    for (int rr = 0; rr < kTileRows; ++rr) s += st_s[rr * kNumStatSums + tid];
    p.stat_partials[(size_t)blockIdx.x * kNumStatSums + tid] = s;
  }
  if (p.head == BT_HEAD_GAUSSIAN && p.dscale_partials) {
    for (int j = tid; j < A; j += kHeadThreads) {
      float s = 0.f;
      for (int rr = 0; rr < kTileRows; ++rr) s += ds_s[rr * JP + j];
      const float sc = p.scale[j];
      const float sgm = 1.f / (1.f + expf(-sc));  // d softplus / d scale
      p.dscale_partials[(size_t)blockIdx.x * A + j] = s * sgm;
    }
  }
}

template <int JP, bool FUSE, int ACT, bool MMA = false>
int launch_heads_inst(const HeadsParams& p, int blocks, size_t smem, cudaStream_t stream) {
  auto kernel = heads_loss_kernel<JP, FUSE, ACT, MMA>;
  static size_t configured = 0;
  if (smem > 48 * 1024 && smem > configured) {
    BT_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    configured = smem;
  }
  BT_CUDA(launch_pdl(kernel, dim3(blocks), dim3(kHeadThreads), smem, stream, p));
  return BT_OK;
}

// The activation of the towers' last layers is a template parameter (one instance per
// activation keeps each kernel's code small); both towers must end in the same one.
template <int JP, bool FUSE, bool MMA = false>
int launch_heads_jp(const HeadsParams& p, int blocks, size_t smem, cudaStream_t stream) {
  switch (p.act_pi) {
    case BT_ACT_TANH: return launch_heads_inst<JP, FUSE, BT_ACT_TANH, MMA>(p, blocks, smem, stream);
    case BT_ACT_RELU: return launch_heads_inst<JP, FUSE, BT_ACT_RELU, MMA>(p, blocks, smem, stream);
    case BT_ACT_SILU: return launch_heads_inst<JP, FUSE, BT_ACT_SILU, MMA>(p, blocks, smem, stream);
    default: return launch_heads_inst<JP, FUSE, BT_ACT_NONE, MMA>(p, blocks, smem, stream);
  }
}

int launch_heads_loss(const HeadsParams& p, int blocks, cudaStream_t stream) {
  const bool shared = p.f_v == p.f_pi;
  const bool fuse = p.dw_pi_partials != nullptr;
  const size_t smem = heads_smem_for(p.F_pi, p.F_v, p.A, shared, fuse);
  BT_CHECK_ARG(p.A >= 1 && p.A <= 63, "heads: action_dim %d outside [1, 63]", p.A);
  BT_CHECK_ARG(p.F_pi % 4 == 0 && p.F_v % 4 == 0, "heads: feature widths %d / %d must be "
               "multiples of 4", p.F_pi, p.F_v);
  BT_CHECK_ARG(shared || p.act_pi == p.act_v, "heads: actor and critic towers must end in the "
               "same activation (%d / %d)", p.act_pi, p.act_v);
  BT_CHECK_ARG(smem <= 227 * 1024, "heads: feature width too large for shared memory");
  const int jp = heads_inst_jp(p.A, fuse);  // the instance below; its layout uses this JP
  if (fuse) {
    BT_CHECK_ARG(heads_fuse_dw(p.F_pi, p.F_v, p.A, shared) && p.dw_v_partials,
                 "heads: fused head weight gradient needs A + 1 <= 16 and widths <= %d, or a "
                 "wide head over a shared torso of width <= %d", kHeadThreads, 2 * kHeadThreads);
    if (jp <= 4) return launch_heads_jp<4, true>(p, blocks, smem, stream);
    if (jp <= 8) return launch_heads_jp<8, true>(p, blocks, smem, stream);
    if (jp <= 12) return launch_heads_jp<12, true>(p, blocks, smem, stream);
    if (jp <= 16) return launch_heads_jp<16, true>(p, blocks, smem, stream);
    if (jp <= 32) return launch_heads_jp<32, true, true>(p, blocks, smem, stream);
    if (jp <= 48) return launch_heads_jp<48, true, true>(p, blocks, smem, stream);
    return launch_heads_jp<64, true, true>(p, blocks, smem, stream);
  }
  if (jp <= 16) return launch_heads_jp<16, false>(p, blocks, smem, stream);
  if (heads_use_mma(p.F_pi, p.F_v, p.A, shared, false)) {
    if (jp <= 32) return launch_heads_jp<32, false, true>(p, blocks, smem, stream);
    if (jp <= 48) return launch_heads_jp<48, false, true>(p, blocks, smem, stream);
    return launch_heads_jp<64, false, true>(p, blocks, smem, stream);
  }
  if (jp <= 32) return launch_heads_jp<32, false>(p, blocks, smem, stream);
  if (jp <= 48) return launch_heads_jp<48, false>(p, blocks, smem, stream);
  return launch_heads_jp<64, false>(p, blocks, smem, stream);
}

bool heads_split_products(int F_pi, int F_v, int A, bool shared) {
  return heads_use_mma(F_pi, F_v, A, shared, heads_fuse_dw(F_pi, F_v, A, shared));
}

// x * w as the split-bf16 product of the wide heads: lo(x) hi(w) + hi(x) lo(w) + hi(x) hi(w),
// each term exact in fp32, added to acc in that order.
__device__ __forceinline__ float split_fma(float x, float w, float acc) {
  const float xh = __bfloat162float(__float2bfloat16_rn(x));
  const float wh = __bfloat162float(__float2bfloat16_rn(w));
  const float xl = __bfloat162float(__float2bfloat16_rn(x - xh));
  const float wl = __bfloat162float(__float2bfloat16_rn(w - wh));
  acc = fmaf(xl, wh, acc);
  acc = fmaf(xh, wl, acc);
  return fmaf(xh, wh, acc);
}

// Head outputs only (bootstrap values, act): one warp per row; the head input is act(f).
__global__ void heads_forward_kernel(const float* f_pi, int F, const float* f_v, int Fv,
                                     const float* w_pi, const float* w_v, int A, int rows,
                                     int act_pi, int act_v, float* out, float* value,
                                     bool split_pi, bool split_v) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float* f = f_pi + (size_t)warp * F;
  if (out) {
    for (int j = 0; j < A; ++j) {
      float acc = 0.f;
      for (int k = lane; k < F; k += 32) {
        const float x = act_forward(f[k], act_pi), w = w_pi[(size_t)k * A + j];
        acc = split_pi ? split_fma(x, w, acc) : fmaf(x, w, acc);
      }
      acc = warp_sum(acc);
      if (lane == 0) out[(size_t)warp * A + j] = acc + w_pi[(size_t)F * A + j];
    }
  }
  if (value) {
    const float* fv = f_v + (size_t)warp * Fv;
    float acc = 0.f;
    for (int k = lane; k < Fv; k += 32) {
      const float x = act_forward(fv[k], act_v), w = w_v[k];
      acc = split_v ? split_fma(x, w, acc) : fmaf(x, w, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) value[warp] = acc + w_v[Fv];
  }
}

int launch_heads_forward(const float* f_pi, int F, const float* f_v, int Fv, const float* w_pi,
                         const float* w_v, int A, int rows, int act_pi, int act_v, float* out,
                         float* value, bool split_pi, bool split_v, cudaStream_t stream) {
  if (rows <= 0) return BT_OK;
  heads_forward_kernel<<<ceil_div(rows * 32, 256), 256, 0, stream>>>(
      f_pi, F, f_v, Fv, w_pi, w_v, A, rows, act_pi, act_v, out, value, split_pi, split_v);
  BT_LAUNCH_CHECK("heads_forward_kernel");
  return BT_OK;
}

}  // namespace bt

namespace bt {

// a14: the sampling of PPO.step (sample_row, ppo_row.cuh) over rows of head outputs.
__global__ void sample_kernel(const float* out, const float* scale, int head, int A, int rows,
                              const float* noise, float temperature, void* action,
                              float* log_prob) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  sample_row(out + (size_t)r * A, scale, head, A, r, noise, temperature, action, log_prob);
}

// Fused act step for the CUDA-core heads: one warp per row evaluates the head outputs (as
// heads_forward_kernel) into the warp's shared-memory row, then samples from it
// (sample_row_warp, bit-identical to sample_kernel).
__global__ void heads_act_kernel(const float* f_pi, int F, const float* f_v, int Fv,
                                 const float* w_pi, const float* w_v, const float* scale,
                                 int head, int A, int rows, int act_pi, int act_v,
                                 bool split_pi, bool split_v, const float* noise,
                                 float temperature, void* action, float* log_prob, float* value) {
  extern __shared__ double act_s[];  // per warp: 64 doubles of sampling scratch, A + 1 floats
  const int wib = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + wib;
  if (row >= rows) return;
  double* es = act_s + (size_t)wib * 64;
  float* o = reinterpret_cast<float*>(act_s + (size_t)warps * 64) + (size_t)wib * (A + 1);
  const float* f = f_pi + (size_t)row * F;
  for (int j = 0; j < A; ++j) {
    float acc = 0.f;
    for (int k = lane; k < F; k += 32) {
      const float x = act_forward(f[k], act_pi), w = w_pi[(size_t)k * A + j];
      acc = split_pi ? split_fma(x, w, acc) : fmaf(x, w, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) o[j] = acc + w_pi[(size_t)F * A + j];
  }
  const float* fv = f_v + (size_t)row * Fv;
  float acc = 0.f;
  for (int k = lane; k < Fv; k += 32) {
    const float x = act_forward(fv[k], act_v), w = w_v[k];
    acc = split_v ? split_fma(x, w, acc) : fmaf(x, w, acc);
  }
  acc = warp_sum(acc);
  if (lane == 0 && value) value[row] = acc + w_v[Fv];
  __syncwarp();
  sample_row_warp(o, scale, head, A, row, noise, temperature, action, log_prob, es, lane);
}

int launch_heads_act(const float* f_pi, int F, const float* f_v, int Fv, const float* w_pi,
                     const float* w_v, const float* scale, int head, int A, int rows, int act_pi,
                     int act_v, bool split_pi, bool split_v, const float* noise,
                     float temperature, void* action, float* log_prob, float* value,
                     cudaStream_t stream) {
  if (rows <= 0) return BT_OK;
  constexpr int kWarps = 8;
  const size_t smem = kWarps * (64 * sizeof(double) + (A + 1) * sizeof(float));
  heads_act_kernel<<<ceil_div(rows, kWarps), 32 * kWarps, smem, stream>>>(f_pi, F, f_v, Fv, w_pi, w_v, scale, head, A, rows, act_pi, act_v,
                               split_pi, split_v, noise, temperature, action, log_prob, value);
  BT_LAUNCH_CHECK("heads_act_kernel");
  return BT_OK;
}

int launch_sample(const float* out, const float* scale, int head, int A, int rows,
                  const float* noise, float temperature, void* action, float* log_prob,
                  cudaStream_t stream) {
  if (rows <= 0) return BT_OK;
  sample_kernel<<<ceil_div(rows, 128), 128, 0, stream>>>(out, scale, head, A, rows, noise,
                                                         temperature, action, log_prob);
  BT_LAUNCH_CHECK("sample_kernel");
  return BT_OK;
}

}  // namespace bt

extern "C" int bt_sample_categorical(const float* logits, const float* uniforms, int32_t rows,
                                     int32_t num_actions, float temperature, int32_t* action,
                                     float* log_prob, void* stream) {
  BT_CHECK_ARG(logits && action && log_prob, "bt_sample_categorical: null argument");
  BT_CHECK_ARG(rows >= 0 && num_actions >= 1, "bt_sample_categorical: bad shape");
  return bt::launch_sample(logits, nullptr, BT_HEAD_CATEGORICAL, num_actions, rows, uniforms,
                           temperature, action, log_prob, (cudaStream_t)stream);
}
