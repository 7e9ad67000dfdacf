// Epilogues of the tensor-core heads (wide categorical heads over a shared tensor-core torso).
//
// Tensor-core heads: with the torso's last activation h = act(y) held as split bf16 pairs
// (hi + lo, written by the last layer's LayerNorm / forward epilogue next to the ones column of
// the bias) and the head kernels packed as W_h [F, 64] (columns 0..A-1 the actor head, column A
// the critic head, the rest zero; split bf16 pairs), one minibatch's heads are three tcgen05
// GEMMs with split-bf16 products (lo*hi + hi*lo + hi*hi, the arithmetic of split_fma):
//   1. O = h W_h ([rows, 64], K = F) with the row-wise epilogue EpiHeadsLoss: one thread per
//      row holds the row's 43 logits and the value, adds the biases, evaluates the PPO loss of
//      boonta/algorithms/ppo.py:77-121 and writes D = dL/dO ([rows, 64], split bf16 pairs) and
//      the block's statistic partial sums;
//   2. dL/dy = (D W_h^T) * act'(y) ([rows, F], K = 64): the dX epilogue of the torso (EpiDx);
//   3. [dW_pi | dw_v] = [h, 1]^T D ([F + 1, 64], K = rows, split-K) with EpiHeadsDw scattering
//      the columns into the head kernels' partial-sum layouts.
#pragma once

#include "gemm_sm100.cuh"
#include "ppo_row.cuh"

namespace bt {
namespace umma {

constexpr int kHeadCols = 64;  // packed head outputs (A actor outputs + the value, padded)

// Row-wise epilogue of the head-output GEMM (split-K kernel, BN = 64, one accumulation chunk):
// thread = row first parks the row's 64 accumulators plus biases in shared memory (rows of
// kLd floats); then the 256 threads of the eight epilogue warps take the tile's 128 rows, two
// adjacent lanes per row, each on 32 of the outputs: max, softmax sum, entropy and log-prob
// combined across the pair by one shuffle (the same value on both; one exponential per output,
// the probabilities as exp(z_j) / sum), the PPO loss terms, D =
// dL/dO stored as split bf16 pairs (16-byte stores), and the statistics summed over the warp
// by a fixed shuffle tree and over the eight warps in order (deterministic).
struct EpiHeadsLoss {
  static constexpr bool kStaged = false;
  static constexpr bool kDeep = true;
  static constexpr bool kTma = false;
  static constexpr bool kRowWise = true;
  static constexpr bool kCoop = true;
  static constexpr int kLd = kHeadCols + 1;
  int A;
  const int* count;  // nullable: live rows
  const int* idx;    // nullable: flat sample index of each row
  const float* b_pi;  // [A] actor bias
  const float* b_v;   // [1] critic bias
  const int* action;
  const float* lp_old;
  const float* v_old;
  const float* adv;
  const float* ret;
  float inv_mb, clip, ent_coef, vf_coef;
  int clip_value;
  __nv_bfloat16* d_hi;  // [rows, 64] dL/dO, split bf16 pairs
  __nv_bfloat16* d_lo;
  double* stat_partials;  // [gridDim.x][kNumStatSums]

  __device__ __forceinline__ void apply_row(int, int, float (&v)[kHeadCols], uint8_t* scr,
                                            int trow) const {
    float* o = reinterpret_cast<float*>(scr) + trow * kLd;
    const float bv = *b_v;
#pragma unroll
    for (int j = 0; j < kHeadCols; ++j) {
      if (j < A) o[j] = v[j] + __ldg(b_pi + j);
      else if (j == A) o[j] = bv + v[j];  // the value
    }
  }

  __device__ __forceinline__ void coop(uint8_t* scr, int m0, int M, int ew, int lane) const {
    // two threads per row (adjacent lanes), thread half h on outputs 32h .. 32h + 31
    const float* rows_s = reinterpret_cast<const float*>(scr);
    double* st_s = reinterpret_cast<double*>(scr + BM * kLd * sizeof(float) + 1024);
    const int t = ew * 32 + lane, r = t >> 1, h = t & 1, jb = 32 * h;
    const int row = m0 + r;
    const int live = count ? min(M, *count) : M;
    const bool on = row < live;
    const float* o = rows_s + r * kLd;
    const int flat = on ? (idx ? idx[row] : row) : 0;
    const int act = on ? action[flat] : 0;
    const float lpo = on ? lp_old[flat] : 0.f;
    const float ad = on ? adv[flat] : 0.f;
    const float rt = on ? ret[flat] : 0.f;
    const float vo = on ? v_old[flat] : 0.f;
    const float value = o[A];
    float x[32];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      x[j] = jb + j < A ? o[jb + j] : -INFINITY;
      mx = fmaxf(mx, x[j]);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    float e[32];  // exp(z_j), each evaluated once
    float se = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      x[j] = x[j] - mx;  // z_j
      e[j] = jb + j < A ? expf(x[j]) : 0.f;
      se += e[j];
    }
    se = se + __shfl_xor_sync(0xffffffffu, se, 1);  // the pair's two halves, same sum on both
    const float lse = logf(se), inv_se = 1.f / se;
    float ent = 0.f, mine = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      e[j] *= inv_se;  // p_j
      if (jb + j < A) {
        const float l = x[j] - lse;
        ent -= e[j] * l;
        if (jb + j == act) mine = l;
      }
    }
    ent = ent + __shfl_xor_sync(0xffffffffu, ent, 1);
    const float lp = mine + __shfl_xor_sync(0xffffffffu, mine, 1);
    const RowLoss rl = ppo_row_loss(lp, lpo, ad, rt, vo, value, on, clip, clip_value, inv_mb,
                                    vf_coef);
    const float g_ent = -ent_coef * inv_mb;
    if (row < M) {
      __nv_bfloat16* dh = d_hi + (size_t)row * kHeadCols + jb;
      __nv_bfloat16* dl = d_lo + (size_t)row * kHeadCols + jb;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float g[2];
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int j = jb + 8 * q + 2 * i + k;
            float gj = 0.f;
            if (j == A) {
              gj = rl.d_value;
            } else if (on && j < A) {
              const float l = x[8 * q + 2 * i + k] - lse;
              const float p = e[8 * q + 2 * i + k];
              gj = rl.g_lp * (((j == act) ? 1.f : 0.f) - p) + g_ent * (-p * (l + ent));
            }
            g[k] = gj;
          }
          const __nv_bfloat162 hp = __floats2bfloat162_rn(g[0], g[1]);
          const __nv_bfloat162 lq = __floats2bfloat162_rn(g[0] - __low2float(hp),
                                                          g[1] - __high2float(hp));
          hw[i] = *reinterpret_cast<const uint32_t*>(&hp);
          lw[i] = *reinterpret_cast<const uint32_t*>(&lq);
        }
        *reinterpret_cast<uint4*>(dh + 8 * q) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(dl + 8 * q) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
    }
    // the row's statistics on its h = 0 thread, summed over the warp by a fixed shuffle tree,
    // then the eight warp sums in warp order by threads 0..11
    double st[kNumStatSums];
#pragma unroll
    for (int k = 0; k < kNumStatSums; ++k) st[k] = 0.0;
    if (on && h == 0) add_row_stats(st, rl, ent, lp, lpo, ad, rt, value, clip);
#pragma unroll
    for (int k = 0; k < kNumStatSums; ++k) st[k] = warp_sum_d(st[k]);
    if (lane == 0) {
#pragma unroll
      for (int k = 0; k < kNumStatSums; ++k) st_s[ew * kNumStatSums + k] = st[k];
    }
    asm volatile("bar.sync 3, 256;" ::: "memory");
    if (t < kNumStatSums) {
      double sum = 0.0;
      for (int w = 0; w < kEpiWarps; ++w) sum += st_s[w * kNumStatSums + t];
      stat_partials[(size_t)blockIdx.x * kNumStatSums + t] = sum;
    }
  }
};

// Row-wise epilogue of the act step's head-output GEMM: thread = row adds the biases, stores
// the value and the row's logits (padded shared-memory rows); then the eight epilogue warps
// sample the tile's rows, one warp per row (sample_row_warp), so the act step needs no
// separate heads or sampling kernel. The logits are the same accumulations the update's loss
// epilogue sees for the same row and parameters.
struct EpiHeadsAct {
  static constexpr bool kStaged = false;
  static constexpr bool kDeep = true;
  static constexpr bool kTma = false;
  static constexpr bool kRowWise = true;
  static constexpr bool kCoop = true;
  static constexpr int kLd = kHeadCols + 1;  // shared row stride (floats)
  int A;
  const float* b_pi;
  const float* b_v;
  const float* noise;  // nullable: [rows, A] uniforms
  float temperature;
  int* action;
  float* log_prob;
  float* value;  // nullable
  __device__ __forceinline__ void apply_row(int row, int M, float (&v)[kHeadCols], uint8_t* scr,
                                            int trow) const {
    float* o = reinterpret_cast<float*>(scr) + trow * kLd;
    float val = *b_v;
#pragma unroll
    for (int j = 0; j < kHeadCols; ++j) {
      if (j < A) o[j] = v[j] + __ldg(b_pi + j);
      else if (j == A) val += v[j];
    }
    if (row < M && value) value[row] = val;
  }
  // after apply_row on every row of the tile (rows m0 .. m0 + 127): epilogue warp ew of 8
  __device__ __forceinline__ void coop(uint8_t* scr, int m0, int M, int ew, int lane) const {
    const float* rows_s = reinterpret_cast<const float*>(scr);
    double* es = reinterpret_cast<double*>(scr + BM * kLd * sizeof(float) + 1024) + ew * 64;
    for (int r = ew; r < BM && m0 + r < M; r += kEpiWarps)
      sample_row_warp(rows_s + r * kLd, nullptr, BT_HEAD_CATEGORICAL, A, m0 + r, noise,
                      temperature, action, log_prob, es, lane);
  }
};

// Head weight-gradient tile [F + 1, 64] (row m = feature, the bias last; column j = output):
// columns j < A go to the actor partials [split][F + 1][A], column A to the critic partials
// [split][F + 1].
struct EpiHeadsDw {
  static constexpr bool kStaged = true;
  static constexpr bool kDeep = true;
  static constexpr bool kTma = false;
  static constexpr bool kRowWise = false;
  float* pi_part;
  float* v_part;
  int A, F;
  __device__ __forceinline__ void apply_col(int row0, int nrows, int col, const float (&v)[32],
                                            int split) const {
    if (col < A) {
      float* o = pi_part + (size_t)split * (F + 1) * A;
#pragma unroll
      for (int r = 0; r < 32; ++r)
        if (r < nrows) o[(size_t)(row0 + r) * A + col] = v[r];
    } else if (col == A) {
      float* o = v_part + (size_t)split * (F + 1);
#pragma unroll
      for (int r = 0; r < 32; ++r)
        if (r < nrows) o[row0 + r] = v[r];
    }
  }
};

}  // namespace umma

int launch_heads_pack(const float* w_pi, const float* w_v, int F, int A, __nv_bfloat16* hi,
                      __nv_bfloat16* lo, cudaStream_t stream);
// Head outputs + loss over `rows` rows (grid: ceil(rows / 128) blocks = statistic partials).
int launch_heads_tc_loss(const umma::Operands& ops, int rows, int F,
                         const umma::EpiHeadsLoss& ep, int* err, cudaStream_t stream);
// Act step: head outputs, value and sampled action of `rows` rows.
int launch_heads_tc_act(const umma::Operands& ops, int rows, int F, const umma::EpiHeadsAct& ep,
                        int* err, cudaStream_t stream);
// Head weight gradient over the live rows, split-K partials.
int launch_heads_tc_dw(const umma::Operands& ops, int F, int rows, int kblocks_per_split,
                       int splits, const int* count, const umma::EpiHeadsDw& ep, int* err,
                       cudaStream_t stream);
// Whether a network's heads run on the tensor-core path (see heads_tc.cuh).
inline bool heads_tc_eligible(int head, bool shared, bool recurrent, bool last_tc, int F, int A) {
  return head == BT_HEAD_CATEGORICAL && shared && !recurrent && last_tc &&
         A + 1 <= umma::kHeadCols && F % umma::BK == 0 && F <= umma::kChunk * umma::BK;
}

}  // namespace bt
