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
// thread = row, holding the row's 64 accumulators.
struct EpiHeadsLoss {
  static constexpr bool kStaged = false;
  static constexpr bool kDeep = true;
  static constexpr bool kTma = false;
  static constexpr bool kRowWise = true;
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

  // All 128 threads of the four row warps call this, also after a failed accumulator wait
  // (they meet at named barrier 1).
  __device__ __forceinline__ void apply_row(int row, int M, float (&v)[kHeadCols], uint8_t* scr,
                                            int trow) const {
    const int live = count ? min(M, *count) : M;
    const bool on = row < live;
    const int flat = on ? (idx ? idx[row] : row) : 0;
    const int act = on ? action[flat] : 0;
    float mx = -INFINITY, value = *b_v;
#pragma unroll
    for (int j = 0; j < kHeadCols; ++j) {
      if (j < A) {
        v[j] += __ldg(b_pi + j);
        mx = fmaxf(mx, v[j]);
      } else if (j == A) {
        value += v[j];
      }
    }
    float se = 0.f;
#pragma unroll
    for (int j = 0; j < kHeadCols; ++j)
      if (j < A) se += expf(v[j] - mx);
    const float lse = logf(se);
    float ent = 0.f, lp = 0.f;
#pragma unroll
    for (int j = 0; j < kHeadCols; ++j) {
      if (j < A) {
        const float l = (v[j] - mx) - lse;
        ent -= expf(l) * l;
        if (j == act) lp = l;
      }
    }
    const float lpo = on ? lp_old[flat] : 0.f;
    const float ad = on ? adv[flat] : 0.f;
    const float rt = on ? ret[flat] : 0.f;
    const float vo = on ? v_old[flat] : 0.f;
    const RowLoss rl = ppo_row_loss(lp, lpo, ad, rt, vo, value, on, clip, clip_value, inv_mb,
                                    vf_coef);
    const float g_ent = -ent_coef * inv_mb;
    // D = dL/dO: the categorical log-prob and entropy gradients, the value gradient in column A
#pragma unroll
    for (int j = 0; j < kHeadCols; ++j) {
      float g = 0.f;
      if (on && j < A) {
        const float l = (v[j] - mx) - lse;
        const float p = expf(l);
        g = rl.g_lp * (((j == act) ? 1.f : 0.f) - p) + g_ent * (-p * (l + ent));
      } else if (j == A) {
        g = rl.d_value;
      }
      v[j] = g;
    }
    if (row < M) {
#pragma unroll
      for (int j = 0; j < kHeadCols; j += 8) {
        uint32_t h[4], l[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const __nv_bfloat162 hp = __floats2bfloat162_rn(v[j + 2 * i], v[j + 2 * i + 1]);
          h[i] = *reinterpret_cast<const uint32_t*>(&hp);
          const __nv_bfloat162 lq = __floats2bfloat162_rn(v[j + 2 * i] - __low2float(hp),
                                                          v[j + 2 * i + 1] - __high2float(hp));
          l[i] = *reinterpret_cast<const uint32_t*>(&lq);
        }
        *reinterpret_cast<uint4*>(d_hi + (size_t)row * kHeadCols + j) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(d_lo + (size_t)row * kHeadCols + j) = make_uint4(l[0], l[1], l[2], l[3]);
      }
    }
    // block statistic partials: rows in tile order, then thread s < 12 adds the 128 rows
    double st[kNumStatSums];
#pragma unroll
    for (int s = 0; s < kNumStatSums; ++s) st[s] = 0.0;
    if (on) add_row_stats(st, rl, ent, lp, lpo, ad, rt, value, clip);
    double* sd = reinterpret_cast<double*>(scr);
#pragma unroll
    for (int s = 0; s < kNumStatSums; ++s) sd[trow * kNumStatSums + s] = st[s];
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (trow < kNumStatSums) {
      double t = 0.0;
      for (int r = 0; r < BM; ++r) t += sd[r * kNumStatSums + trow];
      stat_partials[(size_t)blockIdx.x * kNumStatSums + trow] = t;
    }
  }
};

// Row-wise epilogue of the act step's head-output GEMM: thread = row adds the biases, stores
// the value and samples the action from the logits (sample_row, through a padded shared-memory
// row), so the act step needs no separate heads or sampling kernel. The logits are the same
// accumulations the update's loss epilogue sees for the same row and parameters.
struct EpiHeadsAct {
  static constexpr bool kStaged = false;
  static constexpr bool kDeep = true;
  static constexpr bool kTma = false;
  static constexpr bool kRowWise = true;
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
    float* o = reinterpret_cast<float*>(scr) + trow * (kHeadCols + 1);
    float val = *b_v;
#pragma unroll
    for (int j = 0; j < kHeadCols; ++j) {
      if (j < A) o[j] = v[j] + __ldg(b_pi + j);
      else if (j == A) val += v[j];
    }
    if (row < M) {
      if (value) value[row] = val;
      sample_row(o, nullptr, BT_HEAD_CATEGORICAL, A, row, noise, temperature, action, log_prob);
    }
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
