// Per-row PPO loss terms (boonta/algorithms/ppo.py:90-115) shared by the heads kernels.
#pragma once

#include "common.cuh"
#include "kernels.cuh"

namespace bt {

// The surrogate, value and entropy terms of one row (ppo.py:90-115) and the gradient factors of
// the log-prob and the value, with JAX's balanced tie rule for min / max / clip.
struct RowLoss {
  float g_lp;     // dL / d log_prob (before the 1 / minibatch factor is applied: included)
  float d_value;  // dL / d value (zero for dead rows)
  float mn;       // min(ratio * adv, clip(ratio) * adv)
  float crit;     // the row's value loss
  float ratio;
};

__device__ __forceinline__ RowLoss ppo_row_loss(float lp, float lp_old, float adv, float ret,
                                                float v_old, float value, bool on, float eps,
                                                int clip_value, float inv_mb, float vf_coef) {
  RowLoss o;
  const float ratio = expf(lp - lp_old);
  const float lo = 1.f - eps, hi = 1.f + eps;
  const float u = fmaxf(ratio, lo);
  const float du = (ratio == u) ? ((lo == u) ? 0.5f : 1.f) : 0.f;
  const float clipped = fminf(u, hi);
  const float dm = (u == clipped) ? ((hi == clipped) ? 0.5f : 1.f) : 0.f;
  const float s1 = ratio * adv, s2 = clipped * adv;
  const float mn = fminf(s1, s2);
  const float t1 = (s1 == mn) ? ((s2 == mn) ? 0.5f : 1.f) : 0.f;
  const float t2 = (s2 == mn) ? ((s1 == mn) ? 0.5f : 1.f) : 0.f;
  o.g_lp = -((t1 * adv + t2 * adv * (dm * du)) * ratio) * inv_mb;
  const float c1 = 0.5f * ((value - ret) * (value - ret));
  float crit, dcrit;
  if (clip_value) {
    const float dv = value - v_old;
    const float uu = fmaxf(dv, -eps);
    const float duu = (dv == uu) ? ((-eps == uu) ? 0.5f : 1.f) : 0.f;
    const float cl = fminf(uu, eps);
    const float dcl = (uu == cl) ? ((eps == cl) ? 0.5f : 1.f) : 0.f;
    const float vc = v_old + cl;
    const float c2 = 0.5f * ((vc - ret) * (vc - ret));
    crit = fmaxf(c1, c2);
    const float w1 = (c1 == crit) ? ((c2 == crit) ? 0.5f : 1.f) : 0.f;
    const float w2 = (c2 == crit) ? ((c1 == crit) ? 0.5f : 1.f) : 0.f;
    dcrit = w1 * (value - ret) + w2 * (vc - ret) * (dcl * duu);
  } else {
    crit = c1;
    dcrit = value - ret;
  }
  o.d_value = on ? vf_coef * inv_mb * dcrit : 0.f;
  o.mn = mn;
  o.crit = crit;
  o.ratio = ratio;
  return o;
}

// The twelve statistic sums of one live row (order of the heads kernels' partials).
__device__ __forceinline__ void add_row_stats(double (&st)[kNumStatSums], const RowLoss& r,
                                              float ent, float lp, float lp_old, float adv,
                                              float ret, float value, float eps) {
  st[0] += (double)r.mn;
  st[1] += (double)ent;
  st[2] += (double)(lp_old - lp);
  st[3] += (fabsf(r.ratio - 1.f) > eps) ? 1.0 : 0.0;
  st[4] += (double)adv;
  st[5] += (double)r.crit;
  const double res = (double)ret - (double)value;
  st[6] += res;
  st[7] += res * res;
  st[8] += (double)ret;
  st[9] += (double)ret * (double)ret;
  st[10] += (double)value;
  st[11] += 1.0;
}

constexpr float kLog2Pi = 1.8378770664093453f;

// a14: action sampling of PPO.step (boonta/algorithms/ppo.py:57-74) for row r of head outputs
// o[0..A). Categorical (boonta/networks/distributions.py:8-23): logits = o / temperature
// (greedy argmax at temperature 0), normalised by log_softmax; the action is
// argmax(log_softmax(logits) + gumbel) with gumbel = -log(-log(u)). The noise and the
// log_softmax are evaluated in double and rounded once to float32, and the sum is a float32
// add with the first index winning ties, so the index is a deterministic function of
// (logits, u): the CPU oracle reproduces it bit for bit. Gaussian: action = mean +
// temperature * sigma * noise, and the log-prob of that action.
__device__ inline void sample_row(const float* o, const float* scale, int head, int A, int r,
                                  const float* noise, float temperature, void* action,
                                  float* log_prob) {
  if (head == BT_HEAD_CATEGORICAL) {
    int* act = reinterpret_cast<int*>(action);
    if (!(temperature > 0.f)) {
      int best = 0;
      for (int j = 1; j < A; ++j)
        if (o[j] > o[best]) best = j;
      act[r] = best;
      log_prob[r] = 0.f;
      return;
    }
    double mx = -INFINITY;
    for (int j = 0; j < A; ++j) mx = fmax(mx, (double)(o[j] / temperature));
    double se = 0.0;
    for (int j = 0; j < A; ++j) se += exp((double)(o[j] / temperature) - mx);
    const double lse = log(se) + mx;
    int best = 0;
    float best_v = -INFINITY;
    for (int j = 0; j < A; ++j) {
      const float lj = (float)((double)(o[j] / temperature) - lse);
      float v = lj;
      if (noise) {
        const double u = (double)noise[(size_t)r * A + j];
        v = lj + (float)(-log(-log(u)));
      }
      if (v > best_v || j == 0) {
        best_v = v;
        best = j;
      }
    }
    act[r] = best;
    log_prob[r] = (float)((double)(o[best] / temperature) - lse);
  } else {
    float* act = reinterpret_cast<float*>(action);
    float lp = 0.f;
    for (int j = 0; j < A; ++j) {
      const float s = scale[j];
      const float sig = temperature * ((fmaxf(s, 0.f) + log1pf(expf(-fabsf(s)))) + 1e-3f);
      const float eps = noise ? noise[(size_t)r * A + j] : 0.f;
      const float a = o[j] + sig * eps;
      act[(size_t)r * A + j] = a;
      if (sig > 0.f) lp += -0.5f * eps * eps - logf(sig) - 0.5f * kLog2Pi;
    }
    log_prob[r] = lp;
  }
}

// sample_row for one row by a whole warp (every lane calls it; A <= 64): the categorical case
// evaluates the per-action terms (the scaled logits, their exponentials, the Gumbel noise) on
// lanes j and j + 32 in parallel, adds the exponentials in index order on lane 0 (the order of
// sample_row) and picks the first maximal index with a warp reduction, so the action and the
// log-prob are bit-identical to sample_row's (for non-NaN outputs). `es`: 64 doubles of the
// warp's scratch. Other
// heads and temperature 0 fall back to sample_row on lane 0.
__device__ inline void sample_row_warp(const float* o, const float* scale, int head, int A, int r,
                                       const float* noise, float temperature, void* action,
                                       float* log_prob, double* es, int lane) {
  if (head != BT_HEAD_CATEGORICAL || !(temperature > 0.f) || A > 64) {
    if (lane == 0) sample_row(o, scale, head, A, r, noise, temperature, action, log_prob);
    return;
  }
  const int j0 = lane, j1 = lane + 32;
  const double x0 = j0 < A ? (double)(o[j0] / temperature) : -INFINITY;
  const double x1 = j1 < A ? (double)(o[j1] / temperature) : -INFINITY;
  double mx = fmax(x0, x1);
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, d));
  if (j0 < A) es[j0] = exp(x0 - mx);
  if (j1 < A) es[j1] = exp(x1 - mx);
  __syncwarp();
  double lse = 0.0;
  if (lane == 0) {
    double se = 0.0;
    for (int j = 0; j < A; ++j) se += es[j];
    lse = log(se) + mx;
  }
  lse = __shfl_sync(0xffffffffu, lse, 0);
  float v0 = -INFINITY, v1 = -INFINITY;
  if (j0 < A) {
    v0 = (float)(x0 - lse);
    if (noise) v0 = v0 + (float)(-log(-log((double)noise[(size_t)r * A + j0])));
  }
  if (j1 < A) {
    v1 = (float)(x1 - lse);
    if (noise) v1 = v1 + (float)(-log(-log((double)noise[(size_t)r * A + j1])));
  }
  // first maximal index (sample_row's `v > best_v || j == 0` scan)
  float bv = v0;
  int bj = j0;
  if (v1 > v0) {
    bv = v1;
    bj = j1;
  }
  if (j0 >= A) bj = 1 << 30;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, d);
    const int oj = __shfl_xor_sync(0xffffffffu, bj, d);
    if (ov > bv || (ov == bv && oj < bj)) {
      bv = ov;
      bj = oj;
    }
  }
  if (bj >= A) bj = 0;  // every value -inf or NaN: sample_row keeps index 0
  __syncwarp();
  if (lane == 0) {
    reinterpret_cast<int*>(action)[r] = bj;
    log_prob[r] = (float)((double)(o[bj] / temperature) - lse);
  }
}

}  // namespace bt
