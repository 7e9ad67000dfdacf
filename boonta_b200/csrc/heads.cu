// K5/K6/K7/K13: fused policy/value heads, PPO loss, loss gradient and logged statistics.
//
// One kernel per minibatch computes, for every live row of the minibatch:
//   actor head  out = f_pi [W_pi; b_pi]     (logits, or the gaussian mean)
//   critic head v   = f_v  [W_v; b_v]
//   the clipped-surrogate / clipped-value / entropy loss of
//   boonta/algorithms/ppo.py:77-121 and its gradient dL/d(out), dL/dv (with JAX's
//   balanced tie rule for min/max/clip, ppo.py:95-114), dL/d f_pi and dL/d f_v through
//   the head kernels, multiplied by the derivative of the tower's last activation,
//   and the per-block partial sums behind the eight logged statistics (ppo.py:167-179).
// Rows are processed in tiles of 32 staged in shared memory with the head kernels
// (transposed, row stride = 1 mod 32 so that the dot products are bank-conflict free).
// Per-block partial sums (statistics in double, the gaussian scale gradient in float)
// are written to scratch and summed later in a fixed order, so results are
// deterministic for a fixed grid.
#include "common.cuh"
#include "kernels.cuh"

namespace bt {

constexpr int kHeadRows = 32;
constexpr int kHeadThreads = 256;
constexpr float kLog2Pi = 1.8378770664093453f;

__host__ __device__ inline int head_stride(int f) { return ((f + 31) / 32) * 32 + 1; }

size_t heads_smem_bytes(int F_pi, int F_v, int A, bool shared) {
  const int sp = head_stride(F_pi), sv = head_stride(F_v);
  size_t floats = 0;
  floats += (size_t)(A + (shared ? 1 : 0)) * sp;  // wT (actor rows + critic row if shared)
  floats += shared ? 0 : (size_t)sv;              // critic row of a separate tower
  floats += (size_t)kHeadRows * sp;               // f_pi tile
  floats += shared ? 0 : (size_t)kHeadRows * sv;  // f_v tile
  floats += 2 * (size_t)kHeadRows * (A + 1);      // out_s, dout_s
  floats += 3 * (size_t)A;                        // sigma, 1/sigma, log sigma
  floats += (size_t)(kHeadThreads / 32) * (A + kNumStatSums * 2);  // per-warp reductions
  return floats * 4 + 64;
}

__global__ void __launch_bounds__(kHeadThreads) heads_loss_kernel(HeadsParams p) {
  extern __shared__ __align__(16) float sm[];
  const int A = p.A;
  const bool shared = (p.f_v == p.f_pi);
  const int sp = head_stride(p.F_pi), sv = head_stride(p.F_v);
  float* wT = sm;                                                    // [A(+1)][sp]
  float* wTv = shared ? wT + (size_t)A * sp : wT + (size_t)A * sp;   // critic row
  float* f_s = wT + (size_t)(A + (shared ? 1 : 0)) * sp + (shared ? 0 : sv);
  float* fv_s = shared ? f_s : f_s + (size_t)kHeadRows * sp;
  float* out_s = fv_s + (shared ? (size_t)kHeadRows * sp : (size_t)kHeadRows * sv);
  float* dout_s = out_s + kHeadRows * (A + 1);
  float* sig_s = dout_s + kHeadRows * (A + 1);
  float* isig_s = sig_s + A;
  float* lsig_s = isig_s + A;
  float* red_s = lsig_s + A;  // [8 warps][A] dscale, then doubles for stats
  double* stat_s = reinterpret_cast<double*>(
      (reinterpret_cast<uintptr_t>(red_s + (kHeadThreads / 32) * A) + 7) & ~uintptr_t(7));

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int F = p.F_pi, Fv = p.F_v;
  const int live = live_rows(p.count, p.rows);

  // Stage transposed head kernels (bias in column F).
  for (int i = tid; i < (F + 1) * A; i += kHeadThreads) {
    const int k = i / A, j = i - k * A;
    wT[(size_t)j * sp + k] = p.w_pi[i];
  }
  for (int k = tid; k < Fv + 1; k += kHeadThreads) wTv[k] = p.w_v[k];
  if (p.head == BT_HEAD_GAUSSIAN) {
    for (int j = tid; j < A; j += kHeadThreads) {
      const float s = p.scale[j];
      const float sp_ = fmaxf(s, 0.f) + log1pf(expf(-fabsf(s)));  // softplus
      const float sig = sp_ + 1e-3f;
      sig_s[j] = sig;
      isig_s[j] = 1.f / sig;
      lsig_s[j] = logf(sig);
    }
  }

  double st[kNumStatSums];
#pragma unroll
  for (int s = 0; s < kNumStatSums; ++s) st[s] = 0.0;
  float dscale_acc[2] = {0.f, 0.f};  // lanes own j = lane, lane + 32

  const int num_tiles = ceil_div(live, kHeadRows);
  for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
    const int r0 = tile * kHeadRows;
    __syncthreads();  // previous tile done with f_s / out_s / dout_s (and staging done)
    for (int i = tid; i < kHeadRows * F; i += kHeadThreads) {
      const int r = i / F, k = i - r * F;
      f_s[(size_t)r * sp + k] = (r0 + r < live) ? p.f_pi[(size_t)(r0 + r) * F + k] : 0.f;
    }
    if (!shared) {
      for (int i = tid; i < kHeadRows * Fv; i += kHeadThreads) {
        const int r = i / Fv, k = i - r * Fv;
        fv_s[(size_t)r * sv + k] = (r0 + r < live) ? p.f_v[(size_t)(r0 + r) * Fv + k] : 0.f;
      }
    }
    __syncthreads();
    // Head outputs: out_s[r][j], j < A actor, j == A critic value.
    for (int o = tid; o < kHeadRows * (A + 1); o += kHeadThreads) {
      const int r = o / (A + 1), j = o - r * (A + 1);
      float acc;
      if (j < A) {
        const float* w = wT + (size_t)j * sp;
        const float* f = f_s + (size_t)r * sp;
        acc = w[F];
        for (int k = 0; k < F; ++k) acc = fmaf(f[k], w[k], acc);
      } else {
        const float* f = fv_s + (size_t)r * (shared ? sp : sv);
        acc = wTv[Fv];
        for (int k = 0; k < Fv; ++k) acc = fmaf(f[k], wTv[k], acc);
      }
      out_s[r * (A + 1) + j] = acc;
    }
    __syncthreads();
    // Loss and its gradient, one warp per row.
    for (int r = warp; r < kHeadRows; r += kHeadThreads / 32) {
      const int row = r0 + r;
      float* o = out_s + r * (A + 1);
      float* d = dout_s + r * (A + 1);
      if (row >= live) {
        for (int j = lane; j <= A; j += 32) d[j] = 0.f;
        continue;
      }
      const int flat = p.idx ? p.idx[row] : row;
      const float lp_old = p.lp_old[flat];
      const float adv = p.adv[flat];
      const float ret = p.ret[flat];
      const float v_old = p.v_old[flat];
      const float value = o[A];
      float lp, ent;
      // per-lane pieces for the gradient
      float pj[2] = {0.f, 0.f}, lpj[2] = {0.f, 0.f}, zj[2] = {0.f, 0.f};
      int action = 0;
      if (p.head == BT_HEAD_CATEGORICAL) {
        action = reinterpret_cast<const int*>(p.action)[flat];
        float mx = -INFINITY;
        for (int j = lane; j < A; j += 32) mx = fmaxf(mx, o[j]);
        mx = warp_max(mx);
        float se = 0.f;
        for (int j = lane; j < A; j += 32) se += expf(o[j] - mx);
        se = warp_sum(se);
        const float lse = logf(se);
        float h = 0.f;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int j = lane + 32 * q;
          if (j < A) {
            lpj[q] = (o[j] - mx) - lse;
            pj[q] = expf(lpj[q]);
            h -= pj[q] * lpj[q];
          }
        }
        ent = warp_sum(h);
        lp = (o[action] - mx) - lse;
      } else {
        const float* act = reinterpret_cast<const float*>(p.action) + (size_t)flat * A;
        float acc = 0.f;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int j = lane + 32 * q;
          if (j < A) {
            zj[q] = (act[j] - o[j]) * isig_s[j];
            acc += -0.5f * zj[q] * zj[q] - lsig_s[j] - 0.5f * kLog2Pi;
          }
        }
        lp = warp_sum(acc);
        float e = 0.f;
        for (int j = lane; j < A; j += 32) e += 0.5f + 0.5f * kLog2Pi + lsig_s[j];
        ent = warp_sum(e);
      }
      // Surrogate (ppo.py:90-103).
      const float eps = p.clip;
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
      const float g_lp = -((t1 * adv + t2 * adv * (dm * du)) * ratio) * p.inv_mb;
      const float g_ent = -p.ent_coef * p.inv_mb;
      // Value loss (ppo.py:105-115).
      const float c1 = 0.5f * ((value - ret) * (value - ret));
      float crit, dcrit;
      if (p.clip_value) {
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
      const float d_value = p.vf_coef * p.inv_mb * dcrit;
      // dL/d out
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int j = lane + 32 * q;
        if (j < A) {
          float g;
          if (p.head == BT_HEAD_CATEGORICAL) {
            g = g_lp * (((j == action) ? 1.f : 0.f) - pj[q]) + g_ent * (-pj[q] * (lpj[q] + ent));
          } else {
            g = g_lp * (zj[q] * isig_s[j]);
            dscale_acc[q] += g_lp * ((zj[q] * zj[q] - 1.f) * isig_s[j]) + g_ent * isig_s[j];
          }
          d[j] = g;
          p.d_out[(size_t)row * A + j] = g;
        }
      }
      if (lane == 0) {
        d[A] = d_value;
        p.d_val[row] = d_value;
        st[0] += (double)mn;
        st[1] += (double)ent;
        st[2] += (double)(lp_old - lp);
        st[3] += (fabsf(ratio - 1.f) > eps) ? 1.0 : 0.0;
        st[4] += (double)adv;
        st[5] += (double)crit;
        const double res = (double)ret - (double)value;
        st[6] += res;
        st[7] += res * res;
        st[8] += (double)ret;
        st[9] += (double)ret * (double)ret;
        st[10] += (double)value;
        st[11] += 1.0;
      }
    }
    __syncthreads();
    // dL/d f (times the last activation's derivative).
    for (int i = tid; i < kHeadRows * F; i += kHeadThreads) {
      const int r = i / F, k = i - r * F;
      const int row = r0 + r;
      if (row >= live) continue;
      const float* d = dout_s + r * (A + 1);
      float g = 0.f;
      for (int j = 0; j < A; ++j) g = fmaf(d[j], wT[(size_t)j * sp + k], g);
      if (shared) g = fmaf(d[A], wTv[k], g);
      const size_t gi = (size_t)row * F + k;
      if (p.act_pi != BT_ACT_NONE)
        g *= act_grad(p.pre_pi ? p.pre_pi[gi] : 0.f, p.post_pi ? p.post_pi[gi] : 0.f, p.act_pi);
      p.d_fpi[gi] = g;
    }
    if (!shared) {
      for (int i = tid; i < kHeadRows * Fv; i += kHeadThreads) {
        const int r = i / Fv, k = i - r * Fv;
        const int row = r0 + r;
        if (row >= live) continue;
        float g = dout_s[r * (A + 1) + A] * wTv[k];
        const size_t gi = (size_t)row * Fv + k;
        if (p.act_v != BT_ACT_NONE)
          g *= act_grad(p.pre_v ? p.pre_v[gi] : 0.f, p.post_v ? p.post_v[gi] : 0.f, p.act_v);
        p.d_fv[gi] = g;
      }
    }
  }

  // Block partial sums in a fixed order: warps' lane 0 -> shared -> thread 0.
  __syncthreads();
  if (lane == 0) {
    for (int s = 0; s < kNumStatSums; ++s) stat_s[warp * kNumStatSums + s] = st[s];
  }
  if (p.head == BT_HEAD_GAUSSIAN) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int j = lane + 32 * q;
      if (j < A) red_s[warp * A + j] = dscale_acc[q];
    }
  }
  __syncthreads();
  if (tid < kNumStatSums) {
    double s = 0.0;
    for (int w = 0; w < kHeadThreads / 32; ++w) s += stat_s[w * kNumStatSums + tid];
    p.stat_partials[(size_t)blockIdx.x * kNumStatSums + tid] = s;
  }
  if (p.head == BT_HEAD_GAUSSIAN && p.dscale_partials) {
    for (int j = tid; j < A; j += kHeadThreads) {
      float s = 0.f;
      for (int w = 0; w < kHeadThreads / 32; ++w) s += red_s[w * A + j];
      const float sc = p.scale[j];
      const float sgm = 1.f / (1.f + expf(-sc));  // d softplus / d scale
      p.dscale_partials[(size_t)blockIdx.x * A + j] = s * sgm;
    }
  }
}

int launch_heads_loss(const HeadsParams& p, int blocks, cudaStream_t stream) {
  const bool shared = p.f_v == p.f_pi;
  const size_t smem = heads_smem_bytes(p.F_pi, p.F_v, p.A, shared);
  BT_CHECK_ARG(p.A <= 64, "heads: action_dim %d > 64 is not supported", p.A);
  BT_CHECK_ARG(smem <= 227 * 1024, "heads: feature width too large for shared memory");
  BT_CUDA(cudaFuncSetAttribute(heads_loss_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem));
  heads_loss_kernel<<<blocks, kHeadThreads, smem, stream>>>(p);
  BT_LAUNCH_CHECK("heads_loss_kernel");
  return BT_OK;
}

// Head outputs only (bootstrap values, act): one warp per row.
__global__ void heads_forward_kernel(const float* f_pi, int F, const float* f_v, int Fv,
                                     const float* w_pi, const float* w_v, int A, int rows,
                                     float* out, float* value) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float* f = f_pi + (size_t)warp * F;
  if (out) {
    for (int j = 0; j < A; ++j) {
      float acc = 0.f;
      for (int k = lane; k < F; k += 32) acc = fmaf(f[k], w_pi[(size_t)k * A + j], acc);
      acc = warp_sum(acc);
      if (lane == 0) out[(size_t)warp * A + j] = acc + w_pi[(size_t)F * A + j];
    }
  }
  if (value) {
    const float* fv = f_v + (size_t)warp * Fv;
    float acc = 0.f;
    for (int k = lane; k < Fv; k += 32) acc = fmaf(fv[k], w_v[k], acc);
    acc = warp_sum(acc);
    if (lane == 0) value[warp] = acc + w_v[Fv];
  }
}

int launch_heads_forward(const float* f_pi, int F, const float* f_v, int Fv, const float* w_pi,
                         const float* w_v, int A, int rows, float* out, float* value,
                         cudaStream_t stream) {
  if (rows <= 0) return BT_OK;
  heads_forward_kernel<<<ceil_div(rows * 32, 256), 256, 0, stream>>>(f_pi, F, f_v, Fv, w_pi, w_v,
                                                                     A, rows, out, value);
  BT_LAUNCH_CHECK("heads_forward_kernel");
  return BT_OK;
}

}  // namespace bt

namespace bt {

// a14: action sampling of PPO.step (boonta/algorithms/ppo.py:57-74) for a row of head
// outputs. Categorical (boonta/networks/distributions.py:8-23): logits = out / temperature
// (greedy one-hot of argmax at temperature 0), normalised by log_softmax; the action is
// argmax(log_softmax(logits) + gumbel) with gumbel = -log(-log(u)). The noise and the
// log_softmax are evaluated in double and rounded once to float32, and the sum is a
// float32 add with the first index winning ties, so the index is a deterministic
// function of (logits, u): the CPU oracle reproduces it bit for bit.
// Gaussian: action = mean + temperature * sigma * noise, log-prob of that action.
__global__ void sample_kernel(const float* out, const float* scale, int head, int A, int rows,
                              const float* noise, float temperature, void* action,
                              float* log_prob) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const float* o = out + (size_t)r * A;
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
