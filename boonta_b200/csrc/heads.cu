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

constexpr int kHeadThreads = 256;
constexpr int kHeadWarps = kHeadThreads / 32;
constexpr int kMaxChunks = 4;  // float4 chunks per lane: feature widths up to 512
constexpr float kLog2Pi = 1.8378770664093453f;

// Shared memory: transposed head kernels wT[j][k] (actor rows j < A, then the critic row),
// the biases, per-warp head outputs / output gradients, gaussian constants, reductions.
size_t heads_smem_bytes(int F_pi, int F_v, int A, bool /*shared*/) {
  size_t floats = (size_t)A * F_pi + F_v + (A + 1);  // wT, wTv, biases
  floats += 2 * (size_t)kHeadWarps * (A + 1);         // out / dout per warp
  floats += 3 * (size_t)A;                            // sigma, 1/sigma, log sigma
  floats += (size_t)kHeadWarps * A;                   // dscale reduction
  return floats * 4 + (size_t)kHeadWarps * kNumStatSums * 8 + 64;
}

template <int A>
__device__ __forceinline__ float4 act4(float4 z) {
  return make_float4(act_fwd<A>(z.x), act_fwd<A>(z.y), act_fwd<A>(z.z), act_fwd<A>(z.w));
}

// f = act(pre) for all of a lane's chunks, the activation resolved once.
__device__ __forceinline__ void act_row(const float4 (&z)[kMaxChunks], int act,
                                        float4 (&f)[kMaxChunks]) {
  with_act(act, [&](auto tag) {
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i) f[i] = act4<decltype(tag)::value>(z[i]);
  });
}

__device__ __forceinline__ void load_row(const float* src, int F, int lane, float4 (&v)[kMaxChunks]) {
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int q = lane + 32 * i;
    v[i] = (4 * q < F) ? __ldg(reinterpret_cast<const float4*>(src) + q) : make_float4(0, 0, 0, 0);
  }
}

__device__ __forceinline__ float dot_row(const float4 (&f)[kMaxChunks], const float* w, int F,
                                         int lane) {
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int q = lane + 32 * i;
    if (4 * q < F) {
      const float4 ww = reinterpret_cast<const float4*>(w)[q];
      acc = fmaf(f[i].x, ww.x, acc);
      acc = fmaf(f[i].y, ww.y, acc);
      acc = fmaf(f[i].z, ww.z, acc);
      acc = fmaf(f[i].w, ww.w, acc);
    }
  }
  return warp_sum(acc);
}

// dL/d f for the lane's chunks, times the tower's last activation derivative, stored as
// fp32 or bf16 (hi/lo) at row `row`.
__device__ __forceinline__ void store_df(float4 g, const float4& pre, int act, size_t base, int q,
                                         float* df, __nv_bfloat16* dfb, __nv_bfloat16* dfb_lo) {
  with_act(act, [&](auto tag) {
    constexpr int A = decltype(tag)::value;
    g.x *= act_dz<A>(pre.x);
    g.y *= act_dz<A>(pre.y);
    g.z *= act_dz<A>(pre.z);
    g.w *= act_dz<A>(pre.w);
  });
  const size_t i = base + 4 * (size_t)q;
  if (dfb) {
    store_bf16(dfb, dfb_lo, i, g.x);
    store_bf16(dfb, dfb_lo, i + 1, g.y);
    store_bf16(dfb, dfb_lo, i + 2, g.z);
    store_bf16(dfb, dfb_lo, i + 3, g.w);
  } else {
    *reinterpret_cast<float4*>(df + i) = g;
  }
}

// One warp per row (grid-stride over the minibatch rows). All loads of a row — the
// features of both towers and the pre-activations behind the activation derivative — are
// issued together as float4s before any arithmetic.
__global__ void __launch_bounds__(kHeadThreads) heads_loss_kernel(HeadsParams p) {
  extern __shared__ __align__(16) float sm[];
  const int A = p.A;
  const bool shared = (p.f_v == p.f_pi);
  const int F = p.F_pi, Fv = p.F_v;
  float* wT = sm;                          // [A][F]
  float* wTv = wT + (size_t)A * F;         // [Fv]
  float* bias = wTv + Fv;                  // [A + 1] (actor biases, critic bias)
  float* out_s = bias + (A + 1);           // [warps][A + 1]
  float* dout_s = out_s + kHeadWarps * (A + 1);
  float* sig_s = dout_s + kHeadWarps * (A + 1);
  float* isig_s = sig_s + A;
  float* lsig_s = isig_s + A;
  float* red_s = lsig_s + A;               // [warps][A]
  double* stat_s = reinterpret_cast<double*>(
      (reinterpret_cast<uintptr_t>(red_s + kHeadWarps * A) + 7) & ~uintptr_t(7));

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int live = live_rows(p.count, p.rows);

  for (int i = tid; i < F * A; i += kHeadThreads) {
    const int k = i / A, j = i - k * A;
    wT[(size_t)j * F + k] = p.w_pi[i];
  }
  for (int k = tid; k < Fv; k += kHeadThreads) wTv[k] = p.w_v[k];
  for (int j = tid; j < A; j += kHeadThreads) bias[j] = p.w_pi[(size_t)F * A + j];
  if (tid == 0) bias[A] = p.w_v[Fv];
  if (p.head == BT_HEAD_GAUSSIAN) {
    for (int j = tid; j < A; j += kHeadThreads) {
      const float s = p.scale[j];
      const float sig = (fmaxf(s, 0.f) + log1pf(expf(-fabsf(s)))) + 1e-3f;  // softplus + 1e-3
      sig_s[j] = sig;
      isig_s[j] = 1.f / sig;
      lsig_s[j] = logf(sig);
    }
  }
  __syncthreads();

  double st[kNumStatSums];
#pragma unroll
  for (int s = 0; s < kNumStatSums; ++s) st[s] = 0.0;
  float dscale_acc[2] = {0.f, 0.f};  // lanes own j = lane, lane + 32
  float* o = out_s + warp * (A + 1);
  float* d = dout_s + warp * (A + 1);

  for (int row = blockIdx.x * kHeadWarps + warp; row < live; row += gridDim.x * kHeadWarps) {
    const int flat = p.idx ? p.idx[row] : row;
    // the towers' pre-activations; the head input is act(pre), recomputed here
    float4 f[kMaxChunks], fv[kMaxChunks], zp[kMaxChunks], zv[kMaxChunks];
    load_row(p.f_pi + (size_t)row * F, F, lane, zp);
    if (!shared) load_row(p.f_v + (size_t)row * Fv, Fv, lane, zv);
    act_row(zp, p.act_pi, f);
    if (!shared) act_row(zv, p.act_v, fv);
    const float lp_old = p.lp_old[flat];
    const float adv = p.adv[flat];
    const float ret = p.ret[flat];
    const float v_old = p.v_old[flat];
    int action = 0;
    if (p.head == BT_HEAD_CATEGORICAL) action = reinterpret_cast<const int*>(p.action)[flat];
    float act_j[2] = {0.f, 0.f};
    if (p.head == BT_HEAD_GAUSSIAN) {
      const float* av = reinterpret_cast<const float*>(p.action) + (size_t)flat * A;
      if (lane < A) act_j[0] = av[lane];
      if (lane + 32 < A) act_j[1] = av[lane + 32];
    }
    // Head outputs.
    for (int j = 0; j < A; ++j) {
      const float t = dot_row(f, wT + (size_t)j * F, F, lane);
      if (lane == 0) o[j] = t + bias[j];
    }
    {
      const float t = shared ? dot_row(f, wTv, F, lane) : dot_row(fv, wTv, Fv, lane);
      if (lane == 0) o[A] = t + bias[A];
    }
    __syncwarp();
    const float value = o[A];
    float lp, ent;
    float pj[2] = {0.f, 0.f}, lpj[2] = {0.f, 0.f}, zj[2] = {0.f, 0.f};
    if (p.head == BT_HEAD_CATEGORICAL) {
      float mx = -INFINITY;
      for (int j = lane; j < A; j += 32) mx = fmaxf(mx, o[j]);
      mx = warp_max(mx);
      float se = 0.f;
      for (int j = lane; j < A; j += 32) se += expf(o[j] - mx);
      se = warp_sum(se);
      const float lse = logf(se);
      float h = 0.f;
#pragma unroll
      for (int qq = 0; qq < 2; ++qq) {
        const int j = lane + 32 * qq;
        if (j < A) {
          lpj[qq] = (o[j] - mx) - lse;
          pj[qq] = expf(lpj[qq]);
          h -= pj[qq] * lpj[qq];
        }
      }
      ent = warp_sum(h);
      lp = (o[action] - mx) - lse;
    } else {
      float acc = 0.f, e = 0.f;
#pragma unroll
      for (int qq = 0; qq < 2; ++qq) {
        const int j = lane + 32 * qq;
        if (j < A) {
          zj[qq] = (act_j[qq] - o[j]) * isig_s[j];
          acc += -0.5f * zj[qq] * zj[qq] - lsig_s[j] - 0.5f * kLog2Pi;
          e += 0.5f + 0.5f * kLog2Pi + lsig_s[j];
        }
      }
      lp = warp_sum(acc);
      ent = warp_sum(e);
    }
    // Surrogate (ppo.py:90-103), with JAX's balanced tie rule for min/max/clip.
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
#pragma unroll
    for (int qq = 0; qq < 2; ++qq) {
      const int j = lane + 32 * qq;
      if (j < A) {
        float g;
        if (p.head == BT_HEAD_CATEGORICAL) {
          g = g_lp * (((j == action) ? 1.f : 0.f) - pj[qq]) + g_ent * (-pj[qq] * (lpj[qq] + ent));
        } else {
          g = g_lp * (zj[qq] * isig_s[j]);
          dscale_acc[qq] += g_lp * ((zj[qq] * zj[qq] - 1.f) * isig_s[j]) + g_ent * isig_s[j];
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
    __syncwarp();
    // dL/d f = d_out W_pi^T (+ d_value w_v^T when shared), times act'.
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i) {
      const int q = lane + 32 * i;
      if (4 * q >= F) continue;
      float4 g = make_float4(0, 0, 0, 0);
      for (int j = 0; j < A; ++j) {
        const float dj = d[j];
        const float4 w = reinterpret_cast<const float4*>(wT + (size_t)j * F)[q];
        g.x = fmaf(dj, w.x, g.x);
        g.y = fmaf(dj, w.y, g.y);
        g.z = fmaf(dj, w.z, g.z);
        g.w = fmaf(dj, w.w, g.w);
      }
      if (shared) {
        const float4 w = reinterpret_cast<const float4*>(wTv)[q];
        g.x = fmaf(d[A], w.x, g.x);
        g.y = fmaf(d[A], w.y, g.y);
        g.z = fmaf(d[A], w.z, g.z);
        g.w = fmaf(d[A], w.w, g.w);
      }
      store_df(g, zp[i], p.act_pi, (size_t)row * F, q, p.d_fpi, p.d_fpi_b, p.d_fpi_b_lo);
    }
    if (!shared) {
#pragma unroll
      for (int i = 0; i < kMaxChunks; ++i) {
        const int q = lane + 32 * i;
        if (4 * q >= Fv) continue;
        const float4 w = reinterpret_cast<const float4*>(wTv)[q];
        const float4 g = make_float4(d[A] * w.x, d[A] * w.y, d[A] * w.z, d[A] * w.w);
        store_df(g, zv[i], p.act_v, (size_t)row * Fv, q, p.d_fv, p.d_fv_b, p.d_fv_b_lo);
      }
    }
    __syncwarp();
  }

  // Block partial sums in a fixed order: warps' lane 0 -> shared -> thread 0.
  if (lane == 0) {
    for (int s = 0; s < kNumStatSums; ++s) stat_s[warp * kNumStatSums + s] = st[s];
  }
  if (p.head == BT_HEAD_GAUSSIAN) {
#pragma unroll
    for (int qq = 0; qq < 2; ++qq) {
      const int j = lane + 32 * qq;
      if (j < A) red_s[warp * A + j] = dscale_acc[qq];
    }
  }
  __syncthreads();
  if (tid < kNumStatSums) {
    double s = 0.0;
    for (int w = 0; w < kHeadWarps; ++w) s += stat_s[w * kNumStatSums + tid];
    p.stat_partials[(size_t)blockIdx.x * kNumStatSums + tid] = s;
  }
  if (p.head == BT_HEAD_GAUSSIAN && p.dscale_partials) {
    for (int j = tid; j < A; j += kHeadThreads) {
      float s = 0.f;
      for (int w = 0; w < kHeadWarps; ++w) s += red_s[w * A + j];
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
  BT_CHECK_ARG(p.F_pi % 4 == 0 && p.F_v % 4 == 0 && p.F_pi <= 4 * 32 * kMaxChunks &&
                   p.F_v <= 4 * 32 * kMaxChunks,
               "heads: feature widths %d / %d must be multiples of 4 and at most %d", p.F_pi,
               p.F_v, 4 * 32 * kMaxChunks);
  BT_CHECK_ARG(smem <= 227 * 1024, "heads: feature width too large for shared memory");
  if (smem > 48 * 1024) {
    static size_t configured = 0;
    if (smem > configured) {
      BT_CUDA(cudaFuncSetAttribute(heads_loss_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)smem));
      configured = smem;
    }
  }
  heads_loss_kernel<<<blocks, kHeadThreads, smem, stream>>>(p);
  BT_LAUNCH_CHECK("heads_loss_kernel");
  return BT_OK;
}

// Head outputs only (bootstrap values, act): one warp per row; the head input is act(f).
__global__ void heads_forward_kernel(const float* f_pi, int F, const float* f_v, int Fv,
                                     const float* w_pi, const float* w_v, int A, int rows,
                                     int act_pi, int act_v, float* out, float* value) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float* f = f_pi + (size_t)warp * F;
  if (out) {
    for (int j = 0; j < A; ++j) {
      float acc = 0.f;
      for (int k = lane; k < F; k += 32)
        acc = fmaf(act_forward(f[k], act_pi), w_pi[(size_t)k * A + j], acc);
      acc = warp_sum(acc);
      if (lane == 0) out[(size_t)warp * A + j] = acc + w_pi[(size_t)F * A + j];
    }
  }
  if (value) {
    const float* fv = f_v + (size_t)warp * Fv;
    float acc = 0.f;
    for (int k = lane; k < Fv; k += 32) acc = fmaf(act_forward(fv[k], act_v), w_v[k], acc);
    acc = warp_sum(acc);
    if (lane == 0) value[warp] = acc + w_v[Fv];
  }
}

int launch_heads_forward(const float* f_pi, int F, const float* f_v, int Fv, const float* w_pi,
                         const float* w_v, int A, int rows, int act_pi, int act_v, float* out,
                         float* value, cudaStream_t stream) {
  if (rows <= 0) return BT_OK;
  heads_forward_kernel<<<ceil_div(rows * 32, 256), 256, 0, stream>>>(
      f_pi, F, f_v, Fv, w_pi, w_v, A, rows, act_pi, act_v, out, value);
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
