// K1: generalized advantage estimation as a time-parallel (chunked affine) reverse scan.
//
// Restates boonta/algorithms/advantage_estimators.py:8-56. Per env column n, going from
// t = T-1 down to 0 with carry (advantage = 0, next_value = bootstrap[n]):
//
//   delta     = rho * ((reward + (gamma * (1 - term)) * next_value) - value)
//   delta     = delta * (1 - trunc)
//   advantage = delta + (((gamma*lambda) * c) * (1 - term)) * (1 - trunc)) * advantage
//   returns   = advantage + value;  next_value = value
//
// evaluated in float32 with every product and sum rounded separately (no FMA contraction), in
// the operation order of the reference expression; gamma*lambda is formed in double and
// rounded once, as the reference does with its Python-float hyperparameters. The scan over t
// runs in chunks (gae_chunked_kernel below), so the advantages are composed in a different
// order from the reference's step-by-step one.
//
// Data layout: [T, N] row-major, so for a fixed t consecutive envs are consecutive in memory.
// The HBM roofline bounds it: 18 bytes per env-step (reward 4, terminated 1, truncated 1,
// value 4 read; advantage 4, return 4 written) + 4 per env.
#include "common.cuh"

namespace bt {

struct GaeParams {
  const float* reward;
  const uint8_t* term;
  const uint8_t* trunc;
  const float* value;
  const float* bootstrap;
  const float* rho;  // nullable: 1.0
  const float* c;    // nullable: 1.0
  float* adv;
  float* ret;
  int T, N;
  float gamma;   // float32(gamma)
  float glam;    // float32(gamma * lambda), product formed in double
  int* err;      // nullable error word of the learner (no GAE kernel waits on anything)
};

// The step splits into the part that does not depend on the carried advantage (delta and
// the carry factor k) and the carry itself, advantage = delta + k * advantage.
__device__ __forceinline__ void gae_delta(float r, float v, float next_v, float term_b,
                                          float trunc_b, float rho, float c, float gamma,
                                          float glam, float& delta_out, float& k_out) {
  const float term = __fsub_rn(1.f, term_b);
  const float trunc = __fsub_rn(1.f, trunc_b);
  float delta = __fmul_rn(__fmul_rn(gamma, term), next_v);
  delta = __fsub_rn(__fadd_rn(r, delta), v);
  delta = __fmul_rn(rho, delta);
  delta_out = __fmul_rn(delta, trunc);
  k_out = __fmul_rn(__fmul_rn(__fmul_rn(glam, c), term), trunc);
}

// Time-parallel path. The step is affine in the carried advantage, A_t = delta_t + k_t A_{t+1},
// with delta_t and k_t independent of the carry (gae_delta), and affine maps compose
// associatively. A block owns 32 env columns (lane = column: every load and store is one
// coalesced row segment per warp) and splits the T steps into kGaeChunks chunks, one per warp.
// Each warp folds its chunk, from its last step down to its first, into the map
// A_first = M * A_entering + C (products and sums rounded separately, from a zero carry), the
// maps meet in shared memory, each warp composes the maps of the later chunks (latest first)
// onto the zero advantage past the last step, and rescans its chunk from that carry, storing A
// and R = A + V. oracle/gae.py `gae_chunked` restates this order bit for bit; against the
// reference's sequential order the results differ by a few float32 ulps of A (parity bound
// 1e-5 relative).
constexpr int kGaeChunks = 8;

__device__ __forceinline__ void gae_terms(const GaeParams& p, int t, int n, float& delta,
                                          float& k, float& v) {
  const size_t i = (size_t)t * p.N + n;
  v = p.value[i];
  const float next_v = t + 1 < p.T ? p.value[i + p.N] : p.bootstrap[n];
  gae_delta(p.reward[i], v, next_v, (float)p.term[i], (float)p.trunc[i], p.rho ? p.rho[i] : 1.f,
            p.c ? p.c[i] : 1.f, p.gamma, p.glam, delta, k);
}

// KEEP > 0: chunks of at most KEEP steps, whose inputs are all loaded up front (clamped indices,
// no per-step conditions, so every load is in flight at once) and kept in registers between the
// passes; KEEP = 0: any chunk length, inputs read again in the second pass.
template <int KEEP>
__global__ void __launch_bounds__(32 * kGaeChunks) gae_chunked_kernel(GaeParams p, int chunk) {
  __shared__ float m_s[kGaeChunks][32], c_s[kGaeChunks][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int n = blockIdx.x * 32 + lane;
  const bool col = n < p.N;
  const int t0 = min(p.T, w * chunk), t1 = min(p.T, t0 + chunk);
  constexpr int K = KEEP > 0 ? KEEP : 1;
  float dl[K], kk[K], vv[K];
  float M = 1.f, C = 0.f;
  if (col && KEEP > 0) {
    float rr[K], tm[K], tr[K], ro[K], cw[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const size_t i = (size_t)min(t0 + j, p.T - 1) * p.N + n;
      rr[j] = p.reward[i];
      vv[j] = p.value[i];
      tm[j] = (float)p.term[i];
      tr[j] = (float)p.trunc[i];
      ro[j] = p.rho ? p.rho[i] : 1.f;
      cw[j] = p.c ? p.c[i] : 1.f;
    }
    const float v_end = t1 < p.T ? p.value[(size_t)t1 * p.N + n] : p.bootstrap[n];
#pragma unroll
    for (int j = 0; j < K; ++j)
      gae_delta(rr[j], vv[j], (j + 1 < t1 - t0) ? vv[j + 1 < K ? j + 1 : j] : v_end, tm[j], tr[j],
                ro[j], cw[j], p.gamma, p.glam, dl[j], kk[j]);
#pragma unroll
    for (int j = K - 1; j >= 0; --j) {
      if (t0 + j < t1) {
        C = __fadd_rn(dl[j], __fmul_rn(kk[j], C));
        M = __fmul_rn(kk[j], M);
      }
    }
  } else if (col) {
    for (int t = t1 - 1; t >= t0; --t) {
      float d, k, v;
      gae_terms(p, t, n, d, k, v);
      C = __fadd_rn(d, __fmul_rn(k, C));
      M = __fmul_rn(k, M);
    }
  }
  m_s[w][lane] = M;
  c_s[w][lane] = C;
  __syncthreads();
  if (!col) return;
  float adv = 0.f;  // the advantage past the last step
  for (int c = kGaeChunks - 1; c > w; --c) adv = __fadd_rn(__fmul_rn(m_s[c][lane], adv), c_s[c][lane]);
  if (KEEP > 0) {
#pragma unroll
    for (int j = K - 1; j >= 0; --j) {
      if (t0 + j < t1) {
        adv = __fadd_rn(dl[j], __fmul_rn(kk[j], adv));
        const size_t i = (size_t)(t0 + j) * p.N + n;
        p.adv[i] = adv;
        p.ret[i] = __fadd_rn(adv, vv[j]);
      }
    }
  } else {
    for (int t = t1 - 1; t >= t0; --t) {
      float d, k, v;
      gae_terms(p, t, n, d, k, v);
      adv = __fadd_rn(d, __fmul_rn(k, adv));
      const size_t i = (size_t)t * p.N + n;
      p.adv[i] = adv;
      p.ret[i] = __fadd_rn(adv, v);
    }
  }
}

int launch_gae(const GaeParams& p, cudaStream_t stream) {
  if (p.T == 0 || p.N == 0) return BT_OK;
  const int chunk = ceil_div(p.T, kGaeChunks);
  const dim3 grid(ceil_div(p.N, 32)), block(32 * kGaeChunks);
  if (chunk <= 4) gae_chunked_kernel<4><<<grid, block, 0, stream>>>(p, chunk);
  else if (chunk <= 8) gae_chunked_kernel<8><<<grid, block, 0, stream>>>(p, chunk);
  else if (chunk <= 16) gae_chunked_kernel<16><<<grid, block, 0, stream>>>(p, chunk);
  else gae_chunked_kernel<0><<<grid, block, 0, stream>>>(p, chunk);
  BT_LAUNCH_CHECK("gae_chunked_kernel");
  return BT_OK;
}

GaeParams make_gae_params(const float* reward, const uint8_t* terminated,
                          const uint8_t* truncated, const float* values, const float* bootstrap,
                          const float* rho, const float* c, int T, int N, double gamma,
                          double lam, float* adv, float* ret, int* err) {
  GaeParams p;
  p.reward = reward;
  p.term = terminated;
  p.trunc = truncated;
  p.value = values;
  p.bootstrap = bootstrap;
  p.rho = rho;
  p.c = c;
  p.adv = adv;
  p.ret = ret;
  p.T = T;
  p.N = N;
  p.gamma = (float)gamma;
  p.glam = (float)(gamma * lam);
  p.err = err;
  return p;
}

}  // namespace bt

extern "C" int bt_gae(const float* reward, const uint8_t* terminated, const uint8_t* truncated,
                      const float* values, const float* bootstrap, const float* rho,
                      const float* c, int32_t num_steps, int32_t num_envs, double gamma,
                      double gae_lambda, float* advantages, float* returns, void* stream) {
  BT_CHECK_ARG(num_steps >= 0 && num_envs >= 0, "bt_gae: negative shape (%d, %d)", num_steps,
               num_envs);
  if (num_steps == 0 || num_envs == 0) return BT_OK;
  BT_CHECK_ARG(reward && terminated && truncated && values && bootstrap && advantages && returns,
               "bt_gae: null pointer");
  bt::GaeParams p = bt::make_gae_params(reward, terminated, truncated, values, bootstrap, rho, c,
                                        num_steps, num_envs, gamma, gae_lambda, advantages,
                                        returns, nullptr);
  return bt::launch_gae(p, (cudaStream_t)stream);
}

namespace bt {
int launch_gae_internal(const float* reward, const uint8_t* term, const uint8_t* trunc,
                        const float* values, const float* bootstrap, int T, int N, double gamma,
                        double lam, float* adv, float* ret, int* err, cudaStream_t stream) {
  GaeParams p = make_gae_params(reward, term, trunc, values, bootstrap, nullptr, nullptr, T, N,
                                gamma, lam, adv, ret, err);
  return launch_gae(p, stream);
}
}  // namespace bt
