// K1: generalized advantage estimation as a reverse time scan, one thread per env.
//
// Restates boonta/algorithms/advantage_estimators.py:8-56. Per env column n, going from
// t = T-1 down to 0 with carry (advantage = 0, next_value = bootstrap[n]):
//
//   delta     = rho * ((reward + (gamma * (1 - term)) * next_value) - value)
//   delta     = delta * (1 - trunc)
//   advantage = delta + (((gamma*lambda) * c) * (1 - term)) * (1 - trunc)) * advantage
//   returns   = advantage + value;  next_value = value
//
// evaluated in float32 with every product and sum rounded separately (no FMA
// contraction), the operation order of the reference expression, so the result is
// bit-identical to a non-fused float32 evaluation of it. gamma*lambda is formed in double
// and rounded once, as the reference does with its Python-float hyperparameters.
//
// Data layout: [T, N] row-major, so for a fixed t consecutive envs are consecutive in
// memory. The fast kernel gives each warp 32 env columns: one elected lane arms an
// mbarrier, the warp's lanes issue one bulk (TMA engine) copy per (t, array) row slice
// into shared memory — every load of the block is in flight at once — and after the
// barrier each lane scans its column from shared memory and writes A and R for all t with
// 128-byte coalesced stores. The HBM roofline bounds it: 18 bytes per env-step (reward 4,
// terminated 1, truncated 1, value 4 read; advantage 4, return 4 written) + 4 per env.
#include "common.cuh"
#include "ptx.cuh"

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
  int* err;      // nullable error word (set to 1 when a bounded wait gives up)
};

__device__ __forceinline__ float gae_step(float r, float v, float next_v, float term_b,
                                          float trunc_b, float rho, float c, float adv,
                                          float gamma, float glam) {
  const float term = __fsub_rn(1.f, term_b);
  const float trunc = __fsub_rn(1.f, trunc_b);
  float delta = __fmul_rn(__fmul_rn(gamma, term), next_v);
  delta = __fsub_rn(__fadd_rn(r, delta), v);
  delta = __fmul_rn(rho, delta);
  delta = __fmul_rn(delta, trunc);
  const float k = __fmul_rn(__fmul_rn(__fmul_rn(glam, c), term), trunc);
  return __fadd_rn(delta, __fmul_rn(k, adv));
}

// Plain path: any T, N, alignment. One thread per env, direct loads.
__global__ void gae_plain_kernel(GaeParams p) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= p.N) return;
  float adv = 0.f;
  float next_v = p.bootstrap[n];
  for (int t = p.T - 1; t >= 0; --t) {
    const size_t i = (size_t)t * p.N + n;
    const float v = p.value[i];
    const float rho = p.rho ? p.rho[i] : 1.f;
    const float c = p.c ? p.c[i] : 1.f;
    adv = gae_step(p.reward[i], v, next_v, (float)p.term[i], (float)p.trunc[i], rho, c, adv,
                   p.gamma, p.glam);
    p.adv[i] = adv;
    p.ret[i] = __fadd_rn(adv, v);
    next_v = v;
  }
}

constexpr int kGaeEnvs = 32;  // env columns per warp (block)

// Bulk path: N % 32 == 0 (so every u8 row slice is 32 bytes, 16-byte aligned), rho/c
// absent, T * 32 * 10 bytes of shared memory.
__global__ void __launch_bounds__(32) gae_bulk_kernel(GaeParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int T = p.T;
  float* r_s = reinterpret_cast<float*>(smem);             // [T][32]
  float* v_s = r_s + (size_t)T * kGaeEnvs;                 // [T][32]
  uint8_t* term_s = reinterpret_cast<uint8_t*>(v_s + (size_t)T * kGaeEnvs);  // [T][32]
  uint8_t* trunc_s = term_s + (size_t)T * kGaeEnvs;        // [T][32]
  __shared__ __align__(8) uint64_t bar;

  const int lane = threadIdx.x;
  const int n0 = blockIdx.x * kGaeEnvs;
  if (lane == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (lane == 0) mbar_arrive_expect_tx(&bar, (uint32_t)T * kGaeEnvs * 10u);
  __syncwarp();
  for (int t = lane; t < T; t += 32) {
    const size_t row = (size_t)t * p.N + n0;
    bulk_g2s(r_s + (size_t)t * kGaeEnvs, p.reward + row, kGaeEnvs * 4, &bar);
    bulk_g2s(v_s + (size_t)t * kGaeEnvs, p.value + row, kGaeEnvs * 4, &bar);
    bulk_g2s(term_s + (size_t)t * kGaeEnvs, p.term + row, kGaeEnvs, &bar);
    bulk_g2s(trunc_s + (size_t)t * kGaeEnvs, p.trunc + row, kGaeEnvs, &bar);
  }
  const float boot = p.bootstrap[n0 + lane];
  if (!mbar_wait_bounded(&bar, 0)) {
    // The copies did not land in time: report, poison this block's outputs, and leave
    // without touching shared memory again.
    if (lane == 0 && p.err) atomicExch(p.err, 1);
    for (int t = 0; t < T; ++t) {
      const size_t i = (size_t)t * p.N + n0 + lane;
      p.adv[i] = __int_as_float(0x7fc00000);
      p.ret[i] = __int_as_float(0x7fc00000);
    }
    return;
  }
  float adv = 0.f;
  float next_v = boot;
  for (int t = T - 1; t >= 0; --t) {
    const int s = t * kGaeEnvs + lane;
    const float v = v_s[s];
    adv = gae_step(r_s[s], v, next_v, (float)term_s[s], (float)trunc_s[s], 1.f, 1.f, adv,
                   p.gamma, p.glam);
    const size_t i = (size_t)t * p.N + n0 + lane;
    p.adv[i] = adv;
    p.ret[i] = __fadd_rn(adv, v);
    next_v = v;
  }
}

int launch_gae(const GaeParams& p, cudaStream_t stream) {
  if (p.T == 0 || p.N == 0) return BT_OK;
  const size_t smem = (size_t)p.T * kGaeEnvs * 10;
  const bool aligned =
      (p.N % kGaeEnvs == 0) && ((uintptr_t)p.reward % 16 == 0) &&
      ((uintptr_t)p.value % 16 == 0) && ((uintptr_t)p.term % 16 == 0) &&
      ((uintptr_t)p.trunc % 16 == 0);
  if (aligned && p.rho == nullptr && p.c == nullptr && smem <= 200 * 1024) {
    if (smem > 48 * 1024) {
      BT_CUDA(cudaFuncSetAttribute(gae_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)smem));
    }
    gae_bulk_kernel<<<p.N / kGaeEnvs, kGaeEnvs, smem, stream>>>(p);
    BT_LAUNCH_CHECK("gae_bulk_kernel");
  } else {
    gae_plain_kernel<<<ceil_div(p.N, 128), 128, 0, stream>>>(p);
    BT_LAUNCH_CHECK("gae_plain_kernel");
  }
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
