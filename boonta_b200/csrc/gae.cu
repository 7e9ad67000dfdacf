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
// memory. The fast kernel (gae_tile_kernel below) stages a block's env columns in shared
// memory with asynchronous 16-byte copies issued by all its threads and scans each column
// in one thread, writing A and R with coalesced stores. The HBM roofline bounds it: 18
// bytes per env-step (reward 4, terminated 1, truncated 1, value 4 read; advantage 4,
// return 4 written) + 4 per env.
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

__device__ __forceinline__ float gae_step(float r, float v, float next_v, float term_b,
                                          float trunc_b, float rho, float c, float adv,
                                          float gamma, float glam) {
  float delta, k;
  gae_delta(r, v, next_v, term_b, trunc_b, rho, c, gamma, glam, delta, k);
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

// Tiled path: a block owns NE env columns (NE = 16 or 32) for all T. Every thread of the
// block issues 16-byte asynchronous copies (cp.async, no registers held) of its share of
// the block's reward/value/flag rows into shared memory, in four commit groups that cover
// the time steps from the last one down (the order the scan consumes them); every byte of
// the block is requested before the first wait. The block then waits group by group
// (cp.async.wait_group + a block barrier) and warp 0 scans each quarter while the later
// quarters are still arriving. One thread per column does the scan, so its arithmetic is
// the sequential reference order. Requires N % NE == 0, 16-byte aligned arrays and
// T * NE * 10 bytes of shared memory within kGaeMaxSmem.
constexpr int kGaeGroups = 4;
constexpr size_t kGaeMaxSmem = 200 * 1024;
constexpr int kGaeBatch = 16;  // steps whose inputs are moved to registers at once

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// Wait until at most `pending` of this thread's most recent commit groups are in flight.
__device__ __forceinline__ void cp_async_wait_pending(int pending) {
  switch (pending) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
  }
}

// kGaeBatch steps t = tb - 1 down to tb - kGaeBatch of one column, in three passes so that
// only the carry (one multiply and one add per step) is serial: inputs to registers, the
// carry-independent terms of every step, the carry, then the stores. (Loading first also
// keeps the shared loads clear of the output stores, which go through generic pointers the
// compiler must assume may alias shared memory.)
template <int NE>
__device__ __forceinline__ void gae_scan_batch(const GaeParams& p, const float* r_s,
                                               const float* v_s, const uint8_t* term_s,
                                               const uint8_t* trunc_s, int tb, int n0, int lane,
                                               bool on, float& adv, float& next_v) {
  float rr[kGaeBatch], vv[kGaeBatch], tm[kGaeBatch], tr[kGaeBatch];
#pragma unroll
  for (int k = 0; k < kGaeBatch; ++k) {
    const int s = (tb - 1 - k) * NE + lane;
    rr[k] = r_s[s];
    vv[k] = v_s[s];
    tm[k] = (float)term_s[s];
    tr[k] = (float)trunc_s[s];
  }
  float dl[kGaeBatch], kk[kGaeBatch];
#pragma unroll
  for (int k = 0; k < kGaeBatch; ++k)
    gae_delta(rr[k], vv[k], k == 0 ? next_v : vv[k - 1], tm[k], tr[k], 1.f, 1.f, p.gamma,
              p.glam, dl[k], kk[k]);
#pragma unroll
  for (int k = 0; k < kGaeBatch; ++k) {
    adv = __fadd_rn(dl[k], __fmul_rn(kk[k], adv));
    rr[k] = adv;  // the step's advantage, in place of its reward
  }
  next_v = vv[kGaeBatch - 1];
  if (on) {
    float* pa = p.adv + (size_t)(tb - 1) * p.N + n0 + lane;
    float* pr = p.ret + (size_t)(tb - 1) * p.N + n0 + lane;
#pragma unroll
    for (int k = 0; k < kGaeBatch; ++k) {
      pa[-(ptrdiff_t)k * p.N] = rr[k];
      pr[-(ptrdiff_t)k * p.N] = __fadd_rn(rr[k], vv[k]);
    }
  }
}

template <int NE>
__global__ void __launch_bounds__(NE * 8) gae_tile_kernel(GaeParams p) {
  constexpr int kThreads = NE * 8;
  constexpr int kF = NE / 4, kB = NE / 16;    // 16-byte pieces per row: floats, flags
  constexpr int kRow = 2 * kF + 2 * kB;
  extern __shared__ __align__(128) uint8_t smem[];
  const int T = p.T;
  const int C = (T + kGaeGroups - 1) / kGaeGroups;  // steps per group
  float* r_s = reinterpret_cast<float*>(smem);                 // [T][NE]
  float* v_s = r_s + (size_t)T * NE;                           // [T][NE]
  uint8_t* term_s = reinterpret_cast<uint8_t*>(v_s + (size_t)T * NE);  // [T][NE]
  uint8_t* trunc_s = term_s + (size_t)T * NE;                  // [T][NE]
  const int tid = threadIdx.x;
  const int n0 = blockIdx.x * NE;

  for (int g = 0; g < kGaeGroups; ++g) {  // group g: t in [t_lo, t_hi), latest steps first
    const int t_hi = max(T - g * C, 0);
    const int t_lo = max(t_hi - C, 0);
    const int pieces = (t_hi - t_lo) * kRow;
    for (int i = tid; i < pieces; i += kThreads) {
      const int t = t_lo + i / kRow;
      int j = i - (t - t_lo) * kRow;
      const size_t row = (size_t)t * p.N + n0;
      const int s = t * NE;
      if (j < kF) {
        cp_async16(r_s + s + 4 * j, p.reward + row + 4 * j);
      } else if ((j -= kF) < kF) {
        cp_async16(v_s + s + 4 * j, p.value + row + 4 * j);
      } else if ((j -= kF) < kB) {
        cp_async16(term_s + s + 16 * j, p.term + row + 16 * j);
      } else {
        j -= kB;
        cp_async16(trunc_s + s + 16 * j, p.trunc + row + 16 * j);
      }
    }
    cp_async_commit();  // possibly empty; every thread commits the same four groups
  }

  // Warp 0 scans, all 32 lanes together; with NE = 16, lanes 16..31 shadow lanes 0..15 and
  // store nothing.
  const bool scan = tid < 32;
  const bool on = tid < NE;
  const int lane = tid & (NE - 1);
  float adv = 0.f;
  float next_v = scan ? p.bootstrap[n0 + lane] : 0.f;
  for (int g = 0; g < kGaeGroups; ++g) {
    cp_async_wait_pending(kGaeGroups - 1 - g);
    __syncthreads();  // every thread's copies of group g have landed
    if (!scan) continue;
    const int t_hi = max(T - g * C, 0);
    const int t_lo = max(t_hi - C, 0);
    int tb = t_hi;
    for (; tb - kGaeBatch >= t_lo; tb -= kGaeBatch)
      gae_scan_batch<NE>(p, r_s, v_s, term_s, trunc_s, tb, n0, lane, on, adv, next_v);
    for (; tb > t_lo; --tb) {  // the remainder of a group, one step at a time
      const int s = (tb - 1) * NE + lane;
      const float v = v_s[s];
      adv = gae_step(r_s[s], v, next_v, (float)term_s[s], (float)trunc_s[s], 1.f, 1.f, adv,
                     p.gamma, p.glam);
      if (on) {
        const size_t i = (size_t)(tb - 1) * p.N + n0 + lane;
        p.adv[i] = adv;
        p.ret[i] = __fadd_rn(adv, v);
      }
      next_v = v;
    }
  }
}

template <int NE>
int launch_gae_tile(const GaeParams& p, cudaStream_t stream) {
  const size_t smem = (size_t)p.T * NE * 10;
  if (smem > 48 * 1024) {
    BT_CUDA(cudaFuncSetAttribute(gae_tile_kernel<NE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem));
  }
  gae_tile_kernel<NE><<<p.N / NE, NE * 8, smem, stream>>>(p);
  BT_LAUNCH_CHECK("gae_tile_kernel");
  return BT_OK;
}

int launch_gae(const GaeParams& p, cudaStream_t stream) {
  if (p.T == 0 || p.N == 0) return BT_OK;
  const bool aligned =
      ((uintptr_t)p.reward % 16 == 0) && ((uintptr_t)p.value % 16 == 0) &&
      ((uintptr_t)p.term % 16 == 0) && ((uintptr_t)p.trunc % 16 == 0);
  const bool tiled = aligned && p.rho == nullptr && p.c == nullptr;
  // 32 columns per block when that still gives about two blocks per SM, else 16.
  if (tiled && p.N % 32 == 0 && p.N / 32 >= 2 * kNumSMs && (size_t)p.T * 320 <= kGaeMaxSmem)
    return launch_gae_tile<32>(p, stream);
  if (tiled && p.N % 16 == 0 && (size_t)p.T * 160 <= kGaeMaxSmem)
    return launch_gae_tile<16>(p, stream);
  gae_plain_kernel<<<ceil_div(p.N, 128), 128, 0, stream>>>(p);
  BT_LAUNCH_CHECK("gae_plain_kernel");
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
