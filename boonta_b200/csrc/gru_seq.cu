// K15 as one launch per sequence: the GRU recurrence of a minibatch of env sequences
// (flax GRUCell scanned over time, reset to zero on first.done; boonta/networks/blocks/rnn.py
// :30-59, boonta/algorithms/recurrent_ppo.py:211-223) and its backward through time, each
// as a persistent kernel that walks the T steps with a grid-wide barrier between them,
// instead of two launches (a GEMM and an elementwise kernel) per step.
//
// Work split (both directions): CTA (eb, ub) owns envs [32 eb, 32 eb + 32) of the minibatch
// and hidden units [16 ub, 16 ub + 16); its 256 threads each own two envs x one unit for
// the gate math, so the three gates of a unit (r, z, n) meet in one thread. The CTA keeps
// its slice of W_h in shared memory for the whole sequence.
//
//   forward step t   stage the 32 carry rows hin_t (all H) from L2; hp = hin_t W_h for the
//                    CTA's 48 gate columns (fp32 FMA); gates, h_t, the saved r, z, n,
//                    h W_hn + b_hn; hin_{t+1} = reset ? 0 : h_t; barrier
//   backward step t  gate gradients of the CTA's (env, unit) pairs from dL/dh_t (heads) and
//                    the carry gradient kept in registers; dxp_t, dhp_t written; barrier;
//                    stage the 32 dhp_t rows (all 3H); carry = reset ? 0 : dh z + dhp_t W_h^T
//
// The arithmetic is fp32 with the same gate formulas as the per-step kernels in
// recurrent.cu; only the summation order of the products differs.
//
// The barrier: thread 0 of every CTA adds one to a device counter (zeroed before the launch)
// and spins until it reaches (step + 1) * CTAs. All CTAs must be resident at once: the host
// launches at most one CTA per SM with an occupancy check, and the spin is bounded (2 s of
// %globaltimer), after which the CTA records kErrGruBarrier in the learner's error word
// and leaves; the others then time out at their next barrier.
#include "common.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace bt {

constexpr int kGruSeqThreads = 256;
constexpr int kGruSeqEnvs = 32;   // envs per CTA
constexpr int kGruSeqUnits = 16;  // hidden units per CTA
constexpr int kErrGruBarrier = 21;

struct GruSeqParams {
  int T, H, envs;
  const int* env_count;  // nullable: live envs
  const float* xp;       // [envs * T, 3H] input projections (+ input bias)
  const float* wh;       // [H, 3H]
  const float* bhn;      // [H]
  const uint8_t* reset;  // [envs * T] (row = env * T + t)
  float* hin;            // [envs * T, H] carry entering each step
  float* h;              // [envs * T, H] outputs
  float* gr;
  float* gz;
  float* gn;
  float* ghn;
  const float* dhs;  // [envs * T, H] dL/dh_t from the heads (backward)
  float* dxp;        // [envs * T, 3H] (backward)
  float* dhp;        // [envs * T, 3H] (backward)
  unsigned int* bar;  // zeroed before the launch
  int* err;
};

// Grid-wide step barrier; returns false (after recording the failure) if it gave up.
__device__ __forceinline__ bool gru_grid_barrier(const GruSeqParams& p, unsigned int target,
                                                 int* s_fail) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(p.bar, 1u);
    const uint64_t t0 = global_timer_ns();
    while (true) {
      unsigned int v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.bar) : "memory");
      if (v >= target) break;
      if (global_timer_ns() - t0 > 2000000000ull) {
        *s_fail = 1;
        if (p.err) atomicExch(p.err, kErrGruBarrier);
        break;
      }
    }
    __threadfence();
  }
  __syncthreads();
  return *s_fail == 0;
}

__device__ __forceinline__ float gru_sigmoid(float x) { return 1.f / (1.f + expf(-x)); }

__global__ void __launch_bounds__(kGruSeqThreads, 1) gru_seq_forward_kernel(GruSeqParams p) {
  extern __shared__ __align__(16) float sm[];
  __shared__ int s_fail;
  const int H = p.H, T = p.T, ld = H + 4;
  float* wt_s = sm;                              // [48][H + 4]: W_h columns, transposed
  float* hin_s = sm + 3 * kGruSeqUnits * ld;     // [32][H + 4]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int u_l = 8 * (warp & 1) + (lane & 7);          // unit within the CTA
  const int e_l = 2 * (4 * (warp >> 1) + (lane >> 3));  // first of the thread's two envs
  const int e0 = blockIdx.x * kGruSeqEnvs;
  const int U = blockIdx.y * kGruSeqUnits + u_l;
  const int live = live_rows(p.env_count, p.envs);
  if (tid == 0) s_fail = 0;
  // W_h[:, g H + u] for the CTA's units, gate-major: row c = g * 16 + unit
  for (int i = tid; i < 3 * kGruSeqUnits * H; i += kGruSeqThreads) {
    const int c = i / H, k = i - c * H;
    const int g = c / kGruSeqUnits, u = blockIdx.y * kGruSeqUnits + (c - g * kGruSeqUnits);
    wt_s[c * ld + k] = p.wh[(size_t)k * 3 * H + g * H + u];
  }
  const float bhn = p.bhn[U];
  const int h4 = H / 4;
  for (int t = 0; t < T; ++t) {
    // carry rows of the CTA's envs at step t (written by every CTA in step t - 1)
    for (int i = tid; i < kGruSeqEnvs * h4; i += kGruSeqThreads) {
      const int e = i / h4, k4 = i - e * h4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e0 + e < live)
        v = __ldcg(reinterpret_cast<const float4*>(p.hin + ((size_t)(e0 + e) * T + t) * H) + k4);
      *reinterpret_cast<float4*>(hin_s + e * ld + 4 * k4) = v;
    }
    // the input projections and reset flags of the thread's two outputs
    float x[2][3];
    bool on[2];
    size_t row[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      on[j] = e0 + e_l + j < live;
      row[j] = (size_t)(e0 + e_l + j) * T + t;
#pragma unroll
      for (int g = 0; g < 3; ++g) x[j][g] = on[j] ? p.xp[row[j] * 3 * H + g * H + U] : 0.f;
    }
    __syncthreads();
    float acc[2][3] = {};
    const float* a0 = hin_s + e_l * ld;
    const float* a1 = a0 + ld;
    const float* w0 = wt_s + u_l * ld;
    const float* w1 = w0 + kGruSeqUnits * ld;
    const float* w2 = w1 + kGruSeqUnits * ld;
#pragma unroll 4
    for (int k = 0; k < H; k += 4) {
      const float4 x0 = *reinterpret_cast<const float4*>(a0 + k);
      const float4 x1 = *reinterpret_cast<const float4*>(a1 + k);
      const float4 wr = *reinterpret_cast<const float4*>(w0 + k);
      const float4 wz = *reinterpret_cast<const float4*>(w1 + k);
      const float4 wn = *reinterpret_cast<const float4*>(w2 + k);
#define BT_GRU_FMA4(A, W, ACC)     \
  ACC = fmaf(A.x, W.x, ACC);       \
  ACC = fmaf(A.y, W.y, ACC);       \
  ACC = fmaf(A.z, W.z, ACC);       \
  ACC = fmaf(A.w, W.w, ACC);
      BT_GRU_FMA4(x0, wr, acc[0][0]);
      BT_GRU_FMA4(x0, wz, acc[0][1]);
      BT_GRU_FMA4(x0, wn, acc[0][2]);
      BT_GRU_FMA4(x1, wr, acc[1][0]);
      BT_GRU_FMA4(x1, wz, acc[1][1]);
      BT_GRU_FMA4(x1, wn, acc[1][2]);
#undef BT_GRU_FMA4
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      if (!on[j]) continue;
      const float r = gru_sigmoid(x[j][0] + acc[j][0]);
      const float z = gru_sigmoid(x[j][1] + acc[j][1]);
      const float hn = acc[j][2] + bhn;
      const float n = tanhf(x[j][2] + r * hn);
      const float hi = hin_s[(e_l + j) * ld + U];
      const float out = (1.f - z) * n + z * hi;
      const size_t o = row[j] * H + U;
      p.h[o] = out;
      p.gr[o] = r;
      p.gz[o] = z;
      p.gn[o] = n;
      p.ghn[o] = hn;
      if (t + 1 < T) p.hin[o + H] = p.reset[row[j] + 1] ? 0.f : out;
    }
    if (t + 1 < T && !gru_grid_barrier(p, (unsigned)(t + 1) * gridDim.x * gridDim.y, &s_fail))
      return;
  }
}

// Backward thread layout: thread (env pair, unit pair, kh) with kh = lane & 1; for the
// gate gradients it owns envs 2 ep, 2 ep + 1 of unit 2 up + kh, and in the carry product it
// sums the float4 columns of parity kh for both units of its pair (four accumulators, two
// dhp and two W_h rows per float4 step), the two parities then combined with a shuffle.
__global__ void __launch_bounds__(kGruSeqThreads, 1) gru_seq_backward_kernel(GruSeqParams p) {
  extern __shared__ __align__(16) float sm[];
  __shared__ int s_fail;
  const int H = p.H, T = p.T, H3 = 3 * H, ld = H3 + 4;
  float* w_s = sm;                              // [16][3H + 4]: rows of W_h
  float* d_s = sm + kGruSeqUnits * ld;          // [32][3H + 4]: dhp rows of the step
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kh = lane & 1;
  const int up = ((lane >> 1) & 3) + 4 * (warp & 1);  // unit pair 0..7
  const int u_l = 2 * up + kh;                        // the thread's unit (gate gradients)
  const int e_l = 2 * ((lane >> 3) + 4 * (warp >> 1));
  const int e0 = blockIdx.x * kGruSeqEnvs;
  const int U = blockIdx.y * kGruSeqUnits + u_l;
  const int live = live_rows(p.env_count, p.envs);
  if (tid == 0) s_fail = 0;
  for (int i = tid; i < kGruSeqUnits * H3; i += kGruSeqThreads) {
    const int u = i / H3, c = i - u * H3;
    w_s[u * ld + c] = p.wh[(size_t)(blockIdx.y * kGruSeqUnits + u) * H3 + c];
  }
  float carry[2] = {0.f, 0.f};
  bool on[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) on[j] = e0 + e_l + j < live;
  const int c4 = H3 / 4;
  unsigned int step = 0;
  for (int t = T - 1; t >= 0; --t) {
    float direct[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      if (!on[j]) continue;
      const size_t row = (size_t)(e0 + e_l + j) * T + t;
      const size_t i = row * H + U;
      const float dh = p.dhs[i] + carry[j];
      const float r = p.gr[i], z = p.gz[i], n = p.gn[i], hn = p.ghn[i], hi = p.hin[i];
      const float dn = dh * (1.f - z);
      const float dz = dh * (hi - n);
      const float dan = dn * (1.f - n * n);
      const float dar = (dan * hn) * r * (1.f - r);
      const float daz = dz * z * (1.f - z);
      float* dx = p.dxp + row * H3;
      float* dp = p.dhp + row * H3;
      dx[U] = dar;
      dx[H + U] = daz;
      dx[2 * H + U] = dan;
      dp[U] = dar;
      dp[H + U] = daz;
      dp[2 * H + U] = dan * r;
      direct[j] = dh * z;
    }
    if (t == 0) break;  // no carry into step -1
    ++step;
    if (!gru_grid_barrier(p, step * gridDim.x * gridDim.y, &s_fail)) return;
    for (int i = tid; i < kGruSeqEnvs * c4; i += kGruSeqThreads) {
      const int e = i / c4, q = i - e * c4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e0 + e < live)
        v = __ldcg(reinterpret_cast<const float4*>(p.dhp + ((size_t)(e0 + e) * T + t) * H3) + q);
      *reinterpret_cast<float4*>(d_s + e * ld + 4 * q) = v;
    }
    __syncthreads();
    // acc[env j][unit of the pair v]
    float acc[2][2] = {};
    const float* a0 = d_s + e_l * ld;
    const float* a1 = a0 + ld;
    const float* w0 = w_s + (2 * up) * ld;
    const float* w1 = w0 + ld;
#pragma unroll 4
    for (int c = 4 * kh; c < H3; c += 8) {
      const float4 x0 = *reinterpret_cast<const float4*>(a0 + c);
      const float4 x1 = *reinterpret_cast<const float4*>(a1 + c);
      const float4 v0 = *reinterpret_cast<const float4*>(w0 + c);
      const float4 v1 = *reinterpret_cast<const float4*>(w1 + c);
#define BT_GRU_DOT4(A, W, ACC)  \
  ACC = fmaf(A.x, W.x, ACC);     \
  ACC = fmaf(A.y, W.y, ACC);     \
  ACC = fmaf(A.z, W.z, ACC);     \
  ACC = fmaf(A.w, W.w, ACC);
      BT_GRU_DOT4(x0, v0, acc[0][0]);
      BT_GRU_DOT4(x0, v1, acc[0][1]);
      BT_GRU_DOT4(x1, v0, acc[1][0]);
      BT_GRU_DOT4(x1, v1, acc[1][1]);
#undef BT_GRU_DOT4
    }
    // combine the two column parities; this thread keeps its own unit (2 up + kh)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int v = 0; v < 2; ++v) acc[j][v] += __shfl_xor_sync(0xffffffffu, acc[j][v], 1);
    }
    // the carry gradient into step t - 1 (zero across a reset at step t)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float v = kh ? acc[j][1] : acc[j][0];
      carry[j] = on[j] && !p.reset[(size_t)(e0 + e_l + j) * T + t] ? v + direct[j] : 0.f;
    }
    __syncthreads();  // d_s is restaged in the next step
  }
}

namespace {

size_t fwd_smem(int H) { return (size_t)(3 * kGruSeqUnits + kGruSeqEnvs) * (H + 4) * 4; }
size_t bwd_smem(int H) { return (size_t)(kGruSeqUnits + kGruSeqEnvs) * (3 * H + 4) * 4; }

dim3 seq_grid(int envs, int H) {
  return dim3((unsigned)ceil_div(envs, kGruSeqEnvs), (unsigned)(H / kGruSeqUnits));
}

// Every CTA of the grid must be resident at the same time (they wait on one another).
int seq_fits(const void* kernel, size_t smem, dim3 grid, bool* ok) {
  *ok = false;
  int dev = 0, sms = 0, per_sm = 0;
  BT_CUDA(cudaGetDevice(&dev));
  BT_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  if (smem > 48 * 1024)
    BT_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  BT_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kGruSeqThreads, smem));
  *ok = per_sm >= 1 && (int64_t)grid.x * grid.y <= (int64_t)sms;
  return BT_OK;
}

}  // namespace

// Whether the one-launch kernels serve a sequence of `envs` envs with H hidden units.
int gru_seq_supported(int envs, int H, bool* ok) {
  *ok = false;
  if (H % kGruSeqUnits != 0 || H > 256 || envs < 1) return BT_OK;
  const dim3 grid = seq_grid(envs, H);
  bool f = false, b = false;
  BT_TRY(seq_fits((const void*)gru_seq_forward_kernel, fwd_smem(H), grid, &f));
  BT_TRY(seq_fits((const void*)gru_seq_backward_kernel, bwd_smem(H), grid, &b));
  *ok = f && b;
  return BT_OK;
}

int launch_gru_seq_forward(const GruSeqParams& p, cudaStream_t s) {
  BT_CUDA(cudaMemsetAsync(p.bar, 0, sizeof(unsigned int), s));
  gru_seq_forward_kernel<<<seq_grid(p.envs, p.H), kGruSeqThreads, fwd_smem(p.H), s>>>(p);
  BT_LAUNCH_CHECK("gru_seq_forward_kernel");
  return BT_OK;
}

int launch_gru_seq_backward(const GruSeqParams& p, cudaStream_t s) {
  BT_CUDA(cudaMemsetAsync(p.bar, 0, sizeof(unsigned int), s));
  gru_seq_backward_kernel<<<seq_grid(p.envs, p.H), kGruSeqThreads, bwd_smem(p.H), s>>>(p);
  BT_LAUNCH_CHECK("gru_seq_backward_kernel");
  return BT_OK;
}

}  // namespace bt
