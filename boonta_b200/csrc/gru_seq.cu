// K15 as one launch per sequence: the GRU recurrence of a minibatch of env sequences
// (flax GRUCell scanned over time, reset to zero on first.done; boonta/networks/blocks/rnn.py
// :30-59, boonta/algorithms/recurrent_ppo.py:211-223) and its backward through time, each
// as a persistent kernel that walks the T steps with a grid-wide barrier between them,
// instead of two launches (a GEMM and an elementwise kernel) per step.
//
// Work split (both directions): CTA (eb, ub) owns envs [32 eb, 32 eb + 32) of the minibatch
// and hidden units [16 ub, 16 ub + 16). The per-step products run on the tensor cores as
// warp-level mma.sync (m16n8k16, bf16 operands, fp32 accumulation) in the split-bf16 form
// x = hi + lo with three products (lo hi + hi lo + hi hi, relative error ~1e-5, the scheme
// of BT_PREC_BF16X3); the CTA's W_h fragments stay in registers for the whole sequence and
// the step's fp32 rows are split as they are read from shared memory. Each thread ends a
// product owning one env x two units, with all three gates of those units, so the gate
// math follows in registers.
//
//   forward step t   stage the 32 carry rows hin_t (all H) from L2; hp = hin_t W_h for the
//                    CTA's 48 gate columns; gates, h_t, the saved r, z, n, h W_hn + b_hn;
//                    hin_{t+1} = reset ? 0 : h_t; barrier
//   backward step t  gate gradients of the thread's (env, unit) pairs from dL/dh_t (heads)
//                    and the carry gradient kept in registers; dxp_t, dhp_t written; barrier;
//                    stage the 32 dhp_t rows (all 3H); carry = reset ? 0 : dh z + dhp_t W_h^T
//
// The gate formulas are those of the per-step fp32 kernels in recurrent.cu.
//
// The barrier: thread 0 of every CTA adds one to a device counter (zeroed before the launch)
// and spins until it reaches (step + 1) * CTAs. All CTAs must be resident at once: the host
// launches at most one CTA per SM with an occupancy check, the recurrent path issues all its
// kernels on the caller's stream (no side stream of the learner runs beside these), and the spin
// is bounded (2 s of %globaltimer), after which the CTA records kErrGruBarrier in the learner's
// error word and leaves; the others then time out at their next barrier
// (bt_selftest_gru_barrier makes every barrier give up, on purpose).
#include "common.cuh"
#include "gru_seq.cuh"
#include "kernels.cuh"
#include "mma_sync.cuh"
#include "ptx.cuh"

namespace bt {

constexpr int kGruSeqThreads = 256;
constexpr int kGruSeqEnvs = 32;   // envs per CTA
constexpr int kGruSeqUnits = 16;  // hidden units per CTA

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
      if (v >= target + p.bar_offset) break;
      if (global_timer_ns() - t0 > (p.limit_ns ? p.limit_ns : 2000000000ull)) {
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

// Warp roles (both kernels): warp = mt + 2 * nt + 4 * kh, with m-tile mt (envs 16 mt ..),
// n-tile nt (8 units) and K half kh. After the product the two K halves of a tile meet in
// shared memory (fixed order: half 0 + half 1); a thread then owns env row
// 16 mt + gid + 8 kh and the two units 8 nt + 2 tig + {0, 1} of its tile.
constexpr int kXch = 4 * 32;  // floats per (warp tile, gate) exchange slot

template <int H>
__global__ void __launch_bounds__(kGruSeqThreads, 1) gru_seq_forward_kernel(GruSeqParams p) {
  constexpr int KS = H / 32;  // 16-wide K steps per K half
  constexpr int LD = H + 8;   // row stride of the staged carry rows (conflict-free float2)
  extern __shared__ __align__(16) float sm[];
  __shared__ int s_fail;
  float* hin_s = sm;                                // [32][LD]
  float* xch = sm + kGruSeqEnvs * LD;               // [kh][mt][nt][gate][lane][4]
  const int T = p.T, H3 = 3 * H;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int mt = warp & 1, nt = (warp >> 1) & 1, kh = warp >> 2;
  const int e0 = blockIdx.x * kGruSeqEnvs, u0 = blockIdx.y * kGruSeqUnits;
  const int live = live_rows(p.env_count, p.envs);
  if (tid == 0) s_fail = 0;
  // B fragments of W_h for the whole sequence: gate g, unit u0 + 8 nt + gid, K rows of half kh
  uint32_t bh[3][KS][2], bl[3][KS][2];
#pragma unroll
  for (int g = 0; g < 3; ++g) {
    const float* w = p.wh + g * H + u0 + nt * 8 + gid;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int k = kh * (H / 2) + ks * 16 + tig * 2;
      split_pair(w[(size_t)k * H3], w[(size_t)(k + 1) * H3], bh[g][ks][0], bl[g][ks][0]);
      split_pair(w[(size_t)(k + 8) * H3], w[(size_t)(k + 9) * H3], bh[g][ks][1], bl[g][ks][1]);
    }
  }
  const int r_l = mt * 16 + gid + 8 * kh;  // the thread's env row in the CTA
  const int ub = u0 + nt * 8 + tig * 2;    // its first unit
  const bool on = e0 + r_l < live;
  const float bhn0 = p.bhn[ub], bhn1 = p.bhn[ub + 1];
  constexpr int h4 = H / 4;
  for (int t = 0; t < T; ++t) {
    // carry rows of the CTA's envs at step t (written by every CTA in step t - 1)
    for (int i = tid; i < kGruSeqEnvs * h4; i += kGruSeqThreads) {
      const int e = i / h4, k4 = i - e * h4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e0 + e < live)
        v = __ldcg(reinterpret_cast<const float4*>(p.hin + ((size_t)(e0 + e) * T + t) * H) + k4);
      *reinterpret_cast<float4*>(hin_s + e * LD + 4 * k4) = v;
    }
    const size_t row = (size_t)(e0 + r_l) * T + t;
    float x[2][3];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int g = 0; g < 3; ++g) x[j][g] = on ? p.xp[row * H3 + g * H + ub + j] : 0.f;
    __syncthreads();
    float acc[3][4] = {};
    const float* a0 = hin_s + (mt * 16 + gid) * LD + kh * (H / 2) + tig * 2;
    const float* a1 = a0 + 8 * LD;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      uint32_t ah[4], al[4];
      load_a_split(a0 + ks * 16, a1 + ks * 16, ah, al);
#pragma unroll
      for (int g = 0; g < 3; ++g) mma_split(acc[g], ah, al, bh[g][ks], bl[g][ks]);
    }
#pragma unroll
    for (int g = 0; g < 3; ++g)
      *reinterpret_cast<float4*>(xch + ((warp * 3 + g) * 32 + lane) * 4) =
          make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
    __syncthreads();
    if (on) {
      const int w0 = warp & 3, w1 = w0 + 4;  // the tile's two K halves
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float hp[3];
#pragma unroll
        for (int g = 0; g < 3; ++g)
          hp[g] = xch[((w0 * 3 + g) * 32 + lane) * 4 + 2 * kh + j] +
                  xch[((w1 * 3 + g) * 32 + lane) * 4 + 2 * kh + j];
        const int U = ub + j;
        const float r = gru_sigmoid(x[j][0] + hp[0]);
        const float z = gru_sigmoid(x[j][1] + hp[1]);
        const float hn = hp[2] + (j ? bhn1 : bhn0);
        const float n = tanhf(x[j][2] + r * hn);
        const float hi = hin_s[r_l * LD + U];
        const float out = (1.f - z) * n + z * hi;
        const size_t o = row * H + U;
        p.h[o] = out;
        p.gr[o] = r;
        p.gz[o] = z;
        p.gn[o] = n;
        p.ghn[o] = hn;
        if (t + 1 < T) p.hin[o + H] = p.reset[row + 1] ? 0.f : out;
      }
    }
    if (t + 1 < T && !gru_grid_barrier(p, (unsigned)(t + 1) * gridDim.x * gridDim.y, &s_fail))
      return;
  }
}

template <int H>
__global__ void __launch_bounds__(kGruSeqThreads, 1) gru_seq_backward_kernel(GruSeqParams p) {
  constexpr int H3 = 3 * H;
  constexpr int KS = H3 / 32;  // 16-wide K steps per K half
  constexpr int LD = H3 + 8;
  extern __shared__ __align__(16) float sm[];
  __shared__ int s_fail;
  float* d_s = sm;                        // [32][LD]: dhp rows of the step
  float* xch = sm + kGruSeqEnvs * LD;     // [kh][mt][nt][lane][4]
  const int T = p.T;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int mt = warp & 1, nt = (warp >> 1) & 1, kh = warp >> 2;
  const int e0 = blockIdx.x * kGruSeqEnvs, u0 = blockIdx.y * kGruSeqUnits;
  const int live = live_rows(p.env_count, p.envs);
  if (tid == 0) s_fail = 0;
  // B fragments of W_h^T: unit u0 + 8 nt + gid (a row of W_h), K = the 3H columns of half kh
  uint32_t bh[KS][2], bl[KS][2];
  {
    const float* w = p.wh + (size_t)(u0 + nt * 8 + gid) * H3 + kh * (H3 / 2) + tig * 2;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      split_pair(w[ks * 16], w[ks * 16 + 1], bh[ks][0], bl[ks][0]);
      split_pair(w[ks * 16 + 8], w[ks * 16 + 9], bh[ks][1], bl[ks][1]);
    }
  }
  const int r_l = mt * 16 + gid + 8 * kh;
  const int ub = u0 + nt * 8 + tig * 2;
  const bool on = e0 + r_l < live;
  float carry[2] = {0.f, 0.f};
  constexpr int c4 = H3 / 4;
  unsigned int step = 0;
  for (int t = T - 1; t >= 0; --t) {
    const size_t row = (size_t)(e0 + r_l) * T + t;
    float direct[2] = {0.f, 0.f};
    if (on) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int U = ub + j;
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
    }
    if (t == 0) break;  // no carry into step -1
    ++step;
    if (!gru_grid_barrier(p, step * gridDim.x * gridDim.y, &s_fail)) return;
    for (int i = tid; i < kGruSeqEnvs * c4; i += kGruSeqThreads) {
      const int e = i / c4, q = i - e * c4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e0 + e < live)
        v = __ldcg(reinterpret_cast<const float4*>(p.dhp + ((size_t)(e0 + e) * T + t) * H3) + q);
      *reinterpret_cast<float4*>(d_s + e * LD + 4 * q) = v;
    }
    __syncthreads();
    float acc[4] = {};
    const float* a0 = d_s + (mt * 16 + gid) * LD + kh * (H3 / 2) + tig * 2;
    const float* a1 = a0 + 8 * LD;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      uint32_t ah[4], al[4];
      load_a_split(a0 + ks * 16, a1 + ks * 16, ah, al);
      mma_split(acc, ah, al, bh[ks], bl[ks]);
    }
    *reinterpret_cast<float4*>(xch + (warp * 32 + lane) * 4) =
        make_float4(acc[0], acc[1], acc[2], acc[3]);
    __syncthreads();
    // the carry gradient into step t - 1 (zero across a reset at step t)
    const int w0 = warp & 3, w1 = w0 + 4;
    const bool keep = on && !p.reset[row];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float v = xch[(w0 * 32 + lane) * 4 + 2 * kh + j] + xch[(w1 * 32 + lane) * 4 + 2 * kh + j];
      carry[j] = keep ? v + direct[j] : 0.f;
    }
  }
}

namespace {

size_t fwd_smem(int H) {
  return ((size_t)kGruSeqEnvs * (H + 8) + 8 * 3 * kXch) * sizeof(float);
}
size_t bwd_smem(int H) {
  return ((size_t)kGruSeqEnvs * (3 * H + 8) + 8 * kXch) * sizeof(float);
}

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

template <int H>
int supported_h(int envs, bool* ok) {
  const dim3 grid = seq_grid(envs, H);
  bool f = false, b = false;
  BT_TRY(seq_fits((const void*)gru_seq_forward_kernel<H>, fwd_smem(H), grid, &f));
  BT_TRY(seq_fits((const void*)gru_seq_backward_kernel<H>, bwd_smem(H), grid, &b));
  *ok = f && b;
  return BT_OK;
}

}  // namespace

// Whether the one-launch kernels serve a sequence of `envs` envs with H hidden units
// (H = 64, 128 or 256, every CTA of the grid resident at once).
int gru_seq_supported(int envs, int H, bool* ok) {
  *ok = false;
  if (envs < 1) return BT_OK;
  switch (H) {
    case 64: return supported_h<64>(envs, ok);
    case 128: return supported_h<128>(envs, ok);
    case 256: return supported_h<256>(envs, ok);
    default: return BT_OK;
  }
}

int launch_gru_seq_forward(const GruSeqParams& p, cudaStream_t s) {
  BT_CUDA(cudaMemsetAsync(p.bar, 0, sizeof(unsigned int), s));
  const dim3 grid = seq_grid(p.envs, p.H);
  const size_t smem = fwd_smem(p.H);
  switch (p.H) {
    case 64: gru_seq_forward_kernel<64><<<grid, kGruSeqThreads, smem, s>>>(p); break;
    case 128: gru_seq_forward_kernel<128><<<grid, kGruSeqThreads, smem, s>>>(p); break;
    case 256: gru_seq_forward_kernel<256><<<grid, kGruSeqThreads, smem, s>>>(p); break;
    default: BT_CHECK_ARG(false, "gru sequence kernel: hidden size %d", p.H);
  }
  BT_LAUNCH_CHECK("gru_seq_forward_kernel");
  return BT_OK;
}

int launch_gru_seq_backward(const GruSeqParams& p, cudaStream_t s) {
  BT_CUDA(cudaMemsetAsync(p.bar, 0, sizeof(unsigned int), s));
  const dim3 grid = seq_grid(p.envs, p.H);
  const size_t smem = bwd_smem(p.H);
  switch (p.H) {
    case 64: gru_seq_backward_kernel<64><<<grid, kGruSeqThreads, smem, s>>>(p); break;
    case 128: gru_seq_backward_kernel<128><<<grid, kGruSeqThreads, smem, s>>>(p); break;
    case 256: gru_seq_backward_kernel<256><<<grid, kGruSeqThreads, smem, s>>>(p); break;
    default: BT_CHECK_ARG(false, "gru sequence kernel: hidden size %d", p.H);
  }
  BT_LAUNCH_CHECK("gru_seq_backward_kernel");
  return BT_OK;
}

}  // namespace bt

extern "C" int bt_selftest_gru_barrier(int32_t limit_us, void* stream) {
  using namespace bt;
  BT_CHECK_ARG(limit_us > 0 && limit_us <= 2000000, "limit %d us outside (0, 2 s]", limit_us);
  cudaStream_t s = (cudaStream_t)stream;
  // a 2-step sequence of 32 envs x 64 units (4 CTAs) on zeroed buffers, with every barrier
  // target one above what the grid can reach
  constexpr int kH = 64, kEnvs = 32, kT = 2;
  const size_t rows = (size_t)kEnvs * kT;
  const size_t floats = rows * 3 * kH * 3 + rows * kH * 8 + (size_t)kH * 3 * kH + kH;
  float* buf = nullptr;
  BT_CUDA(cudaMallocAsync(&buf, floats * sizeof(float) + rows + 64, s));
  BT_CUDA(cudaMemsetAsync(buf, 0, floats * sizeof(float) + rows + 64, s));
  float* f = buf;
  auto take = [&](size_t n) { float* q = f; f += n; return q; };
  GruSeqParams p{};
  p.T = kT;
  p.H = kH;
  p.envs = kEnvs;
  p.xp = take(rows * 3 * kH);
  p.dxp = take(rows * 3 * kH);
  p.dhp = take(rows * 3 * kH);
  p.hin = take(rows * kH);
  p.h = take(rows * kH);
  p.gr = take(rows * kH);
  p.gz = take(rows * kH);
  p.gn = take(rows * kH);
  p.ghn = take(rows * kH);
  p.dhs = take(rows * kH);
  p.wh = take((size_t)kH * 3 * kH);
  p.bhn = take(kH);
  take(rows * kH);
  uint8_t* tail = reinterpret_cast<uint8_t*>(f);
  p.reset = tail;
  p.bar = reinterpret_cast<unsigned int*>(tail + ((rows + 15) / 16) * 16);
  p.err = reinterpret_cast<int*>(p.bar + 4);
  p.limit_ns = (unsigned long long)limit_us * 1000ull;
  p.bar_offset = 1;
  bool ok = false;
  BT_TRY(gru_seq_supported(kEnvs, kH, &ok));
  BT_CHECK_ARG(ok, "gru sequence kernel does not fit this device");
  BT_TRY(launch_gru_seq_forward(p, s));
  int code = 0;
  BT_CUDA(cudaMemcpyAsync(&code, p.err, sizeof(int), cudaMemcpyDeviceToHost, s));
  BT_CUDA(cudaFreeAsync(buf, s));
  BT_CUDA(cudaStreamSynchronize(s));
  if (code == kErrGruBarrier) {
    set_error("gru step barrier gave up after %d us (the expected outcome)", limit_us);
    return BT_ERR_TIMEOUT;
  }
  return code ? BT_ERR_CUDA : BT_OK;
}
