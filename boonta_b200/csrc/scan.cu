// K16: the linear recurrence h_t = a_t * h_{t-1} + b_t of the SSM torso, forward and backward,
// as chunked affine scans.
//
// Restates boonta/networks/kernels/scan.py: `_forward` (:13-38) runs the recurrence from
// h_{-1} = init over the steps of each (batch row, feature) column, accumulating in float32 and
// storing h in the dtype of a; `_backward` (:41-68) with the custom VJP (:71-89) gives
//   g_{T-1} = cot_{T-1},  g_t = cot_t + a_{t+1} g_{t+1}   (float32, cot first cast to a's dtype)
//   db = g (stored in a's dtype),  da_t = db_t * h_{t-1} (h_{-1} = init),  dinit = db_0 * a_0,
// the two products taken in a's dtype as the reference's XLA ops do. Layout [batch, steps,
// features], features contiguous; a, b, h, da, db are float32 or bf16 (`dtype`), init / dinit
// float32 or bf16 (`init_dtype`).
//
// Parallel form: both recurrences are affine maps of the carry, x -> m x + c, and affine maps
// compose associatively. A block owns 32 consecutive feature columns of one batch row (lane =
// column, coalesced 128-byte rows for float32) and splits the steps into kChunks chunks, one
// per warp. Each warp folds its chunk into one map (product of the multipliers, scan of the
// offsets from a zero carry), the maps meet in shared memory, each warp composes the maps of
// the chunks before it (in order) onto the initial carry, and rescans its chunk from that carry,
// storing the outputs. The chunk's inputs stay in registers between the two passes when the
// chunk has at most kKeep steps; longer chunks read them again (from L2). Every product and sum
// is rounded separately (no FMA contraction), so a CPU restatement in the same order reproduces
// the outputs bit for bit; against the sequential order the difference is a few float32 ulps of
// the running value. HBM roofline: (2 reads + 1 write) x element size per step forward; the
// backward reads a, h, cot (+ init) and writes da, db.
#include "common.cuh"

namespace bt {

constexpr int kScanChunks = 8;  // warps per block = time chunks
constexpr int kScanKeep = 16;   // chunk steps held in registers between the passes

template <bool BF16>
__device__ __forceinline__ float ld_elem(const void* p, size_t i) {
  if constexpr (BF16) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  } else {
    return reinterpret_cast<const float*>(p)[i];
  }
}
template <bool BF16>
__device__ __forceinline__ void st_elem(void* p, size_t i, float v) {
  if constexpr (BF16) {
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  } else {
    reinterpret_cast<float*>(p)[i] = v;
  }
}
// v rounded to the storage type and back (the value a stored element holds).
template <bool BF16>
__device__ __forceinline__ float rnd(float v) {
  if constexpr (BF16) {
    return __bfloat162float(__float2bfloat16_rn(v));
  } else {
    return v;
  }
}

struct ScanShape {
  int batch, steps, features;
  int chunk;  // steps per chunk (ceil(steps / kScanChunks))
};

// Forward: column (row, f), chunk w = warp covers steps [w * chunk, min(steps, (w+1) * chunk)).
template <bool BF16, bool IBF16>
__global__ void __launch_bounds__(32 * kScanChunks)
    linear_scan_kernel(const void* a, const void* b, const void* init, void* out, ScanShape sh) {
  __shared__ float m_s[kScanChunks][32], c_s[kScanChunks][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int f = blockIdx.x * 32 + lane, row = blockIdx.y;
  const bool col = f < sh.features;
  const int t0 = min(sh.steps, w * sh.chunk), t1 = min(sh.steps, t0 + sh.chunk);
  const size_t base = (size_t)row * sh.steps * sh.features + f;
  float ka[kScanKeep], kb[kScanKeep];
  const bool keep = sh.chunk <= kScanKeep;
  // pass 1: the chunk's map h_end = m * h_start + c
  float m = 1.f, c = 0.f;
  if (col && keep) {
#pragma unroll
    for (int j = 0; j < kScanKeep; ++j) {
      ka[j] = 1.f;
      kb[j] = 0.f;
      if (t0 + j < t1) {
        const size_t i = base + (size_t)(t0 + j) * sh.features;
        ka[j] = ld_elem<BF16>(a, i);
        kb[j] = ld_elem<BF16>(b, i);
      }
    }
#pragma unroll
    for (int j = 0; j < kScanKeep; ++j) {
      if (t0 + j < t1) {
        m = __fmul_rn(ka[j], m);
        c = __fadd_rn(__fmul_rn(ka[j], c), kb[j]);
      }
    }
  } else if (col) {
    for (int t = t0; t < t1; ++t) {
      const size_t i = base + (size_t)t * sh.features;
      const float at = ld_elem<BF16>(a, i), bt = ld_elem<BF16>(b, i);
      m = __fmul_rn(at, m);
      c = __fadd_rn(__fmul_rn(at, c), bt);
    }
  }
  m_s[w][lane] = m;
  c_s[w][lane] = c;
  __syncthreads();
  if (!col) return;
  // the carry entering the chunk: the maps of chunks 0 .. w-1 applied to init, in order
  float h = ld_elem<IBF16>(init, (size_t)row * sh.features + f);
  for (int k = 0; k < w; ++k) h = __fadd_rn(__fmul_rn(m_s[k][lane], h), c_s[k][lane]);
  // pass 2: rescan from the carry
  if (keep) {
#pragma unroll
    for (int j = 0; j < kScanKeep; ++j) {
      if (t0 + j < t1) {
        h = __fadd_rn(__fmul_rn(ka[j], h), kb[j]);
        st_elem<BF16>(out, base + (size_t)(t0 + j) * sh.features, h);
      }
    }
  } else {
    for (int t = t0; t < t1; ++t) {
      const size_t i = base + (size_t)t * sh.features;
      h = __fadd_rn(__fmul_rn(ld_elem<BF16>(a, i), h), ld_elem<BF16>(b, i));
      st_elem<BF16>(out, i, h);
    }
  }
}

// Backward: reverse chunks; the carry entering chunk w comes from chunks w+1 .. last (in
// reverse order), starting from zero past the last step.
template <bool BF16, bool IBF16>
__global__ void __launch_bounds__(32 * kScanChunks)
    linear_scan_backward_kernel(const void* a, const void* h, const void* init, const void* cot,
                                void* da, void* db, void* dinit, ScanShape sh) {
  __shared__ float m_s[kScanChunks][32], c_s[kScanChunks][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int f = blockIdx.x * 32 + lane, row = blockIdx.y;
  const bool col = f < sh.features;
  const int t0 = min(sh.steps, w * sh.chunk), t1 = min(sh.steps, t0 + sh.chunk);
  const size_t base = (size_t)row * sh.steps * sh.features + f;
  const int T = sh.steps;
  // multiplier of the carry at step t: a_{t+1} (none at the last step)
  auto mult = [&](int t) { return t + 1 < T ? ld_elem<BF16>(a, base + (size_t)(t + 1) * sh.features) : 0.f; };
  float m = 1.f, c = 0.f;
  if (col) {
    for (int t = t1 - 1; t >= t0; --t) {
      const float mt = mult(t);
      const float ct = rnd<BF16>(ld_elem<BF16>(cot, base + (size_t)t * sh.features));
      m = __fmul_rn(mt, m);
      c = __fadd_rn(__fmul_rn(mt, c), ct);
    }
  }
  m_s[w][lane] = m;
  c_s[w][lane] = c;
  __syncthreads();
  if (!col) return;
  float g = 0.f;
  for (int k = kScanChunks - 1; k > w; --k) g = __fadd_rn(__fmul_rn(m_s[k][lane], g), c_s[k][lane]);
  for (int t = t1 - 1; t >= t0; --t) {
    const size_t i = base + (size_t)t * sh.features;
    const float ct = rnd<BF16>(ld_elem<BF16>(cot, i));
    g = __fadd_rn(__fmul_rn(mult(t), g), ct);
    const float gs = rnd<BF16>(g);  // db as stored
    st_elem<BF16>(db, i, gs);
    // h_{t-1}, or init itself at t = 0 (the reference concatenates init with h, so an fp32
    // init enters the product unrounded)
    const float hp = t > 0 ? ld_elem<BF16>(h, i - sh.features)
                           : ld_elem<IBF16>(init, (size_t)row * sh.features + f);
    st_elem<BF16>(da, i, __fmul_rn(gs, hp));
    if (t == 0) {
      const float d0 = rnd<BF16>(__fmul_rn(gs, ld_elem<BF16>(a, i)));
      st_elem<IBF16>(dinit, (size_t)row * sh.features + f, d0);
    }
  }
}

static ScanShape scan_shape(int batch, int steps, int features) {
  return {batch, steps, features, ceil_div(steps, kScanChunks)};
}

}  // namespace bt

using bt::ceil_div;

extern "C" int bt_linear_scan(const void* a, const void* b, const void* init, void* out,
                              int32_t batch, int32_t steps, int32_t features, int32_t dtype,
                              int32_t init_dtype, void* stream) {
  BT_CHECK_ARG(batch >= 0 && steps >= 0 && features >= 0, "bt_linear_scan: negative shape");
  BT_CHECK_ARG((dtype == BT_DTYPE_F32 || dtype == BT_DTYPE_BF16) &&
                   (init_dtype == BT_DTYPE_F32 || init_dtype == BT_DTYPE_BF16),
               "bt_linear_scan: dtype %d / init dtype %d", dtype, init_dtype);
  BT_CHECK_ARG(batch <= 65535, "bt_linear_scan: batch %d above 65535", batch);
  if (batch == 0 || steps == 0 || features == 0) return BT_OK;
  BT_CHECK_ARG(a && b && init && out, "bt_linear_scan: null pointer");
  const bt::ScanShape sh = bt::scan_shape(batch, steps, features);
  const dim3 grid(ceil_div(features, 32), batch);
  const cudaStream_t s = (cudaStream_t)stream;
  const bool hb = dtype == BT_DTYPE_BF16, ib = init_dtype == BT_DTYPE_BF16;
  if (hb && ib) bt::linear_scan_kernel<true, true><<<grid, 32 * bt::kScanChunks, 0, s>>>(a, b, init, out, sh);
  else if (hb) bt::linear_scan_kernel<true, false><<<grid, 32 * bt::kScanChunks, 0, s>>>(a, b, init, out, sh);
  else if (ib) bt::linear_scan_kernel<false, true><<<grid, 32 * bt::kScanChunks, 0, s>>>(a, b, init, out, sh);
  else bt::linear_scan_kernel<false, false><<<grid, 32 * bt::kScanChunks, 0, s>>>(a, b, init, out, sh);
  BT_LAUNCH_CHECK("linear_scan_kernel");
  return BT_OK;
}

extern "C" int bt_linear_scan_backward(const void* a, const void* h, const void* init,
                                       const void* cotangent, void* da, void* db, void* dinit,
                                       int32_t batch, int32_t steps, int32_t features,
                                       int32_t dtype, int32_t init_dtype, void* stream) {
  BT_CHECK_ARG(batch >= 0 && steps >= 0 && features >= 0, "bt_linear_scan_backward: negative shape");
  BT_CHECK_ARG((dtype == BT_DTYPE_F32 || dtype == BT_DTYPE_BF16) &&
                   (init_dtype == BT_DTYPE_F32 || init_dtype == BT_DTYPE_BF16),
               "bt_linear_scan_backward: dtype %d / init dtype %d", dtype, init_dtype);
  BT_CHECK_ARG(batch <= 65535, "bt_linear_scan_backward: batch %d above 65535", batch);
  if (batch == 0 || steps == 0 || features == 0) return BT_OK;
  BT_CHECK_ARG(a && h && init && cotangent && da && db && dinit,
               "bt_linear_scan_backward: null pointer");
  const bt::ScanShape sh = bt::scan_shape(batch, steps, features);
  const dim3 grid(ceil_div(features, 32), batch);
  const cudaStream_t s = (cudaStream_t)stream;
  const bool hb = dtype == BT_DTYPE_BF16, ib = init_dtype == BT_DTYPE_BF16;
  if (hb && ib)
    bt::linear_scan_backward_kernel<true, true><<<grid, 32 * bt::kScanChunks, 0, s>>>(a, h, init, cotangent, da, db, dinit, sh);
  else if (hb)
    bt::linear_scan_backward_kernel<true, false><<<grid, 32 * bt::kScanChunks, 0, s>>>(a, h, init, cotangent, da, db, dinit, sh);
  else if (ib)
    bt::linear_scan_backward_kernel<false, true><<<grid, 32 * bt::kScanChunks, 0, s>>>(a, h, init, cotangent, da, db, dinit, sh);
  else
    bt::linear_scan_backward_kernel<false, false><<<grid, 32 * bt::kScanChunks, 0, s>>>(a, h, init, cotangent, da, db, dinit, sh);
  BT_LAUNCH_CHECK("linear_scan_backward_kernel");
  return BT_OK;
}
