// Memory-bound kernels of the learner step:
//   K4  LayerNorm forward/backward fused with the following activation
//   K10 gradient reduction (split-K partials -> gradients, with the global-norm partial
//       sums), clip_by_global_norm + Adam + apply_updates (optax semantics)
//   K12 advantage normalisation;  K13 statistics reductions
//   the multi-GPU minibatch split (global permutation -> this rank's rows)
// Every reduction sums in a fixed order (per-block partials written to scratch, then
// summed in index order), so a fixed input gives bitwise identical results.
#include "kernels.cuh"

namespace bt {

constexpr float kLnEps = 1e-6f;

// ---- LayerNorm -------------------------------------------------------------------------
// flax.linen.LayerNorm(epsilon=1e-6, use_fast_variance=True):
//   mean = E[z], var = max(E[z^2] - mean^2, 0), y = (z - mean) * (rsqrt(var + eps) * scale) + bias
// One warp per row.
__global__ void ln_forward_kernel(const float* z, const float* sb, int rows, int n, int act,
                                  float* y, float* h, __nv_bfloat16* hb, __nv_bfloat16* hb_lo,
                                  int ldhb, float* mean_out, float* rstd_out, const int* count) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();
  if (row >= live_rows(count, rows)) return;
  const float* zr = z + (size_t)row * n;
  float s = 0.f, s2 = 0.f;
  for (int k = lane; k < n; k += 32) {
    const float v = zr[k];
    s += v;
    s2 += v * v;
  }
  s = warp_sum(s);
  s2 = warp_sum(s2);
  const float mean = s / n;
  const float var = fmaxf(s2 / n - mean * mean, 0.f);
  const float r = rsqrtf(var + kLnEps);
  with_act(act, [&](auto tag) {
    for (int k = lane; k < n; k += 32) {
      const float yv = (zr[k] - mean) * (r * sb[k]) + sb[n + k];
      if (y) y[(size_t)row * n + k] = yv;
      const float hv = act_fwd<decltype(tag)::value>(yv);
      if (h) h[(size_t)row * n + k] = hv;
      if (hb) store_bf16(hb, hb_lo, (size_t)row * ldhb + k, hv);
    }
  });
  if (lane == 0) {
    mean_out[row] = mean;
    rstd_out[row] = r;
  }
}

// Vectorised forward for n = 128 NV (NV <= 8): lane `l` owns the float4 columns l, l + 32, ...
// of its warp's row, read once into registers (the scalar kernel above reads each row twice).
template <int NV>
__global__ void __launch_bounds__(256) ln_forward_vec_kernel(
    const float* z, const float* sb, int rows, int n, int act, float* y, float* h,
    __nv_bfloat16* hb, __nv_bfloat16* hb_lo, int ldhb, float* mean_out, float* rstd_out,
    const int* count) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();
  if (row >= live_rows(count, rows)) return;
  const float4* zr = reinterpret_cast<const float4*>(z + (size_t)row * n);
  float4 v[NV];
  float s = 0.f, s2 = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i] = zr[lane + 32 * i];
    s += v[i].x + v[i].y + v[i].z + v[i].w;
    s2 += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
  }
  s = warp_sum(s);
  s2 = warp_sum(s2);
  const float mean = s / n;
  const float var = fmaxf(s2 / n - mean * mean, 0.f);
  const float r = rsqrtf(var + kLnEps);
  const float4* sc = reinterpret_cast<const float4*>(sb);
  const float4* bi = reinterpret_cast<const float4*>(sb + n);
  with_act(act, [&](auto tag) {
    constexpr int A = decltype(tag)::value;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int q = lane + 32 * i;
      const float4 a = __ldg(sc + q), b = __ldg(bi + q);
      float4 yv;
      yv.x = (v[i].x - mean) * (r * a.x) + b.x;
      yv.y = (v[i].y - mean) * (r * a.y) + b.y;
      yv.z = (v[i].z - mean) * (r * a.z) + b.z;
      yv.w = (v[i].w - mean) * (r * a.w) + b.w;
      if (y) reinterpret_cast<float4*>(y + (size_t)row * n)[q] = yv;
      const float4 hv = make_float4(act_fwd<A>(yv.x), act_fwd<A>(yv.y), act_fwd<A>(yv.z),
                                    act_fwd<A>(yv.w));
      if (h) reinterpret_cast<float4*>(h + (size_t)row * n)[q] = hv;
      if (hb) store_bf16x4(hb, hb_lo, (size_t)row * ldhb + 4 * q, hv);
    }
  });
  if (lane == 0) {
    mean_out[row] = mean;
    rstd_out[row] = r;
  }
}

int launch_ln_forward(const float* z, const float* scale_bias, int rows, int n, int act, float* y,
                      float* h, __nv_bfloat16* hb, __nv_bfloat16* hb_lo, int ldhb, float* mean,
                      float* rstd, const int* count, cudaStream_t stream) {
  if (rows <= 0) return BT_OK;
  const dim3 grid(ceil_div(rows * 32, 256));
  const bool vec = n % 128 == 0 && n <= 1024 && (uintptr_t)z % 16 == 0 &&
                   (uintptr_t)scale_bias % 16 == 0 && (uintptr_t)y % 16 == 0 &&
                   (uintptr_t)h % 16 == 0 && (!hb || (ldhb % 4 == 0 && (uintptr_t)hb % 8 == 0 &&
                                                      (uintptr_t)hb_lo % 8 == 0));
  if (vec) {
    switch (n / 128) {
#define BT_LN_FWD(NV)                                                                          \
  case NV:                                                                                     \
    BT_CUDA(launch_pdl(ln_forward_vec_kernel<NV>, grid, dim3(256), 0, stream, z, scale_bias,   \
                       rows, n, act, y, h, hb, hb_lo, ldhb, mean, rstd, count));               \
    return BT_OK;
      BT_LN_FWD(1) BT_LN_FWD(2) BT_LN_FWD(3) BT_LN_FWD(4)
      BT_LN_FWD(5) BT_LN_FWD(6) BT_LN_FWD(7) BT_LN_FWD(8)
#undef BT_LN_FWD
      default: break;
    }
  }
  BT_CUDA(launch_pdl(ln_forward_kernel, grid, dim3(256), 0, stream, z, scale_bias, rows, n, act,
                     y, h, hb, hb_lo, ldhb, mean, rstd, count));
  return BT_OK;
}

// d_z = r * (dxhat - mean(dxhat) - xhat * mean(dxhat * xhat)), dxhat = d_y * scale.
// Grid-stride over rows, one warp per row; lanes keep the (d scale, d bias) partial sums
// of the columns they own; the block sums its warps in order into partials[block].
constexpr int kLnMaxCols = 1024;
__global__ void __launch_bounds__(256) ln_backward_kernel(const float* d_y, const float* z,
                                                          const float* mean, const float* rstd,
                                                          const float* scale, int rows, int n,
                                                          float* d_z, __nv_bfloat16* d_zb,
                                                          __nv_bfloat16* d_zb_lo,
                                                          float* partials, const int* count) {
  __shared__ float red[8][2 * 64];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps_total = gridDim.x * 8;
  const int live = live_rows(count, rows);
  constexpr int kPer = kLnMaxCols / 32;
  float ds[kPer], db[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) ds[i] = db[i] = 0.f;
  for (int row = blockIdx.x * 8 + warp; row < live; row += warps_total) {
    const float* dyr = d_y + (size_t)row * n;
    const float* zr = z + (size_t)row * n;
    const float mu = mean[row], r = rstd[row];
    float m1 = 0.f, m2 = 0.f;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int k = lane + 32 * i;
      if (k < n) {
        const float xhat = (zr[k] - mu) * r;
        const float dy = dyr[k];
        const float dx = dy * scale[k];
        m1 += dx;
        m2 += dx * xhat;
        ds[i] += dy * xhat;
        db[i] += dy;
      }
    }
    m1 = warp_sum(m1) / n;
    m2 = warp_sum(m2) / n;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int k = lane + 32 * i;
      if (k < n) {
        const float xhat = (zr[k] - mu) * r;
        const float dx = dyr[k] * scale[k];
        const float g = r * (dx - m1 - xhat * m2);
        if (d_z) d_z[(size_t)row * n + k] = g;
        if (d_zb) store_bf16(d_zb, d_zb_lo, (size_t)row * n + k, g);
      }
    }
  }
  if (d_zb) {  // rows [live, next 64-row boundary) of the bf16 operand: zeros
    const int end = dz_rows_end(live, rows);
    for (int row = live + blockIdx.x * 8 + warp; row < end; row += warps_total)
      for (int k = lane; k < n; k += 32) store_bf16(d_zb, d_zb_lo, (size_t)row * n + k, 0.f);
  }
  // Block reduction of the column partial sums, 64 columns at a time.
  for (int c0 = 0; c0 < n; c0 += 64) {
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int k = lane + 32 * i;
      if (k >= c0 && k < c0 + 64 && k < n) {
        red[warp][k - c0] = ds[i];
        red[warp][64 + k - c0] = db[i];
      }
    }
    __syncthreads();
    if (threadIdx.x < 128) {
      const int c = threadIdx.x & 63, which = threadIdx.x >> 6;
      if (c0 + c < n) {
        float s = 0.f;
        for (int w = 0; w < 8; ++w) s += red[w][which * 64 + c];
        partials[(size_t)blockIdx.x * 2 * n + which * n + c0 + c] = s;
      }
    }
  }
}

// Vectorised backward for n = 128 NV (NV <= 8): as ln_backward_kernel, with each row's d_y
// and z read once into registers as float4 (lane l owns float4 columns l, l + 32, ...). The
// column partial sums are reduced over the block's warps 128 columns at a time.
template <int NV>
__global__ void __launch_bounds__(256) ln_backward_vec_kernel(
    const float* d_y, const float* z, const float* mean, const float* rstd, const float* scale,
    int rows, int n, float* d_z, __nv_bfloat16* d_zb, __nv_bfloat16* d_zb_lo, float* partials,
    const int* count) {
  __shared__ float4 red[8][2][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps_total = gridDim.x * 8;
  const int live = live_rows(count, rows);
  float4 sc[NV], ds[NV], db[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    sc[i] = __ldg(reinterpret_cast<const float4*>(scale) + lane + 32 * i);
    ds[i] = db[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int row = blockIdx.x * 8 + warp; row < live; row += warps_total) {
    const float4* dyr = reinterpret_cast<const float4*>(d_y + (size_t)row * n);
    const float4* zr = reinterpret_cast<const float4*>(z + (size_t)row * n);
    const float mu = mean[row], r = rstd[row];
    float4 dy[NV], xh[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      dy[i] = dyr[lane + 32 * i];
      xh[i] = zr[lane + 32 * i];
    }
    float m1 = 0.f, m2 = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      xh[i].x = (xh[i].x - mu) * r;
      xh[i].y = (xh[i].y - mu) * r;
      xh[i].z = (xh[i].z - mu) * r;
      xh[i].w = (xh[i].w - mu) * r;
      const float dx0 = dy[i].x * sc[i].x, dx1 = dy[i].y * sc[i].y;
      const float dx2 = dy[i].z * sc[i].z, dx3 = dy[i].w * sc[i].w;
      m1 += dx0 + dx1 + dx2 + dx3;
      m2 += dx0 * xh[i].x + dx1 * xh[i].y + dx2 * xh[i].z + dx3 * xh[i].w;
      ds[i].x += dy[i].x * xh[i].x;
      ds[i].y += dy[i].y * xh[i].y;
      ds[i].z += dy[i].z * xh[i].z;
      ds[i].w += dy[i].w * xh[i].w;
      db[i].x += dy[i].x;
      db[i].y += dy[i].y;
      db[i].z += dy[i].z;
      db[i].w += dy[i].w;
    }
    m1 = warp_sum(m1) / n;
    m2 = warp_sum(m2) / n;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float4 g;
      g.x = r * (dy[i].x * sc[i].x - m1 - xh[i].x * m2);
      g.y = r * (dy[i].y * sc[i].y - m1 - xh[i].y * m2);
      g.z = r * (dy[i].z * sc[i].z - m1 - xh[i].z * m2);
      g.w = r * (dy[i].w * sc[i].w - m1 - xh[i].w * m2);
      const size_t e = (size_t)row * n + 4 * (lane + 32 * i);
      if (d_z) *reinterpret_cast<float4*>(d_z + e) = g;
      if (d_zb) store_bf16x4(d_zb, d_zb_lo, e, g);
    }
  }
  if (d_zb) {  // rows [live, next 64-row boundary) of the bf16 operand: zeros
    const int end = dz_rows_end(live, rows);
    for (int row = live + blockIdx.x * 8 + warp; row < end; row += warps_total)
#pragma unroll
      for (int i = 0; i < NV; ++i)
        store_bf16x4(d_zb, d_zb_lo, (size_t)row * n + 4 * (lane + 32 * i),
                     make_float4(0.f, 0.f, 0.f, 0.f));
  }
  // Block reduction of the column partial sums in warp order, 128 columns at a time: thread
  // t < 64 sums the d-scale float4 of lanes t (columns 4 (t + 32 i) ...), t >= 64 the d-bias.
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    __syncthreads();
    red[warp][0][lane] = ds[i];
    red[warp][1][lane] = db[i];
    __syncthreads();
    if (threadIdx.x < 64) {
      const int which = threadIdx.x >> 5, l = threadIdx.x & 31;
      float4 a = red[0][which][l];
      for (int w = 1; w < 8; ++w) {
        const float4 b = red[w][which][l];
        a.x += b.x;
        a.y += b.y;
        a.z += b.z;
        a.w += b.w;
      }
      reinterpret_cast<float4*>(partials + (size_t)blockIdx.x * 2 * n + which * n)[l + 32 * i] = a;
    }
  }
}

int launch_ln_backward(const float* d_y, const float* z, const float* mean, const float* rstd,
                       const float* scale, int rows, int n, float* d_z, __nv_bfloat16* d_zb,
                       __nv_bfloat16* d_zb_lo, float* partials, int blocks, const int* count,
                       cudaStream_t stream) {
  BT_CHECK_ARG(n <= kLnMaxCols, "layernorm width %d > %d", n, kLnMaxCols);
  const bool vec = n % 128 == 0 && (uintptr_t)d_y % 16 == 0 && (uintptr_t)z % 16 == 0 &&
                   (uintptr_t)scale % 16 == 0 && (uintptr_t)d_z % 16 == 0 &&
                   (uintptr_t)partials % 16 == 0 && (uintptr_t)d_zb % 8 == 0 &&
                   (uintptr_t)d_zb_lo % 8 == 0;
  if (vec) {
    switch (n / 128) {
#define BT_LN_BWD(NV)                                                                         \
  case NV:                                                                                    \
    ln_backward_vec_kernel<NV><<<blocks, 256, 0, stream>>>(d_y, z, mean, rstd, scale, rows, n, \
                                                           d_z, d_zb, d_zb_lo, partials,      \
                                                           count);                            \
    BT_LAUNCH_CHECK("ln_backward_vec_kernel");                                                \
    return BT_OK;
      BT_LN_BWD(1) BT_LN_BWD(2) BT_LN_BWD(3) BT_LN_BWD(4)
      BT_LN_BWD(5) BT_LN_BWD(6) BT_LN_BWD(7) BT_LN_BWD(8)
#undef BT_LN_BWD
      default: break;
    }
  }
  ln_backward_kernel<<<blocks, 256, 0, stream>>>(d_y, z, mean, rstd, scale, rows, n, d_z, d_zb,
                                                 d_zb_lo, partials, count);
  BT_LAUNCH_CHECK("ln_backward_kernel");
  return BT_OK;
}

// ---- gradient reduction + global norm ---------------------------------------------------
__device__ __forceinline__ double block_sum_d(double v, double* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum_d(v);
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  double s = 0.0;
  if (threadIdx.x == 0) {
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += sh[w];
  }
  __syncthreads();
  return s;  // valid in thread 0
}

int count_reduce_chunks(const Segment* segs, int num_segments) {
  int n = 0;
  for (int i = 0; i < num_segments; ++i)
    n += ceil_div(segs[i].len, reduce_chunk_len(segs[i].len, segs[i].nsplit));
  return n;
}

void build_reduce_chunks(const Segment* segs, int num_segments, ReduceChunk* out, int* count) {
  int n = 0;
  for (int i = 0; i < num_segments; ++i) {
    const int c = reduce_chunk_len(segs[i].len, segs[i].nsplit);
    for (int b = 0; b < segs[i].len; b += c)
      out[n++] = {i, b, b + c < segs[i].len ? b + c : segs[i].len};
  }
  *count = n;
}

// Wide chunks (one or more 1024-element pieces): per piece, each thread sums the splits of 4
// elements spaced by the block size, eight splits at a time (32 independent loads in flight
// per thread), in split order.
// Tall chunks (many splits, kTallChunk elements): warp w sums splits w, w + 8, ... of the
// lane's element, then the eight warp sums are added in warp order.
// Narrow segments (fewer elements than a warp has lanes per split pass, e.g. the per-block
// partial sums of the gaussian scale): one warp per element, lanes striding over the
// splits, combined by a fixed shuffle tree. Both orders are fixed, so the result is
// deterministic.
__global__ void __launch_bounds__(256, 4) reduce_segments_kernel(const Segment* segs,
                                                              const ReduceChunk* chunks,
                                                              float* grads,
                                                              double* norm_partials) {
  __shared__ double sh[8];
  pdl_trigger();
  pdl_wait();
  const ReduceChunk ch = chunks[blockIdx.x];
  const Segment sg = segs[ch.seg];
  double sq = 0.0;
  if (sg.len < 256) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = ch.begin + warp; i < ch.end; i += 8) {
      float a = 0.f;
      for (int k = lane; k < sg.nsplit; k += 32) a += __ldg(sg.src + (size_t)k * sg.stride + i);
      a = warp_sum(a);
      if (lane == 0) {
        grads[sg.dst + i] = a;
        sq += (double)a * (double)a;
      }
    }
  } else if (sg.nsplit >= kTallSplits) {
    __shared__ float tall[8][kTallChunk];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int i = ch.begin + lane;
    float a = 0.f;
    if (i < ch.end) {
      int k = warp;
      for (; k + 56 < sg.nsplit; k += 64) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = __ldg(sg.src + (size_t)(k + 8 * u) * sg.stride + i);
#pragma unroll
        for (int u = 0; u < 8; ++u) a += v[u];
      }
      for (; k < sg.nsplit; k += 8) a += __ldg(sg.src + (size_t)k * sg.stride + i);
    }
    tall[warp][lane] = a;
    __syncthreads();
    if (warp == 0 && i < ch.end) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) s += tall[w][lane];
      grads[sg.dst + i] = s;
      sq = (double)s * (double)s;
    }
  } else {
    // one kReduceChunk piece at a time (a block may own several consecutive pieces)
    constexpr int kPer = kReduceChunk / 256;
    for (int c0 = ch.begin; c0 < ch.end; c0 += kReduceChunk) {
      const int c1 = min(ch.end, c0 + kReduceChunk);
      float acc[kPer];
#pragma unroll
      for (int e = 0; e < kPer; ++e) acc[e] = 0.f;
      int k = 0;
      for (; k + 8 <= sg.nsplit; k += 8) {
        float v[8][kPer];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float* src = sg.src + (size_t)(k + u) * sg.stride;
#pragma unroll
          for (int e = 0; e < kPer; ++e) {
            const int i = c0 + threadIdx.x + e * 256;
            v[u][e] = (i < c1) ? __ldg(src + i) : 0.f;
          }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
#pragma unroll
          for (int e = 0; e < kPer; ++e) acc[e] += v[u][e];
      }
      for (; k < sg.nsplit; ++k) {
        const float* src = sg.src + (size_t)k * sg.stride;
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
          const int i = c0 + threadIdx.x + e * 256;
          if (i < c1) acc[e] += __ldg(src + i);
        }
      }
#pragma unroll
      for (int e = 0; e < kPer; ++e) {
        const int i = c0 + threadIdx.x + e * 256;
        if (i < c1) {
          grads[sg.dst + i] = acc[e];
          sq += (double)acc[e] * (double)acc[e];
        }
      }
    }
  }
  if (norm_partials) {
    const double t = block_sum_d(sq, sh);
    if (threadIdx.x == 0) norm_partials[blockIdx.x] = t;
  }
}

int launch_reduce_segments(const Segment* segs, const ReduceChunk* chunks, int num_chunks,
                           float* grads, double* norm_partials, cudaStream_t stream) {
  if (num_chunks <= 0) return BT_OK;
  BT_CUDA(launch_pdl(reduce_segments_kernel, dim3(num_chunks), dim3(256), 0, stream, segs,
                     chunks, grads, norm_partials));
  return BT_OK;
}

__global__ void __launch_bounds__(256) sumsq_kernel(const float* g, int64_t n, double* out) {
  __shared__ double sh[8];
  const int64_t per = ceil_div64(n, kNormBlocks);
  const int64_t b = blockIdx.x * per, e = min(n, b + per);
  double sq = 0.0;
  for (int64_t i = b + threadIdx.x; i < e; i += blockDim.x) sq += (double)g[i] * (double)g[i];
  const double t = block_sum_d(sq, sh);
  if (threadIdx.x == 0) out[blockIdx.x] = t;
}

int launch_sumsq(const float* g, int64_t n, double* norm_partials, cudaStream_t stream) {
  sumsq_kernel<<<kNormBlocks, 256, 0, stream>>>(g, n, norm_partials);
  BT_LAUNCH_CHECK("sumsq_kernel");
  return BT_OK;
}

// ---- clip_by_global_norm + adam + apply_updates ------------------------------------------
// optax: g_norm = ||g||; g <- g if g_norm < max_norm else (g / g_norm) * max_norm;
// mu = (1-b1) g + b1 mu; nu = (1-b2) g^2 + b2 nu; count += 1;
// p += -lr * (mu / (1 - b1^count)) / (sqrt(nu / (1 - b2^count) + eps_root) + eps).
// Every block sums the norm partials itself, in index order (no grid-wide sync needed).
// The moments follow optax's operation order with separately rounded products and sums; the
// per-step constants (1 / g_norm, 1 / (1 - b1^count), 1 / (1 - b2^count)) are formed once per
// block, and the per-element square root and quotient use the hardware approximations
// (sqrt.approx, __fdividef; ~2 ulp), so an element costs a few instructions instead of three
// correctly rounded divisions and a square root. The result agrees with the reference's
// float32 step to ~1e-7 relative in the update.
__device__ __forceinline__ float sqrt_approx(float x) {
  float y;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(256) adam_kernel(AdamParams p) {
  __shared__ double sh[8];
  __shared__ float s_norm;
  pdl_trigger();
  pdl_wait();
  double part = 0.0;
  for (int i = threadIdx.x; i < p.num_norm_partials; i += blockDim.x) part += p.norm_partials[i];
  // fixed-order block sum: thread-strided partial sums, then warps in order
  const double total = block_sum_d(part, sh);
  if (threadIdx.x == 0) s_norm = (float)sqrt(total);
  __syncthreads();
  const float g_norm = s_norm;
  const bool clip = !(g_norm < p.max_norm);
  const int count = (p.count ? *p.count : 0) + p.step + 1;
  const float bc1 = __fsub_rn(1.f, powf(p.b1, (float)count));
  const float bc2 = __fsub_rn(1.f, powf(p.b2, (float)count));
  const float omb1 = __fsub_rn(1.f, p.b1), omb2 = __fsub_rn(1.f, p.b2);
  const float inv_norm = 1.f / g_norm, inv_bc1 = 1.f / bc1, inv_bc2 = 1.f / bc2;
  auto step = [&](float g, float& prm, float& m, float& v) {
    if (clip) g = __fmul_rn(__fmul_rn(g, inv_norm), p.max_norm);
    m = __fadd_rn(__fmul_rn(omb1, g), __fmul_rn(p.b1, m));
    v = __fadd_rn(__fmul_rn(omb2, __fmul_rn(g, g)), __fmul_rn(p.b2, v));
    const float mh = __fmul_rn(m, inv_bc1);
    const float vh = __fmul_rn(v, inv_bc2);
    const float den = __fadd_rn(sqrt_approx(__fadd_rn(vh, p.eps_root)), p.eps);
    const float u = __fmul_rn(-p.lr, __fdividef(mh, den));
    prm = __fadd_rn(prm, u);
  };
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  // four elements per thread and step as float4s (all loads before any store) when every
  // buffer allows it, the remainder past the last multiple of 4 one by one
  const uintptr_t a16 = (uintptr_t)p.params | (uintptr_t)p.mu | (uintptr_t)p.nu |
                        (uintptr_t)p.grads;
  const uintptr_t a8 = (uintptr_t)p.shadow | (uintptr_t)p.shadow_lo;
  const bool vec = (a16 & 15) == 0 && (a8 & 7) == 0;
  const int64_t n4 = vec ? p.n / 4 : 0;
  // two float4 groups per thread and iteration: eight 16-byte loads in flight per thread
  auto update4 = [&](int64_t q, float4 g, float4 prm, float4 m, float4 v) {
    step(g.x, prm.x, m.x, v.x);
    step(g.y, prm.y, m.y, v.y);
    step(g.z, prm.z, m.z, v.z);
    step(g.w, prm.w, m.w, v.w);
    reinterpret_cast<float4*>(p.params)[q] = prm;
    reinterpret_cast<float4*>(p.mu)[q] = m;
    reinterpret_cast<float4*>(p.nu)[q] = v;
    if (p.shadow) store_bf16x4(p.shadow, p.shadow_lo, 4 * q, prm);
    if (p.npush) {
      bool fp32 = true;
      for (int k = 0; k < p.nskip; ++k)
        if (4 * q >= p.skip_lo[k] && 4 * q < p.skip_hi[k]) fp32 = false;
      for (int r = 0; r < p.npush; ++r) {
        if (fp32) reinterpret_cast<float4*>(p.push_params[r])[q] = prm;
        if (p.push_shadow[r]) store_bf16x4(p.push_shadow[r], p.push_shadow_lo[r], 4 * q, prm);
      }
    }
  };
  int64_t q = first;
  for (; q + stride < n4; q += 2 * stride) {
    const int64_t q2 = q + stride;
    const float4 g = __ldg(reinterpret_cast<const float4*>(p.grads) + q);
    const float4 g2 = __ldg(reinterpret_cast<const float4*>(p.grads) + q2);
    const float4 prm = reinterpret_cast<const float4*>(p.params)[q];
    const float4 prm2 = reinterpret_cast<const float4*>(p.params)[q2];
    const float4 m = reinterpret_cast<const float4*>(p.mu)[q];
    const float4 m2 = reinterpret_cast<const float4*>(p.mu)[q2];
    const float4 v = reinterpret_cast<const float4*>(p.nu)[q];
    const float4 v2 = reinterpret_cast<const float4*>(p.nu)[q2];
    update4(q, g, prm, m, v);
    update4(q2, g2, prm2, m2, v2);
  }
  for (; q < n4; q += stride) {
    update4(q, __ldg(reinterpret_cast<const float4*>(p.grads) + q),
            reinterpret_cast<const float4*>(p.params)[q], reinterpret_cast<const float4*>(p.mu)[q],
            reinterpret_cast<const float4*>(p.nu)[q]);
  }
  for (int64_t i = 4 * n4 + first; i < p.n; i += stride) {
    float prm = p.params[i], m = p.mu[i], v = p.nu[i];
    step(p.grads[i], prm, m, v);
    p.params[i] = prm;
    p.mu[i] = m;
    p.nu[i] = v;
    if (p.shadow) store_bf16(p.shadow, p.shadow_lo, i, prm);
    bool fp32 = true;
    for (int k = 0; k < p.nskip; ++k)
      if (i >= p.skip_lo[k] && i < p.skip_hi[k]) fp32 = false;
    for (int r = 0; r < p.npush; ++r) {
      if (fp32) p.push_params[r][i] = prm;
      if (p.push_shadow[r]) store_bf16(p.push_shadow[r], p.push_shadow_lo[r], i, prm);
    }
  }
  // the pushed parameters reach the peers' memory before this thread is done
  if (p.npush) __threadfence_system();
}

int launch_adam(const AdamParams& p, cudaStream_t stream) {
  BT_CUDA(launch_pdl(adam_kernel, dim3(4 * kNumSMs), dim3(256), 0, stream, p));
  return BT_OK;
}

__global__ void __launch_bounds__(256) sumsq_chunks_kernel(const float* g, int64_t n,
                                                           double* out) {
  __shared__ double sh[8];
  const int64_t b = (int64_t)blockIdx.x * kNormChunk;
  const int64_t e = min(n, b + kNormChunk);
  double sq = 0.0;
  for (int64_t i = b + threadIdx.x; i < e; i += blockDim.x) sq += (double)g[i] * (double)g[i];
  const double t = block_sum_d(sq, sh);
  if (threadIdx.x == 0) out[blockIdx.x] = t;
}

int launch_sumsq_chunks(const float* g, int64_t n, double* out, cudaStream_t stream) {
  const int64_t chunks = ceil_div64(n, kNormChunk);
  if (chunks <= 0) return BT_OK;
  sumsq_chunks_kernel<<<(unsigned)chunks, 256, 0, stream>>>(g, n, out);
  BT_LAUNCH_CHECK("sumsq_chunks_kernel");
  return BT_OK;
}

__global__ void increment_kernel(int* count, int by) { *count += by; }

int launch_increment(int* count, int by, cudaStream_t stream) {
  increment_kernel<<<1, 1, 0, stream>>>(count, by);
  BT_LAUNCH_CHECK("increment_kernel");
  return BT_OK;
}

// ---- statistics --------------------------------------------------------------------------
// One warp per statistic: lanes stride over the block partials, then a fixed shuffle tree.
__global__ void stat_reduce_kernel(const double* partials, int blocks, double* out) {
  pdl_trigger();
  pdl_wait();
  const int s = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (s >= kNumStatSums) return;
  double t = 0.0;
  for (int b = lane; b < blocks; b += 32) t += partials[(size_t)b * kNumStatSums + s];
  t = warp_sum_d(t);
  if (lane == 0) out[s] = t;
}

int launch_stat_reduce(const double* partials, int blocks, double* out, cudaStream_t stream) {
  BT_CUDA(launch_pdl(stat_reduce_kernel, dim3(1), dim3(32 * kNumStatSums), 0, stream, partials,
                     blocks, out));
  return BT_OK;
}

// stats[i] = the eight logged values of boonta/algorithms/ppo.py:170-179 for minibatch i.
__global__ void stat_finalize_kernel(const double* sums, int count, float inv_mb, float* stats) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count) return;
  const double* s = sums + (size_t)i * kNumStatSums;
  const double inv = (double)inv_mb;
  float* o = stats + (size_t)i * BT_NUM_STATS;
  o[0] = (float)(-s[0] * inv);
  o[1] = (float)(s[1] * inv);
  o[2] = (float)(s[2] * inv);
  o[3] = (float)(s[3] * inv);
  o[4] = (float)(s[4] * inv);
  o[5] = (float)(s[5] * inv);
  const double mr = s[6] * inv, var_res = fmax(s[7] * inv - mr * mr, 0.0);
  const double mR = s[8] * inv, var_R = fmax(s[9] * inv - mR * mR, 0.0);
  o[6] = (float)(1.0 - var_res / (var_R + 1e-8));
  o[7] = (float)(s[10] * inv);
}

int launch_stat_finalize(const double* sums, int count, float inv_mb, float* stats,
                         cudaStream_t stream) {
  if (count <= 0) return BT_OK;
  stat_finalize_kernel<<<ceil_div(count, 128), 128, 0, stream>>>(sums, count, inv_mb, stats);
  BT_LAUNCH_CHECK("stat_finalize_kernel");
  return BT_OK;
}

// ---- advantage normalisation (ppo.py:220-221) ----------------------------------------------
__global__ void __launch_bounds__(256) adv_moments_kernel(const float* a, int64_t n,
                                                          double* partials) {
  __shared__ double sh[8];
  const int64_t per = ceil_div64(n, kNormBlocks);
  const int64_t b = blockIdx.x * per, e = min(n, b + per);
  double s = 0.0, s2 = 0.0;
  for (int64_t i = b + threadIdx.x; i < e; i += blockDim.x) {
    s += a[i];
    s2 += (double)a[i] * a[i];
  }
  const double t = block_sum_d(s, sh);
  const double t2 = block_sum_d(s2, sh);
  if (threadIdx.x == 0) {
    partials[2 * blockIdx.x] = t;
    partials[2 * blockIdx.x + 1] = t2;
  }
}

int launch_adv_moments(const float* adv, int64_t n, double* partials, cudaStream_t stream) {
  adv_moments_kernel<<<kNormBlocks, 256, 0, stream>>>(adv, n, partials);
  BT_LAUNCH_CHECK("adv_moments_kernel");
  return BT_OK;
}

__global__ void adv_normalize_kernel(float* a, int64_t n, const double* partials, int np,
                                     double total) {
  __shared__ float s_mean, s_den;
  if (threadIdx.x == 0) {
    double s = 0.0, s2 = 0.0;
    for (int i = 0; i < np; ++i) {
      s += partials[2 * i];
      s2 += partials[2 * i + 1];
    }
    const double mean = s / total;
    const double var = fmax(s2 / total - mean * mean, 0.0);
    s_mean = (float)mean;
    s_den = (float)sqrt(var) + 1e-8f;
  }
  __syncthreads();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    a[i] = (a[i] - s_mean) / s_den;
}

int launch_adv_normalize(float* adv, int64_t n, const double* partials, int num_partials,
                         double total, cudaStream_t stream) {
  adv_normalize_kernel<<<2 * kNumSMs, 256, 0, stream>>>(adv, n, partials, num_partials, total);
  BT_LAUNCH_CHECK("adv_normalize_kernel");
  return BT_OK;
}

// ---- multi-GPU minibatch split ---------------------------------------------------------
// Global flat index i = t * N_global + n_global (the flatten order of ppo.py:226-228 over
// the global env axis). Rank r owns n_global in [r*N, (r+1)*N); its local flat index is
// t * N + (n_global - r*N). For env permutations (recurrent) t is 0. One block per slice,
// order-preserving compaction with a block-wide scan.
__global__ void __launch_bounds__(1024) local_indices_kernel(const int* perm, int slice_len,
                                                             int local_units, int rank,
                                                             int global_units, int capacity,
                                                             int* local_idx, int* counts,
                                                             int* err) {
  __shared__ int warp_tot[32];
  __shared__ int base_s;
  const int slice = blockIdx.x;
  const int* src = perm + (size_t)slice * slice_len;
  int* dst = local_idx + (size_t)slice * capacity;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) base_s = 0;
  __syncthreads();
  for (int c0 = 0; c0 < slice_len; c0 += 1024) {
    const int i = c0 + threadIdx.x;
    int local = -1;
    if (i < slice_len) {
      const int g = src[i];
      const int t = g / global_units, ng = g - t * global_units;
      if (ng / local_units == rank) local = t * local_units + (ng - rank * local_units);
    }
    const unsigned ballot = __ballot_sync(0xffffffffu, local >= 0);
    const int before = __popc(ballot & ((1u << lane) - 1u));
    if (lane == 0) warp_tot[warp] = __popc(ballot);
    __syncthreads();
    int off = 0;
    for (int w = 0; w < warp; ++w) off += warp_tot[w];
    const int pos = base_s + off + before;
    if (local >= 0 && pos < capacity) dst[pos] = local;
    __syncthreads();
    if (threadIdx.x == 0) {
      int tot = 0;
      for (int w = 0; w < 32; ++w) tot += warp_tot[w];
      base_s += tot;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const int n = base_s;
    counts[slice] = n < capacity ? n : capacity;
    if (n > capacity && err) atomicExch(err, 2);
  }
  // Pad the tail with a valid index so gathers of padding rows stay in bounds.
  const int n = min(base_s, capacity);
  for (int i = n + threadIdx.x; i < capacity; i += 1024) dst[i] = 0;
}

int launch_local_indices(const int* perm, int num_slices, int slice_len, int /*units_per_row*/,
                         int local_units, int rank, int global_units, int capacity,
                         int* local_idx, int* counts, int* err, cudaStream_t stream) {
  local_indices_kernel<<<num_slices, 1024, 0, stream>>>(perm, slice_len, local_units, rank,
                                                        global_units, capacity, local_idx,
                                                        counts, err);
  BT_LAUNCH_CHECK("local_indices_kernel");
  return BT_OK;
}

// ---- head weight gradients ------------------------------------------------------------------
// [F + 1, n] split partials of [f, 1]^T d for a narrow output gradient d (n <= NMAX <= 64):
// one thread per input feature k (k == F is the constant-one row whose sum is the bias
// gradient), the rows of a split staged 64 at a time in shared memory; each thread keeps
// its n accumulators in registers and sums rows in order.
template <int NMAX, int ACT>
__global__ void __launch_bounds__(128) skinny_dw_kernel(const float* f, int F,
                                                        const float* d, int n, int rows,
                                                        const int* count, int rows_per_split,
                                                        float* out) {
  __shared__ __align__(16) float ds[64][NMAX];
  const int k = blockIdx.x * 128 + threadIdx.x;
  const int live = live_rows(count, rows);
  const int r0 = blockIdx.y * rows_per_split;
  const int r1 = min(live, r0 + rows_per_split);
  float acc[NMAX];
#pragma unroll
  for (int j = 0; j < NMAX; ++j) acc[j] = 0.f;
  for (int rb = r0; rb < r1; rb += 64) {
    __syncthreads();
    for (int i = threadIdx.x; i < 64 * NMAX; i += 128) {
      const int rr = i / NMAX, j = i - rr * NMAX;
      ds[rr][j] = (rb + rr < r1 && j < n) ? d[(size_t)(rb + rr) * n + j] : 0.f;
    }
    __syncthreads();
    const int nr = min(64, r1 - rb);
    // eight rows' loads in flight before their FMAs
    for (int r8 = 0; r8 < nr; r8 += 8) {
      float fk[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int rr = r8 + u;
        fk[u] = (rr < nr && k < F) ? __ldg(f + (size_t)(rb + rr) * F + k)
                                   : ((rr < nr && k == F) ? 1.f : 0.f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (k < F) fk[u] = act_fwd<ACT>(fk[u]);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if constexpr (NMAX % 4 == 0) {
#pragma unroll
          for (int j = 0; j < NMAX; j += 4) {  // broadcast float4 reads of the row's d
            const float4 dd = *reinterpret_cast<const float4*>(&ds[r8 + u][j]);
            acc[j] = fmaf(fk[u], dd.x, acc[j]);
            acc[j + 1] = fmaf(fk[u], dd.y, acc[j + 1]);
            acc[j + 2] = fmaf(fk[u], dd.z, acc[j + 2]);
            acc[j + 3] = fmaf(fk[u], dd.w, acc[j + 3]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < NMAX; ++j) acc[j] = fmaf(fk[u], ds[r8 + u][j], acc[j]);
        }
      }
    }
  }
  if (k <= F) {
    float* o = out + ((size_t)blockIdx.y * (F + 1) + k) * n;
    for (int j = 0; j < n; ++j) o[j] = acc[j];
  }
}

template <int NMAX>
void launch_skinny_n(dim3 grid, const float* f, int F, int act, const float* d, int n, int rows,
                     const int* count, int rps, float* out, cudaStream_t stream) {
  switch (act) {
    case BT_ACT_TANH:
      skinny_dw_kernel<NMAX, BT_ACT_TANH><<<grid, 128, 0, stream>>>(f, F, d, n, rows, count, rps, out);
      break;
    case BT_ACT_RELU:
      skinny_dw_kernel<NMAX, BT_ACT_RELU><<<grid, 128, 0, stream>>>(f, F, d, n, rows, count, rps, out);
      break;
    case BT_ACT_SILU:
      skinny_dw_kernel<NMAX, BT_ACT_SILU><<<grid, 128, 0, stream>>>(f, F, d, n, rows, count, rps, out);
      break;
    default:
      skinny_dw_kernel<NMAX, BT_ACT_NONE><<<grid, 128, 0, stream>>>(f, F, d, n, rows, count, rps, out);
      break;
  }
}

int launch_skinny_dw(const float* f, int F, int act, const float* d, int n, int rows,
                     const int* count, int splits, float* out, cudaStream_t stream) {
  const int rps = ceil_div(rows, splits);
  dim3 grid(ceil_div(F + 1, 128), splits);
  if (n <= 1) {
    launch_skinny_n<1>(grid, f, F, act, d, n, rows, count, rps, out, stream);
  } else if (n <= 8) {
    launch_skinny_n<8>(grid, f, F, act, d, n, rows, count, rps, out, stream);
  } else if (n <= 16) {
    launch_skinny_n<16>(grid, f, F, act, d, n, rows, count, rps, out, stream);
  } else if (n <= 32) {
    launch_skinny_n<32>(grid, f, F, act, d, n, rows, count, rps, out, stream);
  } else if (n <= 48) {
    launch_skinny_n<48>(grid, f, F, act, d, n, rows, count, rps, out, stream);
  } else {
    BT_CHECK_ARG(n <= 64, "skinny dW with %d outputs", n);
    launch_skinny_n<64>(grid, f, F, act, d, n, rows, count, rps, out, stream);
  }
  BT_LAUNCH_CHECK("skinny_dw_kernel");
  return BT_OK;
}

// ---- bf16 operand buffers of the tensor-core path ------------------------------------------
// Minibatch gather of observation rows into a bf16 [rows, ld] operand: columns [0, d) the
// observation, column d = 1 (the bias column of the dW GEMM), (d, ld) zero. One warp per
// row (coalesced along the row). With `table` set, each gathered bf16 row is also stored at
// its own index in the table [*, ld] (the update's bf16 copy of the rollout, filled by the
// first epoch's minibatches, which together read every row once).
__global__ void gather_bf16_kernel(const float* obs, const int* idx, int rows, int d, int ld,
                                   __nv_bfloat16* out, __nv_bfloat16* out_lo, const int* count,
                                   __nv_bfloat16* table) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();
  if (row >= live_rows(count, rows)) return;
  const int r = idx ? idx[row] : row;
  const float* src = obs + (size_t)r * d;
  __nv_bfloat16* trow = table ? table + (size_t)r * ld : nullptr;
  int k0 = 0;
  if ((d & 3) == 0 && (ld & 3) == 0) {
    // float4 loads and 8-byte bf16 stores, four chunks in flight per lane
    const int q4 = d / 4;
    const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll 4
    for (int q = lane; q < q4; q += 32) {
      const float4 v = __ldg(s4 + q);
      store_bf16x4(out, out_lo, (size_t)row * ld + 4 * q, v);
      if (trow) store_bf16x4(trow, nullptr, 4 * q, v);
    }
    k0 = d;
  }
  for (int k = k0 + lane; k < ld; k += 32) {
    const float v = k < d ? src[k] : (k == d ? 1.f : 0.f);
    store_bf16(out, out_lo, (size_t)row * ld + k, v);
    if (trow) store_bf16(trow, nullptr, k, v);
  }
}

// fp32 rows [rows, d] (row stride d) as split bf16 pairs [rows, d]: rows below the live count
// converted, rows from it to the next 64-row boundary zero (the tensor-core dW GEMMs read whole
// 64-row blocks). One warp per row.
__global__ void split_rows_bf16_kernel(const float* src, int rows, int d, __nv_bfloat16* out,
                                       __nv_bfloat16* out_lo, const int* count) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();
  const int live = live_rows(count, rows);
  if (row >= dz_rows_end(live, rows)) return;
  const bool on = row < live;
  const float* r = src + (size_t)row * d;
  if ((d & 3) == 0) {
    const float4* r4 = reinterpret_cast<const float4*>(r);
    for (int q = lane; q < d / 4; q += 32)
      store_bf16x4(out, out_lo, (size_t)row * d + 4 * q,
                   on ? __ldg(r4 + q) : make_float4(0.f, 0.f, 0.f, 0.f));
  } else {
    for (int k = lane; k < d; k += 32) store_bf16(out, out_lo, (size_t)row * d + k, on ? r[k] : 0.f);
  }
}

int launch_split_rows_bf16(const float* src, int rows, int d, __nv_bfloat16* out,
                           __nv_bfloat16* out_lo, const int* count, cudaStream_t stream) {
  if (rows <= 0) return BT_OK;
  BT_CUDA(launch_pdl(split_rows_bf16_kernel, dim3(ceil_div(rows * 32, 256)), dim3(256), 0,
                     stream, src, rows, d, out, out_lo, count));
  return BT_OK;
}

// Rows idx[r] of a bf16 table [*, ld] (ld a multiple of 8) copied to out [rows, ld], one warp
// per row in 16-byte chunks; rows past the live count are left as they are.
__global__ void gather_rows_bf16_kernel(const __nv_bfloat16* src, const int* idx, int rows,
                                        int ld, __nv_bfloat16* out, const int* count) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();
  if (row >= live_rows(count, rows)) return;
  const uint4* s = reinterpret_cast<const uint4*>(src + (size_t)idx[row] * ld);
  uint4* o = reinterpret_cast<uint4*>(out + (size_t)row * ld);
  const int q8 = ld / 8;
#pragma unroll 4
  for (int q = lane; q < q8; q += 32) o[q] = __ldg(s + q);
}

int launch_gather_rows_bf16(const __nv_bfloat16* src, const int* idx, int rows, int ld,
                            __nv_bfloat16* out, const int* count, cudaStream_t stream) {
  if (rows <= 0) return BT_OK;
  BT_CHECK_ARG(ld % 8 == 0, "gather_rows_bf16: row length %d is not a multiple of 8", ld);
  BT_CUDA(launch_pdl(gather_rows_bf16_kernel, dim3(ceil_div(rows * 32, 256)), dim3(256), 0,
                     stream, src, idx, rows, ld, out, count));
  return BT_OK;
}

int launch_gather_bf16(const float* obs, const int* idx, int rows, int d, int ld,
                       __nv_bfloat16* out, __nv_bfloat16* out_lo, const int* count,
                       cudaStream_t stream, __nv_bfloat16* table) {
  if (rows <= 0) return BT_OK;
  BT_CUDA(launch_pdl(gather_bf16_kernel, dim3(ceil_div(rows * 32, 256)), dim3(256), 0, stream,
                     obs, idx, rows, d, ld, out, out_lo, count, table));
  return BT_OK;
}

// Columns [n, ld) of a bf16 [rows, ld] buffer: column n = 1, the rest 0 (set once; the
// forward epilogues only write columns < n).
__global__ void ones_column_kernel(__nv_bfloat16* buf, int rows, int n, int ld, float one) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int w = ld - n;
  if (i >= (int64_t)rows * w) return;
  const int64_t row = i / w;
  const int c = (int)(i - row * w);
  buf[row * ld + n + c] = __float2bfloat16_rn(c == 0 ? one : 0.f);
}

int launch_ones_column(__nv_bfloat16* buf, int rows, int n, int ld, float one,
                       cudaStream_t stream) {
  const int64_t total = (int64_t)rows * (ld - n);
  if (total <= 0) return BT_OK;
  ones_column_kernel<<<(unsigned)ceil_div64(total, 256), 256, 0, stream>>>(buf, rows, n, ld, one);
  BT_LAUNCH_CHECK("ones_column_kernel");
  return BT_OK;
}

// Zero rows [live, rows) of a bf16 [rows, ld] buffer: the tensor-core dW GEMMs read whole
// 64-row K blocks, so the padding rows of a rank's minibatch must contribute nothing.
__global__ void zero_tail_rows_kernel(__nv_bfloat16* buf, __nv_bfloat16* lo, int rows, int ld,
                                      const int* count) {
  const int live = live_rows(count, rows);
  const int64_t n = (int64_t)(rows - live) * ld;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    buf[(int64_t)live * ld + i] = __float2bfloat16_rn(0.f);
    if (lo) lo[(int64_t)live * ld + i] = __float2bfloat16_rn(0.f);
  }
}

int launch_zero_tail_rows(__nv_bfloat16* buf, __nv_bfloat16* lo, int rows, int ld,
                          const int* count, cudaStream_t stream) {
  zero_tail_rows_kernel<<<kNumSMs, 256, 0, stream>>>(buf, lo, rows, ld, count);
  BT_LAUNCH_CHECK("zero_tail_rows_kernel");
  return BT_OK;
}

__global__ void to_bf16_kernel(const float* in, __nv_bfloat16* out, __nv_bfloat16* out_lo,
                               int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    store_bf16(out, out_lo, i, in[i]);
}

int launch_to_bf16(const float* in, __nv_bfloat16* out, __nv_bfloat16* out_lo, int64_t n,
                   cudaStream_t stream) {
  to_bf16_kernel<<<2 * kNumSMs, 256, 0, stream>>>(in, out, out_lo, n);
  BT_LAUNCH_CHECK("to_bf16_kernel");
  return BT_OK;
}

}  // namespace bt
