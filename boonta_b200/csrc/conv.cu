// Conv 3x3, stride 1, SAME padding (flax nn.Conv(features, (3, 3), padding="SAME") in the
// MinAtar-shaped torso) on NHWC observation rows: the forward (z = conv + bias and
// h = act(z)) and the weight gradient over a minibatch. The layer is always the first of
// its tower, so it has no input gradient.
//
// Both kernels stage whole images of the minibatch in shared memory, channel-planar with
// a zero halo (kConvRows images per step, [image][channel][(H + 2) * (W + 2)]), so every
// patch value is a plain shared-memory read and a warp reading one tap of consecutive
// pixels touches consecutive words:
//   forward: one thread per output pixel and group of images computes all NC output
//            channels of that pixel in those images (the weights [9C + 1][NC] are
//            broadcast float4 reads), z and h stored as float4s;
//   dW:      thread t owns patch element k = t % (9C + 1) (k = (dy * 3 + dx) * C + ci,
//            and k = 9C the bias "1") in image phase t / (9C + 1), accumulating
//            sum_pixels patch[k] * dz[c] for all NC channels in registers; the phases
//            (interleaved images) are added in order at the end, one [9C + 1][Cout]
//            partial per block (reduced by the split-K reduction in a fixed order).
// Weight layout: the [9C + 1, Cout] kernel+bias block of the flat parameters (row k as
// above, bias row last), as flax's HWIO kernel flattened.
#include "common.cuh"
#include "kernels.cuh"

namespace bt {

constexpr int kConvThreads = 256;
constexpr int kConvRows = 8;  // images staged per step

struct ConvGeom {
  int H, W, C, Cout;
  __device__ __forceinline__ int hw() const { return H * W; }
  __device__ __forceinline__ int img() const { return (H + 2) * (W + 2) * C; }  // padded
};

// Interior of images [r0, r0 + kConvRows) into x_s (halo already zero), rows past `live`
// as zeros. One thread per (image, pixel): the pixel's C channels are contiguous in the
// observation row.
__device__ __forceinline__ void stage_images(const float* obs, const int* idx, int r0, int live,
                                             const ConvGeom& g, float* x_s) {
  const int hw = g.hw(), wp = g.W + 2, plane = (g.H + 2) * wp;
  for (int i = threadIdx.x; i < kConvRows * hw; i += kConvThreads) {
    const int rr = i / hw, pix = i - rr * hw;
    const int y = pix / g.W, x = pix - y * g.W;
    const int row = r0 + rr;
    float* dst = x_s + rr * g.img() + (y + 1) * wp + (x + 1);
    if (row < live) {
      const float* src = obs + ((size_t)(idx ? idx[row] : row) * hw + pix) * g.C;
      for (int ci = 0; ci < g.C; ++ci) dst[ci * plane] = __ldg(src + ci);
    } else {
      for (int ci = 0; ci < g.C; ++ci) dst[ci * plane] = 0.f;
    }
  }
}

// Forward: thread (pixel p, image group) computes all NC channels of pixel p for IPT
// images of the staged step at once, so each weight row read (broadcast float4s) feeds
// IPT x NC FMAs.
template <int NC, int ACT>
__global__ void __launch_bounds__(kConvThreads) conv_forward_kernel(
    const float* obs, const int* idx, int rows, const int* count, ConvGeom g, const float* w,
    float* z, float* h, __nv_bfloat16* hb, __nv_bfloat16* hb_lo, int ldhb) {
  constexpr int IPT = NC <= 16 ? 4 : 2;  // images per thread
  constexpr int kGroups = kConvRows / IPT;
  extern __shared__ __align__(16) float sm[];
  float* x_s = sm;
  float* w_s = x_s + kConvRows * g.img();  // [9C + 1][NC], channels past Cout zero
  const int kin = 9 * g.C, hw = g.hw(), wp = g.W + 2, plane = (g.H + 2) * wp;
  for (int i = threadIdx.x; i < (kin + 1) * NC; i += kConvThreads) {
    const int k = i / NC, c = i - k * NC;
    w_s[i] = c < g.Cout ? w[(size_t)k * g.Cout + c] : 0.f;
  }
  for (int i = threadIdx.x; i < kConvRows * g.img(); i += kConvThreads) x_s[i] = 0.f;
  __syncthreads();
  const int live = live_rows(count, rows);
  for (int r0 = blockIdx.x * kConvRows; r0 < live; r0 += gridDim.x * kConvRows) {
    stage_images(obs, idx, r0, live, g, x_s);
    __syncthreads();
    for (int task = threadIdx.x; task < kGroups * hw; task += kConvThreads) {
      const int grp = task / hw, pix = task - grp * hw;
      const int y = pix / g.W, x = pix - y * g.W;
      const int i0 = grp * IPT;
      float acc[IPT][NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const float b = w_s[kin * NC + c];
#pragma unroll
        for (int m = 0; m < IPT; ++m) acc[m][c] = b;
      }
      const float* xb = x_s + i0 * g.img() + y * wp + x;
#pragma unroll
      for (int dy = 0; dy < 3; ++dy)
#pragma unroll
        for (int dx = 0; dx < 3; ++dx) {
          const float* xp = xb + dy * wp + dx;
          const float* wr = w_s + ((dy * 3 + dx) * g.C) * NC;
          for (int ci = 0; ci < g.C; ++ci) {
            float v[IPT];
#pragma unroll
            for (int m = 0; m < IPT; ++m) v[m] = xp[m * g.img() + ci * plane];
#pragma unroll
            for (int c = 0; c < NC; c += 4) {
              const float4 ww = *reinterpret_cast<const float4*>(wr + ci * NC + c);
#pragma unroll
              for (int m = 0; m < IPT; ++m) {
                acc[m][c] = fmaf(v[m], ww.x, acc[m][c]);
                acc[m][c + 1] = fmaf(v[m], ww.y, acc[m][c + 1]);
                acc[m][c + 2] = fmaf(v[m], ww.z, acc[m][c + 2]);
                acc[m][c + 3] = fmaf(v[m], ww.w, acc[m][c + 3]);
              }
            }
          }
        }
#pragma unroll
      for (int m = 0; m < IPT; ++m) {
        const int row = r0 + i0 + m;
        if (row >= live) break;
        const size_t o = ((size_t)row * hw + pix) * g.Cout;
        if (g.Cout == NC) {
#pragma unroll
          for (int c = 0; c < NC; c += 4) {
            *reinterpret_cast<float4*>(z + o + c) =
                make_float4(acc[m][c], acc[m][c + 1], acc[m][c + 2], acc[m][c + 3]);
            const float4 hv =
                make_float4(act_fwd<ACT>(acc[m][c]), act_fwd<ACT>(acc[m][c + 1]),
                            act_fwd<ACT>(acc[m][c + 2]), act_fwd<ACT>(acc[m][c + 3]));
            if (h) *reinterpret_cast<float4*>(h + o + c) = hv;
            if (hb) store_bf16x4(hb, hb_lo, (size_t)row * ldhb + (size_t)pix * g.Cout + c, hv);
          }
        } else {
#pragma unroll
          for (int c = 0; c < NC; ++c)
            if (c < g.Cout) {
              z[o + c] = acc[m][c];
              const float hv = act_fwd<ACT>(acc[m][c]);
              if (h) h[o + c] = hv;
              if (hb) store_bf16(hb, hb_lo, (size_t)row * ldhb + (size_t)pix * g.Cout + c, hv);
            }
        }
      }
    }
    __syncthreads();
  }
}

template <int NC>
__global__ void __launch_bounds__(kConvThreads) conv_dw_kernel(
    const float* obs, const int* idx, int rows, const int* count, ConvGeom g, const float* dz,
    int rows_per_block, float* out) {
  extern __shared__ __align__(16) float sm[];
  float* x_s = sm;
  float* dz_s = x_s + kConvRows * g.img();  // [kConvRows * hw][NC]
  const int kin = 9 * g.C, hw = g.hw(), wp = g.W + 2;
  // thread t: patch element kslot = t % (9C + 1) in image phase t / (9C + 1)
  const int groups = kConvThreads / (kin + 1);  // image phases
  const int kslot = threadIdx.x % (kin + 1);
  const int phase = threadIdx.x / (kin + 1);
  const bool active = phase < groups;
  int koff = 0;  // offset of patch element kslot relative to the pixel's top-left tap
  if (kslot < kin) {
    const int tap = kslot / g.C, ci = kslot - tap * g.C;
    koff = ci * (g.H + 2) * wp + (tap / 3) * wp + (tap % 3);
  }
  for (int i = threadIdx.x; i < kConvRows * g.img(); i += kConvThreads) x_s[i] = 0.f;
  __syncthreads();
  float acc[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) acc[c] = 0.f;
  const int live = live_rows(count, rows);
  const int rb = blockIdx.x * rows_per_block;
  const int re = min(live, rb + rows_per_block);
  for (int r0 = rb; r0 < re; r0 += kConvRows) {
    stage_images(obs, idx, r0, re, g, x_s);
    const int nrows = min(kConvRows, re - r0);
    if (g.Cout == NC) {  // the rows' dz are one contiguous block
      const float* src = dz + (size_t)r0 * hw * NC;
      for (int i = threadIdx.x; i < nrows * hw * NC / 4; i += kConvThreads)
        reinterpret_cast<float4*>(dz_s)[i] = reinterpret_cast<const float4*>(src)[i];
    } else {
      for (int i = threadIdx.x; i < nrows * hw * NC; i += kConvThreads) {
        const int p = i / NC, c = i - p * NC;
        dz_s[i] = c < g.Cout ? dz[((size_t)r0 * hw + p) * g.Cout + c] : 0.f;
      }
    }
    __syncthreads();
    if (active) {
      // phase p takes images p, p + groups, ...; pixels in order within an image
      for (int rr = phase; rr < nrows; rr += groups) {
        const float* xi = x_s + rr * g.img() + koff;
        const float* d = dz_s + (size_t)rr * hw * NC;
        for (int y = 0; y < g.H; ++y) {
          for (int x = 0; x < g.W; ++x, d += NC) {
            const float pv = kslot < kin ? xi[y * wp + x] : 1.f;
#pragma unroll
            for (int c = 0; c < NC; c += 4) {
              const float4 dd = *reinterpret_cast<const float4*>(d + c);
              acc[c] = fmaf(pv, dd.x, acc[c]);
              acc[c + 1] = fmaf(pv, dd.y, acc[c + 1]);
              acc[c + 2] = fmaf(pv, dd.z, acc[c + 2]);
              acc[c + 3] = fmaf(pv, dd.w, acc[c + 3]);
            }
          }
        }
      }
    }
    __syncthreads();
  }
  // phases added in order: phase p's sums to shared memory, then phase 0's threads
  float* red = sm;  // [groups][9C + 1][NC] (reuses the image buffers)
  if (active) {
#pragma unroll
    for (int c = 0; c < NC; ++c) red[((size_t)phase * (kin + 1) + kslot) * NC + c] = acc[c];
  }
  __syncthreads();
  if (phase == 0) {
    float* o = out + (size_t)blockIdx.x * (kin + 1) * g.Cout + (size_t)kslot * g.Cout;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      if (c >= g.Cout) break;
      float s = 0.f;
      for (int p = 0; p < groups; ++p) s += red[((size_t)p * (kin + 1) + kslot) * NC + c];
      o[c] = s;
    }
  }
}

namespace {
int conv_nc(int cout) { return cout <= 8 ? 8 : cout <= 16 ? 16 : 32; }

size_t conv_fwd_smem(const ConvGeom& g, int nc) {
  return ((size_t)kConvRows * (g.H + 2) * (g.W + 2) * g.C + (size_t)(9 * g.C + 1) * nc) * 4;
}
size_t conv_dw_smem(const ConvGeom& g, int nc) {
  const size_t stage =
      (size_t)kConvRows * (g.H + 2) * (g.W + 2) * g.C + (size_t)kConvRows * g.H * g.W * nc;
  const size_t red = (size_t)(kConvThreads / (9 * g.C + 1)) * (9 * g.C + 1) * nc;
  return std::max(stage, red) * 4;
}

template <class Kernel>
int set_smem(Kernel k, size_t smem) {
  if (smem > 48 * 1024) BT_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  return BT_OK;
}

struct ConvOut {
  float* z;
  float* h;
  __nv_bfloat16* hb;
  __nv_bfloat16* hb_lo;
  int ldhb;
};

template <int NC, int ACT>
int launch_fwd_nc(const float* obs, const int* idx, int rows, const int* count, ConvGeom g,
                  const float* w, const ConvOut& o, cudaStream_t s) {
  const size_t smem = conv_fwd_smem(g, NC);
  BT_TRY(set_smem(conv_forward_kernel<NC, ACT>, smem));
  const int blocks = std::max(1, std::min(ceil_div(rows, kConvRows), 4 * kNumSMs));
  conv_forward_kernel<NC, ACT><<<blocks, kConvThreads, smem, s>>>(obs, idx, rows, count, g, w,
                                                                  o.z, o.h, o.hb, o.hb_lo, o.ldhb);
  BT_LAUNCH_CHECK("conv_forward_kernel");
  return BT_OK;
}

template <int NC>
int launch_fwd_act(int act, const float* obs, const int* idx, int rows, const int* count,
                   ConvGeom g, const float* w, const ConvOut& o, cudaStream_t s) {
  switch (act) {
    case BT_ACT_TANH: return launch_fwd_nc<NC, BT_ACT_TANH>(obs, idx, rows, count, g, w, o, s);
    case BT_ACT_RELU: return launch_fwd_nc<NC, BT_ACT_RELU>(obs, idx, rows, count, g, w, o, s);
    case BT_ACT_SILU: return launch_fwd_nc<NC, BT_ACT_SILU>(obs, idx, rows, count, g, w, o, s);
    default: return launch_fwd_nc<NC, BT_ACT_NONE>(obs, idx, rows, count, g, w, o, s);
  }
}
}  // namespace

int conv_dw_blocks(int rows) {
  return std::max(1, std::min(2 * kNumSMs, ceil_div(rows, 4 * kConvRows)));
}

int launch_conv_forward(const float* obs, const int* idx, int rows, const int* count, int H,
                        int W, int C, int Cout, const float* w, int act, float* z, float* h,
                        __nv_bfloat16* hb, __nv_bfloat16* hb_lo, int ldhb, cudaStream_t s) {
  BT_CHECK_ARG(Cout >= 1 && Cout <= 32, "conv: %d output channels (at most 32)", Cout);
  const ConvGeom g{H, W, C, Cout};
  BT_CHECK_ARG(conv_fwd_smem(g, conv_nc(Cout)) <= 200 * 1024, "conv: %dx%dx%d images too large", H, W, C);
  BT_CHECK_ARG(!hb || (ldhb % 4 == 0 && Cout % 4 == 0), "conv: bf16 output needs Cout and "
               "its row stride multiples of 4 (%d, %d)", Cout, ldhb);
  if (rows <= 0) return BT_OK;
  const ConvOut o{z, h, hb, hb_lo, ldhb};
  switch (conv_nc(Cout)) {
    case 8: return launch_fwd_act<8>(act, obs, idx, rows, count, g, w, o, s);
    case 16: return launch_fwd_act<16>(act, obs, idx, rows, count, g, w, o, s);
    default: return launch_fwd_act<32>(act, obs, idx, rows, count, g, w, o, s);
  }
}

int launch_conv_dw(const float* obs, const int* idx, int rows, const int* count, int H, int W,
                   int C, int Cout, const float* dz, int blocks, float* out, cudaStream_t s) {
  BT_CHECK_ARG(Cout >= 1 && Cout <= 32, "conv: %d output channels (at most 32)", Cout);
  BT_CHECK_ARG(9 * C + 1 <= kConvThreads, "conv dW: %d input channels (at most %d)", C,
               (kConvThreads - 1) / 9);
  const ConvGeom g{H, W, C, Cout};
  const int nc = conv_nc(Cout);
  const size_t smem = conv_dw_smem(g, nc);
  BT_CHECK_ARG(smem <= 200 * 1024, "conv dW: %dx%dx%d images too large", H, W, C);
  const int rpb = ceil_div(ceil_div(rows, blocks), kConvRows) * kConvRows;
  switch (nc) {
    case 8:
      BT_TRY(set_smem(conv_dw_kernel<8>, smem));
      conv_dw_kernel<8><<<blocks, kConvThreads, smem, s>>>(obs, idx, rows, count, g, dz, rpb, out);
      break;
    case 16:
      BT_TRY(set_smem(conv_dw_kernel<16>, smem));
      conv_dw_kernel<16><<<blocks, kConvThreads, smem, s>>>(obs, idx, rows, count, g, dz, rpb, out);
      break;
    default:
      BT_TRY(set_smem(conv_dw_kernel<32>, smem));
      conv_dw_kernel<32><<<blocks, kConvThreads, smem, s>>>(obs, idx, rows, count, g, dz, rpb, out);
      break;
  }
  BT_LAUNCH_CHECK("conv_dw_kernel");
  return BT_OK;
}

}  // namespace bt
