// Declarations shared by the learner's kernels and its orchestration (learner.cu).
#pragma once

#include "common.cuh"

namespace bt {

// Per-minibatch statistic sums (double), in this order:
//  0 sum min(surr1, surr2)   1 sum entropy        2 sum (lp_old - lp)   3 sum clipped
//  4 sum advantage           5 sum critic term    6 sum (R - v)         7 sum (R - v)^2
//  8 sum R                   9 sum R^2           10 sum v              11 live rows
constexpr int kNumStatSums = 12;

struct HeadsParams {
  int rows;          // capacity rows of the minibatch buffers
  const int* count;  // nullable: live rows
  const int* idx;    // [rows] flat sample index (into [T*N] arrays); nullable = identity
  const float* f_pi;  // pre-activations of the tower outputs; the head input is act(f)
  int F_pi;
  const float* f_v;  // == f_pi when the torso is shared
  int F_v;
  const float* w_pi;   // [F_pi + 1, A]
  const float* w_v;    // [F_v + 1, 1]
  const float* scale;  // gaussian [A]
  int A;
  int head;
  const void* action;
  const float* lp_old;
  const float* v_old;
  const float* adv;
  const float* ret;
  float inv_mb;
  float clip;
  int clip_value;
  float ent_coef;
  float vf_coef;
  float* d_out;  // [rows, A]
  float* d_val;  // [rows]
  float* d_fpi;  // [rows, F_pi]
  float* d_fv;   // [rows, F_v] (separate towers)
  __nv_bfloat16* d_fpi_b;  // when set: dL/d f_pi written as bf16 instead of fp32
  __nv_bfloat16* d_fv_b;
  __nv_bfloat16* d_fpi_b_lo;  // when set: the low halves of split bf16 pairs
  __nv_bfloat16* d_fv_b_lo;
  int act_pi;  // activation of the tower outputs (applied to f, differentiated for dL/dpre)
  int act_v;
  double* stat_partials;   // [gridDim.x][kNumStatSums]
  float* dscale_partials;  // [gridDim.x][A] (gaussian)
  // nullable: fused head weight gradients, per block [gridDim.x][(F_pi + 1) * A] and
  // [gridDim.x][F_v + 1] (allowed when heads_fuse_dw holds)
  float* dw_pi_partials;
  float* dw_v_partials;
};

int launch_heads_loss(const HeadsParams& p, int blocks, cudaStream_t stream);
size_t heads_smem_bytes(int F_pi, int F_v, int A, bool shared);
// Whether the heads kernel can accumulate the head weight gradients itself (small heads).
bool heads_fuse_dw(int F_pi, int F_v, int A, bool shared);
// Whether the heads kernel computes the actor outputs (and, for a shared torso, the value)
// with split-bf16 products (wide heads on warp-level tensor cores).
bool heads_split_products(int F_pi, int F_v, int A, bool shared);
// Head outputs only (act, bootstrap values). split_pi / split_v: evaluate the actor outputs /
// the value with the split-bf16 products of the heads kernel (hi*hi + hi*lo + lo*hi per term,
// fp32 accumulation), so that act and update agree to fp32 rounding.
int launch_heads_forward(const float* f_pi, int F, const float* f_v, int Fv, const float* w_pi,
                         const float* w_v, int A, int rows, int act_pi, int act_v, float* out,
                         float* value, bool split_pi, bool split_v, cudaStream_t stream);
// Fused act step (CUDA-core heads): head outputs and the sample of PPO.step in one kernel;
// action / log_prob per row, value nullable.
int launch_heads_act(const float* f_pi, int F, const float* f_v, int Fv, const float* w_pi,
                     const float* w_v, const float* scale, int head, int A, int rows, int act_pi,
                     int act_v, bool split_pi, bool split_v, const float* noise,
                     float temperature, void* action, float* log_prob, float* value,
                     cudaStream_t stream);

// Conv 3x3 SAME stride 1 on NHWC rows (conv.cu): forward z = conv + bias, h = act(z)
// ([rows, H*W*Cout]); weight gradient as per-block partials [blocks][(9C + 1) * Cout].
int launch_conv_forward(const float* obs, const int* idx, int rows, const int* count, int H,
                        int W, int C, int Cout, const float* w, int act, float* z, float* h,
                        __nv_bfloat16* hb, __nv_bfloat16* hb_lo, int ldhb, cudaStream_t s);
int launch_conv_dw(const float* obs, const int* idx, int rows, const int* count, int H, int W,
                   int C, int Cout, const float* dz, int blocks, float* out, cudaStream_t s);
int conv_dw_blocks(int rows);

// LayerNorm (flax, epsilon 1e-6, fast variance) fused with the following activation.
int launch_ln_forward(const float* z, const float* scale_bias, int rows, int n, int act,
                      float* y, float* h, __nv_bfloat16* hb, __nv_bfloat16* hb_lo, int ldhb,
                      float* mean, float* rstd, const int* count, cudaStream_t stream);
// d_y already carries the activation derivative; writes d_z and per-block partial sums
// [blocks][2n] of (d scale, d bias).
int launch_ln_backward(const float* d_y, const float* z, const float* mean, const float* rstd,
                       const float* scale, int rows, int n, float* d_z, __nv_bfloat16* d_zb,
                       __nv_bfloat16* d_zb_lo, float* partials, int blocks, const int* count,
                       cudaStream_t stream);

// [F + 1, n] split partials [splits][F + 1][n] of [act(f), 1]^T d, for narrow d (n <= 64).
int launch_skinny_dw(const float* f, int F, int act, const float* d, int n, int rows,
                     const int* count, int splits, float* out, cudaStream_t stream);

// bf16 operands of the tensor-core path. Every bf16 writer takes an optional `lo` buffer:
// when set, the value is stored as the pair hi = bf16(x), lo = bf16(x - hi) (the split
// operands of BT_PREC_BF16X3).
__device__ __forceinline__ void store_bf16(__nv_bfloat16* hi, __nv_bfloat16* lo, size_t i,
                                           float x) {
  const __nv_bfloat16 h = __float2bfloat16_rn(x);
  hi[i] = h;
  if (lo) lo[i] = __float2bfloat16_rn(x - __bfloat162float(h));
}
// Four consecutive values (index i a multiple of 4, 8-byte aligned) as bf16, hi and (when
// `lo` is set) the remainders, with paired conversions and 8-byte stores.
__device__ __forceinline__ void store_bf16x4(__nv_bfloat16* hi, __nv_bfloat16* lo, size_t i,
                                             float4 g) {
  const __nv_bfloat162 h01 = __floats2bfloat162_rn(g.x, g.y);
  const __nv_bfloat162 h23 = __floats2bfloat162_rn(g.z, g.w);
  uint2 hv;
  hv.x = *reinterpret_cast<const uint32_t*>(&h01);
  hv.y = *reinterpret_cast<const uint32_t*>(&h23);
  *reinterpret_cast<uint2*>(hi + i) = hv;
  if (lo) {
    const __nv_bfloat162 l01 =
        __floats2bfloat162_rn(g.x - __low2float(h01), g.y - __high2float(h01));
    const __nv_bfloat162 l23 =
        __floats2bfloat162_rn(g.z - __low2float(h23), g.w - __high2float(h23));
    uint2 lv;
    lv.x = *reinterpret_cast<const uint32_t*>(&l01);
    lv.y = *reinterpret_cast<const uint32_t*>(&l23);
    *reinterpret_cast<uint2*>(lo + i) = lv;
  }
}
// Rows idx[r] of a bf16 table [*, ld] to out [rows, ld] (ld a multiple of 8).
int launch_gather_rows_bf16(const __nv_bfloat16* src, const int* idx, int rows, int ld,
                            __nv_bfloat16* out, const int* count, cudaStream_t stream);
int launch_gather_bf16(const float* obs, const int* idx, int rows, int d, int ld,
                       __nv_bfloat16* out, __nv_bfloat16* out_lo, const int* count,
                       cudaStream_t stream, __nv_bfloat16* table = nullptr);
// fp32 [rows, d] -> split bf16 pairs [rows, d]; rows from the live count to the next 64-row
// boundary written as zeros.
int launch_split_rows_bf16(const float* src, int rows, int d, __nv_bfloat16* out,
                           __nv_bfloat16* out_lo, const int* count, cudaStream_t stream);
int launch_ones_column(__nv_bfloat16* buf, int rows, int n, int ld, float one,
                       cudaStream_t stream);
int launch_zero_tail_rows(__nv_bfloat16* buf, __nv_bfloat16* lo, int rows, int ld,
                          const int* count, cudaStream_t stream);
int launch_to_bf16(const float* in, __nv_bfloat16* out, __nv_bfloat16* out_lo, int64_t n,
                   cudaStream_t stream);

// One gradient segment: dst[0:len] = sum over s of src[s * stride + 0:len] (fixed order).
struct Segment {
  const float* src;
  int nsplit;
  int len;
  int64_t stride;
  int64_t dst;  // offset in the flat gradient buffer
};
// A piece of a segment reduced by one block: elements [begin, end) of segment `seg`.
struct ReduceChunk {
  int seg;
  int begin, end;
};
constexpr int kReduceChunk = 1024;
// Segments with at least kTallSplits partials are reduced in chunks of kTallChunk elements,
// the block's eight warps each summing every eighth partial (so the dependent load chain
// per thread is nsplit / 8 long instead of nsplit).
constexpr int kTallSplits = 64;
constexpr int kTallChunk = 32;
// Wide segments with few partials take several kReduceChunk pieces per block (up to 8, about
// 16 partial rows of a piece per block), so a block moves enough bytes to pay for its start
// and its norm reduction.
__host__ __device__ inline int reduce_chunk_len(int len, int nsplit) {
  if (len >= 256 && nsplit >= kTallSplits) return kTallChunk;
  const int reps = nsplit >= 16 ? 1 : (16 / (nsplit < 1 ? 1 : nsplit) > 8 ? 8 : 16 / nsplit);
  return kReduceChunk * reps;
}
// Builds the chunk table of a segment list (host side).
void build_reduce_chunks(const Segment* segs, int num_segments, ReduceChunk* out, int* count);
int count_reduce_chunks(const Segment* segs, int num_segments);
// Sums split partials into the gradient buffer, one block per chunk; when `norm_partials`
// is non-null also writes each block's sum of squares [num_chunks].
int launch_reduce_segments(const Segment* segs, const ReduceChunk* chunks, int num_chunks,
                           float* grads, double* norm_partials, cudaStream_t stream);
// Sum of squares of a flat buffer into norm_partials[kNormBlocks] (multi-GPU path).
constexpr int kNormBlocks = 256;
int launch_sumsq(const float* g, int64_t n, double* norm_partials, cudaStream_t stream);

struct AdamParams {
  float* params;
  float* mu;
  float* nu;
  const float* grads;
  int64_t n;
  const double* norm_partials;
  int num_norm_partials;
  const int* count;  // device adam count before this update block (nullable: 0)
  int step;          // optimizer steps already taken (added to *count)
  float lr, max_norm, b1, b2, eps, eps_root;
  __nv_bfloat16* shadow;     // nullable bf16 copy of params
  __nv_bfloat16* shadow_lo;  // nullable low halves (split bf16 pairs)
  // Other GPUs' copies of the same elements (NVLink peer memory, already offset like params):
  // every new parameter (and its bf16 shadow) is also stored there, and each thread fences its
  // stores system-wide before it finishes. npush = 0: none.
  int npush;
  float* push_params[7];
  __nv_bfloat16* push_shadow[7];
  __nv_bfloat16* push_shadow_lo[7];
  // Element ranges [skip_lo, skip_hi) (relative to params, multiples of 4) whose fp32 values
  // are not pushed (only their bf16 shadow): parameters the peers read through the shadow alone
  // while an update runs.
  int nskip;
  int64_t skip_lo[8], skip_hi[8];
};
int launch_adam(const AdamParams& p, cudaStream_t stream);

// Sum of squares of g in chunks of kNormChunk elements: out[c] = sum over chunk c (one
// block per chunk, fixed order). The standalone optimizer entry points use it.
constexpr int kNormChunk = 8192;
int launch_sumsq_chunks(const float* g, int64_t n, double* out, cudaStream_t stream);

// Per-minibatch statistics.
int launch_stat_reduce(const double* partials, int blocks, double* out, cudaStream_t stream);
int launch_stat_finalize(const double* sums, int count, float inv_mb, float* stats,
                         cudaStream_t stream);

// Advantage normalisation over the whole rollout: (A - mean) / (std + 1e-8).
int launch_adv_moments(const float* adv, int64_t n, double* partials, cudaStream_t stream);
int launch_adv_normalize(float* adv, int64_t n, const double* partials, int num_partials,
                         double total, cudaStream_t stream);

int launch_increment(int* count, int by, cudaStream_t stream);

// Multi-GPU minibatch split: for every (epoch, minibatch) slice of the global
// permutation, keep the indices owned by this rank (in order), mapped to local flat
// indices, and count them. Sets *err = BT_ERR_CAPACITY-style flag when a count exceeds
// `capacity`.
int launch_local_indices(const int* perm, int num_slices, int slice_len, int units_per_row,
                         int local_units, int rank, int global_units, int capacity,
                         int* local_idx, int* counts, int* err, cudaStream_t stream);

}  // namespace bt
