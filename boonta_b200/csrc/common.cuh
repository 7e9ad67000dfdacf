// Shared helpers of the boonta_b200 CUDA library: status reporting, launch checks and
// small device utilities. Every C-ABI entry point returns an int status and leaves a
// message in a thread-local buffer (bt_last_error), mirroring the ffi::Error(code, msg)
// convention of the reference's XLA FFI handlers (boonta/environments/ale/ffi/ffi.cc).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "boonta_b200.h"

namespace bt {

void set_error(const char* fmt, ...);
const char* last_error();

struct Status {
  int code = BT_OK;
  bool ok() const { return code == BT_OK; }
};

}  // namespace bt

#define BT_CHECK_ARG(cond, ...)            \
  do {                                     \
    if (!(cond)) {                         \
      ::bt::set_error(__VA_ARGS__);        \
      return BT_ERR_INVALID;               \
    }                                      \
  } while (0)

#define BT_CUDA(call)                                                                 \
  do {                                                                                \
    cudaError_t err_ = (call);                                                        \
    if (err_ != cudaSuccess) {                                                        \
      ::bt::set_error("%s:%d: %s failed: %s", __FILE__, __LINE__, #call,              \
                      cudaGetErrorString(err_));                                      \
      return BT_ERR_CUDA;                                                             \
    }                                                                                 \
  } while (0)

// After a kernel launch: catch configuration errors without synchronising.
#define BT_LAUNCH_CHECK(name)                                                         \
  do {                                                                                \
    cudaError_t err_ = cudaGetLastError();                                            \
    if (err_ != cudaSuccess) {                                                        \
      ::bt::set_error("%s:%d: launch of %s failed: %s", __FILE__, __LINE__, name,     \
                      cudaGetErrorString(err_));                                      \
      return BT_ERR_CUDA;                                                             \
    }                                                                                 \
  } while (0)

#define BT_TRY(expr)          \
  do {                        \
    int rc_ = (expr);         \
    if (rc_ != BT_OK) return rc_; \
  } while (0)

namespace bt {

constexpr int kNumSMs = 148;  // B200: 2 dies x 74 SMs

__host__ __device__ inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
__host__ __device__ inline int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Activation and its derivative. The derivative is evaluated from the pre-activation
// `z` and the output `h` (tanh uses h, relu and silu use z). The sigmoid inside silu uses
// the hardware exp2-based __expf and the approximate division __fdividef (relative error
// ~2e-7, far inside the learner's 1e-4 gradient tolerance); for z < -88 it tends to 0.
__device__ __forceinline__ float fast_sigmoid(float z) {
  return __fdividef(1.f, 1.f + __expf(-z));
}

// Compile-time activation A (BT_ACT_*): act_fwd<A>(z) and its derivative act_dz<A>(z) from
// the pre-activation alone.
template <int A>
__device__ __forceinline__ float act_fwd(float z) {
  if constexpr (A == BT_ACT_TANH) return tanhf(z);
  if constexpr (A == BT_ACT_RELU) return z > 0.f ? z : 0.f;
  if constexpr (A == BT_ACT_SILU) return z * fast_sigmoid(z);
  return z;
}
template <int A>
__device__ __forceinline__ float act_dz(float z) {
  if constexpr (A == BT_ACT_TANH) {
    const float t = tanhf(z);
    return 1.f - t * t;
  }
  if constexpr (A == BT_ACT_RELU) return z > 0.f ? 1.f : 0.f;
  if constexpr (A == BT_ACT_SILU) {
    const float s = fast_sigmoid(z);
    return s * (1.f + z * (1.f - s));
  }
  return 1.f;
}

// The derivative from the activation's output h = act(z), for the activations where h
// determines it (tanh: 1 - h^2, relu: h > 0, none: 1), bit-identical to act_dz<A>(z).
template <int A>
__device__ __forceinline__ float act_dz_from_out(float h) {
  static_assert(A != BT_ACT_SILU, "silu's derivative needs the pre-activation");
  if constexpr (A == BT_ACT_TANH) return 1.f - h * h;
  if constexpr (A == BT_ACT_RELU) return h > 0.f ? 1.f : 0.f;
  return 1.f;
}

template <int A>
struct ActTag {
  static constexpr int value = A;
};
// Calls f(ActTag<A>{}) with the runtime activation resolved once, so that element loops
// inside f are branch-free and the SFU latencies of their elements overlap.
template <class F>
__device__ __forceinline__ void with_act(int act, F&& f) {
  switch (act) {
    case BT_ACT_TANH: f(ActTag<BT_ACT_TANH>{}); break;
    case BT_ACT_RELU: f(ActTag<BT_ACT_RELU>{}); break;
    case BT_ACT_SILU: f(ActTag<BT_ACT_SILU>{}); break;
    default: f(ActTag<BT_ACT_NONE>{}); break;
  }
}

__device__ __forceinline__ float act_forward(float z, int act) {
  switch (act) {
    case BT_ACT_TANH: return act_fwd<BT_ACT_TANH>(z);
    case BT_ACT_RELU: return act_fwd<BT_ACT_RELU>(z);
    case BT_ACT_SILU: return act_fwd<BT_ACT_SILU>(z);
    default: return z;
  }
}

__device__ __forceinline__ float act_grad(float z, float h, int act) {
  switch (act) {
    case BT_ACT_TANH: return 1.f - h * h;
    case BT_ACT_RELU: return act_dz<BT_ACT_RELU>(z);
    case BT_ACT_SILU: return act_dz<BT_ACT_SILU>(z);
    default: return 1.f;
  }
}

// Programmatic dependent launch. A kernel launched through launch_pdl may start while its
// predecessor in the stream is still finishing; it calls pdl_wait() before reading anything
// that predecessor (or an earlier kernel) writes, and pdl_trigger() to let its own successor
// be scheduled early. Both are no-ops for kernels launched the ordinary way.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <class... KArgs, class... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Effective row count: rows of a padded minibatch that carry data (a device-side count
// when the rank's share of a global minibatch varies, else the static size).
__device__ __forceinline__ int live_rows(const int* count, int rows) {
  if (count == nullptr) return rows;
  int c = *count;
  return c < rows ? c : rows;
}

// End of the rows a bf16 operand of the tensor-core weight-gradient GEMM must hold: its K loop
// reads whole 64-row blocks up to the live count, so the rows [live, dz_rows_end) are written
// as zeros by the kernel that produces the operand (padded multi-rank minibatches).
__device__ __forceinline__ int dz_rows_end(int live, int rows) {
  const int e = (live + 63) / 64 * 64;
  return e < rows ? e : rows;
}

}  // namespace bt
