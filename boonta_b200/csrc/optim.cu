// K10 as a standalone entry point: optax.chain(clip_by_global_norm(max_norm),
// adam(lr, b1, b2, eps, eps_root)) followed by optax.apply_updates, on flat fp32 device
// buffers — the optimizer step of boonta/algorithms/ppo.py:182-191 — for callers that run
// their own forward/backward. The learner handle uses the same kernels inside its update.
//
// The global norm is summed in two fixed-order stages: per-chunk sums of squares (8192
// elements per block) into scratch, then every Adam block adds the chunk sums in index
// order, so the result is deterministic.
#include <cuda.h>

#include <mutex>

#include "kernels.cuh"

using namespace bt;

namespace {

int check_opt_args(float* params, float* mu, float* nu, const float* grads, int64_t n,
                   int32_t count, const bt_optimizer* opt) {
  BT_CHECK_ARG(params && mu && nu && grads && opt, "clip_adam: null argument");
  BT_CHECK_ARG(n >= 0, "clip_adam: negative size %lld", (long long)n);
  BT_CHECK_ARG(count >= 0, "clip_adam: negative step count %d", count);
  return BT_OK;
}

int run_clip_adam(float* params, float* mu, float* nu, const float* grads, int64_t n,
                  int32_t count, const bt_optimizer* opt, double* scratch, cudaStream_t s) {
  BT_TRY(launch_sumsq_chunks(grads, n, scratch, s));
  AdamParams ap{};
  ap.params = params;
  ap.mu = mu;
  ap.nu = nu;
  ap.grads = grads;
  ap.n = n;
  ap.norm_partials = scratch;
  ap.num_norm_partials = (int)ceil_div64(n, kNormChunk);
  ap.count = nullptr;
  ap.step = count;
  ap.lr = opt->lr;
  ap.max_norm = opt->max_grad_norm;
  ap.b1 = opt->b1;
  ap.b2 = opt->b2;
  ap.eps = opt->eps;
  ap.eps_root = opt->eps_root;
  ap.shadow = nullptr;
  ap.shadow_lo = nullptr;
  return launch_adam(ap, s);
}

}  // namespace

// Scratch for the chunk sums comes from CUDA's stream-ordered allocator
// (cudaMallocAsync / cudaFreeAsync on the caller's stream).
extern "C" int bt_clip_adam(float* params, float* mu, float* nu, const float* grads, int64_t n,
                            int32_t count, const bt_optimizer* opt, void* stream) {
  BT_TRY(check_opt_args(params, mu, nu, grads, n, count, opt));
  if (n == 0) return BT_OK;
  cudaStream_t s = (cudaStream_t)stream;
  double* scratch = nullptr;
  BT_CUDA(cudaMallocAsync(&scratch, (size_t)ceil_div64(n, kNormChunk) * sizeof(double), s));
  const int rc = run_clip_adam(params, mu, nu, grads, n, count, opt, scratch, s);
  BT_CUDA(cudaFreeAsync(scratch, s));
  return rc;
}

// ---- the allocation-free variant ----------------------------------------------------------
// Some callers cannot allocate device memory at the point where they run the optimizer: a
// step running inside another framework's memory pool (an XLA FFI custom call runs after
// XLA has reserved most of the device for its own allocator, so a cudaMalloc there can fail
// or fragment memory XLA counts on), or a host with a fixed device-memory budget set at
// start-up. bt_clip_adam_noalloc takes its scratch from a fixed array compiled into this
// library instead.
//
// The array holds one partial sum per 8192-element chunk for up to kNoAllocChunks chunks:
// 128 KB, so at most 134,217,728 elements per call. It lives in device memory of every GPU
// that loads the library until the process exits. Every call writes all the chunk slots it
// reads before reading them, so nothing has to be cleared between calls; the array keeps
// the last call's partial sums. All calls share it: calls whose GPU work overlaps (two
// streams, or two host threads) race on it and must be ordered by the caller.
namespace {

constexpr int kNoAllocChunks = 16384;
constexpr int kNoAllocMaxDevices = 64;
__device__ __align__(256) double g_noalloc_scratch[kNoAllocChunks];

// Device address of g_noalloc_scratch per device, looked up with that device current (host
// code cannot use the symbol itself as a device pointer) and kept together with the id of the
// CUDA context it was looked up in. The lookup happens in the first call on each device, which
// should therefore come before any stream capture there. If the caller tears the context down
// (cudaDeviceReset) and the library's device code is loaded into a new one, the array can sit
// at a new address: a call made in another context than the cached one looks it up again.
struct NoAllocSlot {
  unsigned long long ctx_id = 0;  // cuCtxGetId: unique for the process's lifetime
  void* ptr = nullptr;
};
NoAllocSlot g_noalloc_slot[kNoAllocMaxDevices];
std::mutex g_noalloc_mutex;

// Id of the calling thread's current context, 0 when none is current yet (the runtime makes
// one current on its first call on the thread, e.g. the symbol lookup below).
// The driver entry points come through the runtime (cudaGetDriverEntryPoint), so the library
// does not link libcuda itself.
unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  if (!get_current || !get_id) {
    void* f1 = nullptr;
    void* f2 = nullptr;
    cudaDriverEntryPointQueryResult q1, q2;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault, &q1) != cudaSuccess ||
        cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault, &q2) != cudaSuccess ||
        q1 != cudaDriverEntryPointSuccess || q2 != cudaDriverEntryPointSuccess || !f1 || !f2)
      return 0;
    get_current = reinterpret_cast<GetCurrent>(f1);
    get_id = reinterpret_cast<GetId>(f2);
  }
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

int noalloc_scratch(double** out) {
  int dev = 0;
  BT_CUDA(cudaGetDevice(&dev));
  BT_CHECK_ARG(dev >= 0 && dev < kNoAllocMaxDevices, "device %d out of range", dev);
  const unsigned long long id = current_context_id();
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  NoAllocSlot& slot = g_noalloc_slot[dev];
  if (id == 0 || !slot.ptr || slot.ctx_id != id) {
    void* p = nullptr;
    BT_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    slot.ptr = p;
    slot.ctx_id = current_context_id();
  }
  *out = static_cast<double*>(slot.ptr);
  return BT_OK;
}

}  // namespace

extern "C" int bt_clip_adam_noalloc(float* params, float* mu, float* nu, const float* grads,
                                    int64_t n, int32_t count, const bt_optimizer* opt,
                                    void* stream) {
  BT_TRY(check_opt_args(params, mu, nu, grads, n, count, opt));
  BT_CHECK_ARG(ceil_div64(n, kNormChunk) <= kNoAllocChunks,
               "bt_clip_adam_noalloc: %lld elements exceed the fixed scratch limit of %lld "
               "(use bt_clip_adam)",
               (long long)n, (long long)kNoAllocChunks * kNormChunk);
  if (n == 0) return BT_OK;
  double* scratch = nullptr;
  BT_TRY(noalloc_scratch(&scratch));
  return run_clip_adam(params, mu, nu, grads, n, count, opt, scratch, (cudaStream_t)stream);
}
