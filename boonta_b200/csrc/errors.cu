// Thread-local error messages behind bt_last_error(), and the self-test of the bounded
// waits that every waiting kernel uses.
#include "common.cuh"
#include "ptx.cuh"

namespace bt {

static thread_local char g_last_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

const char* last_error() { return g_last_error; }

}  // namespace bt

extern "C" const char* bt_last_error(void) { return bt::last_error(); }

extern "C" const char* bt_version(void) { return "boonta_b200 0.1 (sm_100a)"; }

namespace {

// One thread waits on an mbarrier that nothing ever arrives at, with the given limit, the way
// every waiting kernel of the library does; when the wait gives up it records the failure
// in *err and returns, leaving the context usable.
__global__ void bounded_wait_selftest_kernel(int* err, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    bt::mbar_init(&bar, 1);
    bt::fence_mbar_init();
    if (!bt::mbar_wait_bounded(&bar, 0, limit_ns)) *err = 1;
  }
}

}  // namespace

extern "C" int bt_selftest_bounded_wait(int32_t limit_us, void* stream) {
  using namespace bt;
  BT_CHECK_ARG(limit_us > 0 && limit_us <= 2000000, "limit %d us outside (0, 2 s]", limit_us);
  cudaStream_t s = (cudaStream_t)stream;
  int* err = nullptr;
  BT_CUDA(cudaMallocAsync(&err, sizeof(int), s));
  BT_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s));
  bounded_wait_selftest_kernel<<<1, 32, 0, s>>>(err, (unsigned long long)limit_us * 1000ull);
  BT_LAUNCH_CHECK("bounded_wait_selftest_kernel");
  int code = 0;
  BT_CUDA(cudaMemcpyAsync(&code, err, sizeof(int), cudaMemcpyDeviceToHost, s));
  BT_CUDA(cudaFreeAsync(err, s));
  BT_CUDA(cudaStreamSynchronize(s));
  if (code) {
    set_error("bounded wait gave up after %d us (the expected outcome)", limit_us);
    return BT_ERR_TIMEOUT;
  }
  return BT_OK;
}
