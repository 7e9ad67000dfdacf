// f2: counter-based random numbers on the device in JAX's threefry conventions, so a caller can
// hand the learner raw PRNG keys instead of host-drawn indices and noise.
//
// threefry2x32 with 20 rounds (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as
// 1, 2, 3", SC 2011; the Random123 reference algorithm): key (k0, k1), key schedule
// ks = (k0, k1, k0 ^ k1 ^ 0x1BD11BDA), x = counter + (ks0, ks1), five groups of four rounds
// (x0 += x1; x1 = rotl(x1, R); x1 ^= x0) with rotations 13 15 26 6 / 17 29 16 24 alternating,
// and after group i (1..5) the injection x0 += ks[i % 3], x1 += ks[(i + 1) % 3] + i.
//
// JAX's key-level operations over it (jax.random with threefry keys in the partitionable mode,
// the default of current JAX; boonta draws with them at boonta/algorithms/ppo.py:200, 230,
// boonta/podracers/anakin.py:106-108 and boonta/networks/distributions.py:21-23):
//   split(key, num)[i]       = threefry(key, (0, i))                  (the counter's 64-bit index
//                                                                     as (hi, lo) words)
//   random_bits(key, n)[i]   = y0 ^ y1 of threefry(key, (hi(i), lo(i)))
//   uniform(key, n, lo, hi)  = max(lo, (bitcast((bits >> 9) | 0x3F800000) - 1) * (hi - lo) + lo)
//   normal(key, n)           = sqrt(2) * erfinv(uniform(key, n, nextafter(-1, 0), 1))
//   permutation(key, n)      = ceil(3 ln n / ln(2^32 - 1)) rounds of: (key, sub) = split(key, 2);
//                              stable sort of the values by random_bits(sub, n)
// and, with partitionable = 0, JAX's original counter layout: the counters 0 .. 2m-1 (m =
// ceil(n / 2), zero-padded) split into halves x0 = 0 .. m-1, x1 = m .. 2m-1, one block per pair,
// outputs concatenated (y0 then y1): random_bits(key, n)[i] = y0 of block i for i < m, y1 of block
// i - m after; split(key, num) takes the 2 num words of that layout pairwise.
// JAX is absent here, so only the threefry block itself is pinned (to the Random123 known-answer
// vectors); XLA's sort is not guaranteed stable, so where two sort keys of a round collide
// (about n^2 / 2^33 pairs) the order of those two values may differ from JAX's.
#include <cub/device/device_radix_sort.cuh>

#include "common.cuh"

namespace bt {

__host__ __device__ __forceinline__ uint32_t rotl32(uint32_t v, int r) {
  return (v << r) | (v >> (32 - r));
}

__host__ __device__ inline void threefry2x32(uint32_t k0, uint32_t k1, uint32_t c0, uint32_t c1,
                                             uint32_t& y0, uint32_t& y1) {
  const uint32_t ks[3] = {k0, k1, k0 ^ k1 ^ 0x1BD11BDAu};
  const int rot[8] = {13, 15, 26, 6, 17, 29, 16, 24};
  uint32_t x0 = c0 + ks[0], x1 = c1 + ks[1];
#pragma unroll
  for (int g = 0; g < 5; ++g) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      x0 += x1;
      x1 = rotl32(x1, rot[(g & 1) * 4 + r]);
      x1 ^= x0;
    }
    const int i = g + 1;
    x0 += ks[i % 3];
    x1 += ks[(i + 1) % 3] + (uint32_t)i;
  }
  y0 = x0;
  y1 = x1;
}

__global__ void threefry_kernel(uint32_t k0, uint32_t k1, const uint32_t* c0, const uint32_t* c1,
                                uint32_t* y0, uint32_t* y1, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    threefry2x32(k0, k1, c0[i], c1[i], y0[i], y1[i]);
}

// Word i of n in either layout.
__host__ __device__ inline uint32_t random_word(uint32_t k0, uint32_t k1, int64_t i, int64_t n,
                                                bool partitionable) {
  uint32_t y0, y1;
  if (partitionable) {
    threefry2x32(k0, k1, (uint32_t)((uint64_t)i >> 32), (uint32_t)i, y0, y1);
    return y0 ^ y1;
  }
  const int64_t m = (n + 1) / 2;
  if (i < m) {
    threefry2x32(k0, k1, (uint32_t)i, i + m < n ? (uint32_t)(i + m) : 0u, y0, y1);
    return y0;
  }
  threefry2x32(k0, k1, (uint32_t)(i - m), (uint32_t)i, y0, y1);
  return y1;
}

__device__ __forceinline__ float uniform_from_bits(uint32_t bits, float lo, float hi) {
  const float f = __uint_as_float((bits >> 9) | 0x3F800000u) - 1.f;
  return fmaxf(lo, f * (hi - lo) + lo);
}

// kind 0: random bits, 1: uniform in [lo, hi), 2: standard normal
__global__ void random_fill_kernel(uint32_t k0, uint32_t k1, int64_t n, int kind, float lo,
                                   float hi, bool partitionable, void* out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t b = random_word(k0, k1, i, n, partitionable);
    if (kind == 0) {
      reinterpret_cast<uint32_t*>(out)[i] = b;
    } else if (kind == 1) {
      reinterpret_cast<float*>(out)[i] = uniform_from_bits(b, lo, hi);
    } else {
      const float u = uniform_from_bits(b, nextafterf(-1.f, 0.f), 1.f);
      reinterpret_cast<float*>(out)[i] = 1.41421356237309515f * erfinvf(u);
    }
  }
}

__global__ void iota_kernel(int32_t* v, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    v[i] = (int32_t)i;
}

static int fill_grid(int64_t n) {
  return (int)std::min<int64_t>(ceil_div64(n, 256), 8 * kNumSMs);
}

void host_split(const uint32_t key[2], int num, bool partitionable, uint32_t* out) {
  if (partitionable) {
    for (int i = 0; i < num; ++i)
      threefry2x32(key[0], key[1], 0u, (uint32_t)i, out[2 * i], out[2 * i + 1]);
    return;
  }
  for (int i = 0; i < 2 * num; ++i) out[i] = random_word(key[0], key[1], i, 2 * num, false);
}

int permutation_rounds(int64_t n) {
  if (n <= 1) return 0;
  return (int)std::ceil(3.0 * std::log((double)n) / std::log(4294967295.0));
}

// Workspace: sort keys twice, values twice (n each, 256-byte aligned) and CUB's temporary
// storage.
static size_t align256(size_t b) { return (b + 255) / 256 * 256; }

int64_t permutation_workspace(int64_t n) {
  size_t temp = 0;
  if (cub::DeviceRadixSort::SortPairs(nullptr, temp, (const uint32_t*)nullptr, (uint32_t*)nullptr,
                                      (const int32_t*)nullptr, (int32_t*)nullptr, (int)n) !=
      cudaSuccess)
    return -1;
  return (int64_t)(2 * align256(n * 4) + 2 * align256(n * 4) + align256(temp));
}

}  // namespace bt

extern "C" void bt_threefry2x32_host(uint32_t k0, uint32_t k1, uint32_t c0, uint32_t c1,
                                     uint32_t* y) {
  bt::threefry2x32(k0, k1, c0, c1, y[0], y[1]);
}

extern "C" int bt_threefry2x32(uint32_t k0, uint32_t k1, const uint32_t* c0, const uint32_t* c1,
                               uint32_t* y0, uint32_t* y1, int64_t n, void* stream) {
  BT_CHECK_ARG(n >= 0, "bt_threefry2x32: negative length");
  if (n == 0) return BT_OK;
  BT_CHECK_ARG(c0 && c1 && y0 && y1, "bt_threefry2x32: null pointer");
  bt::threefry_kernel<<<bt::fill_grid(n), 256, 0, (cudaStream_t)stream>>>(k0, k1, c0, c1, y0, y1, n);
  BT_LAUNCH_CHECK("threefry_kernel");
  return BT_OK;
}

extern "C" int bt_random_split(const uint32_t* key, int32_t num, int32_t partitionable,
                               uint32_t* out) {
  BT_CHECK_ARG(key && out && num >= 0, "bt_random_split: bad argument");
  bt::host_split(key, num, partitionable != 0, out);
  return BT_OK;
}

extern "C" int bt_random_fill(const uint32_t* key, int64_t n, int32_t kind, float minval,
                              float maxval, int32_t partitionable, void* out, void* stream) {
  BT_CHECK_ARG(key && n >= 0, "bt_random_fill: bad argument");
  BT_CHECK_ARG(kind >= 0 && kind <= 2, "bt_random_fill: kind %d", kind);
  if (n == 0) return BT_OK;
  BT_CHECK_ARG(out, "bt_random_fill: null output");
  bt::random_fill_kernel<<<bt::fill_grid(n), 256, 0, (cudaStream_t)stream>>>(
      key[0], key[1], n, kind, minval, maxval, partitionable != 0, out);
  BT_LAUNCH_CHECK("random_fill_kernel");
  return BT_OK;
}

extern "C" int64_t bt_random_permutation_workspace(int64_t n) {
  if (n < 0 || n > INT32_MAX) return -1;
  return bt::permutation_workspace(n);
}

extern "C" int bt_random_permutation(const uint32_t* key, int64_t n, int32_t partitionable,
                                     int32_t* out, void* workspace, int64_t workspace_bytes,
                                     void* stream) {
  BT_CHECK_ARG(key && n >= 0 && n <= INT32_MAX, "bt_random_permutation: bad argument");
  if (n == 0) return BT_OK;
  BT_CHECK_ARG(out, "bt_random_permutation: null output");
  const cudaStream_t s = (cudaStream_t)stream;
  const int rounds = bt::permutation_rounds(n);
  bt::iota_kernel<<<bt::fill_grid(n), 256, 0, s>>>(out, n);
  BT_LAUNCH_CHECK("iota_kernel");
  if (rounds == 0) return BT_OK;
  const int64_t need = bt::permutation_workspace(n);
  BT_CHECK_ARG(workspace && need >= 0 && workspace_bytes >= need,
               "bt_random_permutation: workspace of %lld bytes, %lld needed",
               (long long)workspace_bytes, (long long)need);
  const size_t q = bt::align256((size_t)n * 4);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* keys_a = reinterpret_cast<uint32_t*>(ws);
  uint32_t* keys_b = reinterpret_cast<uint32_t*>(ws + q);
  int32_t* vals_b = reinterpret_cast<int32_t*>(ws + 2 * q);
  void* temp = ws + 4 * q;
  size_t temp_bytes = (size_t)need - 4 * q;
  uint32_t k[2] = {key[0], key[1]};
  int32_t* vals = out;
  for (int r = 0; r < rounds; ++r) {
    uint32_t two[4];
    bt::host_split(k, 2, partitionable != 0, two);  // (key, subkey) = split(key)
    k[0] = two[0];
    k[1] = two[1];
    bt::random_fill_kernel<<<bt::fill_grid(n), 256, 0, s>>>(two[2], two[3], n, 0, 0.f, 0.f,
                                                            partitionable != 0, keys_a);
    BT_LAUNCH_CHECK("random_fill_kernel");
    int32_t* dst = vals == out ? vals_b : out;
    BT_CUDA(cub::DeviceRadixSort::SortPairs(temp, temp_bytes, keys_a, keys_b, vals, dst, (int)n, 0,
                                            32, s));
    vals = dst;
  }
  if (vals != out)
    BT_CUDA(cudaMemcpyAsync(out, vals, (size_t)n * 4, cudaMemcpyDeviceToDevice, s));
  return BT_OK;
}
