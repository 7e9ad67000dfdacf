// Host side of the tcgen05 GEMM: TMA tensor-map encoding (driver entry point resolved
// through the runtime, so the library needs no link-time libcuda) and a diagnostic C-ABI
// entry point that runs one plain GEMM, used by the tests to check every operand-major
// combination against a reference product.
#include <cudaTypedefs.h>

#include "gemm_sm100.cuh"

namespace bt {
namespace umma {

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int resolve_encode() {
  if (g_encode) return BT_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  BT_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
  if (!fn || q != cudaDriverEntryPointSuccess) {
    set_error("cuTensorMapEncodeTiled is unavailable");
    return BT_ERR_CUDA;
  }
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return BT_OK;
}

int encode_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
               uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
  BT_TRY(resolve_encode());
  BT_CHECK_ARG(((uintptr_t)base & 15) == 0, "tensor map base %p not 16-byte aligned", base);
  BT_CHECK_ARG(row_bytes % 16 == 0, "tensor map row stride %llu not a multiple of 16",
               (unsigned long long)row_bytes);
  BT_CHECK_ARG(box_inner * 2 <= 128 && box_outer <= 256, "tensor map box %ux%u", box_inner,
               box_outer);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): dims %llu x %llu, stride %llu, box %u x %u",
              (int)r, (unsigned long long)inner, (unsigned long long)outer,
              (unsigned long long)row_bytes, box_inner, box_outer);
    return BT_ERR_CUDA;
  }
  return BT_OK;
}

int encode_tile_map(CUtensorMap* map, const void* base, bool f32, uint64_t inner,
                    uint64_t outer, uint64_t row_bytes, int swizzle_bytes) {
  BT_TRY(resolve_encode());
  const uint32_t esize = f32 ? 4 : 2;
  BT_CHECK_ARG(((uintptr_t)base & 15) == 0, "tensor map base %p not 16-byte aligned", base);
  BT_CHECK_ARG(row_bytes % 16 == 0, "tensor map row stride %llu not a multiple of 16",
               (unsigned long long)row_bytes);
  BT_CHECK_ARG(32 * esize == (uint32_t)swizzle_bytes, "epilogue tile map: %d-byte swizzle for "
               "%u-byte elements", swizzle_bytes, esize);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                        2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for an epilogue tile map: dims %llu x %llu, "
              "stride %llu", (int)r, (unsigned long long)inner, (unsigned long long)outer,
              (unsigned long long)row_bytes);
    return BT_ERR_CUDA;
  }
  return BT_OK;
}

}  // namespace umma
}  // namespace bt

using namespace bt;

namespace {

int make_operand_maps(const void* A, const void* B, int M, int N, int K, int a_mn, int b_mn,
                      CUtensorMap* ta, CUtensorMap* tb) {
  if (a_mn) {
    BT_TRY(umma::encode_map(ta, A, M, K, (uint64_t)M * 2, 64, 64));
  } else {
    BT_TRY(umma::encode_map(ta, A, K, M, (uint64_t)K * 2, 64, 128));
  }
  if (b_mn) {
    BT_TRY(umma::encode_map(tb, B, N, K, (uint64_t)N * 2, 64, 64));
  } else {
    BT_TRY(umma::encode_map(tb, B, K, N, (uint64_t)K * 2, 64, 128));
  }
  return BT_OK;
}

template <bool X3>
int run_debug_gemm(const umma::Operands& ops, int M, int N, int K, int a_mn, int b_mn, float* D,
                   cudaStream_t s) {
  umma::GemmShape sh{M, N, K, ceil_div(K, umma::BK), nullptr, nullptr, nullptr};
  umma::EpiStore ep{D, N};
  if (a_mn && b_mn) return umma::launch_gemm<128, true, true, X3>(ops, sh, ep, 1, s);
  if (a_mn) return umma::launch_gemm<128, true, false, X3>(ops, sh, ep, 1, s);
  if (b_mn) return umma::launch_gemm<128, false, true, X3>(ops, sh, ep, 1, s);
  return umma::launch_gemm<128, false, false, X3>(ops, sh, ep, 1, s);
}

}  // namespace

// D[M, N] = sum_k A(m, k) B(n, k). A is [M, K] row-major (a_mn = 0) or [K, M] row-major
// (a_mn = 1); B is [N, K] (b_mn = 0) or [K, N] (b_mn = 1). bf16 in, fp32 out.
extern "C" int bt_gemm_bf16(const void* A, const void* B, float* D, int32_t M, int32_t N,
                            int32_t K, int32_t a_mn, int32_t b_mn, int32_t splits, float* partial,
                            void* stream) {
  (void)splits;
  (void)partial;
  BT_CHECK_ARG(A && B && D, "bt_gemm_bf16: null pointer");
  BT_CHECK_ARG(M > 0 && N > 0 && K > 0, "bt_gemm_bf16: bad shape");
  BT_CHECK_ARG(K % 8 == 0 && (a_mn ? M % 8 == 0 : true) && (b_mn ? N % 8 == 0 : true),
               "bt_gemm_bf16: contiguous extents must be multiples of 8");
  umma::Operands ops;
  BT_TRY(make_operand_maps(A, B, M, N, K, a_mn, b_mn, &ops.a, &ops.b));
  ops.a_lo = ops.a;
  ops.b_lo = ops.b;
  return run_debug_gemm<false>(ops, M, N, K, a_mn, b_mn, D, (cudaStream_t)stream);
}

// The split-precision variant: A = A_hi + A_lo, B = B_hi + B_lo (bf16 pairs), D = A_hi B_hi
// + A_hi B_lo + A_lo B_hi.
extern "C" int bt_gemm_bf16x3(const void* A_hi, const void* A_lo, const void* B_hi,
                              const void* B_lo, float* D, int32_t M, int32_t N, int32_t K,
                              int32_t a_mn, int32_t b_mn, void* stream) {
  BT_CHECK_ARG(A_hi && A_lo && B_hi && B_lo && D, "bt_gemm_bf16x3: null pointer");
  BT_CHECK_ARG(M > 0 && N > 0 && K > 0, "bt_gemm_bf16x3: bad shape");
  BT_CHECK_ARG(K % 8 == 0 && (a_mn ? M % 8 == 0 : true) && (b_mn ? N % 8 == 0 : true),
               "bt_gemm_bf16x3: contiguous extents must be multiples of 8");
  umma::Operands ops;
  BT_TRY(make_operand_maps(A_hi, B_hi, M, N, K, a_mn, b_mn, &ops.a, &ops.b));
  BT_TRY(make_operand_maps(A_lo, B_lo, M, N, K, a_mn, b_mn, &ops.a_lo, &ops.b_lo));
  return run_debug_gemm<true>(ops, M, N, K, a_mn, b_mn, D, (cudaStream_t)stream);
}
