// Host side of the tensor-core heads (heads_tc.cuh): the head-kernel packing and the two
// heads-specific GEMM launches (head outputs + loss, head weight gradient).
#include "heads_tc.cuh"

namespace bt {

// W_h [F, 64] as split bf16 pairs: column j < A the actor kernel W_pi[:, j], column A the critic
// kernel w_v, the rest zero (boonta/networks/heads.py: the two Dense heads' kernels).
__global__ void heads_pack_kernel(const float* w_pi, const float* w_v, int F, int A,
                                  __nv_bfloat16* hi, __nv_bfloat16* lo) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= F * umma::kHeadCols) return;
  const int k = i / umma::kHeadCols, j = i - k * umma::kHeadCols;
  const float w = j < A ? w_pi[(size_t)k * A + j] : (j == A ? w_v[k] : 0.f);
  store_bf16(hi, lo, i, w);
}

int launch_heads_pack(const float* w_pi, const float* w_v, int F, int A, __nv_bfloat16* hi,
                      __nv_bfloat16* lo, cudaStream_t stream) {
  const int n = F * umma::kHeadCols;
  heads_pack_kernel<<<ceil_div(n, 256), 256, 0, stream>>>(w_pi, w_v, F, A, hi, lo);
  BT_LAUNCH_CHECK("heads_pack_kernel");
  return BT_OK;
}

int launch_heads_tc_loss(const umma::Operands& ops, int rows, int F,
                         const umma::EpiHeadsLoss& ep, int* err, cudaStream_t stream) {
  umma::GemmShape sh{rows, umma::kHeadCols, F, ceil_div(F, umma::BK), nullptr, nullptr, err};
  return umma::launch_gemm<umma::kHeadCols, false, true, true>(ops, sh, ep, 1, stream);
}

int launch_heads_tc_act(const umma::Operands& ops, int rows, int F, const umma::EpiHeadsAct& ep,
                        int* err, cudaStream_t stream) {
  umma::GemmShape sh{rows, umma::kHeadCols, F, ceil_div(F, umma::BK), nullptr, nullptr, err};
  return umma::launch_gemm<umma::kHeadCols, false, true, true>(ops, sh, ep, 1, stream);
}

int launch_heads_tc_dw(const umma::Operands& ops, int F, int rows, int kblocks_per_split,
                       int splits, const int* count, const umma::EpiHeadsDw& ep, int* err,
                       cudaStream_t stream) {
  umma::GemmShape sh{F + 1, umma::kHeadCols, rows, kblocks_per_split, nullptr, count, err};
  return umma::launch_gemm<umma::kHeadCols, true, true, true>(ops, sh, ep, splits, stream);
}

}  // namespace bt
