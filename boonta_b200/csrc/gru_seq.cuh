// The one-launch GRU sequence kernels (gru_seq.cu): parameters and launchers, shared with the
// recurrent learner path (recurrent.cu).
#pragma once

#include "common.cuh"

namespace bt {

constexpr int kErrGruBarrier = 21;

struct GruSeqParams {
  int T, H, envs;
  const int* env_count;  // nullable: live envs
  const float* xp;       // [envs * T, 3H] input projections (+ input bias)
  const float* wh;       // [H, 3H]
  const float* bhn;      // [H]
  const uint8_t* reset;  // [envs * T] (row = env * T + t)
  float* hin;            // [envs * T, H] carry entering each step
  float* h;              // [envs * T, H] outputs
  float* gr;
  float* gz;
  float* gn;
  float* ghn;
  const float* dhs;  // [envs * T, H] dL/dh_t from the heads (backward)
  float* dxp;        // [envs * T, 3H] (backward)
  float* dhp;        // [envs * T, 3H] (backward)
  unsigned int* bar;  // zeroed before the launch
  int* err;
  // The step barrier gives up after limit_ns (0: 2 s). bar_offset is added to every barrier
  // target (0 in use; the self-test sets it so that no barrier can complete).
  unsigned long long limit_ns;
  unsigned int bar_offset;
};

int gru_seq_supported(int envs, int H, bool* ok);
int launch_gru_seq_forward(const GruSeqParams& p, cudaStream_t s);
int launch_gru_seq_backward(const GruSeqParams& p, cudaStream_t s);

}  // namespace bt
