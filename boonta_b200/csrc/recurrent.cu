// a15: RecurrentPPO.update with a GRU torso (boonta/algorithms/recurrent_ppo.py:98-281,
// boonta/networks/blocks/rnn.py:11-59, flax GRUCell), on the same learner handle.
//
// A minibatch is a set of whole env sequences (recurrent_ppo.py:269-276). Rows are
// env-major, row = e * T + t (the [mb, T] layout of recurrent_ppo.py:217-223), so the live
// rows of a padded minibatch are a prefix and the per-time-step slices are strided views.
//
//   Dense layers      GEMMs over all rows (the obs rows gathered through row -> t*N + n)
//   GRU input proj.   one GEMM over all rows: xp = [x, 1] [W_i; b_i]           [rows, 3H]
//   recurrence        for t = 0..T-1: hp = hin_t W_h (GEMM over the live envs), then one
//                     elementwise kernel: gates r, z, n, h_t, and the next step's
//                     hin_{t+1} = reset_{t+1} ? 0 : h_t (rnn.py:42-45)
//   heads + loss      the fused heads kernel over all rows (features = h_t)
//   BPTT              for t = T-1..0: gate gradients (dxp_t, dhp_t) from dL/dh_t, then the
//                     carry gradient dL/dh_{t-1} = reset_t ? 0 : (dh z + dhp_t W_h^T)
//                     (a GEMM whose epilogue adds dh z and applies the reset)
//   weight grads      GEMMs over all rows: [x,1]^T dxp, hin^T dhp, column sums for b_hn,
//                     and dX of the GRU input feeding the Dense layers' backward
// Everything is fp32 on CUDA cores (the recurrent workload's stated arithmetic).
#include <algorithm>

#include "gemm_simt.cuh"
#include "gru_seq.cuh"
#include "learner.h"

namespace bt {

int comm_allreduce_f64(Comm* c, double* buf, size_t n, cudaStream_t stream);


namespace {

// Row metadata of an env minibatch: idx[e*T + t] = t*N + env[e]; reset flags from
// first.done (or the explicit flags of the tail sequence); live rows = count * T.
__global__ void rnn_rows_kernel(const int* env, int envs, const int* env_count, int T, int N,
                                const uint8_t* first_done, int* idx, uint8_t* reset,
                                int* rows_live) {
  const int live = live_rows(env_count, envs);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i == 0) *rows_live = live * T;
  if (i >= (int64_t)live * T) return;
  const int e = (int)(i / T), t = (int)(i - (int64_t)e * T);
  const int n = env ? env[e] : e;
  const int flat = t * N + n;
  idx[i] = flat;
  reset[i] = first_done[flat];
}

__global__ void set_int_kernel(int* p, int v) {
  if (blockIdx.x == 0 && threadIdx.x == 0) *p = v;
}

// Tail sequence (recurrent_ppo.py:188-198): rows e*2 + {0, 1}; resets first.done[T-1] and
// second.done[T-1] = terminated | truncated at T-1.
__global__ void tail_rows_kernel(int N, int T, const uint8_t* first_done, const uint8_t* term,
                                 const uint8_t* trunc, uint8_t* reset, int* idx) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= N) return;
  const size_t last = (size_t)(T - 1) * N + e;
  reset[2 * e] = first_done[last];
  reset[2 * e + 1] = (uint8_t)(term[last] | trunc[last]);
  idx[2 * e] = 2 * e;
  idx[2 * e + 1] = 2 * e + 1;
}

// hin for step 0: reset ? 0 : carry[env].
__global__ void gru_init_kernel(const float* carry, const int* env, const int* env_count,
                                int envs, int T, int H, const uint8_t* reset, float* hin) {
  const int live = live_rows(env_count, envs);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)live * H) return;
  const int e = (int)(i / H), k = (int)(i - (int64_t)e * H);
  const int n = env ? env[e] : e;
  const size_t row = (size_t)e * T;
  hin[row * H + k] = reset[row] ? 0.f : carry[(size_t)n * H + k];
}

// Gates of step t (flax GRUCell): r = s(xr + hr), z = s(xz + hz), n = tanh(xn + r (hn + b_hn)),
// h = (1 - z) n + z hin; saves r, z, n, hn + b_hn; writes hin of step t + 1.
__global__ void gru_fwd_step_kernel(int t, int T, int H, int envs, const int* env_count,
                                    const float* xp, const float* hp, const float* bhn,
                                    const uint8_t* reset, float* hin, float* h, float* gr,
                                    float* gz, float* gn, float* ghn) {
  const int live = live_rows(env_count, envs);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)live * H) return;
  const int e = (int)(i / H), k = (int)(i - (int64_t)e * H);
  const size_t row = (size_t)e * T + t;
  const float* x = xp + row * 3 * H;
  const float* p = hp + (size_t)e * 3 * H;
  const float r = 1.f / (1.f + expf(-(x[k] + p[k])));
  const float z = 1.f / (1.f + expf(-(x[H + k] + p[H + k])));
  const float hn = p[2 * H + k] + bhn[k];
  const float n = tanhf(x[2 * H + k] + r * hn);
  const float hi = hin[row * H + k];
  const float out = (1.f - z) * n + z * hi;
  h[row * H + k] = out;
  gr[row * H + k] = r;
  gz[row * H + k] = z;
  gn[row * H + k] = n;
  ghn[row * H + k] = hn;
  if (t + 1 < T) hin[(row + 1) * H + k] = reset[row + 1] ? 0.f : out;
}

// Gate gradients of step t from dh = dL/dh_t (heads) + the carry gradient from step t+1.
__global__ void gru_bwd_step_kernel(int t, int T, int H, int envs, const int* env_count,
                                    const float* dhs, const float* dh_carry, const float* hin,
                                    const float* gr, const float* gz, const float* gn,
                                    const float* ghn, float* dxp, float* dhp, float* dh_direct) {
  const int live = live_rows(env_count, envs);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)live * H) return;
  const int e = (int)(i / H), k = (int)(i - (int64_t)e * H);
  const size_t row = (size_t)e * T + t;
  const size_t j = row * H + k;
  const float dh = dhs[j] + (t + 1 < T ? dh_carry[(size_t)e * H + k] : 0.f);
  const float r = gr[j], z = gz[j], n = gn[j], hn = ghn[j], hi = hin[j];
  const float dn = dh * (1.f - z);
  const float dz = dh * (hi - n);
  const float dan = dn * (1.f - n * n);
  const float dar = (dan * hn) * r * (1.f - r);
  const float daz = dz * z * (1.f - z);
  float* dx = dxp + row * 3 * H;
  float* dp = dhp + row * 3 * H;
  dx[k] = dar;
  dx[H + k] = daz;
  dx[2 * H + k] = dan;
  dp[k] = dar;
  dp[H + k] = daz;
  dp[2 * H + k] = dan * r;
  dh_direct[(size_t)e * H + k] = dh * z;
}

// Epilogue of the per-step dhp W_h^T GEMM: carry gradient into step t - 1.
struct EpiCarry {
  float* out;             // dh_carry [envs, H]
  const float* direct;    // dh * z [envs, H]
  const uint8_t* reset;   // row flags
  int T, t, H;
  __device__ __forceinline__ void store(int m, int n, float v, int) const {
    const size_t i = (size_t)m * H + n;
    out[i] = reset[(size_t)m * T + t] ? 0.f : v + direct[i];
  }
};

template <class K, class... A>
int launch_elementwise(K kernel, int64_t n, cudaStream_t s, A... args) {
  if (n <= 0) return BT_OK;
  kernel<<<(unsigned)ceil_div64(n, 256), 256, 0, s>>>(args...);
  BT_LAUNCH_CHECK("recurrent elementwise kernel");
  return BT_OK;
}

int pick_splits_k(int M, int N, int K) {
  const int tiles = ceil_div(M, kBM) * ceil_div(N, kBN);
  int s = std::max(1, (2 * kNumSMs) / tiles);
  return std::min(s, std::max(1, K / 256));
}

LayerPlan& gru_layer(bt_learner* L) { return L->towers[0].layers.back(); }

GruSeqParams seq_params(bt_learner* L, LayerPlan& g, const int* env_count, int envs, int T) {
  GruSeqParams q{};
  q.T = T;
  q.H = g.hidden;
  q.envs = envs;
  q.env_count = env_count;
  q.xp = g.xp;
  q.wh = L->params + g.wh_off;
  q.bhn = L->params + g.bhn_off;
  q.reset = L->rnn_reset;
  q.hin = g.hin;
  q.h = g.h;
  q.gr = g.gr;
  q.gz = g.gz;
  q.gn = g.gn;
  q.ghn = g.ghn;
  q.dhs = g.d_pre;
  q.dxp = g.dxp;
  q.dhp = g.dhp;
  q.bar = g.seq_bar;
  q.err = L->err_d;
  return q;
}

// Forward of the GRU over `envs` sequences of length T (rows e*T + t), input x [rows, kin].
int gru_forward(bt_learner* L, LayerPlan& g, const float* x, const float* carry, const int* env,
                const int* env_count, const int* rows_live, int envs, int T, cudaStream_t s) {
  const int H = g.hidden, rows = envs * T;
  // xp = [x, 1] [W_i; b_i]
  if (g.tc_proj) {
    BT_K(L, kProfMisc, s, launch_gather_bf16(x, nullptr, rows, g.kin, g.ldxg, g.xb, g.xb_lo,
                                             rows_live, s));
    umma::GemmShape sh{rows, 3 * H, g.kin, ceil_div(g.kin, umma::BK), rows_live, nullptr,
                       L->err_d};
    umma::EpiFwd ep;
    ep.f32_map = g.map_xp;
    ep.hi_map = g.map_xp;
    ep.lo_map = g.map_xp;
    ep.bias = L->params + g.wi_off + (size_t)g.kin * 3 * H;
    ep.act = BT_ACT_NONE;
    ep.has_f32 = true;
    ep.has_hi = ep.has_lo = false;
    BT_K(L, kProfGemmFwd, s, umma::launch_gemm<128, false, true, true>(g.proj_ops, sh, ep, 1, s));
  } else {
    ARows a{x, nullptr, g.kin, g.kin};
    BRows b{L->params + g.wi_off, 3 * H, g.kin + 1};
    EpiForward ep{g.xp, nullptr, 3 * H, BT_ACT_NONE};
    BT_K(L, kProfGemmFwd, s, launch_gemm_simt(a, b, ep, rows, 3 * H, g.kin + 1, 1, s, rows_live, nullptr));
  }
  BT_K(L, kProfMisc, s, launch_elementwise(gru_init_kernel, (int64_t)envs * H, s, carry, env,
                                           env_count, envs, T, H, (const uint8_t*)L->rnn_reset,
                                           g.hin));
  if (envs == L->units_cap ? g.seq_mb : (envs == L->N && T == 2 && g.seq_tail)) {
    // the whole recurrence in one launch
    BT_K(L, kProfGemmFwd, s, launch_gru_seq_forward(seq_params(L, g, env_count, envs, T), s));
    return BT_OK;
  }
  for (int t = 0; t < T; ++t) {
    ARows a{g.hin + (size_t)t * H, nullptr, T * H, H};
    BRows b{L->params + g.wh_off, 3 * H, H};
    EpiForward ep{g.hp, nullptr, 3 * H, BT_ACT_NONE};
    BT_K(L, kProfGemmFwd, s, launch_gemm_simt_small<32>(a, b, ep, envs, 3 * H, H, s, env_count));
    BT_K(L, kProfMisc, s, launch_elementwise(gru_fwd_step_kernel, (int64_t)envs * H, s, t, T, H,
                                             envs, env_count, (const float*)g.xp,
                                             (const float*)g.hp,
                                             (const float*)(L->params + g.bhn_off),
                                             (const uint8_t*)L->rnn_reset, g.hin, g.h, g.gr, g.gz,
                                             g.gn, g.ghn));
  }
  return BT_OK;
}

int gru_backward_steps(bt_learner* L, LayerPlan& g, const int* env_count, int envs, int T,
                       cudaStream_t s);
int gru_weight_grads(bt_learner* L, LayerPlan& g, LayerPlan& prev, const int* rows_live,
                     int rows, cudaStream_t s);

int gru_backward(bt_learner* L, LayerPlan& g, LayerPlan& prev, const int* env_count,
                 const int* rows_live, int envs, int T, cudaStream_t s) {
  const int H = g.hidden, rows = envs * T;
  if (envs == L->units_cap && g.seq_mb) {
    // backward through time in one launch
    BT_K(L, kProfGemmDx, s, launch_gru_seq_backward(seq_params(L, g, env_count, envs, T), s));
  } else {
    BT_TRY(gru_backward_steps(L, g, env_count, envs, T, s));
  }
  BT_TRY(gru_weight_grads(L, g, prev, rows_live, rows, s));
  return BT_OK;
}

int gru_backward_steps(bt_learner* L, LayerPlan& g, const int* env_count, int envs, int T,
                       cudaStream_t s) {
  const int H = g.hidden;
  for (int t = T - 1; t >= 0; --t) {
    BT_K(L, kProfMisc, s, launch_elementwise(gru_bwd_step_kernel, (int64_t)envs * H, s, t, T, H,
                                             envs, env_count, (const float*)g.d_pre,
                                             (const float*)g.dh_carry, (const float*)g.hin,
                                             (const float*)g.gr, (const float*)g.gz,
                                             (const float*)g.gn, (const float*)g.ghn, g.dxp,
                                             g.dhp, g.dh_direct));
    if (t > 0) {
      ARows a{g.dhp + (size_t)t * 3 * H, nullptr, T * 3 * H, 3 * H};
      BCols b{L->params + g.wh_off, 3 * H, 3 * H};
      EpiCarry ep{g.dh_carry, g.dh_direct, L->rnn_reset, T, t, H};
      BT_K(L, kProfGemmDx, s, launch_gemm_simt_small<16>(a, b, ep, envs, H, 3 * H, s, env_count));
    }
  }
  return BT_OK;
}

int gru_weight_grads(bt_learner* L, LayerPlan& g, LayerPlan& prev, const int* rows_live,
                     int rows, cudaStream_t s) {
  const int H = g.hidden;
  if (g.tc_proj) {
    // the projection gradients and the carries as split bf16 pairs (the x operand is still
    // in place from the forward), then three tcgen05 GEMMs
    const int H3 = 3 * H;
    BT_K(L, kProfMisc, s, launch_split_rows_bf16(g.dxp, rows, H3, g.dxpb, g.dxpb_lo, rows_live, s));
    BT_K(L, kProfMisc, s, launch_split_rows_bf16(g.dhp, rows, H3, g.dhpb, g.dhpb_lo, rows_live, s));
    BT_K(L, kProfMisc, s, launch_split_rows_bf16(g.hin, rows, H, g.hinb, g.hinb_lo, rows_live, s));
    {
      umma::GemmShape sh{g.kin + 1, H3, rows, g.wi_kbps, nullptr, rows_live, L->err_d};
      umma::EpiDw ep{g.wi_part, H3, (size_t)(g.kin + 1) * H3};
      BT_K(L, kProfGemmDw, s, umma::launch_gemm<128, true, true, true>(g.wi_ops, sh, ep, g.wi_splits, s));
    }
    {
      umma::GemmShape sh{H, H3, rows, g.wh_kbps, nullptr, rows_live, L->err_d};
      umma::EpiDw ep{g.wh_part, H3, (size_t)H * H3};
      BT_K(L, kProfGemmDw, s, umma::launch_gemm<128, true, true, true>(g.wh_ops, sh, ep, g.wh_splits, s));
    }
    {
      ACols a{g.hin, nullptr, H, 0};  // ones row only: column sums of dhp's n part -> b_hn
      BRows b{g.dhp + 2 * H, 3 * H, rows};
      EpiPartial ep{g.bhn_part, H, (size_t)H};
      BT_K(L, kProfGemmDw, s, launch_gemm_simt(a, b, ep, 1, H, rows, g.bhn_splits, s, nullptr,
                                               rows_live));
    }
    {
      umma::GemmShape sh{rows, g.kin, H3, ceil_div(H3, umma::BK), rows_live, nullptr, L->err_d};
      umma::EpiDx epx;
      epx.in_map = prev.map_pre;
      epx.f32_map = prev.map_dpre;
      epx.hi_map = prev.map_dpre;
      epx.lo_map = prev.map_dpre;
      epx.act = prev.act;
      epx.has_f32 = true;
      epx.has_hi = epx.has_lo = false;
      BT_K(L, kProfGemmDx, s, umma::launch_gemm<128, false, false, true>(g.gdx_ops, sh, epx, 1, s));
    }
    return BT_OK;
  }
  // weight gradients over all live rows
  {
    ACols a{prev.h, nullptr, g.kin, g.kin};  // [x, 1]^T dxp -> [W_i; b_i]
    BRows b{g.dxp, 3 * H, rows};
    EpiPartial ep{g.wi_part, 3 * H, (size_t)(g.kin + 1) * 3 * H};
    BT_K(L, kProfGemmDw, s, launch_gemm_simt(a, b, ep, g.kin + 1, 3 * H, rows, g.wi_splits, s, nullptr,
                                             rows_live));
  }
  {
    ACols a{g.hin, nullptr, H, H};  // hin^T dhp -> W_h (no bias row: M = H)
    BRows b{g.dhp, 3 * H, rows};
    EpiPartial ep{g.wh_part, 3 * H, (size_t)H * 3 * H};
    BT_K(L, kProfGemmDw, s, launch_gemm_simt(a, b, ep, H, 3 * H, rows, g.wh_splits, s, nullptr,
                                             rows_live));
  }
  {
    ACols a{g.hin, nullptr, H, 0};  // ones row only: column sums of dhp's n part -> b_hn
    BRows b{g.dhp + 2 * H, 3 * H, rows};
    EpiPartial ep{g.bhn_part, H, (size_t)H};
    BT_K(L, kProfGemmDw, s, launch_gemm_simt(a, b, ep, 1, H, rows, g.bhn_splits, s, nullptr,
                                             rows_live));
  }
  // dL/d x = dxp W_i^T, times the previous layer's activation derivative
  {
    ARows a{g.dxp, nullptr, 3 * H, 3 * H};
    BCols b{L->params + g.wi_off, 3 * H, 3 * H};
    EpiActGrad ep{prev.d_pre, prev.pre(), prev.h, prev.kout, prev.act};
    BT_K(L, kProfGemmDx, s, launch_gemm_simt(a, b, ep, rows, g.kin, 3 * H, 1, s, rows_live, nullptr));
  }
  return BT_OK;
}

int recurrent_heads(bt_learner* L, LayerPlan& g, const MinibatchInputs& in, const int* rows_live,
                    double* stat_slot, cudaStream_t s) {
  const bt_learner_config& c = L->cfg;
  HeadsParams hp{};
  hp.rows = L->rows_cap;
  hp.count = rows_live;
  hp.idx = in.idx;
  hp.f_pi = g.h;
  hp.F_pi = L->F_pi;
  hp.f_v = g.h;
  hp.F_v = L->F_v;
  hp.w_pi = L->params + L->head_pi_off;
  hp.w_v = L->params + L->head_v_off;
  hp.scale = L->head_scale_off >= 0 ? L->params + L->head_scale_off : nullptr;
  hp.A = L->A;
  hp.head = c.network.head;
  hp.action = in.action;
  hp.lp_old = in.lp_old;
  hp.v_old = in.v_old;
  hp.adv = in.adv;
  hp.ret = in.ret;
  hp.inv_mb = in.inv_mb;
  hp.clip = c.ppo.clip_coefficient;
  hp.clip_value = c.ppo.clip_value_loss;
  hp.ent_coef = c.ppo.entropy_coefficient;
  hp.vf_coef = c.ppo.value_coefficient;
  hp.d_out = L->d_out;
  hp.d_val = L->d_val;
  hp.d_fpi = g.d_pre;  // dL/dh_t, no activation after the GRU
  hp.act_pi = BT_ACT_NONE;
  hp.act_v = BT_ACT_NONE;
  hp.stat_partials = L->stat_part;
  hp.dscale_partials = L->dscale_part;
  if (L->heads_fused_dw) {
    hp.dw_pi_partials = L->head_pi_part;
    hp.dw_v_partials = L->head_v_part;
  }
  BT_K(L, kProfHeads, s, launch_heads_loss(hp, L->heads_blocks, s));
  BT_K(L, kProfStats, s, launch_stat_reduce(L->stat_part, L->heads_blocks, stat_slot, s));
  if (!L->heads_fused_dw) {
    BT_K(L, kProfHeadDw, s, launch_skinny_dw(g.h, L->F_pi, BT_ACT_NONE, L->d_out, L->A,
                                             L->rows_cap, rows_live, L->head_pi_splits,
                                             L->head_pi_part, s));
    BT_K(L, kProfHeadDw, s, launch_skinny_dw(g.h, L->F_v, BT_ACT_NONE, L->d_val, 1, L->rows_cap,
                                             rows_live, L->head_v_splits, L->head_v_part, s));
  }
  return BT_OK;
}

}  // namespace

int allocate_gru(bt_learner* L, LayerPlan& g) {
  const int H = g.hidden, R = L->act_rows, E = L->units_cap;
  const size_t rh = (size_t)R * H, r3 = (size_t)R * 3 * H;
  BT_TRY(dalloc(L, &g.xp, r3));
  BT_TRY(dalloc(L, &g.dxp, r3));
  BT_TRY(dalloc(L, &g.dhp, r3));
  BT_TRY(dalloc(L, &g.h, rh));
  BT_TRY(dalloc(L, &g.hin, rh));
  BT_TRY(dalloc(L, &g.gr, rh));
  BT_TRY(dalloc(L, &g.gz, rh));
  BT_TRY(dalloc(L, &g.gn, rh));
  BT_TRY(dalloc(L, &g.ghn, rh));
  BT_TRY(dalloc(L, &g.d_pre, rh));
  g.z = g.h;  // no separate pre-activation
  g.d_z = g.d_pre;
  const int envs = std::max(E, L->N);
  BT_TRY(dalloc(L, &g.hp, (size_t)envs * 3 * H));
  BT_TRY(dalloc(L, &g.dh_direct, (size_t)envs * H));
  BT_TRY(dalloc(L, &g.dh_carry, (size_t)envs * H));
  BT_CUDA(cudaMemset(g.dh_carry, 0, (size_t)envs * H * 4));
  const int rows = L->rows_cap;
  g.wi_splits = pick_splits_k(g.kin + 1, 3 * H, rows);
  g.wh_splits = pick_splits_k(H, 3 * H, rows);
  {
    // the input projection, the GRU weight gradients and the dX into the previous (Dense)
    // layer on the tcgen05 GEMM in split bf16, the recurrence's own arithmetic
    std::vector<LayerPlan>& layers = L->towers[0].layers;
    const LayerPlan* prev = layers.size() >= 2 ? &layers[layers.size() - 2] : nullptr;
    g.tc_proj = prev && prev->kind == BT_LAYER_DENSE && !prev->tc && prev->kout == g.kin &&
                g.kin % 32 == 0 && H % 64 == 0;
    if (g.tc_proj) {
      const int nkb = ceil_div(rows, umma::BK);
      auto split_k = [&](int M, int* kbps, int* splits) {
        const int tiles = ceil_div(M, umma::BM) * ceil_div(3 * H, 128);
        const int sp = std::max(1, std::min(kNumSMs / tiles, nkb / 8));
        *kbps = ceil_div(nkb, sp);
        *splits = ceil_div(nkb, *kbps);
      };
      split_k(g.kin + 1, &g.wi_kbps, &g.wi_splits);
      split_k(H, &g.wh_kbps, &g.wh_splits);
    }
  }
  g.bhn_splits = pick_splits_k(1, H, rows);
  BT_TRY(dalloc(L, &g.wi_part, (size_t)g.wi_splits * (g.kin + 1) * 3 * H));
  BT_TRY(dalloc(L, &g.wh_part, (size_t)g.wh_splits * H * 3 * H));
  BT_TRY(dalloc(L, &g.bhn_part, (size_t)g.bhn_splits * H));
  L->segs_h.push_back({g.wi_part, g.wi_splits, (g.kin + 1) * 3 * H,
                       (int64_t)(g.kin + 1) * 3 * H, g.wi_off});
  L->segs_h.push_back({g.wh_part, g.wh_splits, H * 3 * H, (int64_t)H * 3 * H, g.wh_off});
  L->segs_h.push_back({g.bhn_part, g.bhn_splits, H, (int64_t)H, g.bhn_off});
  // one-launch sequence kernels where every CTA of their grid fits on the GPU at once
  BT_TRY(gru_seq_supported(E, H, &g.seq_mb));
  BT_TRY(gru_seq_supported(L->N, H, &g.seq_tail));
  BT_TRY(dalloc(L, &g.seq_bar, 1));
  // row metadata
  BT_TRY(dalloc(L, &L->rnn_idx, R));
  BT_TRY(dalloc(L, &L->rnn_reset, R));
  BT_TRY(dalloc(L, &L->rnn_rows, 1));
  BT_TRY(dalloc(L, &L->tail_obs, (size_t)2 * L->N * L->cfg.network.obs_dim));
  return BT_OK;
}

// Buffers and tensor maps of the GRU's tensor-core projections (after the parameter layout and
// the tensor-core path of the other layers are set up).
int allocate_gru_tc(bt_learner* L) {
  if (!L->recurrent) return BT_OK;
  std::vector<LayerPlan>& layers = L->towers[0].layers;
  LayerPlan& g = layers.back();
  if (!g.tc_proj) return BT_OK;
  LayerPlan& prev = layers[layers.size() - 2];
  const int H = g.hidden, K = g.kin, H3 = 3 * H, R = L->act_rows;
  auto pair = [&](__nv_bfloat16** hi, __nv_bfloat16** lo, size_t n) -> int {
    BT_TRY(dalloc(L, hi, n));
    BT_TRY(dalloc(L, lo, n));
    BT_CUDA(cudaMemset(*hi, 0, n * 2));
    BT_CUDA(cudaMemset(*lo, 0, n * 2));
    return BT_OK;
  };
  // the bf16 shadow of the parameters (refreshed when an update starts, written by every Adam
  // step) serves W_i
  if (!L->params_b) BT_TRY(pair(&L->params_b, &L->params_b_lo, L->num_params));
  g.ldxg = (K + 1 + 7) / 8 * 8;
  BT_TRY(pair(&g.xb, &g.xb_lo, (size_t)R * g.ldxg));
  BT_TRY(pair(&g.hinb, &g.hinb_lo, (size_t)R * H));
  BT_TRY(pair(&g.dxpb, &g.dxpb_lo, (size_t)R * H3));
  BT_TRY(pair(&g.dhpb, &g.dhpb_lo, (size_t)R * H3));
  const uint64_t ldx = (uint64_t)g.ldxg * 2, l3 = (uint64_t)H3 * 2, lh = (uint64_t)H * 2;
  for (int part = 0; part < 2; ++part) {
    const __nv_bfloat16* w = (part ? L->params_b_lo : L->params_b) + g.wi_off;
    const __nv_bfloat16* x = part ? g.xb_lo : g.xb;
    const __nv_bfloat16* hin = part ? g.hinb_lo : g.hinb;
    const __nv_bfloat16* dx = part ? g.dxpb_lo : g.dxpb;
    const __nv_bfloat16* dh = part ? g.dhpb_lo : g.dhpb;
    umma::Operands& pj = g.proj_ops;
    umma::Operands& wi = g.wi_ops;
    umma::Operands& wh = g.wh_ops;
    umma::Operands& gx = g.gdx_ops;
    // xp = x W_i (+ b_i in the epilogue): A = x (K-major over the K inputs), B = W_i ([K][3H])
    BT_TRY(umma::encode_map(part ? &pj.a_lo : &pj.a, x, K, R, ldx, 64, 128));
    BT_TRY(umma::encode_map(part ? &pj.b_lo : &pj.b, w, H3, K, l3, 64, 64));
    // [W_i; b_i] gradient = [x, 1]^T dxp: both MN-major over the rows
    BT_TRY(umma::encode_map(part ? &wi.a_lo : &wi.a, x, K + 1, R, ldx, 64, 64));
    BT_TRY(umma::encode_map(part ? &wi.b_lo : &wi.b, dx, H3, R, l3, 64, 64));
    // W_h gradient = hin^T dhp
    BT_TRY(umma::encode_map(part ? &wh.a_lo : &wh.a, hin, H, R, lh, 64, 64));
    BT_TRY(umma::encode_map(part ? &wh.b_lo : &wh.b, dh, H3, R, l3, 64, 64));
    // dL/dx = dxp W_i^T: A = dxp (K-major over 3H), B = W_i as [N = K][K = 3H]
    BT_TRY(umma::encode_map(part ? &gx.a_lo : &gx.a, dx, H3, R, l3, 64, 128));
    BT_TRY(umma::encode_map(part ? &gx.b_lo : &gx.b, w, H3, K, l3, 64, 128));
  }
  BT_TRY(umma::encode_tile_map(&g.map_xp, g.xp, true, H3, R, (uint64_t)H3 * 4, 128));
  const uint64_t lp4 = (uint64_t)prev.kout * 4;
  BT_TRY(umma::encode_tile_map(&prev.map_pre, prev.pre(), true, prev.kout, R, lp4, 128));
  BT_TRY(umma::encode_tile_map(&prev.map_dpre, prev.d_pre, true, prev.kout, R, lp4, 128));
  BT_CUDA(cudaDeviceSynchronize());
  return BT_OK;
}

int recurrent_update(bt_learner* L, const bt_batch* b, const int32_t* perm, float* stats,
                     cudaStream_t s) {
  BT_CHECK_ARG(b->first_done && b->carry && b->last_carry,
               "recurrent update needs first_done, carry and last_carry");
  const int world = std::max(1, L->cfg.world_size);
  BT_CHECK_ARG(world == 1 || L->comm, "world_size %d needs bt_learner_comm_init", world);
  const int E = L->cfg.ppo.update_epochs, M = L->cfg.ppo.num_minibatches;
  const int T = L->T, N = L->N, D = L->cfg.network.obs_dim;
  TowerPlan& tp = L->towers[0];
  LayerPlan& g = gru_layer(L);
  const int gi = (int)tp.layers.size() - 1;
  LayerPlan& prev = tp.layers[gi - 1];

  // ---- tail bootstrap (recurrent_ppo.py:188-198) ----
  BT_CUDA(cudaMemcpy2DAsync(L->tail_obs, 2 * D * 4, b->obs + (size_t)(T - 1) * N * D, D * 4, D * 4,
                            N, cudaMemcpyDeviceToDevice, s));
  BT_CUDA(cudaMemcpy2DAsync(L->tail_obs + D, 2 * D * 4, b->bootstrap_obs, D * 4, D * 4, N,
                            cudaMemcpyDeviceToDevice, s));
  BT_K(L, kProfMisc, s, launch_elementwise(tail_rows_kernel, N, s, N, T, b->first_done,
                                           b->terminated, b->truncated, L->rnn_reset, L->rnn_idx));
  BT_K(L, kProfMisc, s, launch_elementwise(set_int_kernel, 1, s, L->rnn_rows, 2 * N));
  BT_TRY(forward_tower(L, tp, L->tail_obs, nullptr, 2 * N, L->rnn_rows, s));
  BT_TRY(gru_forward(L, g, prev.h, b->last_carry, nullptr, nullptr, L->rnn_rows, N, 2, s));
  BT_K(L, kProfHeadsFwd, s, launch_heads_forward(g.h, L->F_v, g.h, L->F_v,
                                                 L->params + L->head_pi_off,
                                                 L->params + L->head_v_off, L->A, 2 * N,
                                                 BT_ACT_NONE, BT_ACT_NONE, nullptr, L->act_val,
                                                 L->split_pi, L->split_v, s));
  BT_CUDA(cudaMemcpy2DAsync(L->boot, 4, L->act_val + 1, 8, 4, N, cudaMemcpyDeviceToDevice, s));
  BT_K(L, kProfGae, s, launch_gae_internal(b->reward, b->terminated, b->truncated, b->value,
                                           L->boot, T, N, L->cfg.ppo.gamma, L->cfg.ppo.gae_lambda,
                                           L->adv, L->ret, L->err_d, s));
  if (L->cfg.ppo.normalize_advantage) {
    BT_K(L, kProfMisc, s, launch_adv_moments(L->adv, L->B, L->adv_part, s));
    if (L->comm) BT_TRY(comm_allreduce_f64(L->comm, L->adv_part, 2 * kNormBlocks, s));
    BT_K(L, kProfMisc, s, launch_adv_normalize(L->adv, L->B, L->adv_part, kNormBlocks,
                                               (double)L->B * world, s));
  }
  if (world > 1) {
    BT_K(L, kProfMisc, s, launch_local_indices(perm, E * M, L->mb, 0, N, L->cfg.rank, N * world,
                                               L->units_cap, L->local_idx, L->local_counts,
                                               L->err_d, s));
  }

  // ---- epochs x env-minibatches ----
  MinibatchInputs in{};
  in.obs = b->obs;
  in.action = b->action;
  in.lp_old = b->log_prob;
  in.v_old = b->value;
  in.adv = L->adv;
  in.ret = L->ret;
  in.idx = L->rnn_idx;
  in.inv_mb = 1.0f / (float)((double)L->mb * T);
  const int envs = L->units_cap;
  for (int e = 0; e < E; ++e) {
    for (int m = 0; m < M; ++m) {
      const int i = e * M + m;
      const int* env = world > 1 ? L->local_idx + (size_t)i * envs
                                 : perm + (size_t)e * N * world + (size_t)m * L->mb;
      const int* env_count = world > 1 ? L->local_counts + i : nullptr;
      BT_K(L, kProfMisc, s, launch_elementwise(rnn_rows_kernel, (int64_t)envs * T, s, env, envs,
                                               env_count, T, N, b->first_done, L->rnn_idx,
                                               L->rnn_reset, L->rnn_rows));
      BT_TRY(forward_tower(L, tp, b->obs, L->rnn_idx, L->rows_cap, L->rnn_rows, s));
      BT_TRY(gru_forward(L, g, prev.h, b->carry, env, env_count, L->rnn_rows, envs, T, s));
      double* slot = L->stat_sums + (size_t)i * kNumStatSums;
      BT_TRY(recurrent_heads(L, g, in, L->rnn_rows, slot, s));
      BT_TRY(gru_backward(L, g, prev, env_count, L->rnn_rows, envs, T, s));
      BT_TRY(backward_tower(L, tp, b->obs, L->rnn_idx, L->rows_cap, L->rnn_rows, s, gi - 1));
      BT_K(L, kProfReduce, s, launch_reduce_segments(L->segs_d, L->chunks_d, L->num_chunks,
                                                     L->grads, world == 1 ? L->norm_part : nullptr,
                                                     s));
      BT_TRY(optimizer_step(L, i, s));
    }
  }
  if (exchange_active(L)) BT_TRY(exchange_gather_moments(L, s));
  BT_K(L, kProfMisc, s, launch_increment(L->count_d, E * M, s));
  if (L->comm) BT_TRY(comm_allreduce_f64(L->comm, L->stat_sums, (size_t)E * M * kNumStatSums, s));
  if (stats) {
    BT_K(L, kProfStats, s, launch_stat_finalize(L->stat_sums, E * M,
                                                1.0f / (float)((double)L->mb * T), stats, s));
  }
  return BT_OK;
}


// a14 for GRU networks (RecurrentPPO.step, boonta/algorithms/recurrent_ppo.py:72-96): one
// time step of the network on `num` envs from the caller's carry (zero where reset, the
// rnn.py:42-45 rule), the heads, and the sample; the new carry goes to carry_out.
int recurrent_act(bt_learner* L, const float* obs, const uint8_t* reset, const float* carry,
                  int num, const float* noise, float temperature, void* action, float* log_prob,
                  float* value, float* carry_out, cudaStream_t s) {
  TowerPlan& tp = L->towers[0];
  LayerPlan& g = gru_layer(L);
  const int gi = (int)tp.layers.size() - 1;
  LayerPlan& prev = tp.layers[gi - 1];
  const int H = g.hidden;
  BT_CUDA(cudaMemcpyAsync(L->rnn_reset, reset, (size_t)num, cudaMemcpyDeviceToDevice, s));
  BT_K(L, kProfMisc, s, launch_elementwise(set_int_kernel, 1, s, L->rnn_rows, num));
  BT_TRY(forward_tower(L, tp, obs, nullptr, num, L->rnn_rows, s));
  BT_TRY(gru_forward(L, g, prev.h, carry, nullptr, nullptr, L->rnn_rows, num, 1, s));
  // head outputs and the sample in one kernel
  BT_K(L, kProfHeadsFwd, s,
       launch_heads_act(g.h, L->F_pi, g.h, L->F_v, L->params + L->head_pi_off,
                        L->params + L->head_v_off,
                        L->head_scale_off >= 0 ? L->params + L->head_scale_off : nullptr,
                        L->cfg.network.head, L->A, num, BT_ACT_NONE, BT_ACT_NONE, L->split_pi,
                        L->split_v, noise, temperature, action, log_prob, value, s));
  // rows are env-major with T = 1, so the step's outputs are the carry rows in env order
  BT_CUDA(cudaMemcpyAsync(carry_out, g.h, (size_t)num * H * sizeof(float),
                          cudaMemcpyDeviceToDevice, s));
  return BT_OK;
}

}  // namespace bt
