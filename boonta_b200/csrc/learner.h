// Internal state of a learner handle (one per GPU and stream).
#pragma once

#include <cuda.h>

#include <string>
#include <vector>

#include "gemm_sm100.cuh"
#include "kernels.cuh"

struct ParamEntryC {
  std::string name;
  int64_t offset;
  std::vector<int64_t> shape;
};

struct LayerPlan {
  int kind = BT_LAYER_DENSE;
  int act = BT_ACT_NONE;
  int ln = 0;
  int kin = 0;    // input width (dense), 9*C (conv patch)
  int kout = 0;   // output width per row (conv: H*W*Cout)
  int ncol = 0;   // GEMM N: dense kout, conv Cout
  int H = 0, W = 0, C = 0;
  int64_t w_off = 0, ln_off = 0;
  float* z = nullptr;     // pre-activation (pre-LayerNorm)
  float* y = nullptr;     // LayerNorm output (LN layers)
  float* h = nullptr;     // layer output
  float* mean = nullptr;  // LN row statistics
  float* rstd = nullptr;
  float* d_pre = nullptr;  // dL/d(pre-activation): d y for LN layers, d z otherwise
  float* d_z = nullptr;    // dL/dz (== d_pre without LayerNorm)
  float* dw_part = nullptr;
  int dw_splits = 1;
  float* ln_part = nullptr;
  int ln_blocks = 0;
  // tensor-core (bf16) path
  bool tc = false;
  bool out_b = false;  // (conv) also writes its output as the bf16 operand hb/hb_lo
  __nv_bfloat16* xin_b = nullptr;  // bf16 input operand [rows, ldx], ones column at kin
  int ldx = 0;
  __nv_bfloat16* hb = nullptr;  // bf16 output [rows, ldh], ones column at kout
  int ldh = 0;
  __nv_bfloat16* dzb = nullptr;  // bf16 dL/dz [rows, kout]
  __nv_bfloat16* hb_lo = nullptr;   // split mode: low halves of hb / dzb / xin_b
  __nv_bfloat16* dzb_lo = nullptr;
  __nv_bfloat16* xin_lo = nullptr;
  bt::umma::Operands fwd_ops, dx_ops, dw_ops;
  // epilogue tile maps (32 x 32 boxes): z and pre() (fp32), hb / hb_lo and dzb / dzb_lo (bf16),
  // d_pre (fp32, LayerNorm layers)
  CUtensorMap map_z, map_pre, map_hb, map_hb_lo, map_dzb, map_dzb_lo, map_dpre;
  int fwd_bn = 128;
  int dw_bn = 128;
  int dw_kbps = 1;
  // GRU (recurrent torso); rows are env-major (row = env * T + t)
  int hidden = 0;
  int64_t wi_off = 0, wh_off = 0, bhn_off = 0;
  float* xp = nullptr;    // input projections [rows, 3H] (+ input bias)
  float* hin = nullptr;   // carry entering each step (after the reset) [rows, H]
  float* gr = nullptr;    // saved gates r, z, n and (h W_hn + b_hn) [rows, H] each
  float* gz = nullptr;
  float* gn = nullptr;
  float* ghn = nullptr;
  float* hp = nullptr;    // one step's hidden projection [envs, 3H]
  float* dxp = nullptr;   // dL/d input projections [rows, 3H]
  float* dhp = nullptr;   // dL/d hidden projections [rows, 3H]
  float* dh_direct = nullptr;  // dh * z of the current step [envs, H]
  float* dh_carry = nullptr;   // gradient flowing into the previous step's output [envs, H]
  // one-launch sequence kernels (gru_seq.cu) usable for the minibatch / the tail sequence
  bool seq_mb = false, seq_tail = false;
  unsigned int* seq_bar = nullptr;  // their step-barrier counter
  float* wi_part = nullptr;    // split partials of d[W_i; b_i], dW_h, db_hn
  float* wh_part = nullptr;
  float* bhn_part = nullptr;
  int wi_splits = 1, wh_splits = 1, bhn_splits = 1;
  // GRU projections on the tcgen05 GEMM in split bf16 (tc_proj): the input x, the carries and
  // the projection gradients as split bf16 pairs, the maps of the four GEMMs
  bool tc_proj = false;
  int ldxg = 0, wi_kbps = 1, wh_kbps = 1;
  __nv_bfloat16 *xb = nullptr, *xb_lo = nullptr;      // [rows, ldxg], ones column at kin
  __nv_bfloat16 *hinb = nullptr, *hinb_lo = nullptr;  // [rows, H]
  __nv_bfloat16 *dxpb = nullptr, *dxpb_lo = nullptr;  // [rows, 3H]
  __nv_bfloat16 *dhpb = nullptr, *dhpb_lo = nullptr;  // [rows, 3H]
  bt::umma::Operands proj_ops{}, wi_ops{}, wh_ops{}, gdx_ops{};
  CUtensorMap map_xp;
  // LayerNorm + ReLU tensor-core layer whose consumers take relu'(y) from the bf16 output hb
  // (the next layer's dX epilogue, or the tensor-core heads): the update's minibatch forward
  // does not write y
  bool relu_from_hb = false;
  const float* pre() const { return ln ? y : z; }
};

struct TowerPlan {
  std::vector<LayerPlan> layers;
  int in_dim = 0;
  int out_dim = 0;
};

struct Comm;      // NCCL communicator (comm.cu)
struct Exchange;  // NVLink peer-memory gradient exchange (exchange.cu)

// Kernel classes of the per-class device-time profile (bt_learner_profile_read).
enum ProfClass {
  kProfGae = 0, kProfGemmFwd, kProfGemmDx, kProfGemmDw, kProfHeads, kProfHeadsFwd, kProfLnFwd,
  kProfLnBwd, kProfReduce, kProfAdam, kProfStats, kProfAllreduce, kProfMisc, kProfHeadDw,
  kProfNumClasses
};
extern const char* const kProfNames[kProfNumClasses];

struct ProfRecord {
  int cls;
  cudaEvent_t a, b;
};

// CUDA-event timing of every launch of the learner, by kernel class (off by default).
struct Profiler {
  bool on = false;
  std::vector<cudaEvent_t> pool;
  size_t used = 0;
  std::vector<ProfRecord> recs;
  int64_t launches = 0;  // kernels (and collectives) enqueued since creation
};

struct bt_learner {
  bt_learner_config cfg{};
  int device = 0;
  std::vector<ParamEntryC> entries;
  int64_t num_params = 0;
  // state (flat layout)
  float* params = nullptr;
  float* grads = nullptr;
  float* mu = nullptr;
  float* nu = nullptr;
  int* count_d = nullptr;   // adam count
  int* err_d = nullptr;     // device error word
  int* mb_count_d = nullptr;  // live rows for bt_learner_loss_grads
  // tensor-core path
  bool tc_any = false;
  bool tc_first = false;  // some tower starts with a tensor-core layer (reads L->xg)
  bool x3 = false;                    // split-bf16 (BT_PREC_BF16X3) operands
  __nv_bfloat16* params_b = nullptr;  // bf16 shadow of params (written by every Adam step)
  __nv_bfloat16* params_b_lo = nullptr;
  __nv_bfloat16* xg = nullptr;        // gathered minibatch observations [rows, ldx0]
  // bf16 copy of the rollout's observations [T*N, ldx0] (wide bf16 inputs): each update
  // minibatch gathers its rows from it (gather_rows, set per minibatch)
  __nv_bfloat16* obs_b = nullptr;
  bool gather_rows = false;
  bool fill_obs_b = false;  // first epoch: gather from the fp32 rollout and fill obs_b
  __nv_bfloat16* xg_lo = nullptr;
  int ldx0 = 0;
  // network
  TowerPlan towers[2];
  int ntowers = 1;
  bool shared = true;
  int A = 0;
  int F_pi = 0, F_v = 0;
  int64_t head_pi_off = 0, head_scale_off = -1, head_v_off = 0;
  // sizes
  int T = 0, N = 0;
  int64_t B = 0;     // T*N on this rank
  int mb = 0;        // global minibatch size (rows, or envs for recurrent)
  int units_cap = 0; // local minibatch capacity in permutation units (rows, or envs)
  int rows_cap = 0;  // local minibatch capacity (rows)
  bool recurrent = false;
  // recurrent path: per-minibatch row metadata
  int* rnn_idx = nullptr;       // [rows] flat sample index t*N + n of row env*T + t
  uint8_t* rnn_reset = nullptr; // [rows] reset the carry before this step
  int* rnn_rows = nullptr;      // live rows (device) = live envs * T
  float* tail_obs = nullptr;    // [2N, obs_dim] (first.obs[T-1], second.obs[T-1]) per env
  int act_rows = 0;  // rows of the activation buffers
  // heads
  float* d_out = nullptr;
  float* d_val = nullptr;
  float* head_pi_part = nullptr;
  int head_pi_splits = 1;
  float* head_v_part = nullptr;
  int head_v_splits = 1;
  float* dscale_part = nullptr;
  double* stat_part = nullptr;
  int heads_blocks = 0;
  bool heads_fused_dw = false;  // the heads kernel writes the head weight-gradient partials
  bool split_pi = false, split_v = false;  // heads evaluated with split-bf16 products
  // tensor-core heads (heads_tc.cuh): packed head kernels W_h [F, 64], the head-output
  // gradient D [act_rows, 64] (split bf16 pairs), the maps of the three head GEMMs
  bool tc_heads = false;
  __nv_bfloat16 *whb = nullptr, *whb_lo = nullptr;
  __nv_bfloat16 *dhb = nullptr, *dhb_lo = nullptr;
  bt::umma::Operands head_o_ops{}, head_dx_ops{}, head_dw_ops{};
  int head_dw_kbps = 1;
  // targets
  float* adv = nullptr;
  float* ret = nullptr;
  float* boot = nullptr;
  float* act_out = nullptr;  // act: [rows, A] head outputs
  float* act_val = nullptr;
  // reductions
  std::vector<bt::Segment> segs_h;
  bt::Segment* segs_d = nullptr;
  bt::ReduceChunk* chunks_d = nullptr;
  int num_chunks = 0;
  double* norm_part = nullptr;
  double* stat_sums = nullptr;  // [E*M + 1][kNumStatSums]
  double* adv_part = nullptr;
  // multi-GPU
  int* local_idx = nullptr;
  int* local_counts = nullptr;
  Comm* comm = nullptr;
  Exchange* xchg = nullptr;  // set up with the communicator when every peer can be mapped
  bool use_xchg = true;
  std::vector<void*> allocations;
  Profiler prof;
  // Side streams for independent work inside one update (the critic tower next to the
  // actor's; dW GEMMs next to the dX chain). Work forks from and joins back into the
  // caller's stream through events, so the call keeps the caller's stream order.
  cudaStream_t side[4] = {nullptr, nullptr, nullptr, nullptr};
  std::vector<cudaEvent_t> fork_events;
  // CUDA-graph replay of bt_learner_update: the first call with a given set of batch
  // pointers runs eagerly, the second captures the update into a graph, later calls with
  // the same pointers replay it. Permutations and statistics pass through the stable
  // buffers perm_d / stats_d so that they do not change the captured arguments.
  bool graphs_on = true;
  cudaStream_t cap_stream = nullptr;  // captures run here (the caller's may be the legacy stream)
  cudaGraphExec_t graph = nullptr;
  int64_t graph_launches = 0;  // kernels and collectives in the graph
  const void* graph_key[12] = {};
  const void* seen_key[12] = {};
  int32_t* perm_d = nullptr;
  float* stats_d = nullptr;
  size_t next_event = 0;
};


cudaEvent_t prof_event(bt_learner* L);

// Side stream i for work that may overlap the caller's stream s. While profiling, every
// launch stays on s, so that each recorded event pair times one kernel alone on the GPU.
inline cudaStream_t side_stream(bt_learner* L, int i, cudaStream_t s) {
  return L->prof.on ? s : L->side[i];
}

template <class T>
int dalloc(bt_learner* L, T** p, size_t count) {
  if (count == 0) count = 1;
  void* q = nullptr;
  BT_CUDA(cudaMalloc(&q, count * sizeof(T)));
  L->allocations.push_back(q);
  *p = static_cast<T*>(q);
  return BT_OK;
}

struct MinibatchInputs {
  const float* obs;
  const void* action;
  const float* lp_old;
  const float* v_old;
  const float* adv;
  const float* ret;
  const int* idx;
  const int* count;  // nullable
  float inv_mb;
};

namespace bt {
// Make `to` wait for all work enqueued so far on `from`.
int stream_dep(bt_learner* L, cudaStream_t from, cudaStream_t to);
int forward_tower(bt_learner* L, TowerPlan& tp, const float* obs, const int* idx, int rows,
                  const int* count, cudaStream_t s, bool keep_pre = true);
int backward_tower(bt_learner* L, TowerPlan& tp, const float* obs, const int* idx, int rows,
                   const int* count, cudaStream_t s, int top, cudaStream_t s_dw = nullptr);
int optimizer_step(bt_learner* L, int step, cudaStream_t s);
int launch_gae_internal(const float* reward, const uint8_t* term, const uint8_t* trunc,
                        const float* values, const float* bootstrap, int T, int N, double gamma,
                        double lam, float* adv, float* ret, int* err, cudaStream_t stream);
int allocate_gru(bt_learner* L, LayerPlan& lp);
int recurrent_update(bt_learner* L, const bt_batch* b, const int32_t* perm, float* stats,
                     cudaStream_t s);
bool exchange_active(const bt_learner* L);
int exchange_optimizer_step(bt_learner* L, int step, cudaStream_t s);
int exchange_gather_moments(bt_learner* L, cudaStream_t s);
int exchange_create(bt_learner* L, int (*allgather)(void* ctx, const void* send, void* recv,
                                                    size_t bytes),
                    void* ctx);
void exchange_destroy(Exchange* x);
}  // namespace bt

// Enqueue one kernel (or collective) launch `call`, counting it and, when profiling is
// on, bracketing it with CUDA events on stream `s`.
#define BT_K(L, cls, s, ...)                                    \
  do {                                                          \
    cudaEvent_t a_ = nullptr;                                   \
    if ((L)->prof.on) {                                         \
      a_ = prof_event(L);                                       \
      cudaEventRecord(a_, s);                                   \
    }                                                           \
    BT_TRY((__VA_ARGS__));                                      \
    (L)->prof.launches++;                                       \
    if ((L)->prof.on) {                                         \
      cudaEvent_t b_ = prof_event(L);                           \
      cudaEventRecord(b_, s);                                   \
      (L)->prof.recs.push_back({cls, a_, b_});                  \
    }                                                           \
  } while (0)
#define BT_C(L, cls, s, ...) BT_K(L, cls, s, __VA_ARGS__)
