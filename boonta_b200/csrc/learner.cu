// The learner handle: one PPO learner step per call, enqueued on one stream.
//
// Restates the control flow of boonta/algorithms/ppo.py:76-233 (PPO.update):
//   1. bootstrap value V(second.obs[T-1])                        (:208-212)
//   2. GAE over [T, N] (gae.cu)                                   (:213-219)
//   3. optional advantage normalisation                           (:220-221)
//   4. for each epoch e, minibatch m: the rows permutation[e][m*mb:(m+1)*mb] of the
//      flattened rollout (index t*N + n, :199-203, :226-228):
//        forward -> fused heads + loss + loss gradient -> backward -> gradient
//        reduction (+ NCCL all-reduce across ranks) -> clip + Adam  (:148-197)
// with every buffer allocated once at create. Parameters, gradients and both Adam
// moments live in one flat fp32 buffer each (layout below), so the optimizer is a
// single elementwise pass and the cross-GPU gradient mean is one all-reduce.
//
// Flat layout (must match boonta_b200/spec.py:param_layout): for every tower (shared
// torso, or actor then critic), for every layer, a group [kernel [K, N]; bias [N]]
// (+ [ln_scale [N]; ln_bias [N]]); conv kernels [3, 3, Cin, Cout] + bias; then
// actor_head [F, A] + bias [A], gaussian scale [A], critic_head [F, 1] + bias [1].
// Each group starts on a 64-float boundary.
#include <algorithm>
#include <cstring>

#include "gemm_simt.cuh"
#include "gemm_sm100.cuh"
#include "heads_tc.cuh"
#include "learner.h"

namespace bt {

int launch_gae_internal(const float* reward, const uint8_t* term, const uint8_t* trunc,
                        const float* values, const float* bootstrap, int T, int N, double gamma,
                        double lam, float* adv, float* ret, int* err, cudaStream_t stream);
int comm_allreduce_f32(Comm* c, float* buf, size_t n, cudaStream_t stream);
int comm_allreduce_f64(Comm* c, double* buf, size_t n, cudaStream_t stream);
void comm_destroy(Comm* c);

namespace {

constexpr int64_t kAlign = 64;
int64_t align_up(int64_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

int layer_out_dim(const bt_layer& l) {
  if (l.kind == BT_LAYER_CONV3X3) return l.height * l.width * l.features;
  return l.features;
}

struct LayoutBuilder {
  std::vector<ParamEntryC>& out;
  int64_t off = 0;
  void part(const std::string& name, std::vector<int64_t> shape) {
    int64_t n = 1;
    for (auto s : shape) n *= s;
    out.push_back({name, off, shape});
    off += n;
  }
  void end() { off = align_up(off); }
};

int check_layer(const bt_layer& l, int in_dim, bool first, bool last, bool shared,
                int precision) {
  BT_CHECK_ARG(l.features > 0, "layer with %d features", l.features);
  BT_CHECK_ARG(l.activation >= BT_ACT_NONE && l.activation <= BT_ACT_SILU, "bad activation %d",
               l.activation);
  if (l.kind == BT_LAYER_CONV3X3) {
    BT_CHECK_ARG(first, "a Conv3x3 layer is only supported as the first layer of a tower");
    BT_CHECK_ARG(l.height * l.width * l.in_channels == in_dim,
                 "conv input %dx%dx%d does not match obs_dim %d", l.height, l.width, l.in_channels,
                 in_dim);
    BT_CHECK_ARG(!l.layernorm, "LayerNorm after a conv is not supported");
  } else if (l.kind == BT_LAYER_GRU) {
    if (!last || !shared || first || precision != BT_PREC_FP32) {
      ::bt::set_error(
          "a GRU layer is supported as the last layer of a shared torso after a Dense layer, "
          "in fp32");
      return BT_ERR_UNSUPPORTED;
    }
  } else {
    BT_CHECK_ARG(l.kind == BT_LAYER_DENSE, "bad layer kind %d", l.kind);
  }
  return BT_OK;
}

}  // namespace

int build_layout(bt_learner* L) {
  const bt_network& net = L->cfg.network;
  LayoutBuilder b{L->entries};
  L->shared = net.num_critic == 0;
  L->ntowers = L->shared ? 1 : 2;
  const char* names[2] = {L->shared ? "torso" : "actor", "critic"};
  for (int t = 0; t < L->ntowers; ++t) {
    const bt_layer* layers = t == 0 ? net.torso : net.critic;
    const int n = t == 0 ? net.num_torso : net.num_critic;
    BT_CHECK_ARG(n >= 1 && n <= BT_MAX_LAYERS, "tower %d has %d layers", t, n);
    TowerPlan& tp = L->towers[t];
    tp.layers.clear();
    tp.in_dim = net.obs_dim;
    int dim = net.obs_dim;
    for (int i = 0; i < n; ++i) {
      const bt_layer& l = layers[i];
      BT_TRY(check_layer(l, dim, i == 0, i == n - 1, L->shared, L->cfg.precision));
      LayerPlan lp;
      lp.kind = l.kind;
      lp.act = l.activation;
      lp.ln = l.layernorm ? 1 : 0;
      // Dense layers take the precision's tensor-core path; a Conv3x3 (always the first
      // layer) stays on its fp32 kernels and hands bf16 operands to the tensor-core layer
      // after it.
      lp.tc = L->cfg.precision != BT_PREC_FP32 && l.kind == BT_LAYER_DENSE;
      std::string p = std::string(names[t]) + "/" + std::to_string(i);
      if (l.kind == BT_LAYER_GRU) {
        const int H = l.features;
        lp.kin = dim;
        lp.kout = H;
        lp.ncol = 3 * H;
        lp.hidden = H;
        lp.wi_off = b.off;
        b.part(p + "/input_kernel", {dim, 3 * H});
        b.part(p + "/input_bias", {3 * H});
        b.end();
        lp.wh_off = b.off;
        b.part(p + "/recurrent_kernel", {H, 3 * H});
        b.end();
        lp.bhn_off = b.off;
        b.part(p + "/hn_bias", {H});
        b.end();
        lp.w_off = lp.wi_off;
        L->recurrent = true;
      } else if (l.kind == BT_LAYER_CONV3X3) {
        lp.H = l.height;
        lp.W = l.width;
        lp.C = l.in_channels;
        lp.kin = 9 * l.in_channels;
        lp.ncol = l.features;
        lp.kout = layer_out_dim(l);
        lp.w_off = b.off;
        b.part(p + "/kernel", {3, 3, l.in_channels, l.features});
        b.part(p + "/bias", {l.features});
        b.end();
      } else {
        lp.kin = dim;
        lp.kout = l.features;
        lp.ncol = l.features;
        lp.w_off = b.off;
        b.part(p + "/kernel", {dim, l.features});
        b.part(p + "/bias", {l.features});
        b.end();
        if (lp.ln) {
          lp.ln_off = b.off;
          b.part(p + "/ln_scale", {l.features});
          b.part(p + "/ln_bias", {l.features});
          b.end();
        }
      }
      dim = lp.kout;
      tp.layers.push_back(lp);
    }
    tp.out_dim = dim;
  }
  L->F_pi = L->towers[0].out_dim;
  L->F_v = L->shared ? L->F_pi : L->towers[1].out_dim;
  L->A = net.action_dim;
  BT_CHECK_ARG(L->A >= 1 && L->A <= 64, "action_dim %d outside [1, 64]", L->A);
  BT_CHECK_ARG(net.head == BT_HEAD_CATEGORICAL || net.head == BT_HEAD_GAUSSIAN, "bad head %d",
               net.head);
  L->head_pi_off = b.off;
  b.part("actor_head/kernel", {L->F_pi, L->A});
  b.part("actor_head/bias", {L->A});
  b.end();
  if (net.head == BT_HEAD_GAUSSIAN) {
    L->head_scale_off = b.off;
    b.part("actor_head/scale", {L->A});
    b.end();
  }
  L->head_v_off = b.off;
  b.part("critic_head/kernel", {L->F_v, 1});
  b.part("critic_head/bias", {1});
  b.end();
  L->num_params = b.off;
  return BT_OK;
}

namespace {

// Split-K factor for a dW GEMM: enough CTAs for ~2 waves on 148 SMs, at least 256
// reduction rows per split.
int pick_splits(int M, int N, int K) {
  const int tiles = ceil_div(M, kBM) * ceil_div(N, kBN);
  int s = std::max(1, (2 * kNumSMs) / tiles);
  s = std::min(s, std::max(1, K / 256));
  return s;
}

}  // namespace

int allocate_tensor_core(bt_learner* L);
int allocate_gru_tc(bt_learner* L);

int allocate(bt_learner* L) {
  const bt_learner_config& c = L->cfg;
  const int E = c.ppo.update_epochs, M = c.ppo.num_minibatches;
  const int world = std::max(1, c.world_size);
  L->T = c.num_steps;
  L->N = c.num_envs;
  L->B = (int64_t)L->T * L->N;
  BT_CHECK_ARG(M >= 1 && E >= 1, "num_minibatches %d / update_epochs %d", M, E);
  // Minibatches are over samples (t, n), or over whole env sequences for a recurrent torso
  // (recurrent_ppo.py:269-276); `units` is what the permutation runs over.
  const int64_t units_local = L->recurrent ? L->N : L->B;
  const int64_t units_global = units_local * world;
  BT_CHECK_ARG(units_global % M == 0, "%lld %s not divisible by num_minibatches %d",
               (long long)units_global, L->recurrent ? "envs" : "samples", M);
  L->mb = (int)(units_global / M);
  int units_cap;
  if (world == 1) {
    units_cap = L->mb;
  } else {
    // Hypergeometric share of a global minibatch: mean mb/world, std < sqrt(mb/world).
    const double mean = (double)L->mb / world;
    int cap = (int)std::ceil(mean + 16.0 * std::sqrt(mean) + 64.0);
    units_cap = (int)std::min<int64_t>(std::min<int64_t>(cap, L->mb), units_local);
  }
  L->units_cap = units_cap;
  L->rows_cap = L->recurrent ? units_cap * L->T : units_cap;
  L->act_rows = std::max(L->rows_cap, L->recurrent ? 2 * L->N : L->N);
  const int R = L->act_rows;

  const int64_t P = L->num_params;
  BT_TRY(dalloc(L, &L->params, P));
  BT_TRY(dalloc(L, &L->grads, P));
  BT_TRY(dalloc(L, &L->mu, P));
  BT_TRY(dalloc(L, &L->nu, P));
  BT_CUDA(cudaMemset(L->params, 0, P * 4));
  BT_CUDA(cudaMemset(L->grads, 0, P * 4));
  BT_CUDA(cudaMemset(L->mu, 0, P * 4));
  BT_CUDA(cudaMemset(L->nu, 0, P * 4));
  BT_TRY(dalloc(L, &L->count_d, 4));
  BT_CUDA(cudaMemset(L->count_d, 0, 16));
  L->err_d = L->count_d + 1;
  L->mb_count_d = L->count_d + 2;

  L->segs_h.clear();
  for (int t = 0; t < L->ntowers; ++t) {
    for (size_t i = 0; i < L->towers[t].layers.size(); ++i) {
      LayerPlan& lp = L->towers[t].layers[i];
      if (lp.kind == BT_LAYER_GRU) {
        BT_TRY(allocate_gru(L, lp));
        continue;
      }
      const size_t n = (size_t)R * lp.kout;
      BT_TRY(dalloc(L, &lp.z, n));
      BT_TRY(dalloc(L, &lp.h, n));
      BT_TRY(dalloc(L, &lp.d_pre, n));
      if (lp.ln) {
        BT_TRY(dalloc(L, &lp.y, n));
        BT_TRY(dalloc(L, &lp.d_z, n));
        BT_TRY(dalloc(L, &lp.mean, R));
        BT_TRY(dalloc(L, &lp.rstd, R));
        lp.ln_blocks = 2 * kNumSMs;
        BT_TRY(dalloc(L, &lp.ln_part, (size_t)lp.ln_blocks * 2 * lp.kout));
      } else {
        lp.d_z = lp.d_pre;
      }
      // dW GEMM: [kin + 1, ncol] over K = rows (dense) or rows * H*W (conv)
      const int dm = lp.kin + 1, dn = lp.ncol;
      const int dk = L->rows_cap;
      if (lp.tc) {
        // tcgen05 dW: tiles of 128 x BN over [kin + 1, kout] (M runs over the wide input side,
        // so the large input operand is re-read only kout / BN times), split over K (the rows)
        // to fill one wave of CTAs with at least 8 K blocks (512 rows) per split.
        lp.dw_bn = (L->cfg.precision == BT_PREC_BF16 && lp.kout % 256 == 0) ? 256 : 128;
        const int tiles = ceil_div(lp.kin + 1, 128) * ceil_div(lp.kout, lp.dw_bn);
        const int nkb = ceil_div(L->rows_cap, 64);
        int splits = std::max(1, std::min(kNumSMs / tiles, nkb / 8));
        lp.dw_kbps = ceil_div(nkb, splits);
        lp.dw_splits = ceil_div(nkb, lp.dw_kbps);
      } else if (lp.kind == BT_LAYER_CONV3X3) {
        lp.dw_splits = conv_dw_blocks(L->rows_cap);  // one partial per conv dW block
      } else {
        lp.dw_splits = pick_splits(dm, dn, dk);
      }
      BT_TRY(dalloc(L, &lp.dw_part, (size_t)lp.dw_splits * dm * dn));
      L->segs_h.push_back({lp.dw_part, lp.dw_splits, dm * dn, (int64_t)dm * dn, lp.w_off});
      if (lp.ln) {
        L->segs_h.push_back(
            {lp.ln_part, lp.ln_blocks, 2 * lp.kout, (int64_t)2 * lp.kout, lp.ln_off});
      }
    }
  }
  // heads
  const int A = L->A;
  BT_TRY(dalloc(L, &L->d_out, (size_t)R * A));
  BT_TRY(dalloc(L, &L->d_val, R));
  // heads kernel: tiles of 32 rows, up to two blocks per SM (shared memory allowing), the
  // tiles spread evenly over the blocks
  {
    const size_t hs = heads_smem_bytes(L->F_pi, L->F_v, A, L->shared);
    const int per_sm = std::max<int>(1, std::min<int>(2, (int)((226 * 1024) / (hs + 1024))));
    const int tiles = ceil_div(L->rows_cap, 32);
    const int rounds = ceil_div(tiles, kNumSMs * per_sm);
    L->heads_blocks = ceil_div(tiles, rounds);
  }
  {
    const LayerPlan* last = L->towers[0].layers.empty() ? nullptr : &L->towers[0].layers.back();
    L->tc_heads = last && last->kind == BT_LAYER_DENSE &&
                  heads_tc_eligible(c.network.head, L->shared, L->recurrent, last->tc, L->F_pi, A);
  }
  L->heads_fused_dw = !L->tc_heads && heads_fuse_dw(L->F_pi, L->F_v, A, L->shared);
  // act and the bootstrap evaluate the heads with the update's product arithmetic
  L->split_pi = L->tc_heads || heads_split_products(L->F_pi, L->F_v, A, L->shared);
  L->split_v = L->split_pi && L->shared;
  if (L->tc_heads) {
    // tensor-core heads: one statistic partial per 128-row tile; the head dW GEMM split over
    // the rows to fill one wave of CTAs with at least 8 K blocks per split
    L->heads_blocks = ceil_div(L->rows_cap, umma::BM);
    const int tiles = ceil_div(L->F_pi + 1, umma::BM);
    const int nkb = ceil_div(L->rows_cap, umma::BK);
    const int splits = std::max(1, std::min(kNumSMs / tiles, nkb / 8));
    L->head_dw_kbps = ceil_div(nkb, splits);
    L->head_pi_splits = L->head_v_splits = ceil_div(nkb, L->head_dw_kbps);
  } else if (L->heads_fused_dw) {
    // the heads kernel accumulates the head weight gradients, one partial per block
    L->head_pi_splits = L->head_v_splits = L->heads_blocks;
  } else {
    // skinny head dW: up to 8 blocks of 128 threads per SM (enough loads in flight), at
    // least 128 rows per split (fewer partials for the reduction to read)
    L->head_pi_splits = std::max(1, std::min(ceil_div(L->rows_cap, 128),
                                             8 * kNumSMs / ceil_div(L->F_pi + 1, 128)));
    L->head_v_splits = std::max(1, std::min(ceil_div(L->rows_cap, 128),
                                            8 * kNumSMs / ceil_div(L->F_v + 1, 128)));
  }
  BT_TRY(dalloc(L, &L->head_pi_part, (size_t)L->head_pi_splits * (L->F_pi + 1) * A));
  BT_TRY(dalloc(L, &L->head_v_part, (size_t)L->head_v_splits * (L->F_v + 1)));
  L->segs_h.push_back({L->head_pi_part, L->head_pi_splits, (L->F_pi + 1) * A,
                       (int64_t)(L->F_pi + 1) * A, L->head_pi_off});
  BT_TRY(dalloc(L, &L->stat_part, (size_t)L->heads_blocks * kNumStatSums));
  if (c.network.head == BT_HEAD_GAUSSIAN) {
    BT_TRY(dalloc(L, &L->dscale_part, (size_t)L->heads_blocks * A));
    L->segs_h.push_back({L->dscale_part, L->heads_blocks, A, (int64_t)A, L->head_scale_off});
  }
  L->segs_h.push_back(
      {L->head_v_part, L->head_v_splits, L->F_v + 1, (int64_t)(L->F_v + 1), L->head_v_off});
  BT_TRY(dalloc(L, &L->segs_d, L->segs_h.size()));
  BT_CUDA(cudaMemcpy(L->segs_d, L->segs_h.data(), L->segs_h.size() * sizeof(Segment),
                     cudaMemcpyHostToDevice));
  {
    std::vector<ReduceChunk> chunks(
        count_reduce_chunks(L->segs_h.data(), (int)L->segs_h.size()));
    build_reduce_chunks(L->segs_h.data(), (int)L->segs_h.size(), chunks.data(), &L->num_chunks);
    BT_TRY(dalloc(L, &L->chunks_d, chunks.size()));
    BT_CUDA(cudaMemcpy(L->chunks_d, chunks.data(), chunks.size() * sizeof(ReduceChunk),
                       cudaMemcpyHostToDevice));
  }
  BT_TRY(dalloc(L, &L->norm_part, std::max<size_t>(L->num_chunks, kNormBlocks)));
  BT_TRY(dalloc(L, &L->stat_sums, (size_t)(E * M + 1) * kNumStatSums));
  BT_TRY(dalloc(L, &L->adv_part, 2 * kNormBlocks));
  // targets
  BT_TRY(dalloc(L, &L->adv, L->B));
  BT_TRY(dalloc(L, &L->ret, L->B));
  BT_TRY(dalloc(L, &L->boot, L->N));
  BT_TRY(dalloc(L, &L->act_out, (size_t)R * A));
  BT_TRY(dalloc(L, &L->act_val, R));
  if (world > 1) {
    BT_TRY(dalloc(L, &L->local_idx, (size_t)E * M * L->units_cap));
    BT_TRY(dalloc(L, &L->local_counts, (size_t)E * M));
  }
  BT_TRY(allocate_tensor_core(L));
  return allocate_gru_tc(L);
}

// ---- tensor-core (bf16) operand buffers and TMA tensor maps -------------------------------
int allocate_tensor_core(bt_learner* L) {
  L->tc_any = L->tc_first = false;
  for (int t = 0; t < L->ntowers; ++t) {
    for (LayerPlan& lp : L->towers[t].layers) L->tc_any |= lp.tc;
    L->tc_first |= !L->towers[t].layers.empty() && L->towers[t].layers[0].tc;
  }
  if (!L->tc_any) return BT_OK;
  L->x3 = L->cfg.precision == BT_PREC_BF16X3;
  const int R = L->act_rows;
  auto ru8 = [](int x) { return (x + 7) / 8 * 8; };
  auto pair = [&](__nv_bfloat16** hi, __nv_bfloat16** lo, size_t n) -> int {
    BT_TRY(dalloc(L, hi, n));
    BT_CUDA(cudaMemset(*hi, 0, n * 2));
    if (L->x3) {
      BT_TRY(dalloc(L, lo, n));
      BT_CUDA(cudaMemset(*lo, 0, n * 2));
    }
    return BT_OK;
  };
  BT_TRY(pair(&L->params_b, &L->params_b_lo, L->num_params));
  L->ldx0 = ru8(L->cfg.network.obs_dim + 1);
  BT_TRY(pair(&L->xg, &L->xg_lo, (size_t)R * L->ldx0));
  if (L->tc_first && !L->x3 && !L->recurrent && L->cfg.network.obs_dim >= 1024) {
    // wide bf16 observations: the update converts the rollout once and gathers each
    // minibatch's rows from the bf16 copy
    BT_TRY(dalloc(L, &L->obs_b, (size_t)L->B * L->ldx0));
  }
  for (int t = 0; t < L->ntowers; ++t) {
    std::vector<LayerPlan>& layers = L->towers[t].layers;
    for (size_t i = 0; i < layers.size(); ++i) {
      LayerPlan& lp = layers[i];
      if (!lp.tc) continue;
      BT_CHECK_ARG(lp.kout % 8 == 0, "tensor-core layer width %d is not a multiple of 8", lp.kout);
      lp.ldh = ru8(lp.kout + 1);
      BT_TRY(pair(&lp.hb, &lp.hb_lo, (size_t)R * lp.ldh));
      BT_TRY(launch_ones_column(lp.hb, R, lp.kout, lp.ldh, 1.f, 0));
      if (L->tc_heads && t == 0 && i + 1 == layers.size() && !lp.hb_lo) {
        // the tensor-core heads read the torso output as split bf16 pairs
        BT_TRY(dalloc(L, &lp.hb_lo, (size_t)R * lp.ldh));
        BT_CUDA(cudaMemset(lp.hb_lo, 0, (size_t)R * lp.ldh * 2));
      }
      BT_TRY(pair(&lp.dzb, &lp.dzb_lo, (size_t)R * lp.kout));
      if (i == 0) {
        lp.xin_b = L->xg;
        lp.xin_lo = L->xg_lo;
        lp.ldx = L->ldx0;
      } else {
        LayerPlan& prev = layers[i - 1];
        BT_CHECK_ARG(prev.tc || prev.kind == BT_LAYER_CONV3X3,
                     "a tensor-core layer must follow a tensor-core or Conv3x3 layer");
        if (!prev.tc) {
          // the conv writes its output as the bf16 operand of this layer, and this layer's
          // dX epilogue writes the conv's dL/dz in fp32 (maps for both)
          prev.out_b = true;
          prev.ldh = ru8(prev.kout + 1);
          BT_TRY(pair(&prev.hb, &prev.hb_lo, (size_t)R * prev.ldh));
          BT_TRY(launch_ones_column(prev.hb, R, prev.kout, prev.ldh, 1.f, 0));
          const uint64_t f32_ld = (uint64_t)prev.kout * 4;
          BT_TRY(umma::encode_tile_map(&prev.map_pre, prev.pre(), true, prev.kout, R, f32_ld, 128));
          BT_TRY(umma::encode_tile_map(&prev.map_dpre, prev.d_pre, true, prev.kout, R, f32_ld,
                                       128));
        }
        lp.xin_b = prev.hb;
        lp.xin_lo = prev.hb_lo;
        lp.ldx = prev.ldh;
      }
      const int mtiles = ceil_div(L->rows_cap, umma::BM);
      lp.fwd_bn = (!L->x3 && lp.kout % 256 == 0 && mtiles * (lp.kout / 256) >= kNumSMs) ? 256 : 128;
      // hi maps, then (split mode) the same maps over the lo halves
      for (int part = 0; part < (L->x3 ? 2 : 1); ++part) {
        const __nv_bfloat16* w = (part ? L->params_b_lo : L->params_b) + lp.w_off;
        const __nv_bfloat16* xin = part ? lp.xin_lo : lp.xin_b;
        const __nv_bfloat16* dz = part ? lp.dzb_lo : lp.dzb;
        CUtensorMap* fa = part ? &lp.fwd_ops.a_lo : &lp.fwd_ops.a;
        CUtensorMap* fb = part ? &lp.fwd_ops.b_lo : &lp.fwd_ops.b;
        CUtensorMap* xa = part ? &lp.dx_ops.a_lo : &lp.dx_ops.a;
        CUtensorMap* xb = part ? &lp.dx_ops.b_lo : &lp.dx_ops.b;
        CUtensorMap* wa = part ? &lp.dw_ops.a_lo : &lp.dw_ops.a;
        CUtensorMap* wb = part ? &lp.dw_ops.b_lo : &lp.dw_ops.b;
        BT_TRY(umma::encode_map(fa, xin, lp.kin, R, (uint64_t)lp.ldx * 2, 64, 128));
        BT_TRY(umma::encode_map(fb, w, lp.kout, lp.kin, (uint64_t)lp.kout * 2, 64, 64));
        BT_TRY(umma::encode_map(xa, dz, lp.kout, R, (uint64_t)lp.kout * 2, 64, 128));
        BT_TRY(umma::encode_map(xb, w, lp.kout, lp.kin, (uint64_t)lp.kout * 2, 64, 128));
        // dW = [x, 1]^T dz: A = the layer input over (kin + 1, rows), B = dz over (kout, rows)
        BT_TRY(umma::encode_map(wa, xin, lp.kin + 1, R, (uint64_t)lp.ldx * 2, 64, 64));
        BT_TRY(umma::encode_map(wb, dz, lp.kout, R, (uint64_t)lp.kout * 2, 64, 64));
      }
      const uint64_t rows = (uint64_t)R, f32_ld = (uint64_t)lp.kout * 4;
      BT_TRY(umma::encode_tile_map(&lp.map_z, lp.z, true, lp.kout, rows, f32_ld, 128));
      BT_TRY(umma::encode_tile_map(&lp.map_pre, lp.pre(), true, lp.kout, rows, f32_ld, 128));
      BT_TRY(umma::encode_tile_map(&lp.map_dpre, lp.d_pre, true, lp.kout, rows, f32_ld, 128));
      BT_TRY(umma::encode_tile_map(&lp.map_hb, lp.hb, false, lp.kout, rows,
                                   (uint64_t)lp.ldh * 2, 64));
      BT_TRY(umma::encode_tile_map(&lp.map_dzb, lp.dzb, false, lp.kout, rows,
                                   (uint64_t)lp.kout * 2, 64));
      lp.map_hb_lo = lp.map_hb;
      lp.map_dzb_lo = lp.map_dzb;
      if (lp.hb_lo) {
        BT_TRY(umma::encode_tile_map(&lp.map_hb_lo, lp.hb_lo, false, lp.kout, rows,
                                     (uint64_t)lp.ldh * 2, 64));
      }
      if (L->x3) {
        BT_TRY(umma::encode_tile_map(&lp.map_dzb_lo, lp.dzb_lo, false, lp.kout, rows,
                                     (uint64_t)lp.kout * 2, 64));
      }
      if (!L->x3) {
        lp.fwd_ops.a_lo = lp.fwd_ops.a;
        lp.fwd_ops.b_lo = lp.fwd_ops.b;
        lp.dx_ops.a_lo = lp.dx_ops.a;
        lp.dx_ops.b_lo = lp.dx_ops.b;
        lp.dw_ops.a_lo = lp.dw_ops.a;
        lp.dw_ops.b_lo = lp.dw_ops.b;
      }
    }
  }
  // LayerNorm + ReLU tensor-core layers whose every consumer of y takes relu'(y) from hb
  for (int t = 0; t < L->ntowers; ++t) {
    std::vector<LayerPlan>& layers = L->towers[t].layers;
    for (size_t i = 0; i < layers.size(); ++i) {
      LayerPlan& lp = layers[i];
      const bool last = i + 1 == layers.size();
      lp.relu_from_hb = lp.tc && lp.ln && lp.act == BT_ACT_RELU &&
                        (last ? (L->tc_heads && t == 0) : layers[i + 1].tc);
    }
  }
  if (L->tc_heads) {
    // maps of the three head GEMMs (heads_tc.cuh); every operand is a split bf16 pair
    const LayerPlan& last = L->towers[0].layers.back();
    const int F = L->F_pi, H = umma::kHeadCols;
    BT_TRY(dalloc(L, &L->whb, (size_t)F * H));
    BT_TRY(dalloc(L, &L->whb_lo, (size_t)F * H));
    BT_TRY(dalloc(L, &L->dhb, (size_t)R * H));
    BT_TRY(dalloc(L, &L->dhb_lo, (size_t)R * H));
    BT_CUDA(cudaMemset(L->dhb, 0, (size_t)R * H * 2));
    BT_CUDA(cudaMemset(L->dhb_lo, 0, (size_t)R * H * 2));
    const uint64_t hld = (uint64_t)last.ldh * 2, dld = (uint64_t)H * 2;
    for (int part = 0; part < 2; ++part) {
      const __nv_bfloat16* h = part ? last.hb_lo : last.hb;
      const __nv_bfloat16* w = part ? L->whb_lo : L->whb;
      const __nv_bfloat16* d = part ? L->dhb_lo : L->dhb;
      umma::Operands& o = L->head_o_ops;
      umma::Operands& x = L->head_dx_ops;
      umma::Operands& g = L->head_dw_ops;
      // outputs O = h W_h: A = h (K-major, K = F), B = W_h (MN-major, [K = F][N = 64])
      BT_TRY(umma::encode_map(part ? &o.a_lo : &o.a, h, F, R, hld, 64, 128));
      BT_TRY(umma::encode_map(part ? &o.b_lo : &o.b, w, H, F, dld, 64, 64));
      // dL/dy = D W_h^T: A = D (K-major, K = 64), B = W_h (K-major, [N = F][K = 64])
      BT_TRY(umma::encode_map(part ? &x.a_lo : &x.a, d, H, R, dld, 64, 128));
      BT_TRY(umma::encode_map(part ? &x.b_lo : &x.b, w, H, F, dld, 64, 128));
      // head dW = [h, 1]^T D: A = h with its ones column (MN-major over F + 1), B = D (MN-major)
      BT_TRY(umma::encode_map(part ? &g.a_lo : &g.a, h, F + 1, R, hld, 64, 64));
      BT_TRY(umma::encode_map(part ? &g.b_lo : &g.b, d, H, R, dld, 64, 64));
    }
  }
  BT_CUDA(cudaDeviceSynchronize());
  return BT_OK;
}

// ---- forward / backward of one tower --------------------------------------------------
// Layers marked `tc` run on the tcgen05 tensor-core GEMM with bf16 operands (activations
// and dz stored as bf16 row-major buffers, weights from the bf16 shadow of the params);
// the others run on the fp32 CUDA-core GEMM. A tensor-core tower's first layer reads the
// minibatch gathered into L->xg (gather_obs).
int gather_obs(bt_learner* L, const float* obs, const int* idx, int rows, const int* count,
               cudaStream_t s) {
  if (!L->tc_first) return BT_OK;
  if (L->gather_rows && idx) {
    if (L->fill_obs_b) {
      // a first-epoch minibatch: its fp32 rows to the GEMM operand, and (when later epochs
      // follow) into the update's bf16 copy of the rollout at their own indices
      BT_K(L, kProfMisc, s, launch_gather_bf16(obs, idx, rows, L->cfg.network.obs_dim, L->ldx0,
                                               L->xg, nullptr, count, s,
                                               L->cfg.ppo.update_epochs > 1 ? L->obs_b : nullptr));
      return BT_OK;
    }
    // a later epoch: its rows from the update's bf16 copy of the rollout
    BT_K(L, kProfMisc, s, launch_gather_rows_bf16(L->obs_b, idx, rows, L->ldx0, L->xg, count, s));
    return BT_OK;
  }
  BT_K(L, kProfMisc, s, launch_gather_bf16(obs, idx, rows, L->cfg.network.obs_dim, L->ldx0, L->xg,
                                           L->xg_lo, count, s));
  return BT_OK;
}

// keep_pre = false (the update's minibatch forward): layers whose y is read only through
// relu'(y) (relu_from_hb) skip writing it.
int forward_tower(bt_learner* L, TowerPlan& tp, const float* obs, const int* idx, int rows,
                  const int* count, cudaStream_t s, bool keep_pre) {
  const float* in = obs;
  const int* gather = idx;
  int in_ld = tp.in_dim;
  for (size_t i = 0; i < tp.layers.size(); ++i) {
    LayerPlan& lp = tp.layers[i];
    if (lp.kind == BT_LAYER_GRU) break;  // the recurrent path runs the GRU (recurrent.cu)
    const float* w = L->params + lp.w_off;
    if (lp.tc) {
      umma::GemmShape sh{rows, lp.kout, lp.kin, ceil_div(lp.kin, umma::BK), count, nullptr,
                         L->err_d};
      // The last layer's output is consumed through its pre-activation (the heads apply
      // the activation), so only z is stored for it; the bf16 outputs feed the next layer.
      const bool last = i + 1 == tp.layers.size();
      // (the tensor-core heads read the last layer's output as split bf16 pairs)
      const bool out_b = !last || (L->tc_heads && &tp == &L->towers[0]);
      umma::EpiFwd ep;
      ep.f32_map = lp.map_z;
      ep.hi_map = lp.map_hb;
      ep.lo_map = lp.map_hb_lo;
      ep.bias = w + (size_t)lp.kin * lp.kout;
      ep.act = lp.act;
      ep.has_f32 = true;
      ep.has_hi = !lp.ln && out_b;
      ep.has_lo = ep.has_hi && lp.hb_lo != nullptr;
      if (L->x3) {
        BT_K(L, kProfGemmFwd, s, umma::launch_gemm<128, false, true, true>(lp.fwd_ops, sh, ep, 1, s));
      } else if (lp.fwd_bn == 256) {
        BT_K(L, kProfGemmFwd, s, umma::launch_gemm<256, false, true, false>(lp.fwd_ops, sh, ep, 1, s));
      } else {
        BT_K(L, kProfGemmFwd, s, umma::launch_gemm<128, false, true, false>(lp.fwd_ops, sh, ep, 1, s));
      }
      if (lp.ln) {
        BT_K(L, kProfLnFwd, s, launch_ln_forward(lp.z, L->params + lp.ln_off, rows, lp.kout, lp.act,
                                                 (keep_pre || !lp.relu_from_hb) ? lp.y : nullptr,
                                                 nullptr, out_b ? lp.hb : nullptr,
                                                 out_b ? lp.hb_lo : nullptr, lp.ldh, lp.mean,
                                                 lp.rstd, count, s));
      }
    } else if (lp.kind == BT_LAYER_CONV3X3) {
      BT_K(L, kProfGemmFwd, s, launch_conv_forward(in, gather, rows, count, lp.H, lp.W, lp.C,
                                                   lp.ncol, w, lp.act, lp.z,
                                                   lp.out_b ? nullptr : lp.h,
                                                   lp.out_b ? lp.hb : nullptr, lp.hb_lo,
                                                   lp.ldh, s));
    } else {
      ARows a{in, gather, in_ld, lp.kin};
      BRows b{w, lp.ncol, lp.kin + 1};
      EpiForward ep{lp.z, lp.ln ? nullptr : lp.h, lp.ncol, lp.ln ? BT_ACT_NONE : lp.act};
      BT_K(L, kProfGemmFwd, s, launch_gemm_simt(a, b, ep, rows, lp.ncol, lp.kin + 1, 1, s, count, nullptr));
      if (lp.ln) {
        BT_K(L, kProfLnFwd, s, launch_ln_forward(lp.z, L->params + lp.ln_off, rows, lp.kout, lp.act, lp.y, lp.h,
                                 nullptr, nullptr, 0, lp.mean, lp.rstd, count, s));
      }
    }
    in = lp.h;
    gather = nullptr;
    in_ld = lp.kout;
  }
  return BT_OK;
}

int stream_dep(bt_learner* L, cudaStream_t from, cudaStream_t to) {
  if (from == to) return BT_OK;
  cudaEvent_t e = L->fork_events[L->next_event++ % L->fork_events.size()];
  BT_CUDA(cudaEventRecord(e, from));
  BT_CUDA(cudaStreamWaitEvent(to, e, 0));
  return BT_OK;
}

// Backward of layers top..0 of a tower. When s_dw is given, each layer's weight-gradient
// GEMM runs on s_dw (after the layer's dz is ready) while the dX chain continues on s; s
// waits for s_dw before returning.
int backward_tower(bt_learner* L, TowerPlan& tp, const float* obs, const int* idx, int rows,
                   const int* count, cudaStream_t s, int top, cudaStream_t s_dw) {
  if (top < 0) top = (int)tp.layers.size() - 1;
  const cudaStream_t sw = s_dw ? s_dw : s;
  for (int i = top; i >= 0; --i) {
    LayerPlan& lp = tp.layers[i];
    const float* w = L->params + lp.w_off;
    if (lp.ln) {
      BT_K(L, kProfLnBwd, s, launch_ln_backward(lp.d_pre, lp.z, lp.mean, lp.rstd, L->params + lp.ln_off, rows,
                                lp.kout, lp.tc ? nullptr : lp.d_z, lp.tc ? lp.dzb : nullptr,
                                lp.tc ? lp.dzb_lo : nullptr, lp.ln_part, lp.ln_blocks, count, s));
    }
    BT_TRY(stream_dep(L, s, sw));  // dz of this layer is ready
    const int dm = lp.kin + 1, dn = lp.ncol;
    if (lp.tc) {
      // dW [kin + 1, kout] = [x, 1]^T dz, split-K partials in the parameter layout
      umma::GemmShape sh{lp.kin + 1, lp.kout, rows, lp.dw_kbps, nullptr, count, L->err_d};
      umma::EpiDw ep{lp.dw_part, lp.kout, (size_t)dm * dn};
      if (L->x3) {
        BT_K(L, kProfGemmDw, sw, umma::launch_gemm<128, true, true, true>(lp.dw_ops, sh, ep, lp.dw_splits, sw));
      } else if (lp.dw_bn == 256) {
        BT_K(L, kProfGemmDw, sw, umma::launch_gemm<256, true, true, false>(lp.dw_ops, sh, ep, lp.dw_splits, sw));
      } else {
        BT_K(L, kProfGemmDw, sw, umma::launch_gemm<128, true, true, false>(lp.dw_ops, sh, ep, lp.dw_splits, sw));
      }
      if (i > 0) {
        LayerPlan& prev = tp.layers[i - 1];
        umma::GemmShape shx{rows, lp.kin, lp.kout, ceil_div(lp.kout, umma::BK), count, nullptr,
                            L->err_d};
        umma::EpiDx epx;
        epx.in_map = prev.relu_from_hb ? prev.map_hb : prev.map_pre;
        epx.in_bf16 = prev.relu_from_hb;
        epx.f32_map = prev.map_dpre;
        epx.hi_map = prev.map_dzb;
        epx.lo_map = prev.map_dzb_lo;
        epx.act = prev.act;
        // fp32 dL/dz for a LayerNorm or non-tensor-core (conv) previous layer
        epx.has_f32 = prev.ln || !prev.tc;
        epx.has_hi = !epx.has_f32;
        epx.has_lo = epx.has_hi && L->x3;
        if (L->x3) {
          BT_K(L, kProfGemmDx, s, umma::launch_gemm<128, false, false, true>(lp.dx_ops, shx, epx, 1, s));
        } else {
          BT_K(L, kProfGemmDx, s, umma::launch_gemm<128, false, false, false>(lp.dx_ops, shx, epx, 1, s));
        }
      }
      continue;
    }
    EpiPartial ep{lp.dw_part, dn, (size_t)dm * dn};
    if (lp.kind == BT_LAYER_CONV3X3) {
      BT_K(L, kProfGemmDw, sw, launch_conv_dw(obs, idx, rows, count, lp.H, lp.W, lp.C, lp.ncol,
                                              lp.d_z, lp.dw_splits, lp.dw_part, sw));
    } else {
      const float* in = i == 0 ? obs : tp.layers[i - 1].h;
      const int* gather = i == 0 ? idx : nullptr;
      ACols a{in, gather, lp.kin, lp.kin};
      BRows b{lp.d_z, lp.ncol, rows};
      BT_K(L, kProfGemmDw, sw, launch_gemm_simt(a, b, ep, dm, dn, rows, lp.dw_splits, sw, nullptr, count));
    }
    if (i > 0) {
      LayerPlan& prev = tp.layers[i - 1];
      ARows a{lp.d_z, nullptr, lp.ncol, lp.ncol};
      BCols b{w, lp.ncol, lp.ncol};
      EpiActGrad ep2{prev.d_pre, prev.pre(), prev.h, prev.kout, prev.act};
      BT_K(L, kProfGemmDx, s, launch_gemm_simt(a, b, ep2, rows, lp.kin, lp.ncol, 1, s, count, nullptr));
    }
  }
  BT_TRY(stream_dep(L, sw, s));
  return BT_OK;
}

// Forward + loss + backward + gradient reduction for one minibatch. Leaves the
// (unreduced across ranks) gradients in L->grads and the statistic sums in stat_slot.
int loss_grads(bt_learner* L, const MinibatchInputs& in, double* stat_slot, bool with_norm,
               cudaStream_t s) {
  const int rows = L->rows_cap;
  const bt_learner_config& c = L->cfg;
  BT_TRY(gather_obs(L, in.obs, in.idx, rows, in.count, s));
  // separate actor and critic towers run side by side (the critic on a side stream)
  const cudaStream_t sc = side_stream(L, 0, s);
  if (L->ntowers > 1) {
    BT_TRY(stream_dep(L, s, sc));
    BT_TRY(forward_tower(L, L->towers[1], in.obs, in.idx, rows, in.count, sc, false));
  }
  BT_TRY(forward_tower(L, L->towers[0], in.obs, in.idx, rows, in.count, s, false));
  if (L->ntowers > 1) BT_TRY(stream_dep(L, sc, s));
  TowerPlan& t0 = L->towers[0];
  TowerPlan& tv = L->towers[L->ntowers - 1];
  LayerPlan& last_pi = t0.layers.back();
  LayerPlan& last_v = tv.layers.back();
  cudaStream_t sh = side_stream(L, 3, s);
  if (L->tc_heads) {
    // head outputs + loss + dL/dO (one 128-row tile per block), then on a side stream the
    // statistics and the head weight gradient next to dL/dy and the torso's backward
    BT_K(L, kProfHeads, s, launch_heads_pack(L->params + L->head_pi_off, L->params + L->head_v_off,
                                             L->F_pi, L->A, L->whb, L->whb_lo, s));
    umma::EpiHeadsLoss eh{};
    eh.A = L->A;
    eh.count = in.count;
    eh.idx = in.idx;
    eh.b_pi = L->params + L->head_pi_off + (size_t)L->F_pi * L->A;
    eh.b_v = L->params + L->head_v_off + L->F_v;
    eh.action = static_cast<const int*>(in.action);
    eh.lp_old = in.lp_old;
    eh.v_old = in.v_old;
    eh.adv = in.adv;
    eh.ret = in.ret;
    eh.inv_mb = in.inv_mb;
    eh.clip = c.ppo.clip_coefficient;
    eh.clip_value = c.ppo.clip_value_loss;
    eh.ent_coef = c.ppo.entropy_coefficient;
    eh.vf_coef = c.ppo.value_coefficient;
    eh.d_hi = L->dhb;
    eh.d_lo = L->dhb_lo;
    eh.stat_partials = L->stat_part;
    BT_K(L, kProfHeads, s, launch_heads_tc_loss(L->head_o_ops, rows, L->F_pi, eh, L->err_d, s));
    BT_TRY(stream_dep(L, s, sh));
    BT_K(L, kProfStats, sh, launch_stat_reduce(L->stat_part, L->heads_blocks, stat_slot, sh));
    umma::EpiHeadsDw ed{L->head_pi_part, L->head_v_part, L->A, L->F_pi};
    BT_K(L, kProfHeadDw, sh, launch_heads_tc_dw(L->head_dw_ops, L->F_pi, rows, L->head_dw_kbps,
                                                L->head_pi_splits, in.count, ed, L->err_d, sh));
    umma::GemmShape shx{rows, L->F_pi, umma::kHeadCols, 1, in.count, nullptr, L->err_d};
    umma::EpiDx epx;
    epx.in_map = last_pi.relu_from_hb ? last_pi.map_hb : last_pi.map_pre;
    epx.in_bf16 = last_pi.relu_from_hb;
    epx.f32_map = last_pi.map_dpre;
    epx.hi_map = last_pi.map_dzb;
    epx.lo_map = last_pi.map_dzb_lo;
    epx.act = last_pi.act;
    epx.has_f32 = last_pi.ln;
    epx.has_hi = !epx.has_f32;
    epx.has_lo = epx.has_hi && L->x3;
    BT_K(L, kProfHeads, s,
         umma::launch_gemm<128, false, false, true>(L->head_dx_ops, shx, epx, 1, s));
  } else {
  HeadsParams hp{};
  hp.rows = rows;
  hp.count = in.count;
  hp.idx = in.idx;
  hp.f_pi = last_pi.pre();  // the heads apply the activation themselves
  hp.F_pi = L->F_pi;
  hp.f_v = last_v.pre();
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
  // the head outputs' gradients are needed only by the separate head dW kernels
  hp.d_out = L->heads_fused_dw ? nullptr : L->d_out;
  hp.d_val = L->heads_fused_dw ? nullptr : L->d_val;
  hp.d_fpi = last_pi.d_pre;
  hp.d_fv = L->shared ? nullptr : last_v.d_pre;
  hp.d_fpi_b = (last_pi.tc && !last_pi.ln) ? last_pi.dzb : nullptr;
  hp.d_fv_b = (!L->shared && last_v.tc && !last_v.ln) ? last_v.dzb : nullptr;
  hp.d_fpi_b_lo = hp.d_fpi_b ? last_pi.dzb_lo : nullptr;
  hp.d_fv_b_lo = hp.d_fv_b ? last_v.dzb_lo : nullptr;
  hp.act_pi = last_pi.act;
  hp.act_v = last_v.act;
  hp.stat_partials = L->stat_part;
  hp.dscale_partials = L->dscale_part;
  if (L->heads_fused_dw) {
    hp.dw_pi_partials = L->head_pi_part;
    hp.dw_v_partials = L->head_v_part;
  }
  BT_K(L, kProfHeads, s, launch_heads_loss(hp, L->heads_blocks, s));
  // The statistics reduction and the head weight gradients (when not fused: [F + 1, A] =
  // [f, 1]^T d_out and [F + 1, 1] = [f, 1]^T d_value) run on a side stream next to the
  // towers' backward; it joins the caller's stream before the gradient reduction, so the
  // next minibatch's heads kernel finds the partial sums consumed.
  BT_TRY(stream_dep(L, s, sh));
  BT_K(L, kProfStats, sh, launch_stat_reduce(L->stat_part, L->heads_blocks, stat_slot, sh));
  if (!L->heads_fused_dw) {
    BT_K(L, kProfHeadDw, sh, launch_skinny_dw(last_pi.pre(), L->F_pi, last_pi.act, L->d_out,
                                              L->A, rows, in.count, L->head_pi_splits,
                                              L->head_pi_part, sh));
    BT_K(L, kProfHeadDw, sh, launch_skinny_dw(last_v.pre(), L->F_v, last_v.act, L->d_val, 1,
                                              rows, in.count, L->head_v_splits,
                                              L->head_v_part, sh));
  }
  }
  // Padded minibatches (multi-GPU, bt_learner_loss_grads): the tensor-core dW GEMMs read whole
  // 64-row blocks up to the live count, and the kernels writing their bf16 dz operands (the
  // heads, the dX epilogues, LayerNorm backward) write the rows past the count up to the next
  // 64-row boundary as zeros.
  if (L->ntowers > 1) {
    BT_TRY(stream_dep(L, s, sc));
    BT_TRY(backward_tower(L, L->towers[1], in.obs, in.idx, rows, in.count, sc, -1,
                          side_stream(L, 2, s)));
  }
  BT_TRY(backward_tower(L, L->towers[0], in.obs, in.idx, rows, in.count, s, -1,
                        side_stream(L, 1, s)));
  if (L->ntowers > 1) BT_TRY(stream_dep(L, sc, s));
  BT_TRY(stream_dep(L, sh, s));
  BT_K(L, kProfReduce, s, launch_reduce_segments(L->segs_d, L->chunks_d, L->num_chunks, L->grads,
                                with_norm ? L->norm_part : nullptr, s));
  return BT_OK;
}

int check_batch(bt_learner* L, const bt_batch* b) {
  BT_CHECK_ARG(b != nullptr, "null batch");
  BT_CHECK_ARG(b->obs && b->bootstrap_obs && b->action && b->reward && b->terminated &&
                   b->truncated && b->log_prob && b->value,
               "batch has a null field");
  return BT_OK;
}

int bootstrap_and_gae(bt_learner* L, const bt_batch* b, cudaStream_t s) {
  // V(second.obs[T-1]) through the critic's tower (or the shared torso).
  TowerPlan& tv = L->towers[L->ntowers - 1];
  BT_TRY(gather_obs(L, b->bootstrap_obs, nullptr, L->N, nullptr, s));
  BT_TRY(forward_tower(L, tv, b->bootstrap_obs, nullptr, L->N, nullptr, s));
  BT_K(L, kProfHeadsFwd, s, launch_heads_forward(tv.layers.back().pre(), L->F_v, tv.layers.back().pre(), L->F_v,
                              L->params + L->head_pi_off, L->params + L->head_v_off, L->A, L->N,
                              tv.layers.back().act, tv.layers.back().act, nullptr, L->boot,
                              L->split_pi, L->split_v, s));
  BT_K(L, kProfGae, s, launch_gae_internal(b->reward, b->terminated, b->truncated, b->value, L->boot, L->T,
                             L->N, L->cfg.ppo.gamma, L->cfg.ppo.gae_lambda, L->adv, L->ret,
                             L->err_d, s));
  if (L->cfg.ppo.normalize_advantage) {
    BT_K(L, kProfMisc, s, launch_adv_moments(L->adv, L->B, L->adv_part, s));
    if (L->comm) BT_TRY(comm_allreduce_f64(L->comm, L->adv_part, 2 * kNormBlocks, s));
    BT_K(L, kProfMisc, s, launch_adv_normalize(L->adv, L->B, L->adv_part, kNormBlocks,
                                (double)L->B * std::max(1, L->cfg.world_size), s));
  }
  return BT_OK;
}

int optimizer_step(bt_learner* L, int step, cudaStream_t s) {
  if (exchange_active(L)) return exchange_optimizer_step(L, step, s);
  const bt_optimizer& o = L->cfg.optimizer;
  AdamParams ap{};
  ap.params = L->params;
  ap.mu = L->mu;
  ap.nu = L->nu;
  ap.grads = L->grads;
  ap.n = L->num_params;
  if (L->comm) {
    BT_C(L, kProfAllreduce, s, comm_allreduce_f32(L->comm, L->grads, (size_t)L->num_params, s));
    BT_K(L, kProfReduce, s, launch_sumsq(L->grads, L->num_params, L->norm_part, s));
    ap.num_norm_partials = kNormBlocks;
  } else {
    ap.num_norm_partials = L->num_chunks;
  }
  ap.norm_partials = L->norm_part;
  ap.count = L->count_d;
  ap.step = step;
  ap.lr = o.lr;
  ap.max_norm = o.max_grad_norm;
  ap.b1 = o.b1;
  ap.b2 = o.b2;
  ap.eps = o.eps;
  ap.eps_root = o.eps_root;
  ap.shadow = L->params_b;
  ap.shadow_lo = L->params_b_lo;
  BT_K(L, kProfAdam, s, launch_adam(ap, s));
  return BT_OK;
}

}  // namespace bt

using namespace bt;

// ---- C ABI -------------------------------------------------------------------------------
extern "C" int bt_learner_create(const bt_learner_config* cfg, bt_learner** out) {
  BT_CHECK_ARG(cfg && out, "bt_learner_create: null argument");
  *out = nullptr;
  BT_CHECK_ARG(cfg->num_steps > 0 && cfg->num_envs > 0, "num_steps %d / num_envs %d",
               cfg->num_steps, cfg->num_envs);
  BT_CHECK_ARG(cfg->network.obs_dim > 0, "obs_dim %d", cfg->network.obs_dim);
  BT_CHECK_ARG(cfg->precision == BT_PREC_FP32 || cfg->precision == BT_PREC_BF16 ||
                   cfg->precision == BT_PREC_BF16X3,
               "precision %d is not available in this build", cfg->precision);
  BT_CHECK_ARG(cfg->world_size >= 1 && cfg->rank >= 0 && cfg->rank < cfg->world_size,
               "rank %d / world_size %d", cfg->rank, cfg->world_size);
  bt_learner* L = new bt_learner();
  L->cfg = *cfg;
  int rc = cudaGetDevice(&L->device) == cudaSuccess ? BT_OK : BT_ERR_CUDA;
  for (int i = 0; i < 4 && rc == BT_OK; ++i)
    if (cudaStreamCreateWithFlags(&L->side[i], cudaStreamNonBlocking) != cudaSuccess) rc = BT_ERR_CUDA;
  for (int i = 0; i < 64 && rc == BT_OK; ++i) {
    cudaEvent_t e;
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
      rc = BT_ERR_CUDA;
    } else {
      L->fork_events.push_back(e);
    }
  }
  if (rc != BT_OK) set_error("bt_learner_create: stream/event creation failed");
  if (rc == BT_OK) rc = build_layout(L);
  if (rc == BT_OK) rc = allocate(L);
  if (rc != BT_OK) {
    bt_learner_destroy(L);
    return rc;
  }
  *out = L;
  return BT_OK;
}

extern "C" void bt_learner_destroy(bt_learner* L) {
  if (!L) return;
  if (L->graph) cudaGraphExecDestroy(L->graph);  // before the communicator it may use
  if (L->cap_stream) cudaStreamDestroy(L->cap_stream);
  if (L->xchg) exchange_destroy(L->xchg);
  if (L->comm) comm_destroy(L->comm);
  for (cudaEvent_t e : L->prof.pool) cudaEventDestroy(e);
  for (cudaEvent_t e : L->fork_events) cudaEventDestroy(e);
  for (cudaStream_t st : L->side)
    if (st) cudaStreamDestroy(st);
  for (void* p : L->allocations) cudaFree(p);
  delete L;
}

extern "C" int64_t bt_learner_num_params(const bt_learner* L) { return L ? L->num_params : -1; }

extern "C" int32_t bt_learner_param_count(const bt_learner* L) {
  return L ? (int32_t)L->entries.size() : -1;
}

extern "C" int bt_learner_param_info(const bt_learner* L, int32_t index, char* name,
                                     int32_t name_len, int64_t* offset, int32_t* ndim,
                                     int64_t* shape) {
  BT_CHECK_ARG(L, "null learner");
  BT_CHECK_ARG(index >= 0 && index < (int32_t)L->entries.size(), "param index %d", index);
  const ParamEntryC& e = L->entries[index];
  if (name && name_len > 0) {
    std::strncpy(name, e.name.c_str(), name_len - 1);
    name[name_len - 1] = 0;
  }
  if (offset) *offset = e.offset;
  if (ndim) *ndim = (int32_t)e.shape.size();
  if (shape)
    for (size_t i = 0; i < e.shape.size() && i < 4; ++i) shape[i] = e.shape[i];
  return BT_OK;
}

extern "C" int bt_learner_set_state(bt_learner* L, const float* params, const float* mu,
                                    const float* nu, int32_t count, void* stream) {
  BT_CHECK_ARG(L && params, "bt_learner_set_state: null argument");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t bytes = (size_t)L->num_params * 4;
  BT_CUDA(cudaMemcpyAsync(L->params, params, bytes, cudaMemcpyDefault, s));
  if (L->params_b)
    BT_K(L, kProfMisc, s, launch_to_bf16(L->params, L->params_b, L->params_b_lo, L->num_params, s));
  if (mu) {
    BT_CUDA(cudaMemcpyAsync(L->mu, mu, bytes, cudaMemcpyDefault, s));
  } else {
    BT_CUDA(cudaMemsetAsync(L->mu, 0, bytes, s));
  }
  if (nu) {
    BT_CUDA(cudaMemcpyAsync(L->nu, nu, bytes, cudaMemcpyDefault, s));
  } else {
    BT_CUDA(cudaMemsetAsync(L->nu, 0, bytes, s));
  }
  static thread_local int host_count;
  host_count = count;
  BT_CUDA(cudaMemcpyAsync(L->count_d, &host_count, 4, cudaMemcpyHostToDevice, s));
  BT_CUDA(cudaStreamSynchronize(s));  // host_count must outlive the copy
  return BT_OK;
}

extern "C" int bt_learner_get_state(bt_learner* L, float* params, float* mu, float* nu,
                                    int32_t* count, void* stream) {
  BT_CHECK_ARG(L, "null learner");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t bytes = (size_t)L->num_params * 4;
  if (params) BT_CUDA(cudaMemcpyAsync(params, L->params, bytes, cudaMemcpyDefault, s));
  if (mu) BT_CUDA(cudaMemcpyAsync(mu, L->mu, bytes, cudaMemcpyDefault, s));
  if (nu) BT_CUDA(cudaMemcpyAsync(nu, L->nu, bytes, cudaMemcpyDefault, s));
  if (count) {
    BT_CUDA(cudaMemcpyAsync(count, L->count_d, 4, cudaMemcpyDefault, s));
    BT_CUDA(cudaStreamSynchronize(s));
  }
  return BT_OK;
}

extern "C" int bt_learner_load_state(bt_learner* L, const float* params, const float* mu,
                                     const float* nu, const int32_t* count, void* stream) {
  BT_CHECK_ARG(L && params, "bt_learner_load_state: null argument");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t bytes = (size_t)L->num_params * 4;
  if (params != L->params) BT_CUDA(cudaMemcpyAsync(L->params, params, bytes, cudaMemcpyDeviceToDevice, s));
  if (L->params_b)
    BT_K(L, kProfMisc, s, launch_to_bf16(L->params, L->params_b, L->params_b_lo, L->num_params, s));
  if (mu && mu != L->mu) BT_CUDA(cudaMemcpyAsync(L->mu, mu, bytes, cudaMemcpyDeviceToDevice, s));
  if (nu && nu != L->nu) BT_CUDA(cudaMemcpyAsync(L->nu, nu, bytes, cudaMemcpyDeviceToDevice, s));
  if (count) BT_CUDA(cudaMemcpyAsync(L->count_d, count, 4, cudaMemcpyDeviceToDevice, s));
  return BT_OK;
}

extern "C" int bt_learner_store_state(bt_learner* L, float* params, float* mu, float* nu,
                                      int32_t* count, void* stream) {
  BT_CHECK_ARG(L, "null learner");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t bytes = (size_t)L->num_params * 4;
  if (params) BT_CUDA(cudaMemcpyAsync(params, L->params, bytes, cudaMemcpyDeviceToDevice, s));
  if (mu) BT_CUDA(cudaMemcpyAsync(mu, L->mu, bytes, cudaMemcpyDeviceToDevice, s));
  if (nu) BT_CUDA(cudaMemcpyAsync(nu, L->nu, bytes, cudaMemcpyDeviceToDevice, s));
  if (count) BT_CUDA(cudaMemcpyAsync(count, L->count_d, 4, cudaMemcpyDeviceToDevice, s));
  return BT_OK;
}

extern "C" int bt_learner_check(bt_learner* L, void* stream) {
  BT_CHECK_ARG(L, "null learner");
  BT_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  int code = 0;
  BT_CUDA(cudaMemcpy(&code, L->err_d, sizeof(int), cudaMemcpyDeviceToHost));
  if (code == 0) return BT_OK;
  BT_CUDA(cudaMemset(L->err_d, 0, sizeof(int)));
  if (code == 2) {
    set_error("a rank's share of a global minibatch exceeded the learner's capacity");
    return BT_ERR_CAPACITY;
  }
  if (code == 31) {  // kErrExchange (exchange.cu)
    set_error("a barrier of the NVLink gradient exchange gave up (a peer did not arrive); the "
              "update's results are invalid");
    return BT_ERR_TIMEOUT;
  }
  if (code == 21) {  // kErrGruBarrier (gru_seq.cu)
    set_error("a step barrier of the recurrent sequence kernels gave up; its results are invalid");
    return BT_ERR_TIMEOUT;
  }
  const char* what = code == umma::kErrTimeoutFull    ? "a stage of TMA loads never arrived"
                     : code == umma::kErrTimeoutEmpty ? "a stage was never released by the MMAs"
                     : code == umma::kErrTimeoutAcc   ? "an accumulator was never committed or released"
                     : code == umma::kErrTimeoutEpiIn ? "an epilogue input tile never arrived"
                                                      : "unknown";
  set_error("a bounded wait in a tensor-core GEMM gave up (code %d: %s); its results are invalid",
            code, what);
  return BT_ERR_TIMEOUT;
}

namespace {

// The body of one PPO.update (non-recurrent), enqueued on s (and side streams joined back).
int update_body(bt_learner* L, const bt_batch* batch, const int32_t* perm, float* stats,
                cudaStream_t s) {
  const int world = std::max(1, L->cfg.world_size);
  const int E = L->cfg.ppo.update_epochs, M = L->cfg.ppo.num_minibatches;
  const int64_t Bg = L->B * world;
  BT_TRY(bootstrap_and_gae(L, batch, s));
  // (with a bf16 copy of the rollout, the first epoch's minibatch gathers fill it: an epoch
  // reads every row once, so the later epochs' gathers move half the bytes)
  if (world > 1) {
    BT_K(L, kProfMisc, s, launch_local_indices(perm, E * M, L->mb, 0, L->N, L->cfg.rank, L->N * world,
                                L->rows_cap, L->local_idx, L->local_counts, L->err_d, s));
  }
  MinibatchInputs in{};
  in.obs = batch->obs;
  in.action = batch->action;
  in.lp_old = batch->log_prob;
  in.v_old = batch->value;
  in.adv = L->adv;
  in.ret = L->ret;
  in.inv_mb = 1.0f / (float)L->mb;
  for (int e = 0; e < E; ++e) {
    for (int m = 0; m < M; ++m) {
      const int i = e * M + m;
      if (world > 1) {
        in.idx = L->local_idx + (size_t)i * L->units_cap;
        in.count = L->local_counts + i;
      } else {
        in.idx = perm + (size_t)e * Bg + (size_t)m * L->mb;
        in.count = nullptr;
      }
      L->gather_rows = L->obs_b != nullptr;
      L->fill_obs_b = e == 0;
      const int rc = loss_grads(L, in, L->stat_sums + (size_t)i * kNumStatSums, world == 1, s);
      L->gather_rows = false;
      BT_TRY(rc);
      BT_TRY(optimizer_step(L, i, s));
    }
  }
  if (exchange_active(L)) BT_TRY(exchange_gather_moments(L, s));
  BT_K(L, kProfMisc, s, launch_increment(L->count_d, E * M, s));
  if (L->comm) BT_TRY(comm_allreduce_f64(L->comm, L->stat_sums, (size_t)E * M * kNumStatSums, s));
  if (stats) BT_K(L, kProfStats, s, launch_stat_finalize(L->stat_sums, E * M, 1.0f / (float)L->mb, stats, s));
  return BT_OK;
}

constexpr int kKey = 12;

void batch_key(const bt_batch* b, bool stats, const void* (&key)[kKey]) {
  const void* k[kKey] = {b->obs,        b->bootstrap_obs, b->action,     b->reward,
                         b->terminated, b->truncated,     b->log_prob,   b->value,
                         b->first_done, b->carry,         b->last_carry,
                         stats ? (const void*)1 : nullptr};
  for (int i = 0; i < kKey; ++i) key[i] = k[i];
}

bool same_key(const void* const (&a)[kKey], const void* const (&b)[kKey]) {
  for (int i = 0; i < kKey; ++i)
    if (a[i] != b[i]) return false;
  return true;
}

// One full update, recurrent or not, enqueued on s.
int run_update(bt_learner* L, const bt_batch* batch, const int32_t* perm, float* stats,
               cudaStream_t s) {
  if (L->recurrent) return recurrent_update(L, batch, perm, stats, s);
  return update_body(L, batch, perm, stats, s);
}

// Captures update_body into L->graph (updating the existing executable graph in place when
// the topology allows it). The capture enqueues nothing: the launches it counted are
// recorded as the graph's and removed from the live count.
int capture_update(bt_learner* L, const bt_batch* batch, bool stats) {
  const int64_t n0 = L->prof.launches;
  if (!L->cap_stream) BT_CUDA(cudaStreamCreateWithFlags(&L->cap_stream, cudaStreamNonBlocking));
  const cudaStream_t cs = L->cap_stream;
  BT_CUDA(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
  const int rc = run_update(L, batch, L->perm_d, stats ? L->stats_d : nullptr, cs);
  cudaGraph_t g = nullptr;
  const cudaError_t e = cudaStreamEndCapture(cs, &g);
  L->graph_launches = L->prof.launches - n0;
  L->prof.launches = n0;
  if (rc != BT_OK || e != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    if (rc != BT_OK) return rc;
    set_error("bt_learner_update: stream capture failed: %s", cudaGetErrorString(e));
    return BT_ERR_CUDA;
  }
  if (L->graph) {
    cudaGraphExecUpdateResultInfo info;
    if (cudaGraphExecUpdate(L->graph, g, &info) != cudaSuccess) {
      cudaGetLastError();
      cudaGraphExecDestroy(L->graph);
      L->graph = nullptr;
    }
  }
  cudaError_t ie = cudaSuccess;
  if (!L->graph) ie = cudaGraphInstantiate(&L->graph, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) {
    L->graph = nullptr;
    set_error("bt_learner_update: graph instantiation failed: %s", cudaGetErrorString(ie));
    return BT_ERR_CUDA;
  }
  return BT_OK;
}

}  // namespace

extern "C" int bt_learner_update(bt_learner* L, const bt_batch* batch, const int32_t* perm,
                                 float* stats, void* stream) {
  BT_CHECK_ARG(L && perm, "bt_learner_update: null argument");
  BT_TRY(check_batch(L, batch));
  const int world = std::max(1, L->cfg.world_size);
  BT_CHECK_ARG(world == 1 || L->comm, "world_size %d needs bt_learner_comm_init", world);
  cudaStream_t s = (cudaStream_t)stream;
  if (!L->graphs_on || L->prof.on) return run_update(L, batch, perm, stats, s);
  const int E = L->cfg.ppo.update_epochs, M = L->cfg.ppo.num_minibatches;
  // permutations: [E, T*N*world] samples, or [E, N*world] environments (recurrent)
  const size_t perm_bytes =
      (size_t)E * (L->recurrent ? (int64_t)L->N : L->B) * world * sizeof(int32_t);
  if (!L->perm_d) {
    BT_TRY(dalloc(L, &L->perm_d, perm_bytes / sizeof(int32_t)));
    BT_TRY(dalloc(L, &L->stats_d, (size_t)E * M * 8));
  }
  BT_CUDA(cudaMemcpyAsync(L->perm_d, perm, perm_bytes, cudaMemcpyDeviceToDevice, s));
  const void* key[kKey];
  batch_key(batch, stats != nullptr, key);
  if (L->graph && same_key(key, L->graph_key)) {
    BT_CUDA(cudaGraphLaunch(L->graph, s));
    L->prof.launches += L->graph_launches;
  } else if (same_key(key, L->seen_key)) {
    BT_TRY(capture_update(L, batch, stats != nullptr));
    for (int i = 0; i < kKey; ++i) L->graph_key[i] = key[i];
    BT_CUDA(cudaGraphLaunch(L->graph, s));
    L->prof.launches += L->graph_launches;
  } else {
    for (int i = 0; i < kKey; ++i) L->seen_key[i] = key[i];
    BT_TRY(run_update(L, batch, L->perm_d, stats ? L->stats_d : nullptr, s));
  }
  if (stats)
    BT_CUDA(cudaMemcpyAsync(stats, L->stats_d, (size_t)E * M * 8 * sizeof(float),
                            cudaMemcpyDeviceToDevice, s));
  return BT_OK;
}

extern "C" int bt_learner_use_graphs(bt_learner* L, int32_t enable) {
  BT_CHECK_ARG(L, "null learner");
  L->graphs_on = enable != 0;
  return BT_OK;
}

extern "C" int bt_learner_targets(bt_learner* L, float* advantages, float* returns,
                                  float* bootstrap, void* stream) {
  BT_CHECK_ARG(L, "null learner");
  cudaStream_t s = (cudaStream_t)stream;
  if (advantages)
    BT_CUDA(cudaMemcpyAsync(advantages, L->adv, L->B * 4, cudaMemcpyDeviceToDevice, s));
  if (returns) BT_CUDA(cudaMemcpyAsync(returns, L->ret, L->B * 4, cudaMemcpyDeviceToDevice, s));
  if (bootstrap)
    BT_CUDA(cudaMemcpyAsync(bootstrap, L->boot, L->N * 4, cudaMemcpyDeviceToDevice, s));
  return BT_OK;
}

extern "C" int bt_learner_loss_grads(bt_learner* L, const bt_batch* batch, const float* adv,
                                     const float* ret, const int32_t* indices, int32_t count,
                                     float* grads, float* stats, void* stream) {
  BT_CHECK_ARG(L && indices && adv && ret, "bt_learner_loss_grads: null argument");
  if (L->recurrent) {
    set_error("bt_learner_loss_grads: recurrent networks train through bt_learner_update");
    return BT_ERR_UNSUPPORTED;
  }
  BT_TRY(check_batch(L, batch));
  BT_CHECK_ARG(count >= 1 && count <= L->rows_cap, "count %d outside [1, %d]", count,
               L->rows_cap);
  cudaStream_t s = (cudaStream_t)stream;
  static thread_local int host_count;
  host_count = count;
  BT_CUDA(cudaMemcpyAsync(L->mb_count_d, &host_count, 4, cudaMemcpyHostToDevice, s));
  BT_CUDA(cudaStreamSynchronize(s));
  MinibatchInputs in{};
  in.obs = batch->obs;
  in.action = batch->action;
  in.lp_old = batch->log_prob;
  in.v_old = batch->value;
  in.adv = adv;
  in.ret = ret;
  in.idx = indices;
  in.count = L->mb_count_d;
  in.inv_mb = 1.0f / (float)count;
  const int E = L->cfg.ppo.update_epochs, M = L->cfg.ppo.num_minibatches;
  double* slot = L->stat_sums + (size_t)E * M * kNumStatSums;
  BT_TRY(loss_grads(L, in, slot, true, s));
  if (grads)
    BT_CUDA(cudaMemcpyAsync(grads, L->grads, (size_t)L->num_params * 4, cudaMemcpyDeviceToDevice,
                            s));
  if (stats) BT_K(L, kProfStats, s, launch_stat_finalize(slot, 1, 1.0f / (float)count, stats, s));
  return BT_OK;
}

namespace bt {
}

namespace bt {
int recurrent_act(bt_learner* L, const float* obs, const uint8_t* reset, const float* carry,
                  int num, const float* noise, float temperature, void* action, float* log_prob,
                  float* value, float* carry_out, cudaStream_t s);
}

extern "C" int bt_learner_act_recurrent(bt_learner* L, const float* obs, const uint8_t* reset,
                                        const float* carry, int32_t num, const float* noise,
                                        float temperature, void* action, float* log_prob,
                                        float* value, float* carry_out, void* stream) {
  BT_CHECK_ARG(L && obs && reset && carry && action && log_prob && carry_out,
               "bt_learner_act_recurrent: null argument");
  if (!L->recurrent) {
    set_error("bt_learner_act_recurrent: the network has no GRU layer (use bt_learner_act)");
    return BT_ERR_INVALID;
  }
  const int cap = std::min(L->act_rows, L->N);
  BT_CHECK_ARG(num >= 0 && num <= cap, "bt_learner_act_recurrent: %d rows > capacity %d", num,
               cap);
  if (num == 0) return BT_OK;
  return bt::recurrent_act(L, obs, reset, carry, num, noise, temperature, action, log_prob, value,
                           carry_out, (cudaStream_t)stream);
}

extern "C" int bt_learner_act(bt_learner* L, const float* obs, int32_t num, const float* noise,
                              float temperature, void* action, float* log_prob, float* value,
                              void* stream) {
  BT_CHECK_ARG(L && obs && action && log_prob, "bt_learner_act: null argument");
  if (L->recurrent) {
    set_error("bt_learner_act: recurrent networks need a carry (use bt_learner_act_recurrent)");
    return BT_ERR_UNSUPPORTED;
  }
  BT_CHECK_ARG(num >= 0 && num <= L->act_rows, "bt_learner_act: %d rows > capacity %d", num,
               L->act_rows);
  cudaStream_t s = (cudaStream_t)stream;
  BT_TRY(gather_obs(L, obs, nullptr, num, nullptr, s));
  for (int t = 0; t < L->ntowers; ++t)
    BT_TRY(forward_tower(L, L->towers[t], obs, nullptr, num, nullptr, s));
  TowerPlan& t0 = L->towers[0];
  TowerPlan& tv = L->towers[L->ntowers - 1];
  if (L->tc_heads) {
    // head outputs on the tensor cores (the update's arithmetic), sampled in the epilogue
    BT_K(L, kProfHeadsFwd, s, launch_heads_pack(L->params + L->head_pi_off,
                                                L->params + L->head_v_off, L->F_pi, L->A,
                                                L->whb, L->whb_lo, s));
    umma::EpiHeadsAct ea{};
    ea.A = L->A;
    ea.b_pi = L->params + L->head_pi_off + (size_t)L->F_pi * L->A;
    ea.b_v = L->params + L->head_v_off + L->F_v;
    ea.noise = noise;
    ea.temperature = temperature;
    ea.action = static_cast<int*>(action);
    ea.log_prob = log_prob;
    ea.value = value;
    BT_K(L, kProfHeadsFwd, s, launch_heads_tc_act(L->head_o_ops, num, L->F_pi, ea, L->err_d, s));
    return BT_OK;
  }
  // head outputs and the sample in one kernel
  BT_K(L, kProfHeadsFwd, s,
       launch_heads_act(t0.layers.back().pre(), L->F_pi, tv.layers.back().pre(), L->F_v,
                        L->params + L->head_pi_off, L->params + L->head_v_off,
                        L->head_scale_off >= 0 ? L->params + L->head_scale_off : nullptr,
                        L->cfg.network.head, L->A, num, t0.layers.back().act,
                        tv.layers.back().act, L->split_pi, L->split_v, noise, temperature,
                        action, log_prob, value, s));
  return BT_OK;
}

// ---- profiling ---------------------------------------------------------------------------
const char* const kProfNames[kProfNumClasses] = {
    "gae", "gemm_fwd", "gemm_dx", "gemm_dw", "heads_loss", "heads_fwd", "ln_fwd",
    "ln_bwd", "grad_reduce", "clip_adam", "stats", "allreduce", "misc", "head_dw"};

cudaEvent_t prof_event(bt_learner* L) {
  Profiler& p = L->prof;
  if (p.used == p.pool.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    p.pool.push_back(e);
  }
  return p.pool[p.used++];
}

extern "C" int bt_learner_profile(bt_learner* L, int32_t enable) {
  BT_CHECK_ARG(L, "null learner");
  L->prof.on = enable != 0;
  if (enable) {
    L->prof.recs.clear();
    L->prof.used = 0;
  }
  return BT_OK;
}

extern "C" int bt_learner_profile_read(bt_learner* L, int32_t cls, char* name, int32_t name_len,
                                       double* total_ms, int64_t* launches) {
  BT_CHECK_ARG(L, "null learner");
  BT_CHECK_ARG(cls >= 0 && cls < kProfNumClasses, "profile class %d", cls);
  double ms = 0.0;
  int64_t n = 0;
  for (const ProfRecord& r : L->prof.recs) {
    if (r.cls != cls) continue;
    BT_CUDA(cudaEventSynchronize(r.b));
    float t = 0.f;
    BT_CUDA(cudaEventElapsedTime(&t, r.a, r.b));
    ms += t;
    ++n;
  }
  if (name && name_len > 0) {
    std::strncpy(name, kProfNames[cls], name_len - 1);
    name[name_len - 1] = 0;
  }
  if (total_ms) *total_ms = ms;
  if (launches) *launches = n;
  return BT_OK;
}

extern "C" int64_t bt_learner_launch_count(const bt_learner* L) {
  return L ? L->prof.launches : -1;
}
