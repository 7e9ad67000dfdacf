// K9 + K10 over NVLink: the per-minibatch gradient mean fused with the optimizer step, in
// peer memory.
//
// The reference's cross-device step is an all-reduce of the gradient that XLA inserts
// (boonta/podracers/anakin.py:165-186), followed by optax's clip_by_global_norm + adam on every
// device (boonta/algorithms/ppo.py:182-191). On one NVSwitch box every GPU can load and store
// every peer's memory directly, so instead of an all-reduce followed by a full optimizer pass
// on each GPU, rank r of G:
//   1. barrier: every rank's gradient for the minibatch is complete;
//   2. reduces its 1/G slice of the flat gradient by reading that slice from every peer
//      (NVLink loads, ranks summed in rank order) into its own buffer, with the slice's sum of
//      squares;
//   3. publishes the sum of squares into every peer's mailbox, barrier; every rank now holds
//      the G partial sums and adds them in rank order (the same global norm everywhere);
//   4. runs clip + Adam on its slice only (1/G of the optimizer's memory traffic), storing each
//      new parameter and its bf16 shadow into its own buffers and into every peer's (NVLink
//      stores, fenced system-wide by each thread); the tensor-core layers' weight matrices,
//      which the peers read only through the shadow during the update, go as the shadow alone;
//   5. barrier: every slice is updated everywhere.
// The gradient crosses NVLink once inbound per rank ((G-1)/G of it) and the parameters once
// outbound ((G-1)/G), the volume of one all-reduce, with the optimizer step on 1/G of the
// parameters in between. Adam's moments stay sharded during the update (each rank owns its slice's mu / nu)
// and are gathered the same way once the update ends (with those weights' fp32 values), so every
// rank holds the full state
// between updates. The mailboxes and the peers' buffers are CUDA IPC mappings set up when the
// communicator is created (bt_learner_comm_init).
//
// Barriers: a single thread stores this rank's barrier count into a flag slot of every rank's
// mailbox (system-scope release) and waits until every slot of its own mailbox has reached that
// count (system-scope acquire). The wait is bounded (10 s): a rank that gives up records
// kErrExchange in the learner's error word and returns, and bt_learner_check reports it.
#include <algorithm>
#include <vector>

#include "learner.h"

namespace bt {

constexpr int kXchgMaxRanks = 8;
constexpr int kErrExchange = 31;
constexpr int kXchgBlocks = 4 * kNumSMs;
// A barrier gives up after 10 s: ranks can start an update seconds apart (process start-up,
// lazy module loading), far beyond any wait inside a running update.
constexpr uint64_t kXchgWaitNs = 10000000000ull;

struct XchgBox {
  unsigned long long flag[kXchgMaxRanks];  // the last barrier count rank p reached
  double sums[kXchgMaxRanks];              // rank p's sum of squares of its reduced slice
  unsigned long long count;                // this rank's barriers so far
};

struct XchgPeers {
  float* buf[kXchgMaxRanks];
};

struct XchgBoxes {
  XchgBox* box[kXchgMaxRanks];
};

}  // namespace bt

struct Exchange {
  int rank = 0, world = 1;
  int64_t n = 0, slice = 0;
  bt::XchgPeers grads{}, params{}, mu{}, nu{};
  __nv_bfloat16* shadow[bt::kXchgMaxRanks] = {};     // peers' bf16 parameter copies
  __nv_bfloat16* shadow_lo[bt::kXchgMaxRanks] = {};  // (and low halves, split mode)
  bt::XchgBoxes boxes{};
  bt::XchgBox* own = nullptr;
  double* block_sums = nullptr;
  std::vector<void*> opened;  // IPC mappings of the peers' buffers
};

namespace bt {

namespace {

__device__ __forceinline__ void store_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long load_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// One warp; lane p < world talks to rank p. With `sums` set, the warp first adds the block
// partial sums of squares and lane p stores the total into rank p's mailbox slot `rank`. Then the barrier: lane p stores this rank's barrier count into rank
// p's flag slot (release, system scope: ordered after the lane's own stores) and waits until
// rank p's slot in this rank's mailbox has reached it (acquire). The data the peers read next
// (gradients, or parameters pushed by an earlier kernel that fenced its stores) was complete
// when this kernel started.
__global__ void xchg_barrier_kernel(XchgBoxes boxes, XchgBox* own, int rank, int world,
                                    const double* sums, int nsums, int* err) {
  const int p = threadIdx.x;
  const unsigned long long c = own->count + 1;
  double t = 0.0;
  if (sums) {  // fixed lane order and tree: the same total on every launch
    for (int i = p; i < nsums; i += 32) t += sums[i];
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  }
  if (p < world) {
    if (sums) boxes.box[p]->sums[rank] = t;
    store_release_sys(&boxes.box[p]->flag[rank], c);
    const uint64_t t0 = global_timer_ns();
    while (load_acquire_sys(&own->flag[p]) < c) {
      if (global_timer_ns() - t0 > kXchgWaitNs) {
        atomicExch(err, kErrExchange);
        break;
      }
    }
  }
  __syncwarp();
  if (p == 0) own->count = c;
}

// The rank's slice [lo, hi) of the gradient summed over the ranks (rank order), written over
// its own gradient, with per-block sums of squares. lo, hi are multiples of 4.
__global__ void __launch_bounds__(256) xchg_reduce_kernel(XchgPeers g, int world, int64_t lo,
                                                          int64_t hi, float* out,
                                                          double* block_sums) {
  __shared__ double sh[8];
  double sq = 0.0;
  const int64_t q0 = lo / 4, q1 = hi / 4;
  for (int64_t q = q0 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < q1;
       q += (int64_t)gridDim.x * blockDim.x) {
    float4 v[kXchgMaxRanks];
#pragma unroll
    for (int p = 0; p < kXchgMaxRanks; ++p)
      if (p < world) v[p] = __ldcg(reinterpret_cast<const float4*>(g.buf[p]) + q);
    float4 a = v[0];
#pragma unroll
    for (int p = 1; p < kXchgMaxRanks; ++p) {
      if (p < world) {
        a.x += v[p].x;
        a.y += v[p].y;
        a.z += v[p].z;
        a.w += v[p].w;
      }
    }
    reinterpret_cast<float4*>(out)[q] = a;
    sq += (double)a.x * a.x + (double)a.y * a.y + (double)a.z * a.z + (double)a.w * a.w;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if (lane == 0) sh[warp] = sq;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += sh[w];
    block_sums[blockIdx.x] = t;
  }
}

// Every slice but the rank's own copied from its owner into `out` (and, for the parameters,
// the bf16 shadow written). Slices are `slice` long, the last one ends at n; multiples of 4.
__global__ void __launch_bounds__(256) xchg_gather_kernel(XchgPeers src, int rank, int world,
                                                          int64_t slice, int64_t n, float* out,
                                                          __nv_bfloat16* shadow,
                                                          __nv_bfloat16* shadow_lo) {
  const int64_t q4 = slice / 4;
  const int64_t total = q4 * (world - 1);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int p = (int)(i / q4);
    p += p >= rank ? 1 : 0;
    const int64_t q = (int64_t)p * q4 + i % q4;
    if (4 * q >= n) continue;
    const float4 v = __ldcg(reinterpret_cast<const float4*>(src.buf[p]) + q);
    reinterpret_cast<float4*>(out)[q] = v;
    if (shadow) store_bf16x4(shadow, shadow_lo, 4 * q, v);
  }
}

int launch_barrier(const Exchange* x, const double* sums, int nsums, int* err, cudaStream_t s) {
  xchg_barrier_kernel<<<1, 32, 0, s>>>(x->boxes, x->own, x->rank, x->world, sums, nsums, err);
  BT_LAUNCH_CHECK("xchg_barrier_kernel");
  return BT_OK;
}

int launch_reduce(const Exchange* x, int64_t lo, int64_t hi, float* out, cudaStream_t s) {
  xchg_reduce_kernel<<<kXchgBlocks, 256, 0, s>>>(x->grads, x->world, lo, hi, out, x->block_sums);
  BT_LAUNCH_CHECK("xchg_reduce_kernel");
  return BT_OK;
}

int launch_gather(const Exchange* x, const XchgPeers& src, float* out, __nv_bfloat16* shadow,
                  __nv_bfloat16* shadow_lo, cudaStream_t s) {
  xchg_gather_kernel<<<kXchgBlocks, 256, 0, s>>>(src, x->rank, x->world, x->slice, x->n, out,
                                                 shadow, shadow_lo);
  BT_LAUNCH_CHECK("xchg_gather_kernel");
  return BT_OK;
}

}  // namespace

bool exchange_active(const bt_learner* L) { return L->xchg != nullptr && L->use_xchg; }

// The gradient exchange and optimizer step of one minibatch (replaces the all-reduce and the
// full Adam pass). Enqueued on s.
int exchange_optimizer_step(bt_learner* L, int step, cudaStream_t s) {
  Exchange* x = L->xchg;
  const int64_t lo = std::min<int64_t>(x->n, (int64_t)x->rank * x->slice);
  const int64_t hi = std::min<int64_t>(x->n, lo + x->slice);
  BT_K(L, kProfAllreduce, s, launch_barrier(x, nullptr, 0, L->err_d, s));
  BT_K(L, kProfAllreduce, s, launch_reduce(x, lo, hi, L->grads, s));
  BT_K(L, kProfAllreduce, s, launch_barrier(x, x->block_sums, kXchgBlocks, L->err_d, s));
  const bt_optimizer& o = L->cfg.optimizer;
  AdamParams ap{};
  ap.params = L->params + lo;
  ap.mu = L->mu + lo;
  ap.nu = L->nu + lo;
  ap.grads = L->grads + lo;
  ap.n = hi - lo;
  ap.norm_partials = x->own->sums;
  ap.num_norm_partials = x->world;
  ap.count = L->count_d;
  ap.step = step;
  ap.lr = o.lr;
  ap.max_norm = o.max_grad_norm;
  ap.b1 = o.b1;
  ap.b2 = o.b2;
  ap.eps = o.eps;
  ap.eps_root = o.eps_root;
  ap.shadow = L->params_b ? L->params_b + lo : nullptr;
  ap.shadow_lo = L->params_b_lo ? L->params_b_lo + lo : nullptr;
  // the tensor-core layers' weight matrices are read through the bf16 shadow alone while the
  // update runs: their fp32 values are not pushed (exchange_gather_moments copies them at the
  // update's end)
  if (L->params_b) {
    for (int t = 0; t < L->ntowers; ++t) {
      for (const LayerPlan& lp : L->towers[t].layers) {
        if (!lp.tc || lp.kind != BT_LAYER_DENSE || ap.nskip == 8) continue;
        const int64_t a = std::max<int64_t>(lp.w_off, lo);
        const int64_t b = std::min<int64_t>(lp.w_off + (int64_t)lp.kin * lp.kout, hi);
        if (a < b) {
          ap.skip_lo[ap.nskip] = a - lo;
          ap.skip_hi[ap.nskip] = b - lo;
          ++ap.nskip;
        }
      }
    }
  }
  for (int p = 0; p < x->world; ++p) {
    if (p == x->rank) continue;
    ap.push_params[ap.npush] = x->params.buf[p] + lo;
    ap.push_shadow[ap.npush] = x->shadow[p] ? x->shadow[p] + lo : nullptr;
    ap.push_shadow_lo[ap.npush] = x->shadow_lo[p] ? x->shadow_lo[p] + lo : nullptr;
    ++ap.npush;
  }
  if (hi > lo) BT_K(L, kProfAdam, s, launch_adam(ap, s));
  BT_K(L, kProfAllreduce, s, launch_barrier(x, nullptr, 0, L->err_d, s));
  return BT_OK;
}

// After the update's last minibatch: every rank gathers the other ranks' slices of Adam's
// moments and of the fp32 parameters (the weights pushed only as their bf16 shadow), so the full
// state is replicated between updates.
int exchange_gather_moments(bt_learner* L, cudaStream_t s) {
  Exchange* x = L->xchg;
  BT_K(L, kProfAllreduce, s, launch_barrier(x, nullptr, 0, L->err_d, s));
  BT_K(L, kProfAllreduce, s, launch_gather(x, x->mu, L->mu, nullptr, nullptr, s));
  BT_K(L, kProfAllreduce, s, launch_gather(x, x->nu, L->nu, nullptr, nullptr, s));
  BT_K(L, kProfAllreduce, s, launch_gather(x, x->params, L->params, nullptr, nullptr, s));
  // no rank's moments change again before every rank has finished copying them
  BT_K(L, kProfAllreduce, s, launch_barrier(x, nullptr, 0, L->err_d, s));
  return BT_OK;
}

// Set-up (host): the mailbox, then the IPC handles of the gradient, parameter, moment and
// mailbox buffers exchanged through `allgather` (the communicator's all-gather of `bytes` per
// rank, blocking) and opened. Returns BT_OK with L->xchg left null when the peers cannot be
// mapped (the learner then uses the NCCL all-reduce).
int exchange_create(bt_learner* L, int (*allgather)(void* ctx, const void* send, void* recv,
                                                    size_t bytes),
                    void* ctx) {
  const int world = L->cfg.world_size, rank = L->cfg.rank;
  if (world < 2 || world > kXchgMaxRanks) return BT_OK;
  Exchange* x = new Exchange();
  x->rank = rank;
  x->world = world;
  x->n = L->num_params;
  x->slice = ((x->n + world - 1) / world + 63) / 64 * 64;
  int rc = dalloc(L, &x->own, 1);
  if (rc == BT_OK) rc = dalloc(L, &x->block_sums, kXchgBlocks);
  if (rc == BT_OK && cudaMemset(x->own, 0, sizeof(XchgBox)) != cudaSuccess) rc = BT_ERR_CUDA;
  if (rc == BT_OK && cudaDeviceSynchronize() != cudaSuccess) rc = BT_ERR_CUDA;
  constexpr int kBufs = 7;
  void* local[kBufs] = {L->grads, L->params, L->mu, L->nu, x->own, L->params_b, L->params_b_lo};
  std::vector<cudaIpcMemHandle_t> mine(kBufs), all((size_t)kBufs * world);
  for (int i = 0; i < kBufs && rc == BT_OK; ++i)
    if (local[i] && cudaIpcGetMemHandle(&mine[i], local[i]) != cudaSuccess) rc = BT_ERR_CUDA;
  // every rank takes part in the all-gather, mapped or not (a failed handle is sent as zeros
  // and makes every rank fall back together)
  int ok = rc == BT_OK ? 1 : 0;
  if (!ok) {
    cudaGetLastError();
    std::fill(mine.begin(), mine.end(), cudaIpcMemHandle_t{});
  }
  std::vector<int> oks(world);
  BT_TRY(allgather(ctx, &ok, oks.data(), sizeof(int)));
  BT_TRY(allgather(ctx, mine.data(), all.data(), sizeof(cudaIpcMemHandle_t) * kBufs));
  for (int p = 0; p < world; ++p) ok &= oks[p];
  for (int p = 0; p < world && ok; ++p) {
    for (int i = 0; i < kBufs; ++i) {
      void* ptr = local[i];
      if (!ptr) continue;  // no bf16 shadow (fp32 learner) or no low halves
      if (p != rank) {
        if (cudaIpcOpenMemHandle(&ptr, all[(size_t)p * kBufs + i],
                                 cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
          cudaGetLastError();
          ok = 0;
          break;
        }
        x->opened.push_back(ptr);
      }
      float* f = static_cast<float*>(ptr);
      switch (i) {
        case 0: x->grads.buf[p] = f; break;
        case 1: x->params.buf[p] = f; break;
        case 2: x->mu.buf[p] = f; break;
        case 3: x->nu.buf[p] = f; break;
        case 4: x->boxes.box[p] = static_cast<XchgBox*>(ptr); break;
        case 5: x->shadow[p] = static_cast<__nv_bfloat16*>(ptr); break;
        default: x->shadow_lo[p] = static_cast<__nv_bfloat16*>(ptr); break;
      }
    }
  }
  // agree: every rank uses the exchange or none does
  int agreed = ok;
  BT_TRY(allgather(ctx, &agreed, oks.data(), sizeof(int)));
  for (int p = 0; p < world; ++p) ok &= oks[p];
  if (!ok) {
    for (void* p : x->opened) cudaIpcCloseMemHandle(p);
    delete x;
    return BT_OK;
  }
  L->xchg = x;
  return BT_OK;
}

void exchange_destroy(Exchange* x) {
  if (!x) return;
  for (void* p : x->opened) cudaIpcCloseMemHandle(p);
  delete x;
}

}  // namespace bt

using namespace bt;

// Diagnostic (no counterpart in the reference): `iters` repetitions of a part of the exchange on
// the learner's current buffers, enqueued on `stream`, for timing the parts on their own. mode 0:
// the whole gradient exchange + optimizer step; 1: its three barriers alone; 2: the slice
// reduction alone; 3: the parameter gather alone. Every rank must make the same calls.
extern "C" int bt_learner_exchange_probe(bt_learner* L, int32_t mode, int32_t iters,
                                         void* stream) {
  BT_CHECK_ARG(L && L->xchg, "bt_learner_exchange_probe: no NVLink exchange on this learner");
  BT_CHECK_ARG(mode >= 0 && mode <= 3 && iters >= 0, "bt_learner_exchange_probe: mode %d", mode);
  cudaStream_t s = (cudaStream_t)stream;
  Exchange* x = L->xchg;
  const int64_t lo = std::min<int64_t>(x->n, (int64_t)x->rank * x->slice);
  const int64_t hi = std::min<int64_t>(x->n, lo + x->slice);
  for (int i = 0; i < iters; ++i) {
    if (mode == 0) {
      BT_TRY(exchange_optimizer_step(L, 0, s));
    } else if (mode == 1) {
      BT_TRY(launch_barrier(x, nullptr, 0, L->err_d, s));
      BT_TRY(launch_barrier(x, x->block_sums, kXchgBlocks, L->err_d, s));
      BT_TRY(launch_barrier(x, nullptr, 0, L->err_d, s));
    } else if (mode == 2) {
      BT_TRY(launch_reduce(x, lo, hi, L->grads, s));
    } else {
      BT_TRY(launch_gather(x, x->params, L->params, L->params_b, L->params_b_lo, s));
    }  // (mode 3 times the pull-based parameter gather, for comparison with the push)
  }
  return BT_OK;
}

extern "C" int bt_learner_use_p2p(bt_learner* L, int32_t enable) {
  BT_CHECK_ARG(L, "null learner");
  L->use_xchg = enable != 0;
  return L->xchg ? BT_OK : (enable ? BT_ERR_UNSUPPORTED : BT_OK);
}
