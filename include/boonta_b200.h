/*
 * boonta_b200 — C-ABI of the B200-native PPO learner step.
 *
 * This header is the drop-in boundary for boonta's Anakin PPO learner path. Every entry
 * point takes plain pointers and sizes (device pointers unless stated), an opaque
 * `void* stream` (a cudaStream_t; NULL = the legacy default stream) and returns an int
 * status (0 = ok, negative = error, with a message in `bt_last_error()`). Calls only
 * enqueue work on the given stream and never synchronise the device, which is the stream
 * contract of an XLA FFI custom call.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   bt_gae                  boonta/algorithms/advantage_estimators.py:8-56
 *                           (generalized_advantage_estimator, incl. rho/c V-trace weights)
 *   bt_learner_create       boonta/algorithms/ppo.py:37-55 (PPO(cfg, network, optimizer),
 *                           PPO.init) and recurrent_ppo.py:37-69 for GRU networks; the
 *                           network and optimizer are described by value, not as flax /
 *                           optax objects
 *   bt_learner_update       boonta/algorithms/ppo.py:76-233 (PPO.update) and
 *                           recurrent_ppo.py:98-281 (RecurrentPPO.update), including the
 *                           implicit gradient mean across devices inserted for
 *                           boonta/podracers/anakin.py:165-186
 *   bt_learner_act          boonta/algorithms/ppo.py:57-74 (PPO.step) with
 *                           boonta/networks/distributions.py:21-23 (Gumbel-argmax sample)
 *   bt_learner_act_recurrent
 *                           boonta/algorithms/recurrent_ppo.py:72-96 (RecurrentPPO.step)
 *   bt_learner_set_state /
 *   bt_learner_get_state    the PPOState pytree (ppo.py:30-34): params and the optax
 *                           chain state (clip: empty; adam: count, mu, nu)
 *   bt_linear_scan /
 *   bt_linear_scan_backward boonta/networks/kernels/scan.py:13-89 (the SSM torso's linear
 *                           recurrence and its custom VJP; the Pallas Mosaic-GPU kernel)
 *   bt_random_*             jax.random's threefry key operations behind ppo.py:200, 230
 *                           (permutation, split) and distributions.py:21-23 (uniform draws)
 *   bt_learner_comm_init    the NCCL communicator behind jax.distributed / XLA's
 *                           all-reduce (hangar/train.py:17-18, anakin.py:165-186)
 *
 * The XLA FFI handlers a JAX host would register (jax.ffi.register_ffi_target, the
 * mechanism of boonta/environments/__init__.py:10-15,38-43) wrap these functions one to
 * one (boonta_b200/csrc/xla_ffi.cc, built when jaxlib's headers are available).
 */
#ifndef BOONTA_B200_H_
#define BOONTA_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define BT_API __attribute__((visibility("default")))
#else
#define BT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------------------ */
#define BT_OK 0
#define BT_ERR_INVALID (-1)     /* bad argument: null pointer, shape, alignment, config */
#define BT_ERR_CUDA (-2)        /* a CUDA runtime call failed                            */
#define BT_ERR_NCCL (-3)        /* an NCCL call failed or the communicator is missing     */
#define BT_ERR_TIMEOUT (-4)     /* a bounded wait gave up                                 */
#define BT_ERR_CAPACITY (-5)    /* a rank's share of a global minibatch exceeded capacity */
#define BT_ERR_UNSUPPORTED (-6) /* a network or option this build does not implement      */

/* ---- enums --------------------------------------------------------------------------- */
#define BT_LAYER_DENSE 0
#define BT_LAYER_CONV3X3 1 /* flax Conv(features, (3,3), padding="SAME"), NHWC, then flatten */
#define BT_LAYER_GRU 2     /* flax GRUCell scanned over time, reset to zero on first.done   */

#define BT_ACT_NONE 0
#define BT_ACT_TANH 1
#define BT_ACT_RELU 2
#define BT_ACT_SILU 3

#define BT_HEAD_CATEGORICAL 0 /* distrax Categorical over the logits (distributions.py:8-38) */
#define BT_HEAD_GAUSSIAN 1    /* MultivariateNormalDiag(mean, softplus(scale) + 1e-3) with a
                                 learned state-independent scale (distributions.py:49-57)    */

#define BT_PREC_FP32 0   /* fp32 operands, fp32 accumulation (CUDA cores)                 */
#define BT_PREC_BF16 1   /* bf16 operands, fp32 accumulation (tcgen05 tensor cores)       */
#define BT_PREC_BF16X3 2 /* fp32 split into bf16 hi + lo, three tcgen05 products          */

#define BT_MAX_LAYERS 8
#define BT_NUM_STATS 8 /* actor/loss, actor/entropy, actor/approximate_kl,
                          actor/clip_fraction, actor/advantage, critic/loss,
                          critic/explained_variance, critic/value (ppo.py:170-179) */

/* ---- configuration -------------------------------------------------------------------- */
typedef struct bt_layer {
  int32_t kind;       /* BT_LAYER_*                                          */
  int32_t features;   /* Dense/GRU output width; Conv3x3 output channels      */
  int32_t activation; /* BT_ACT_* (Dense, Conv3x3)                           */
  int32_t layernorm;  /* Dense: 1 = LayerNorm(eps 1e-6) before the activation */
  int32_t height, width, in_channels; /* Conv3x3 input image (NHWC)          */
} bt_layer;

typedef struct bt_network {
  int32_t obs_dim;    /* features per observation row (flattened)               */
  int32_t num_torso;  /* layers of the shared torso, or of the actor's tower       */
  bt_layer torso[BT_MAX_LAYERS];
  int32_t num_critic; /* 0: the torso is shared; else the critic's own tower        */
  bt_layer critic[BT_MAX_LAYERS];
  int32_t head;       /* BT_HEAD_*                                               */
  int32_t action_dim; /* logits (categorical) or mean dimensions (gaussian)       */
} bt_network;

typedef struct bt_ppo_config { /* boonta/algorithms/ppo.py:17-27 */
  int32_t num_minibatches;
  int32_t update_epochs;
  float clip_coefficient;
  int32_t clip_value_loss;
  float entropy_coefficient;
  float value_coefficient;
  double gamma;      /* python floats in the reference: gamma*gae_lambda is formed in */
  double gae_lambda; /* double and rounded once to float32                           */
  int32_t normalize_advantage;
} bt_ppo_config;

typedef struct bt_optimizer { /* optax.chain(clip_by_global_norm, adam) */
  float lr, max_grad_norm, b1, b2, eps, eps_root;
} bt_optimizer;

typedef struct bt_learner_config {
  bt_network network;
  bt_ppo_config ppo;
  bt_optimizer optimizer;
  int32_t num_steps; /* T                                  */
  int32_t num_envs;  /* N envs on this rank                 */
  int32_t precision; /* BT_PREC_* for the torso GEMMs       */
  int32_t world_size;/* ranks the env batch is sharded over */
  int32_t rank;
} bt_learner_config;

/* One rollout in boonta's Transition layout, leaves [T, N, ...] (utils/transition.py). */
typedef struct bt_batch {
  const float* obs;           /* first.obs        [T, N, obs_dim]                     */
  const float* bootstrap_obs; /* second.obs[T-1]  [N, obs_dim]                        */
  const void* action;         /* second.action    int32 [T, N] | float [T, N, A]       */
  const float* reward;        /* second.reward    [T, N]                              */
  const uint8_t* terminated;  /* second.terminated [T, N] (0/1)                        */
  const uint8_t* truncated;   /* second.truncated  [T, N] (0/1)                        */
  const float* log_prob;      /* aux.log_prob     [T, N]                              */
  const float* value;         /* aux.value        [T, N]                              */
  const uint8_t* first_done;  /* recurrent: first.done [T, N]                          */
  const float* carry;         /* recurrent: carry entering step 0   [N, H]             */
  const float* last_carry;    /* recurrent: carry entering step T-1 [N, H]             */
} bt_batch;

typedef struct bt_learner bt_learner;

/* ---- error reporting -------------------------------------------------------------------- */
BT_API const char* bt_last_error(void); /* thread-local message of the last failing call */
BT_API const char* bt_version(void);

/* ---- GAE (boonta/algorithms/advantage_estimators.py:8-56) ----------------------------------
 * advantages/returns [T, N] float32; rho and c may be NULL (= 1.0). Device pointers. */
BT_API int bt_gae(const float* reward, const uint8_t* terminated, const uint8_t* truncated,
           const float* values, const float* bootstrap, const float* rho, const float* c,
           int32_t num_steps, int32_t num_envs, double gamma, double gae_lambda,
           float* advantages, float* returns, void* stream);

/* ---- linear recurrence scan (boonta/networks/kernels/scan.py:13-89) -----------------------
 * h[b, t, f] = a[b, t, f] * h[b, t-1, f] + bx[b, t, f] with h[b, -1, f] = init[b, f], over
 * [batch, steps, features] arrays (features contiguous), accumulated in float32 and stored in
 * `dtype` (the dtype of a; BT_DTYPE_*); init in `init_dtype`. The backward is the reference's
 * custom VJP: db = reverse scan of the cotangent with multipliers a[t+1], da = db * h[t-1]
 * (init at t = 0), dinit = db[:, 0] * a[:, 0]. batch <= 65535. Device pointers. */
#define BT_DTYPE_F32 0
#define BT_DTYPE_BF16 1
BT_API int bt_linear_scan(const void* a, const void* b, const void* init, void* out,
                   int32_t batch, int32_t steps, int32_t features, int32_t dtype,
                   int32_t init_dtype, void* stream);
BT_API int bt_linear_scan_backward(const void* a, const void* h, const void* init,
                            const void* cotangent, void* da, void* db, void* dinit,
                            int32_t batch, int32_t steps, int32_t features, int32_t dtype,
                            int32_t init_dtype, void* stream);

/* ---- counter-based random numbers in JAX's threefry conventions ---------------------------
 * (jax.random with threefry2x32 keys; boonta/algorithms/ppo.py:200, 230,
 * boonta/networks/distributions.py:21-23). Keys are two uint32 words (jax.random.key_data);
 * `partitionable` selects JAX's counter layout (1: jax_threefry_partitionable, the default of
 * current JAX; 0: the original layout).
 *   bt_threefry2x32_host / bt_threefry2x32: the raw block cipher (Random123 threefry2x32-20) on
 *     one counter pair (host) or n pairs (device arrays).
 *   bt_random_split: jax.random.split(key, num) on the host: out[2*i], out[2*i+1].
 *   bt_random_fill: n values of jax.random.bits (kind 0, uint32), uniform(minval, maxval)
 *     (kind 1, float32) or normal (kind 2, float32) into device memory.
 *   bt_random_permutation: jax.random.permutation(key, n) as int32 (device), with a device
 *     workspace of bt_random_permutation_workspace(n) bytes (-1: n unsupported). */
BT_API void bt_threefry2x32_host(uint32_t k0, uint32_t k1, uint32_t c0, uint32_t c1, uint32_t* y);
BT_API int bt_threefry2x32(uint32_t k0, uint32_t k1, const uint32_t* c0, const uint32_t* c1,
                    uint32_t* y0, uint32_t* y1, int64_t n, void* stream);
BT_API int bt_random_split(const uint32_t* key, int32_t num, int32_t partitionable, uint32_t* out);
BT_API int bt_random_fill(const uint32_t* key, int64_t n, int32_t kind, float minval,
                   float maxval, int32_t partitionable, void* out, void* stream);
BT_API int64_t bt_random_permutation_workspace(int64_t n);
BT_API int bt_random_permutation(const uint32_t* key, int64_t n, int32_t partitionable,
                          int32_t* out, void* workspace, int64_t workspace_bytes, void* stream);

/* ---- learner ---------------------------------------------------------------------------- */
BT_API int bt_learner_create(const bt_learner_config* cfg, bt_learner** out);
BT_API void bt_learner_destroy(bt_learner* learner);

/* Flat parameter layout (floats). Entries are (name, offset, shape). */
BT_API int64_t bt_learner_num_params(const bt_learner* learner); /* length of the flat buffer */
BT_API int32_t bt_learner_param_count(const bt_learner* learner);
BT_API int bt_learner_param_info(const bt_learner* learner, int32_t index, char* name,
                          int32_t name_len, int64_t* offset, int32_t* ndim, int64_t* shape);

/* Copy state in/out (device pointers, flat layout; mu/nu/count = optax adam state). */
BT_API int bt_learner_set_state(bt_learner* learner, const float* params, const float* mu,
                         const float* nu, int32_t count, void* stream);
BT_API int bt_learner_get_state(bt_learner* learner, float* params, float* mu, float* nu,
                         int32_t* count, void* stream);

/* The same state moves without any host synchronisation (only stream-ordered device-to-device
 * copies, the XLA FFI stream contract): all pointers are device pointers, count an int32 in
 * device memory. load_state needs params and leaves mu / nu / count as they are where NULL;
 * store_state skips the NULL ones. These carry
 * the functional PPOState of a jitted PPO.update (ppo.py:30-34, 76-233) in and out of the
 * handle around each update. */
BT_API int bt_learner_load_state(bt_learner* learner, const float* params, const float* mu,
                                 const float* nu, const int32_t* count, void* stream);
BT_API int bt_learner_store_state(bt_learner* learner, float* params, float* mu, float* nu,
                                  int32_t* count, void* stream);

/* One full learner step. permutations: device int32 [E, T*N*world_size] (or
 * [E, N*world_size] env permutations for recurrent networks); stats: device float
 * [E, M, BT_NUM_STATS] or NULL. */
BT_API int bt_learner_update(bt_learner* learner, const bt_batch* batch, const int32_t* permutations,
                      float* stats, void* stream);

/* Synchronises `stream` and reports a failure that kernels of earlier calls recorded on the
 * device (a bounded wait that gave up: BT_ERR_TIMEOUT; a rank's minibatch share beyond
 * capacity: BT_ERR_CAPACITY), clearing it. Updates only enqueue work, so their device-side
 * failures surface here (no counterpart in the reference, where XLA reports them). */
BT_API int bt_learner_check(bt_learner* learner, void* stream);

/* Self-test of the bounded waits every waiting kernel uses: one thread waits on an mbarrier
 * that nothing arrives at, for limit_us microseconds (at most 2 s), then gives up and records
 * the failure; returns BT_ERR_TIMEOUT when it did (the expected result) with the context still
 * usable. No counterpart in the reference. */
BT_API int bt_selftest_bounded_wait(int32_t limit_us, void* stream);
/* The GRU sequence kernels' grid-wide step barrier with an unreachable target and the given
 * limit (microseconds, at most 2 s): returns BT_ERR_TIMEOUT when every CTA gave up, as designed.
 * Synchronises the stream. */
BT_API int bt_selftest_gru_barrier(int32_t limit_us, void* stream);

/* CUDA-graph replay of bt_learner_update (on by default; no counterpart in the reference,
 * where XLA compiles the update into one program). The first update with a given set of
 * batch pointers runs eagerly, the second is captured into a CUDA graph, and later updates
 * with the same batch pointers replay it (the permutations and statistics are copied through
 * internal buffers, so they may change between calls). While profiling, updates run eagerly. */
BT_API int bt_learner_use_graphs(bt_learner* learner, int32_t enable);

/* Targets of the last update: advantages/returns [T, N], bootstrap values [N]. */
BT_API int bt_learner_targets(bt_learner* learner, float* advantages, float* returns,
                       float* bootstrap, void* stream);

/* Loss gradients of one minibatch without an optimizer step (parity testing):
 * indices [count] into the flattened rollout; advantages/returns as in the rollout
 * layout; grads: flat [num_params]; stats: [BT_NUM_STATS]. */
BT_API int bt_learner_loss_grads(bt_learner* learner, const bt_batch* batch,
                          const float* advantages, const float* returns,
                          const int32_t* indices, int32_t count, float* grads, float* stats,
                          void* stream);

/* Act (PPO.step): obs [num, obs_dim]. Categorical: noise = uniform draws u in (0, 1)
 * [num, A] (the Gumbel noise is -log(-log(u))), NULL = no noise; temperature 0 = greedy
 * argmax; action int32 [num]. Gaussian: noise = standard normal draws [num, A],
 * action float [num, A] = mean + temperature * scale * noise. log_prob [num],
 * value [num] (nullable). */
BT_API int bt_learner_act(bt_learner* learner, const float* obs, int32_t num, const float* noise,
                   float temperature, void* action, float* log_prob, float* value,
                   void* stream);

/* Act for GRU networks (RecurrentPPO.step, boonta/algorithms/recurrent_ppo.py:72-96): one time
 * step on num envs. obs [num, obs_dim]; reset u8 [num] (1 = the episode starts at this step:
 * the carry is zeroed first, boonta/networks/blocks/rnn.py:42-45); carry [num, H] entering the
 * step; noise, temperature, action, log_prob, value as in bt_learner_act; carry_out [num, H]
 * the carry leaving the step. num is at most N (the learner's envs per rank). */
BT_API int bt_learner_act_recurrent(bt_learner* learner, const float* obs, const uint8_t* reset,
                                    const float* carry, int32_t num, const float* noise,
                                    float temperature, void* action, float* log_prob,
                                    float* value, float* carry_out, void* stream);

/* Categorical sampling alone (boonta/networks/distributions.py:8-23): action =
 * argmax(log_softmax(logits / temperature) + (-log(-log(u)))), first index on ties; the
 * noise and log_softmax are evaluated in double and rounded once to float32, so the index
 * is a deterministic function of (logits, u). logits, uniforms [rows, num_actions]. */
BT_API int bt_sample_categorical(const float* logits, const float* uniforms, int32_t rows,
                                 int32_t num_actions, float temperature, int32_t* action,
                                 float* log_prob, void* stream);

/* ---- diagnostics ---------------------------------------------------------------------------
 * One tcgen05 tensor-core GEMM, D[M, N] (fp32, row-major) = sum_k A(m, k) B(n, k), bf16
 * operands: A is [M, K] row-major (a_mn = 0) or [K, M] row-major (a_mn = 1); B is [N, K]
 * (b_mn = 0) or [K, N] (b_mn = 1). Contiguous extents must be multiples of 8. The learner
 * runs the same kernel with fused epilogues; this entry point lets tests check the operand
 * layouts against a reference product. `splits`/`partial` are reserved (pass 1 / NULL). */
BT_API int bt_gemm_bf16(const void* A, const void* B, float* D, int32_t M, int32_t N, int32_t K,
                        int32_t a_mn, int32_t b_mn, int32_t splits, float* partial, void* stream);
/* Split-precision variant (the BT_PREC_BF16X3 arithmetic): fp32 operands given as bf16
 * pairs x = hi + lo; D = A_hi B_hi + A_hi B_lo + A_lo B_hi, accumulated in fp32. */
BT_API int bt_gemm_bf16x3(const void* A_hi, const void* A_lo, const void* B_hi, const void* B_lo,
                          float* D, int32_t M, int32_t N, int32_t K, int32_t a_mn, int32_t b_mn,
                          void* stream);

/* ---- tracing ----------------------------------------------------------------------------
 * The reference profiles with jax.profiler traces (hangar/scripts/profile_boonta.py:25-65);
 * here every kernel the learner enqueues can be bracketed with CUDA events on its stream.
 * bt_learner_profile(1) clears and starts recording, (0) stops. profile_read returns, for
 * kernel class `cls` (0 .. until it returns BT_ERR_INVALID), its name, the summed device
 * time in ms and the number of launches recorded (it synchronises on the events). While
 * recording, the work that otherwise overlaps on side streams runs on the caller's stream,
 * so each recorded time is one kernel alone on the GPU.
 * bt_learner_launch_count: kernels and collectives enqueued since creation. */
BT_API int bt_learner_profile(bt_learner* learner, int32_t enable);
BT_API int bt_learner_profile_read(bt_learner* learner, int32_t cls, char* name,
                                   int32_t name_len, double* total_ms, int64_t* launches);
BT_API int64_t bt_learner_launch_count(const bt_learner* learner);

/* ---- optimizer step (boonta/algorithms/ppo.py:182-191) ------------------------------------
 * optax.chain(clip_by_global_norm(opt->max_grad_norm), adam(opt->lr, b1, b2, eps, eps_root))
 * then optax.apply_updates, on flat fp32 device buffers of n elements, in place: params,
 * mu, nu updated from grads. `count` = Adam steps already taken (the optax count before
 * this step). Scratch (8 bytes per 8192 elements) comes from the stream-ordered allocator
 * on `stream`. */
BT_API int bt_clip_adam(float* params, float* mu, float* nu, const float* grads, int64_t n,
                        int32_t count, const bt_optimizer* opt, void* stream);

/* The same optimizer step without allocating anything (no counterpart in the reference).
 * For callers that cannot allocate device memory where they run the optimizer, e.g. an XLA
 * FFI custom call, which runs after XLA has reserved most of the GPU for its own pool.
 * Scratch is a fixed 128 KB array compiled into the library (resident on every GPU that
 * loads it until exit), so n is limited to 134,217,728 elements; larger n is rejected with
 * BT_ERR_INVALID. The first call on a device looks the array's address up (a CUDA runtime
 * query), so make that first call before any stream capture on the device; the address is
 * kept per device and CUDA context, and looked up again in a new context (after a
 * cudaDeviceReset). All calls share the array: calls whose GPU work overlaps race and must be
 * ordered by the caller. */
BT_API int bt_clip_adam_noalloc(float* params, float* mu, float* nu, const float* grads,
                                int64_t n, int32_t count, const bt_optimizer* opt, void* stream);

/* ---- multi-GPU (NCCL over NVLink) -------------------------------------------------------- */
BT_API int bt_nccl_unique_id(void* out, int32_t size); /* size >= 128 bytes */
BT_API int bt_learner_comm_init(bt_learner* learner, const void* unique_id, int32_t size);
/* The per-minibatch gradient mean and optimizer step over NVLink peer memory (on by default
 * when bt_learner_comm_init could map every peer's buffers): each rank reduces its 1/world
 * slice of the gradient from its peers' memory, runs clip + Adam on that slice and copies the
 * other slices' new parameters from their owners; 0 switches back to an NCCL all-reduce and
 * the full optimizer step on every rank (the same results up to the order of the ranks'
 * sum). Returns BT_ERR_UNSUPPORTED when enabling it without a mapping. The reference's
 * counterpart is the all-reduce XLA inserts for anakin.py:165-186. */
BT_API int bt_learner_use_p2p(bt_learner* learner, int32_t enable);
/* Timing diagnostic of the NVLink exchange (no counterpart in the reference): `iters`
 * repetitions of one part on the learner's current buffers (mode 0: the whole gradient
 * exchange + optimizer step; 1: its three barriers; 2: the slice reduction; 3: the parameter
 * gather). Every rank must make the same calls; the buffers' contents become meaningless. */
BT_API int bt_learner_exchange_probe(bt_learner* learner, int32_t mode, int32_t iters,
                                     void* stream);

#ifdef __cplusplus
}
#endif
#endif /* BOONTA_B200_H_ */
