// XLA FFI handlers: the learner path as jax.ffi custom calls on the CUDA platform.
//
// boonta binds native code to JAX as XLA FFI custom calls: C++ handlers declared with
// XLA_FFI_DEFINE_HANDLER_SYMBOL, exported through extern "C" getters, wrapped in a PyCapsule
// and registered with jax.ffi.register_ffi_target (boonta/environments/__init__.py:10-15,
// 38-43; handlers in boonta/environments/ale/ffi/ffi.cc:283-339). These handlers bind the
// learner path the same way, each one a thin wrapper over the C-ABI of include/boonta_b200.h:
//
//   boonta_gae                 bt_gae                       advantage_estimators.py:8-56
//   boonta_ppo_update          bt_learner_load_state ->     ppo.py:76-233 (PPO.update, a
//                              bt_learner_update ->         pure function of the PPOState)
//                              bt_learner_store_state
//   boonta_recurrent_ppo_update  the same for GRU networks   recurrent_ppo.py:98-281
//   boonta_ppo_act             bt_learner_load_state (params only) -> bt_learner_act
//                                                           ppo.py:57-74 (PPO.step)
//
// The learner handle (its workspace, created once per device by bt_learner_create from the
// network and PPO config) travels as the int64 attribute "learner"; the PPOState (flat params,
// Adam mu / nu and count) comes in as buffers and goes out as results, so the custom call is
// a pure function as XLA expects. Every handler only enqueues work on XLA's stream.
//
// Built only when JAXLIB_INCLUDE names jaxlib's FFI headers (jax.ffi.include_dir(), which
// holds xla/ffi/api/ffi.h); `python -m boonta_b200.build` then compiles this file into the
// same library. No such header exists in this image, so this file is not compiled or tested
// here.
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "boonta_b200.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

ffi::Error status(int rc) {
  if (rc == BT_OK) return ffi::Error::Success();
  const ffi::ErrorCode code = rc == BT_ERR_INVALID || rc == BT_ERR_CAPACITY
                                  ? ffi::ErrorCode::kInvalidArgument
                              : rc == BT_ERR_UNSUPPORTED ? ffi::ErrorCode::kUnimplemented
                                                         : ffi::ErrorCode::kInternal;
  return ffi::Error(code, std::string("boonta_b200: ") + bt_last_error());
}

ffi::Error invalid(const char* what) {
  return ffi::Error(ffi::ErrorCode::kInvalidArgument, std::string("boonta_b200: ") + what);
}

bt_learner* handle(int64_t learner) { return reinterpret_cast<bt_learner*>(learner); }

// ---- GAE ------------------------------------------------------------------------------------
ffi::Error GaeCuda(cudaStream_t stream, ffi::Buffer<ffi::F32> reward, ffi::Buffer<ffi::PRED> terminated,
                   ffi::Buffer<ffi::PRED> truncated, ffi::Buffer<ffi::F32> values,
                   ffi::Buffer<ffi::F32> bootstrap, double gamma, double gae_lambda,
                   ffi::ResultBuffer<ffi::F32> advantages, ffi::ResultBuffer<ffi::F32> returns) {
  const auto dims = reward.dimensions();
  if (dims.size() != 2) return invalid("gae: reward must be [T, N]");
  const int64_t t = dims[0], n = dims[1];
  if (bootstrap.element_count() != (size_t)n) return invalid("gae: bootstrap must be [N]");
  return status(bt_gae(reward.typed_data(),
                       reinterpret_cast<const uint8_t*>(terminated.typed_data()),
                       reinterpret_cast<const uint8_t*>(truncated.typed_data()),
                       values.typed_data(), bootstrap.typed_data(), nullptr, nullptr, (int32_t)t,
                       (int32_t)n, gamma, gae_lambda, advantages->typed_data(),
                       returns->typed_data(), stream));
}

// ---- PPO.update ------------------------------------------------------------------------------
ffi::Error UpdateCommon(cudaStream_t stream, int64_t learner, bt_batch& b,
                        ffi::Buffer<ffi::S32> permutations, ffi::Buffer<ffi::F32> params,
                        ffi::Buffer<ffi::F32> mu, ffi::Buffer<ffi::F32> nu,
                        ffi::Buffer<ffi::S32> count, ffi::ResultBuffer<ffi::F32> params_out,
                        ffi::ResultBuffer<ffi::F32> mu_out, ffi::ResultBuffer<ffi::F32> nu_out,
                        ffi::ResultBuffer<ffi::S32> count_out,
                        ffi::ResultBuffer<ffi::F32> stats) {
  bt_learner* L = handle(learner);
  if (!L) return invalid("ppo_update: null learner handle");
  const int64_t p = bt_learner_num_params(L);
  if ((int64_t)params.element_count() != p || (int64_t)mu.element_count() != p ||
      (int64_t)nu.element_count() != p)
    return invalid("ppo_update: params / mu / nu do not match the learner's flat layout");
  if (count.element_count() != 1) return invalid("ppo_update: count must be a scalar");
  int rc = bt_learner_load_state(L, params.typed_data(), mu.typed_data(), nu.typed_data(),
                                 count.typed_data(), stream);
  if (rc == BT_OK) rc = bt_learner_update(L, &b, permutations.typed_data(), stats->typed_data(), stream);
  if (rc == BT_OK)
    rc = bt_learner_store_state(L, params_out->typed_data(), mu_out->typed_data(),
                                nu_out->typed_data(), count_out->typed_data(), stream);
  return status(rc);
}

ffi::Error PpoUpdateCuda(cudaStream_t stream, ffi::Buffer<ffi::F32> obs,
                         ffi::Buffer<ffi::F32> bootstrap_obs, ffi::AnyBuffer action,
                         ffi::Buffer<ffi::F32> reward, ffi::Buffer<ffi::PRED> terminated,
                         ffi::Buffer<ffi::PRED> truncated, ffi::Buffer<ffi::F32> log_prob,
                         ffi::Buffer<ffi::F32> value, ffi::Buffer<ffi::S32> permutations,
                         ffi::Buffer<ffi::F32> params, ffi::Buffer<ffi::F32> mu,
                         ffi::Buffer<ffi::F32> nu, ffi::Buffer<ffi::S32> count, int64_t learner,
                         ffi::ResultBuffer<ffi::F32> params_out,
                         ffi::ResultBuffer<ffi::F32> mu_out, ffi::ResultBuffer<ffi::F32> nu_out,
                         ffi::ResultBuffer<ffi::S32> count_out,
                         ffi::ResultBuffer<ffi::F32> stats) {
  bt_batch b{};
  b.obs = obs.typed_data();
  b.bootstrap_obs = bootstrap_obs.typed_data();
  b.action = action.untyped_data();
  b.reward = reward.typed_data();
  b.terminated = reinterpret_cast<const uint8_t*>(terminated.typed_data());
  b.truncated = reinterpret_cast<const uint8_t*>(truncated.typed_data());
  b.log_prob = log_prob.typed_data();
  b.value = value.typed_data();
  return UpdateCommon(stream, learner, b, permutations, params, mu, nu, count, params_out, mu_out,
                      nu_out, count_out, stats);
}

ffi::Error RecurrentPpoUpdateCuda(
    cudaStream_t stream, ffi::Buffer<ffi::F32> obs, ffi::Buffer<ffi::F32> bootstrap_obs,
    ffi::AnyBuffer action, ffi::Buffer<ffi::F32> reward, ffi::Buffer<ffi::PRED> terminated,
    ffi::Buffer<ffi::PRED> truncated, ffi::Buffer<ffi::F32> log_prob, ffi::Buffer<ffi::F32> value,
    ffi::Buffer<ffi::PRED> first_done, ffi::Buffer<ffi::F32> carry,
    ffi::Buffer<ffi::F32> last_carry, ffi::Buffer<ffi::S32> permutations,
    ffi::Buffer<ffi::F32> params, ffi::Buffer<ffi::F32> mu, ffi::Buffer<ffi::F32> nu,
    ffi::Buffer<ffi::S32> count, int64_t learner, ffi::ResultBuffer<ffi::F32> params_out,
    ffi::ResultBuffer<ffi::F32> mu_out, ffi::ResultBuffer<ffi::F32> nu_out,
    ffi::ResultBuffer<ffi::S32> count_out, ffi::ResultBuffer<ffi::F32> stats) {
  bt_batch b{};
  b.obs = obs.typed_data();
  b.bootstrap_obs = bootstrap_obs.typed_data();
  b.action = action.untyped_data();
  b.reward = reward.typed_data();
  b.terminated = reinterpret_cast<const uint8_t*>(terminated.typed_data());
  b.truncated = reinterpret_cast<const uint8_t*>(truncated.typed_data());
  b.log_prob = log_prob.typed_data();
  b.value = value.typed_data();
  b.first_done = reinterpret_cast<const uint8_t*>(first_done.typed_data());
  b.carry = carry.typed_data();
  b.last_carry = last_carry.typed_data();
  return UpdateCommon(stream, learner, b, permutations, params, mu, nu, count, params_out, mu_out,
                      nu_out, count_out, stats);
}

// ---- PPO.step ----------------------------------------------------------------------------------
ffi::Error PpoActCuda(cudaStream_t stream, ffi::Buffer<ffi::F32> obs, ffi::Buffer<ffi::F32> noise,
                      ffi::Buffer<ffi::F32> params, int64_t learner, float temperature,
                      ffi::Result<ffi::AnyBuffer> action, ffi::ResultBuffer<ffi::F32> log_prob,
                      ffi::ResultBuffer<ffi::F32> value) {
  bt_learner* L = handle(learner);
  if (!L) return invalid("ppo_act: null learner handle");
  const auto dims = obs.dimensions();
  if (dims.size() != 2) return invalid("ppo_act: obs must be [num, obs_dim]");
  if ((int64_t)params.element_count() != bt_learner_num_params(L))
    return invalid("ppo_act: params do not match the learner's flat layout");
  int rc = bt_learner_load_state(L, params.typed_data(), nullptr, nullptr, nullptr, stream);
  if (rc == BT_OK)
    rc = bt_learner_act(L, obs.typed_data(), (int32_t)dims[0],
                        noise.element_count() ? noise.typed_data() : nullptr, temperature,
                        action->untyped_data(), log_prob->typed_data(), value->typed_data(),
                        stream);
  return status(rc);
}

}  // namespace

XLA_FFI_DEFINE_HANDLER_SYMBOL(kGae, GaeCuda,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()   // reward [T, N]
                                  .Arg<ffi::Buffer<ffi::PRED>>()  // terminated
                                  .Arg<ffi::Buffer<ffi::PRED>>()  // truncated
                                  .Arg<ffi::Buffer<ffi::F32>>()   // values
                                  .Arg<ffi::Buffer<ffi::F32>>()   // bootstrap [N]
                                  .Attr<double>("gamma")
                                  .Attr<double>("gae_lambda")
                                  .Ret<ffi::Buffer<ffi::F32>>()   // advantages
                                  .Ret<ffi::Buffer<ffi::F32>>()); // returns

#define BT_FFI_STATE_ARGS                  \
  .Arg<ffi::Buffer<ffi::S32>>() /* perms */ \
      .Arg<ffi::Buffer<ffi::F32>>()         \
      .Arg<ffi::Buffer<ffi::F32>>()         \
      .Arg<ffi::Buffer<ffi::F32>>()         \
      .Arg<ffi::Buffer<ffi::S32>>()         \
      .Attr<int64_t>("learner")             \
      .Ret<ffi::Buffer<ffi::F32>>()         \
      .Ret<ffi::Buffer<ffi::F32>>()         \
      .Ret<ffi::Buffer<ffi::F32>>()         \
      .Ret<ffi::Buffer<ffi::S32>>()         \
      .Ret<ffi::Buffer<ffi::F32>>()

XLA_FFI_DEFINE_HANDLER_SYMBOL(kPpoUpdate, PpoUpdateCuda,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()   // first.obs
                                  .Arg<ffi::Buffer<ffi::F32>>()   // second.obs[-1]
                                  .Arg<ffi::AnyBuffer>()          // second.action
                                  .Arg<ffi::Buffer<ffi::F32>>()   // second.reward
                                  .Arg<ffi::Buffer<ffi::PRED>>()  // second.terminated
                                  .Arg<ffi::Buffer<ffi::PRED>>()  // second.truncated
                                  .Arg<ffi::Buffer<ffi::F32>>()   // aux.log_prob
                                  .Arg<ffi::Buffer<ffi::F32>>()   // aux.value
                                      BT_FFI_STATE_ARGS);

XLA_FFI_DEFINE_HANDLER_SYMBOL(kRecurrentPpoUpdate, RecurrentPpoUpdateCuda,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()   // first.obs
                                  .Arg<ffi::Buffer<ffi::F32>>()   // second.obs[-1]
                                  .Arg<ffi::AnyBuffer>()          // second.action
                                  .Arg<ffi::Buffer<ffi::F32>>()   // second.reward
                                  .Arg<ffi::Buffer<ffi::PRED>>()  // second.terminated
                                  .Arg<ffi::Buffer<ffi::PRED>>()  // second.truncated
                                  .Arg<ffi::Buffer<ffi::F32>>()   // aux.log_prob
                                  .Arg<ffi::Buffer<ffi::F32>>()   // aux.value
                                  .Arg<ffi::Buffer<ffi::PRED>>()  // first.done
                                  .Arg<ffi::Buffer<ffi::F32>>()   // carry entering step 0
                                  .Arg<ffi::Buffer<ffi::F32>>()   // carry entering step T-1
                                      BT_FFI_STATE_ARGS);

XLA_FFI_DEFINE_HANDLER_SYMBOL(kPpoAct, PpoActCuda,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()  // obs [num, obs_dim]
                                  .Arg<ffi::Buffer<ffi::F32>>()  // noise (empty: none)
                                  .Arg<ffi::Buffer<ffi::F32>>()  // params
                                  .Attr<int64_t>("learner")
                                  .Attr<float>("temperature")
                                  .Ret<ffi::AnyBuffer>()          // action
                                  .Ret<ffi::Buffer<ffi::F32>>()   // log_prob
                                  .Ret<ffi::Buffer<ffi::F32>>()); // value

// Handler getters for jax.ffi.register_ffi_target(name, PyCapsule(getter()), platform="CUDA").
extern "C" {
BT_API void* bt_xla_gae_handler() { return reinterpret_cast<void*>(kGae); }
BT_API void* bt_xla_ppo_update_handler() { return reinterpret_cast<void*>(kPpoUpdate); }
BT_API void* bt_xla_recurrent_ppo_update_handler() {
  return reinterpret_cast<void*>(kRecurrentPpoUpdate);
}
BT_API void* bt_xla_ppo_act_handler() { return reinterpret_cast<void*>(kPpoAct); }
}
