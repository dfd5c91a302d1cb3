// levo_ops.hpp — C++ face of liblevo_b200.so for the reference's C++ callers.
//
// Header-only wrappers over the C ABI of levo_ops.h.  They keep the names and
// the error behaviour of the reference's operators, so a call site in
// LeVo2.cpp changes its arguments (device pointers instead of ggml_tensor*),
// not its structure or its exception handling:
//   invalid arguments  -> std::invalid_argument("LeVo audio graph: ...")   (src/levo-audio-ops.cpp:10-12)
//   norm failures      -> std::runtime_error("LeVo LM: ...") for RMSNorm    (src/levo-lm.cpp:50-52),
//                         std::runtime_error("LeVo Flow estimator: ...") for LayerNorm
//                                                                          (src/levo-flow-estimator.cpp:35-37)
//   Flow-side checks   -> std::invalid_argument with the reference's wording (src/levo-renderer-pattern.cpp:127-130)
//   non-finite Euler   -> std::runtime_error("LeVo Flow renderer: ...")    (src/levo-flow-renderer.cpp:13-15,24-28)
//   cancellation       -> levo::b200::operation_cancelled                 (include/levo.h:21-24)
//   anything else      -> std::runtime_error with the library's message
// All tensors are device pointers in the reference's layouts (activations
// [channels][time], rows [rows][dim], Flow state [frames][latent_dim]).
#ifndef LEVO_OPS_HPP
#define LEVO_OPS_HPP

#include <cstddef>
#include <cstdint>
#include <exception>
#include <functional>
#include <memory>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

#include "levo_ops.h"

namespace levo::b200 {

class operation_cancelled : public std::runtime_error {
   public:
    operation_cancelled() : std::runtime_error("LeVo operation cancelled") {}
};

namespace detail {
inline void check(int rc, const char *domain) {
    if (rc == LEVO_OPS_OK) return;
    const std::string msg = std::string(domain) + levo_ops_last_error();
    if (rc == LEVO_OPS_EINVAL) throw std::invalid_argument(msg);
    if (rc == LEVO_OPS_ECANCELLED) throw operation_cancelled();
    throw std::runtime_error(msg);
}
// The reference's LM and Flow estimator report every failure (shapes included)
// through their own fail(), as std::runtime_error with their own prefix.
inline void check_runtime(int rc, const char *domain) {
    if (rc == LEVO_OPS_OK) return;
    if (rc == LEVO_OPS_ECANCELLED) throw operation_cancelled();
    throw std::runtime_error(std::string(domain) + levo_ops_last_error());
}
constexpr const char *kAudio = "LeVo audio graph: ";
constexpr const char *kLm = "LeVo LM: ";
constexpr const char *kFlowEstimator = "LeVo Flow estimator: ";
constexpr const char *kFlow = "LeVo Flow renderer: ";
constexpr const char *kVae = "LeVo VAE: ";
}  // namespace detail

// levo::detail::snake_beta (src/levo-audio-ops.cpp:125-152): y = x + sin(x*e^a)^2 / (e^b + 1e-9).
inline void snake_beta(const float *x, const float *alpha_log, const float *beta_log, float *y,
                       int64_t channels, int64_t time, levo_stream_t stream = nullptr) {
    detail::check(levo_snakebeta_f32(x, time, alpha_log, beta_log, LEVO_DTYPE_F32, y, time, channels, time,
                                     stream),
                  detail::kAudio);
}

// Per-channel alpha = exp(alpha_log) and 1/beta, computed once per weight load
// (levo_snake_params_prepare); snake_beta_prepared then gives snake_beta's exact bits.
inline void snake_params_prepare(const float *alpha_log, const float *beta_log, float *alpha, float *inv_beta,
                                 int64_t channels, levo_stream_t stream = nullptr) {
    detail::check(levo_snake_params_prepare(alpha_log, beta_log, LEVO_DTYPE_F32, channels, alpha, inv_beta, stream),
                  detail::kAudio);
}

inline void snake_beta_prepared(const float *x, const float *alpha, const float *inv_beta, float *y,
                                int64_t channels, int64_t time, levo_stream_t stream = nullptr) {
    detail::check(levo_snakebeta_f32(x, time, alpha, inv_beta, LEVO_DTYPE_SNAKE_PREPARED, y, time, channels, time,
                                     stream),
                  detail::kAudio);
}

// One run_residual / stage node run (src/levo-vae.cpp:90-101), fused.
inline void fused_unit(const levo_fused_unit &unit, levo_stream_t stream = nullptr) {
    detail::check(levo_vae_fused_unit_f32(&unit, stream), detail::kAudio);
}

// rms_norm_weighted + residual add (src/levo-lm.cpp:131-138,198-202), F16 activations.
inline void add_rms_norm_f16(const void *x, const void *residual, const float *gamma, void *h_out, void *y_out,
                             int64_t rows, int64_t dim, float eps, bool f16_boundary,
                             levo_stream_t stream = nullptr) {
    detail::check_runtime(levo_add_rmsnorm_f16(x, residual, gamma, h_out, y_out, rows, dim, eps,
                                               f16_boundary ? LEVO_NORM_F16_BOUNDARY : 0u, stream),
                          detail::kLm);
}

// layer_norm + residual add (src/levo-flow-estimator.cpp:106-109,221-227), F32 activations.
inline void add_layer_norm_f32(const float *x, const float *residual, const float *gamma, const float *beta,
                               float *h_out, float *y_out, int64_t rows, int64_t dim, float eps = 1.0e-5f,
                               levo_stream_t stream = nullptr) {
    detail::check_runtime(levo_add_layernorm_f32(x, residual, gamma, beta, h_out, y_out, rows, dim, eps, 0u, stream),
                          detail::kFlowEstimator);
}

// combine_renderer_cfg (src/levo-renderer-pattern.cpp:123-135), device vectors.
inline void combine_renderer_cfg(const float *unconditional, const float *conditional, float *out, int64_t n,
                                 float guidance_scale, levo_stream_t stream = nullptr) {
    const int rc = levo_cfg_combine_f32(unconditional, conditional, out, n, guidance_scale, stream);
    if (rc == LEVO_OPS_EINVAL) {
        // the reference's own messages, without a domain prefix
        if (n <= 0) throw std::invalid_argument("CFG vectors must have equal non-empty lengths");
        throw std::invalid_argument("CFG guidance scale must be finite");
    }
    detail::check(rc, detail::kFlow);
}

// solve_flow_euler (src/levo-flow-renderer.cpp:57-120) on device state
// [frames][latent_dim]: per step the in-context interpolation, the caller's
// velocity callback (the estimator), the fused CFG combine + Euler update and
// the reference's finiteness checks, then the final context restore; the work
// runs in levo_flow_euler_solve_f32.  `velocity(state, step)` returns a device
// pointer to [2][frames*latent_dim] (row 0 unconditional, row 1 conditional)
// when cfg, else [frames*latent_dim]; `cancelled()` is polled before each step.
// Errors carry the reference's exception types and messages: a non-finite
// velocity / state or an invalid input throws std::runtime_error("LeVo Flow
// renderer: ..."), cancellation operation_cancelled; an exception thrown by a
// callback propagates unchanged.  With a checkpoint (the reference's
// euler_resume_state, its state a caller-owned device buffer), the solve keeps
// the state before each step there: after a failure or a cancellation `state`
// holds the reference's resume state and checkpoint->completed_steps its step.
struct euler_device_input {
    float *state;              // in/out
    const float *noise;        // [frames*latent_dim]
    const float *context;      // [frames*latent_dim]
    int64_t frames = 0;
    int64_t latent_dim = 0;
    int64_t incontext_frames = 0;
    float sigma_min = 1.0e-4f;
};

struct euler_device_checkpoint {
    float *state = nullptr;  // device [frames*latent_dim], caller-owned
    int64_t completed_steps = 0;
};

template <class Velocity, class Cancelled>
void solve_flow_euler(const euler_device_input &in, int64_t steps, bool cfg, float guidance,
                      Velocity &&velocity, Cancelled &&cancelled, int32_t *status_dev,
                      int64_t completed_steps = 0, levo_stream_t stream = nullptr,
                      euler_device_checkpoint *checkpoint = nullptr) {
    using V = std::remove_reference_t<Velocity>;
    using C = std::remove_reference_t<Cancelled>;
    struct callbacks {
        V *velocity;
        C *cancelled;
        std::exception_ptr error;
    } cb{&velocity, &cancelled, nullptr};
    const levo_velocity_fn on_velocity = [](void *user, const float *state, int64_t step, float,
                                            levo_stream_t) -> const float * {
        auto *c = static_cast<callbacks *>(user);
        try {
            return (*c->velocity)(state, step);
        } catch (...) {
            c->error = std::current_exception();
            return nullptr;
        }
    };
    const levo_cancel_fn on_cancel = [](void *user) -> int {
        auto *c = static_cast<callbacks *>(user);
        try {
            return (*c->cancelled)() ? 1 : 0;
        } catch (...) {
            c->error = std::current_exception();
            return 1;
        }
    };
    int64_t done = completed_steps;
    const int rc = levo_flow_euler_solve_f32(in.state, in.noise, in.context, in.frames, in.latent_dim,
                                             in.incontext_frames, in.sigma_min, steps, completed_steps, cfg ? 1 : 0,
                                             guidance, on_velocity, &cb, on_cancel, &cb,
                                             checkpoint ? checkpoint->state : nullptr, status_dev, &done, stream);
    if (checkpoint) checkpoint->completed_steps = done;
    if (cb.error) std::rethrow_exception(cb.error);
    if (rc == LEVO_OPS_OK) return;
    if (rc == LEVO_OPS_ECANCELLED) throw operation_cancelled();
    std::string msg = levo_ops_last_error();
    const std::string own = "levo_flow_euler_solve_f32: ";
    if (msg.rfind(own, 0) == 0) msg.erase(0, own.size());
    const std::size_t step_note = msg.find(" (step");  // the reference names no step
    if (rc == LEVO_OPS_ENONFINITE && step_note != std::string::npos) msg.erase(step_note);
    throw std::runtime_error(std::string(detail::kFlow) + msg);
}

// vae_decode_result (src/levo-vae.h:12-19).
struct vae_decode_result {
    std::size_t frames = 0;
    std::size_t samples_per_channel = 0;
    std::vector<float> audio;                       // planar [audio_channels][samples_per_channel]
    std::vector<std::vector<float>> stage_outputs;  // capture_stages: stage s as [stage_width[s]][L_s]
};

// vae_decoder (src/levo-vae.h:21-43) over the elementwise chain.
class vae_decoder {
   public:
    vae_decoder(const levo_vae_topology &topology, const std::vector<float> &packed_params, int64_t max_frames,
                int device = 0, levo_conv_fn conv = nullptr, void *conv_user = nullptr) {
        levo_vae_chain *chain = nullptr;
        detail::check(levo_vae_chain_create(&chain, &topology, packed_params.data(), max_frames, conv, conv_user,
                                            device),
                      detail::kVae);
        chain_.reset(chain);
        topology_ = topology;
    }

    // vae_decoder::decode (src/levo-vae.cpp:172-276): host latent [latent_dim][frames] -> host audio
    // [audio_channels][frames * prod(strides)].  capture_stages also returns every stage's output;
    // `cancelled` is polled before the work and after it, as the reference polls around its graph
    // (src/levo-vae.cpp:248-255).  `tanh` is the BASELINE epilogue (the reference has none).
    vae_decode_result decode(const std::vector<float> &latent, std::size_t frames, bool capture_stages = false,
                             const std::function<bool()> &cancelled = {}, bool tanh = false,
                             levo_stream_t stream = nullptr) const {
        if (frames == 0 || latent.size() != frames * static_cast<std::size_t>(topology_.latent_dim))
            throw std::runtime_error("LeVo VAE: latent payload does not have shape [64,frames]");
        vae_decode_result result;
        result.frames = frames;
        std::size_t length = frames;
        if (capture_stages) result.stage_outputs.resize(static_cast<std::size_t>(topology_.n_stages));
        std::vector<float *> dest;
        for (int s = 0; s < topology_.n_stages; ++s) {
            length *= static_cast<std::size_t>(topology_.stage_stride[s]);
            if (capture_stages) {
                auto &stage = result.stage_outputs[static_cast<std::size_t>(s)];
                stage.resize(static_cast<std::size_t>(topology_.stage_width[s]) * length);
                dest.push_back(stage.data());
            }
        }
        result.samples_per_channel = length;
        result.audio.resize(static_cast<std::size_t>(topology_.audio_channels) * length);
        struct capture_scope {  // capture stays on for this call only
            levo_vae_chain *chain;
            ~capture_scope() { levo_vae_chain_set_stage_capture(chain, nullptr, 0); }
        } scope{chain_.get()};
        if (capture_stages)
            detail::check(levo_vae_chain_set_stage_capture(chain_.get(), dest.data(), topology_.n_stages),
                          detail::kVae);
        const levo_cancel_fn poll = cancelled ? &poll_cancel : nullptr;
        void *user = cancelled ? const_cast<std::function<bool()> *>(&cancelled) : nullptr;
        detail::check(levo_vae_chain_decode_windows(chain_.get(), latent.data(), 1, static_cast<int64_t>(frames),
                                                    result.audio.data(), tanh ? LEVO_CHAIN_TANH : 0u, poll, user,
                                                    stream),
                      detail::kVae);
        if (cancelled && cancelled()) throw operation_cancelled();
        return result;
    }

    levo_vae_chain *handle() const noexcept { return chain_.get(); }

   private:
    static int poll_cancel(void *user) { return (*static_cast<std::function<bool()> *>(user))() ? 1 : 0; }
    struct deleter {
        void operator()(levo_vae_chain *c) const noexcept { levo_vae_chain_destroy(c); }
    };
    std::unique_ptr<levo_vae_chain, deleter> chain_;
    levo_vae_topology topology_{};
};

}  // namespace levo::b200

#endif  // LEVO_OPS_HPP
