// ref_shim.cpp — extern "C" wrappers over the reference's own GGML-free
// renderer functions, compiled together with the reference sources where they
// lie (src/levo-flow-renderer.cpp, src/levo-renderer-pattern.cpp) into
// oracle/_ref/libref_levo.so.  TEST INFRASTRUCTURE ONLY: used by tests/ to
// pin the oracle and the CUDA kernels against the reference's real code for
// the CFG combine, the Euler solver and the window schedule / crossfade.
#include <cstdint>
#include <cstring>
#include <exception>
#include <stdexcept>
#include <string>
#include <vector>

#include "levo-flow-renderer.h"
#include "levo-renderer-pattern.h"
#include "levo-sampling.h"

#define REF_API extern "C" __attribute__((visibility("default")))

namespace {
thread_local std::string g_error;

int fail(const std::exception &e) {
    g_error = e.what();
    return -1;
}
}  // namespace

REF_API const char *ref_last_error() { return g_error.c_str(); }

// combine_renderer_cfg (src/levo-renderer-pattern.cpp:123-135).
REF_API int ref_combine_renderer_cfg(const float *u, const float *c, int64_t n, float g, float *out) {
    try {
        std::vector<float> uu(u, u + n), cc(c, c + n);
        const std::vector<float> r = levo::combine_renderer_cfg(uu, cc, g);
        std::memcpy(out, r.data(), r.size() * sizeof(float));
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}

// solve_flow_euler (src/levo-flow-renderer.cpp:57-120) with a velocity
// callback that returns the CFG combine of precomputed per-step velocities
// (uncond/cond [steps][frames*latent_dim], indexed by absolute step).
//   resume_step >= 0: resume from {resume_step, resume_state}.
//   pause_after >= 0: the cancel callback fires on poll number pause_after
//                     (0-based), emulating a pause at that boundary.
//   seen (optional) [steps][n]: the state passed to each velocity call.
// Returns 0 when solved, 1 when paused (checkpoint in out_state /
// out_completed), -2 when the solver threw after its loop began (a non-finite
// velocity or state, src/levo-flow-renderer.cpp:104,106: the checkpoint of the
// last completed step in out_state / out_completed, the message in
// ref_last_error()), -1 on any other error (ref_last_error()).
REF_API int ref_solve_flow_euler(const float *noise, const float *context, int64_t frames,
                                 int64_t latent_dim, int64_t incontext_frames, float sigma_min,
                                 int64_t steps, const float *uncond, const float *cond, int cfg,
                                 float guidance, int64_t resume_step, const float *resume_state,
                                 int64_t pause_after, float *seen, float *out_state,
                                 int64_t *out_completed) {
    try {
        const std::size_t n = static_cast<std::size_t>(frames * latent_dim);
        levo::flow::euler_input in;
        in.initial_noise.assign(noise, noise + n);
        in.normalized_incontext.assign(context, context + n);
        in.frames = static_cast<std::size_t>(frames);
        in.latent_dim = static_cast<std::size_t>(latent_dim);
        in.incontext_frames = static_cast<std::size_t>(incontext_frames);
        in.sigma_min = sigma_min;
        std::size_t call = 0;
        const std::size_t first = resume_step >= 0 ? static_cast<std::size_t>(resume_step) : 0;
        auto velocity = [&](const std::vector<float> &state, float) {
            const std::size_t step = first + call++;
            if (seen) std::memcpy(seen + step * n, state.data(), n * sizeof(float));
            std::vector<float> u(uncond + step * n, uncond + (step + 1) * n);
            if (!cfg) return u;
            std::vector<float> c(cond + step * n, cond + (step + 1) * n);
            return levo::combine_renderer_cfg(u, c, guidance);
        };
        std::size_t polls = 0;
        levo::cancellation_callback cancelled;
        if (pause_after >= 0)
            cancelled = [&] { return polls++ >= static_cast<std::size_t>(pause_after); };
        levo::flow::euler_resume_state resume;
        if (resume_step >= 0) {
            resume.completed_steps = first;
            resume.normalized_state.assign(resume_state, resume_state + n);
        }
        levo::flow::euler_resume_state checkpoint;
        try {
            const std::vector<float> out = levo::flow::solve_flow_euler(
                in, static_cast<std::size_t>(steps), velocity, {}, cancelled,
                resume_step >= 0 ? &resume : nullptr, &checkpoint);
            std::memcpy(out_state, out.data(), n * sizeof(float));
            *out_completed = static_cast<int64_t>(checkpoint.completed_steps);
            return 0;
        } catch (const levo::operation_cancelled &) {
            std::memcpy(out_state, checkpoint.normalized_state.data(), n * sizeof(float));
            *out_completed = static_cast<int64_t>(checkpoint.completed_steps);
            return 1;
        } catch (const std::runtime_error &e) {
            if (checkpoint.normalized_state.size() != n) throw;  // thrown before the step loop
            std::memcpy(out_state, checkpoint.normalized_state.data(), n * sizeof(float));
            *out_completed = static_cast<int64_t>(checkpoint.completed_steps);
            g_error = e.what();
            return -2;
        }
    } catch (const std::exception &e) {
        return fail(e);
    }
}

// make_renderer_schedule (src/levo-renderer-pattern.cpp:57-107).
// desc receives 5 values per window: input_offset_frames,
// output_offset_samples, decoded_samples, overlap_left, overlap_right.
REF_API int ref_make_renderer_schedule(int64_t source_frames, int64_t *padded_frames,
                                       int64_t *target_samples, int64_t *windows, int64_t *desc,
                                       int64_t max_windows) {
    try {
        const levo::renderer_schedule s = levo::make_renderer_schedule(static_cast<std::size_t>(source_frames));
        *padded_frames = static_cast<int64_t>(s.padded_frames);
        *target_samples = static_cast<int64_t>(s.target_samples);
        *windows = static_cast<int64_t>(s.windows.size());
        for (std::size_t i = 0; i < s.windows.size() && static_cast<int64_t>(i) < max_windows; ++i) {
            const levo::renderer_window &w = s.windows[i];
            desc[5 * i + 0] = static_cast<int64_t>(w.input_offset_frames);
            desc[5 * i + 1] = static_cast<int64_t>(w.output_offset_samples);
            desc[5 * i + 2] = static_cast<int64_t>(w.decoded_samples);
            desc[5 * i + 3] = static_cast<int64_t>(w.overlap_left_samples);
            desc[5 * i + 4] = static_cast<int64_t>(w.overlap_right_samples);
        }
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}

// assemble_renderer_audio (src/levo-renderer-pattern.cpp:137-203).
// left/right: [windows][decoded_samples]; outputs hold target_samples each.
REF_API int ref_assemble_renderer_audio(int64_t source_frames, const float *left,
                                        const float *right, float *out_left, float *out_right) {
    try {
        const levo::renderer_schedule s = levo::make_renderer_schedule(static_cast<std::size_t>(source_frames));
        std::vector<levo::renderer_stereo_audio> decoded(s.windows.size());
        for (std::size_t i = 0; i < s.windows.size(); ++i) {
            const std::size_t n = s.windows[i].decoded_samples;
            decoded[i].left.assign(left + i * n, left + (i + 1) * n);
            decoded[i].right.assign(right + i * n, right + (i + 1) * n);
        }
        const levo::renderer_stereo_audio out = levo::assemble_renderer_audio(s, decoded);
        std::memcpy(out_left, out.left.data(), out.left.size() * sizeof(float));
        std::memcpy(out_right, out.right.data(), out.right.size() * sizeof(float));
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}

// make_renderer_euler_schedule (src/levo-renderer-pattern.cpp:109-121).
REF_API int ref_make_renderer_euler_schedule(int64_t steps, float *times, float *dt) {
    try {
        const levo::renderer_euler_schedule s = levo::make_renderer_euler_schedule(static_cast<std::size_t>(steps));
        std::memcpy(times, s.times.data(), s.times.size() * sizeof(float));
        *dt = s.dt;
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}

// Sampler::sample_streams with use_sampling = false (src/levo-sampling.cpp:129-152).
// recent: [rows][recent_len] (entries < 0 are dropped, so rows may be padded),
// the repetition window is recent_len; ignore applies to stream 0.
REF_API int ref_sample_streams_greedy(const float *logits, int64_t rows, int64_t vocab, const int64_t *recent,
                                      int64_t recent_len, float penalty, const int64_t *ignore,
                                      int64_t n_ignore, int64_t *out) {
    try {
        std::vector<levo::logits> streams(static_cast<std::size_t>(rows));
        std::vector<std::vector<int64_t>> rec;
        for (int64_t r = 0; r < rows; ++r) {
            streams[r].assign(logits + r * vocab, logits + (r + 1) * vocab);
            if (recent) {
                std::vector<int64_t> row;
                for (int64_t k = 0; k < recent_len; ++k)
                    if (recent[r * recent_len + k] >= 0) row.push_back(recent[r * recent_len + k]);
                rec.push_back(row);
            }
        }
        levo::sampling_config config;
        config.use_sampling = false;
        config.repetition_penalty = penalty;
        config.repetition_window = static_cast<std::size_t>(recent_len);
        if (ignore) config.ignore_tokens.assign(ignore, ignore + n_ignore);
        levo::Sampler sampler(0);
        const std::vector<int64_t> tokens = sampler.sample_streams(streams, config, rec);
        std::memcpy(out, tokens.data(), tokens.size() * sizeof(int64_t));
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}

// apply_cfg (src/levo-sampling.cpp:21-27): unconditional + scale * (conditional - unconditional).
REF_API int ref_apply_cfg(const float *cond, const float *uncond, int64_t n, float scale, float *out) {
    try {
        const levo::logits r = levo::apply_cfg(levo::logits(cond, cond + n), levo::logits(uncond, uncond + n), scale);
        std::memcpy(out, r.data(), r.size() * sizeof(float));
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}
