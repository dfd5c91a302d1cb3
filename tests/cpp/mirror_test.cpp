// C++ parity program for include/levo_ops.hpp, in the style of the reference's
// own tests (plain main(), a check per known answer).  Built and run by
// tests/test_gpu_cpp_mirror.py on a GPU box.
#include <cmath>
#include <cstdio>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "levo_ops.hpp"

static int failures = 0;
#define CHECK(cond)                                                      \
    do {                                                                 \
        if (!(cond)) {                                                   \
            std::fprintf(stderr, "FAILED %s:%d: %s\n", __FILE__, __LINE__, #cond); \
            ++failures;                                                  \
        }                                                                \
    } while (0)

template <class T>
static T *to_device(const std::vector<T> &h) {
    T *d = nullptr;
    cudaMalloc(&d, h.size() * sizeof(T) + 16);
    cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice);
    return d;
}
template <class T>
static std::vector<T> to_host(const T *d, size_t n) {
    std::vector<T> h(n);
    cudaDeviceSynchronize();
    cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost);
    return h;
}

int main() {
    using namespace levo::b200;

    // SnakeBeta known answer (tests/test-audio-ops.cpp:163-215), CUDA tolerance 2e-5.
    const std::vector<float> x = {-1.0F, 0.0F, 1.0F, -0.5F, 0.5F, 1.5F};
    const std::vector<float> a = {std::log(2.0F), std::log(0.5F)}, b = {std::log(1.5F), std::log(0.75F)};
    float *dx = to_device(x), *da = to_device(a), *db = to_device(b), *dy = to_device(std::vector<float>(6));
    snake_beta(dx, da, db, dy, 2, 3);
    const std::vector<float> y = to_host(dy, 6);
    for (int c = 0; c < 2; ++c)
        for (int t = 0; t < 3; ++t) {
            const float v = x[c * 3 + t], s = std::sin(v * std::exp(a[c]));
            CHECK(std::fabs(y[c * 3 + t] - (v + s * s / (std::exp(b[c]) + 1.0e-9F))) < 2.0e-5F);
        }

    // Prepared parameters give the same bits.
    float *dal = to_device(std::vector<float>(2)), *dib = to_device(std::vector<float>(2));
    float *dy2 = to_device(std::vector<float>(6));
    snake_params_prepare(da, db, dal, dib, 2);
    snake_beta_prepared(dx, dal, dib, dy2, 2, 3);
    CHECK(to_host(dy2, 6) == y);

    // Errors keep the reference's exception types and prefixes.
    bool thrown = false;
    try {
        snake_beta(dx, nullptr, db, dy, 2, 3);
    } catch (const std::invalid_argument &e) {
        thrown = std::string(e.what()).rfind("LeVo audio graph: ", 0) == 0;
    }
    CHECK(thrown);

    // combine_renderer_cfg known answer (tests/test-renderer-pattern.cpp:88-91).
    float *du = to_device(std::vector<float>{1.0F, 2.0F}), *dc = to_device(std::vector<float>{3.0F, 6.0F});
    float *dv = to_device(std::vector<float>(2));
    combine_renderer_cfg(du, dc, dv, 2, 1.5F);
    const std::vector<float> v = to_host(dv, 2);
    CHECK(std::fabs(v[0] - 4.0F) < 1e-6F && std::fabs(v[1] - 8.0F) < 1e-6F);
    thrown = false;
    try {
        combine_renderer_cfg(du, dc, dv, 0, 1.5F);
    } catch (const std::invalid_argument &e) {
        thrown = std::string(e.what()) == "CFG vectors must have equal non-empty lengths";
    }
    CHECK(thrown);

    // solve_flow_euler known answer (tests/test-flow-renderer.cpp:33-65): 3 frames x 2,
    // 1 in-context frame, sigma_min 0.1, 2 steps of velocity 1, final context restore.
    const std::vector<float> noise = {1.0F, 2.0F, 10.0F, 20.0F, 30.0F, 40.0F};
    const std::vector<float> ctx = {4.0F, 8.0F, 0.0F, 0.0F, 0.0F, 0.0F};
    float *dstate = to_device(noise), *dnoise = to_device(noise), *dctx = to_device(ctx);
    float *dones = to_device(std::vector<float>(6, 1.0F));
    int32_t *dstatus = to_device(std::vector<int32_t>{0});
    euler_device_input in{dstate, dnoise, dctx, 3, 2, 1, 0.1F};
    std::vector<std::vector<float>> seen;
    solve_flow_euler(
        in, 2, /*cfg=*/false, 1.0F,
        [&](const float *state, int64_t) {
            seen.push_back(to_host(state, 6));
            return static_cast<const float *>(dones);
        },
        [] { return false; }, dstatus);
    const std::vector<float> solved = to_host(dstate, 6);
    CHECK(seen.size() == 2);
    CHECK(std::fabs(seen[0][0] - 1.0F) < 1e-6F && std::fabs(seen[0][1] - 2.0F) < 1e-6F);
    CHECK(std::fabs(seen[1][0] - 2.55F) < 1e-6F && std::fabs(seen[1][1] - 5.10F) < 1e-6F);
    const float want[6] = {4, 8, 11, 21, 31, 41};
    for (int i = 0; i < 6; ++i) CHECK(std::fabs(solved[i] - want[i]) < 1e-6F);
    CHECK(to_host(dstatus, 1)[0] == 0);
    // cancellation before the first velocity evaluation (tests/test-flow-renderer.cpp:111-127)
    thrown = false;
    try {
        solve_flow_euler(in, 2, false, 1.0F, [&](const float *, int64_t) { return static_cast<const float *>(dones); },
                         [] { return true; }, dstatus);
    } catch (const operation_cancelled &) {
        thrown = true;
    }
    CHECK(thrown);
    // A non-finite velocity at step 1 throws the reference's message (src/levo-flow-renderer.cpp:104)
    // and, with a checkpoint, leaves the state after step 0 (its euler_resume_state, :107-110).
    float *dbad = to_device(std::vector<float>{1.0F, 1.0F, 1.0F, NAN, 1.0F, 1.0F});
    float *dckpt = to_device(std::vector<float>(6));
    float *dstate2 = to_device(noise);
    euler_device_input in2{dstate2, dnoise, dctx, 3, 2, 1, 0.1F};
    euler_device_checkpoint ckpt{dckpt, 0};
    std::vector<float> after_step0;
    thrown = false;
    try {
        solve_flow_euler(
            in2, 2, false, 1.0F,
            [&](const float *state, int64_t step) {
                if (step == 1) after_step0 = to_host(state, 6);  // after the step-1 interpolation
                return static_cast<const float *>(step == 0 ? dones : dbad);
            },
            [] { return false; }, dstatus, 0, nullptr, &ckpt);
    } catch (const std::runtime_error &e) {
        thrown = std::string(e.what()) == "LeVo Flow renderer: Euler velocity contains a non-finite value";
    }
    CHECK(thrown);
    CHECK(ckpt.completed_steps == 1);
    const std::vector<float> resumed = to_host(dstate2, 6);
    // the checkpoint is the state before the step-1 interpolation: noise + 1 * dt for every element
    const float ck[6] = {1.5F, 2.5F, 10.5F, 20.5F, 30.5F, 40.5F};
    for (int i = 0; i < 6; ++i) CHECK(std::fabs(resumed[i] - ck[i]) < 1e-6F);
    CHECK(to_host(dckpt, 6) == resumed);
    (void)after_step0;
    // Non-finite noise is rejected before any step (src/levo-flow-renderer.cpp:71), state untouched.
    std::vector<float> bad_noise = noise;
    bad_noise[4] = NAN;
    float *dnoise_bad = to_device(bad_noise);
    float *dstate3 = to_device(bad_noise);
    euler_device_input in3{dstate3, dnoise_bad, dctx, 3, 2, 1, 0.1F};
    int calls = 0;
    thrown = false;
    try {
        solve_flow_euler(
            in3, 2, false, 1.0F,
            [&](const float *, int64_t) {
                ++calls;
                return static_cast<const float *>(dones);
            },
            [] { return false; }, dstatus);
    } catch (const std::runtime_error &e) {
        thrown = std::string(e.what()) == "LeVo Flow renderer: Euler noise contains a non-finite value";
    }
    CHECK(thrown);
    CHECK(calls == 0);
    const std::vector<float> untouched = to_host(dstate3, 6);
    CHECK(std::isnan(untouched[4]) && untouched[0] == bad_noise[0] && untouched[5] == bad_noise[5]);

    // Norm errors carry the prefixes of the reference's LM and Flow estimator (std::runtime_error).
    thrown = false;
    try {
        add_rms_norm_f16(dx, nullptr, nullptr, nullptr, dy, 1, 8, 1e-6F, false);
    } catch (const std::runtime_error &e) {
        thrown = std::string(e.what()).rfind("LeVo LM: ", 0) == 0;
    }
    CHECK(thrown);
    thrown = false;
    try {
        add_layer_norm_f32(dx, nullptr, dx, nullptr, nullptr, dy, 1, 4);
    } catch (const std::runtime_error &e) {
        thrown = std::string(e.what()).rfind("LeVo Flow estimator: ", 0) == 0;
    }
    CHECK(thrown);

    // vae_decoder over a reduced topology: deterministic, finite, bounded by tanh.
    levo_vae_topology topo{};
    topo.latent_dim = 4;
    topo.audio_channels = 2;
    topo.entry_width = 16;
    topo.n_stages = 2;
    topo.stage_width[0] = 8;
    topo.stage_stride[0] = 3;
    topo.stage_width[1] = 4;
    topo.stage_stride[1] = 2;
    topo.n_residual = 1;
    topo.dilation[0] = 1;
    const int64_t nparams = levo_vae_param_count(&topo);
    std::vector<float> params(static_cast<size_t>(nparams));
    for (size_t i = 0; i < params.size(); ++i) params[i] = 0.01F * static_cast<float>(static_cast<int>(i % 17) - 8);
    vae_decoder dec(topo, params, 16);
    std::vector<float> latent(4 * 10);
    for (size_t i = 0; i < latent.size(); ++i) latent[i] = std::sin(0.3F * static_cast<float>(i));
    const vae_decode_result r1 = dec.decode(latent, 10, false, {}, true), r2 = dec.decode(latent, 10, true, {}, true);
    const std::vector<float> &a1 = r1.audio;
    CHECK(r1.frames == 10 && r1.samples_per_channel == 60);
    CHECK(a1.size() == static_cast<size_t>(2 * 10 * 6) && a1 == r2.audio);
    for (float s : a1) CHECK(std::isfinite(s) && std::fabs(s) <= 1.0F);
    // capture_stages: stage outputs [8][30] and [4][60]; none for the plain decode
    CHECK(r1.stage_outputs.empty() && r2.stage_outputs.size() == 2);
    CHECK(r2.stage_outputs.size() == 2 && r2.stage_outputs[0].size() == 8 * 30 && r2.stage_outputs[1].size() == 4 * 60);
    for (const auto &stage : r2.stage_outputs)
        for (float v : stage) CHECK(std::isfinite(v));
    thrown = false;
    try {
        (void)dec.decode(latent, 9);
    } catch (const std::runtime_error &e) {
        thrown = std::string(e.what()).rfind("LeVo VAE: ", 0) == 0;
    }
    CHECK(thrown);
    // a non-finite latent is rejected like vae_decoder::decode (src/levo-vae.cpp:189-191)
    std::vector<float> bad = latent;
    bad[7] = std::nanf("");
    thrown = false;
    try {
        (void)dec.decode(bad, 10);
    } catch (const std::runtime_error &e) {
        thrown = std::string(e.what()).find("non-finite") != std::string::npos;
    }
    CHECK(thrown);
    // cancellation before the work
    thrown = false;
    try {
        (void)dec.decode(latent, 10, false, [] { return true; });
    } catch (const operation_cancelled &) {
        thrown = true;
    }
    CHECK(thrown);

    if (failures == 0) std::printf("mirror ok\n");
    return failures == 0 ? 0 : 1;
}
