// Host-side VibeVoice DPM-Solver++ schedule: timesteps, sigmas and the per-step
// coefficients VibeVoiceDPMSolverScheduler applies.  fp32 scalar math in the
// same order as the reference so the coefficients are bit-identical:
//   cosine betas / alphas_cumprod      src/models/vibevoice/scheduler.cpp:15-53
//   linspace timesteps + sigmas        scheduler.cpp:55-91, 106-116
//   alpha/sigma of sigma               scheduler.cpp:93-96
//   first / second order coefficients  scheduler.cpp:182-238
//   order selection in step()          scheduler.cpp:240-274 (kSolverOrder == 2 makes
//                                      every middle step second order)
#include <cmath>
#include <cstdint>
#include <vector>

#include "../../include/b200diff.h"

namespace {

constexpr float kPi = 3.14159265358979323846F;

float alpha_bar_cosine(float t) {
    const float value = std::cos((t + 0.008F) / 1.008F * kPi * 0.5F);
    return value * value;
}

void alpha_sigma(float sigma, float& alpha_t, float& sigma_t) {
    alpha_t = 1.0F / std::sqrt(sigma * sigma + 1.0F);
    sigma_t = sigma * alpha_t;
}

}  // namespace

extern "C" b2d_status b2d_vv_schedule(int64_t ddpm_num_steps, int64_t steps, b2d_vv_step* out) {
    if (ddpm_num_steps <= 0 || steps <= 0 || out == nullptr) return B2D_EINVAL;
    std::vector<float> alphas_cumprod;
    alphas_cumprod.reserve(static_cast<size_t>(ddpm_num_steps));
    float cumulative = 1.0F;
    for (int64_t i = 0; i < ddpm_num_steps; ++i) {
        const float t1 = static_cast<float>(i) / static_cast<float>(ddpm_num_steps);
        const float t2 = static_cast<float>(i + 1) / static_cast<float>(ddpm_num_steps);
        float beta = 1.0F - alpha_bar_cosine(t2) / alpha_bar_cosine(t1);
        if (beta > 0.999F) beta = 0.999F;
        cumulative *= (1.0F - beta);
        alphas_cumprod.push_back(cumulative);
    }
    std::vector<int64_t> forward;
    for (int64_t i = 0; i <= steps; ++i) {
        const double value = 0.0 + (static_cast<double>(ddpm_num_steps - 1) - 0.0) * static_cast<double>(i) /
                                       static_cast<double>(steps);
        forward.push_back(static_cast<int64_t>(std::nearbyint(value)));
    }
    std::vector<int64_t> timesteps;
    for (int64_t i = steps; i >= 1; --i) timesteps.push_back(forward[static_cast<size_t>(i)]);
    std::vector<float> sigmas;
    for (int64_t t : timesteps) {
        const float a = alphas_cumprod[static_cast<size_t>(t)];
        sigmas.push_back(std::sqrt((1.0F - a) / a));
    }
    sigmas.push_back(0.0F);

    int64_t lower_order_nums = 0;
    for (int64_t idx = 0; idx < steps; ++idx) {
        b2d_vv_step& s = out[idx];
        s.timestep = timesteps[static_cast<size_t>(idx)];
        s.sigma = sigmas[static_cast<size_t>(idx)];
        s.sigma_next = sigmas[static_cast<size_t>(idx + 1)];
        alpha_sigma(s.sigma, s.alpha_s, s.sigma_s);
        const bool lower_order_final = idx == steps - 1;
        s.order = (lower_order_nums < 1 || lower_order_final) ? 1 : 2;
        float alpha_t, sigma_t, alpha_s0, sigma_s0;
        alpha_sigma(sigmas[static_cast<size_t>(idx + 1)], alpha_t, sigma_t);
        alpha_sigma(sigmas[static_cast<size_t>(idx)], alpha_s0, sigma_s0);
        const float lambda_t = std::log(alpha_t) - std::log(sigma_t);
        const float lambda_s0 = std::log(alpha_s0) - std::log(sigma_s0);
        const float h = lambda_t - lambda_s0;
        const float exp_neg_h = std::exp(-h);
        s.sample_coeff = sigma_t / sigma_s0;
        s.d0_coeff = -alpha_t * (exp_neg_h - 1.0F);
        s.inv_r0 = 0.0F;
        if (s.order == 2) {
            float alpha_s1, sigma_s1;
            alpha_sigma(sigmas[static_cast<size_t>(idx - 1)], alpha_s1, sigma_s1);
            const float lambda_s1 = std::log(alpha_s1) - std::log(sigma_s1);
            const float h0 = lambda_s0 - lambda_s1;
            const float r0 = h0 / h;
            s.inv_r0 = 1.0F / r0;
        }
        if (lower_order_nums < 2) ++lower_order_nums;
    }
    return B2D_OK;
}
