// Per-episode plant stress variation (physics_domain.hpp:43-157) and its
// episode seed (sim_domain_episode_seed, sim.metal:50-54), for the episode
// reset. Same operations and order as the reference, so the drawn plant is
// bit-identical (IEEE division and square root, no contraction).
#pragma once
#include "mdn_shared.h"

namespace mdn {

__device__ __forceinline__ uint32_t domain_episode_seed(const mdn_runtime_config& rt, uint32_t cfg_seed, uint32_t env,
                                                        uint32_t episode) {
    uint32_t seed = rt.domain_seed ^ cfg_seed ^ ((env + 1u) * 0x9e3779b9u) ^ ((episode + 1u) * 0x85ebca6bu);
    seed ^= seed >> 16;
    seed *= 0x7feb352du;
    seed ^= seed >> 15;
    seed *= 0x846ca68bu;
    seed ^= seed >> 16;
    return seed ? seed : 1u;
}

// xorshift32 that never returns zero (rl_physics_domain_next).
__device__ __forceinline__ uint32_t domain_next(uint32_t& state) {
    uint32_t v = state ? state : 1u;
    v ^= v << 13;
    v ^= v >> 17;
    v ^= v << 5;
    state = v ? v : 1u;
    return state;
}

__device__ __forceinline__ float domain_scale(uint32_t& state, float low, float high, float amplitude) {
    const float u = float(domain_next(state) >> 8) * (1.0f / 16777216.0f);
    const float draw = low + (high - low) * u;
    return 1.0f + amplitude * (draw - 1.0f);
}

// Inverse of a symmetric positive-definite 3x3 by cofactors; false when the
// matrix is not finite, not symmetric or not positive definite.
__device__ __forceinline__ bool domain_inverse3(const float* m, float* inv) {
    const float a = m[0], b = m[1], c = m[2], d = m[3], e = m[4], f = m[5], g = m[6], h = m[7], i = m[8];
    for (int j = 0; j < 9; j++)
        if (!isfinite(m[j])) return false;
    if (fabsf(b - d) > 1.0e-6f || fabsf(c - g) > 1.0e-6f || fabsf(f - h) > 1.0e-6f) return false;
    const float minor2 = a * e - b * d;
    const float det = a * (e * i - f * h) - b * (d * i - f * g) + c * (d * h - e * g);
    if (!(a > 0.0f) || !(minor2 > 0.0f) || !(det > 0.0f) || !isfinite(det)) return false;
    const float rcp = 1.0f / det;
    inv[0] = (e * i - f * h) * rcp;
    inv[1] = (c * h - b * i) * rcp;
    inv[2] = (b * f - c * e) * rcp;
    inv[3] = (f * g - d * i) * rcp;
    inv[4] = (a * i - c * g) * rcp;
    inv[5] = (c * d - a * f) * rcp;
    inv[6] = (d * h - e * g) * rcp;
    inv[7] = (b * g - a * h) * rcp;
    inv[8] = (a * e - b * d) * rcp;
    for (int j = 0; j < 9; j++)
        if (!isfinite(inv[j])) return false;
    return true;
}

// Maximum vertical thrust over weight at action_max.
__device__ __forceinline__ float domain_thrust_to_weight(const mdn_physics_params& p) {
    float thrust = 0.0f;
    const float action = p.action_max;
    for (int rotor = 0; rotor < 4; rotor++) {
        const float* k = p.rotor_thrust_coefficients + 3 * rotor;
        const float magnitude = k[0] + k[1] * action + k[2] * action * action;
        thrust += p.rotor_thrust_directions[3 * rotor + 2] * magnitude;
    }
    const float weight = p.mass * fabsf(p.gravity_world[2]);
    return weight > 0.0f ? thrust / weight : 0.0f;
}

// rl_physics_sample_domain: `varied` starts as the nominal plant; with a
// positive amplitude the draws are mass, 3 inertia axes, then per rotor thrust
// gain, rising and falling lag. Returns false for an invalid range/amplitude,
// a non-invertible inertia or a thrust-to-weight below the range's minimum.
__device__ __noinline__ bool sample_domain(const mdn_physics_params& nominal, uint32_t& rng, float amplitude,
                                           const mdn_domain_range& r, mdn_physics_params& varied) {
    if (!isfinite(amplitude) || amplitude < 0.0f || amplitude > 1.0f || !isfinite(r.minimum_thrust_to_weight) ||
        r.minimum_thrust_to_weight < 1.0f || !isfinite(r.mass_scale_min) || !isfinite(r.mass_scale_max) ||
        !isfinite(r.inertia_axis_scale_min) || !isfinite(r.inertia_axis_scale_max) || !isfinite(r.thrust_gain_min) ||
        !isfinite(r.thrust_gain_max) || !isfinite(r.rising_lag_scale_min) || !isfinite(r.rising_lag_scale_max) ||
        !isfinite(r.falling_lag_scale_min) || !isfinite(r.falling_lag_scale_max) ||
        !(r.mass_scale_min > 0.0f && r.mass_scale_min <= r.mass_scale_max) ||
        !(r.inertia_axis_scale_min > 0.0f && r.inertia_axis_scale_min <= r.inertia_axis_scale_max) ||
        !(r.thrust_gain_min > 0.0f && r.thrust_gain_min <= r.thrust_gain_max) ||
        !(r.rising_lag_scale_min > 0.0f && r.rising_lag_scale_min <= r.rising_lag_scale_max) ||
        !(r.falling_lag_scale_min > 0.0f && r.falling_lag_scale_min <= r.falling_lag_scale_max))
        return false;
    varied = nominal;
    if (amplitude > 0.0f) {
        const float mass_scale = domain_scale(rng, r.mass_scale_min, r.mass_scale_max, amplitude);
        float axis[3];
        for (int k = 0; k < 3; k++) axis[k] = domain_scale(rng, r.inertia_axis_scale_min, r.inertia_axis_scale_max, amplitude);
        float gain[4], rising[4], falling[4];
        for (int rotor = 0; rotor < 4; rotor++) {
            gain[rotor] = domain_scale(rng, r.thrust_gain_min, r.thrust_gain_max, amplitude);
            rising[rotor] = domain_scale(rng, r.rising_lag_scale_min, r.rising_lag_scale_max, amplitude);
            falling[rotor] = domain_scale(rng, r.falling_lag_scale_min, r.falling_lag_scale_max, amplitude);
        }
        varied.mass = nominal.mass * mass_scale;
        float root[3];
        for (int k = 0; k < 3; k++) root[k] = sqrtf(axis[k]);
        for (int row = 0; row < 3; row++)
            for (int col = 0; col < 3; col++)
                varied.inertia[3 * row + col] = nominal.inertia[3 * row + col] * mass_scale * root[row] * root[col];
        if (!domain_inverse3(varied.inertia, varied.inertia_inverse)) return false;
        for (int rotor = 0; rotor < 4; rotor++) {
            for (int k = 0; k < 3; k++)
                varied.rotor_thrust_coefficients[3 * rotor + k] = nominal.rotor_thrust_coefficients[3 * rotor + k] * gain[rotor];
            varied.rotor_time_constants_rising[rotor] = nominal.rotor_time_constants_rising[rotor] * rising[rotor];
            varied.rotor_time_constants_falling[rotor] = nominal.rotor_time_constants_falling[rotor] * falling[rotor];
        }
    }
    return domain_thrust_to_weight(varied) >= r.minimum_thrust_to_weight;
}

}  // namespace mdn
