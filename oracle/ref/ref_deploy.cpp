/*
 * TEST INFRASTRUCTURE ONLY - never linked into, or called by, the product.
 *
 * The reference's deployment readers and writer (deployment.hpp,
 * navigation_wide_deployment.hpp, unmodified) behind C entry points, built by
 * oracle/Makefile into oracle/_ref/libref_deploy.so. The tests check libmdn's
 * policy export against them: byte-identical NAVPOL1 files from the same
 * weights, and NAVWID4 files that the reference's loader accepts and evaluates.
 */
#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "navigation_wide_deployment.hpp"

extern "C" {

// NavigationPolicy::write_file (deployment.hpp:166-201) with default metadata
// and the given max speed.
int refd_write_navpol(const char* path, const float* weights, float max_speed, const char* source) {
    nav_deployment::Metadata m{};
    m.max_speed_mps = max_speed;
    return nav_deployment::NavigationPolicy::write_file(path, weights, nav_deployment::actor_weight_count, m, source)
               ? 1
               : 0;
}

// Load a NAVPOL1 file; weights_out[12104], hash_out, max_speed_out.
int refd_load_navpol(const char* path, float* weights_out, uint64_t* hash_out, float* max_speed_out) {
    auto p = std::make_unique<nav_deployment::NavigationPolicy>();
    if (!p->load(path)) return 0;
    std::memcpy(weights_out, p->weights().data(), sizeof(float) * nav_deployment::actor_weight_count);
    *hash_out = p->source_checkpoint_hash();
    *max_speed_out = p->metadata().max_speed_mps;
    return 1;
}

// Load a NAVWID4 file and evaluate raw_mean / infer on `rows` observations.
// Returns the hidden width (0 = rejected).
uint32_t refd_wide_eval(const char* path, const float* obs, uint32_t rows, float* mean_out, float* velocity_out,
                        uint64_t* hash_out) {
    nav_deployment::WideNavigationPolicy p;
    if (!p.load(path)) return 0;
    for (uint32_t r = 0; r < rows; r++) {
        if (!p.raw_mean(obs + size_t(r) * 184, mean_out + size_t(r) * 4)) return 0;
        nav_deployment::NavigationAction a;
        if (!p.infer(obs + size_t(r) * 184, a)) return 0;
        for (int j = 0; j < 3; j++) velocity_out[size_t(r) * 4 + j] = a.body_velocity_mps[j];
        velocity_out[size_t(r) * 4 + 3] = a.yaw_rate_rps;
    }
    *hash_out = p.source_checkpoint_hash();
    return p.metadata().hidden_count_value;
}

// Load a NAVPOL1 file and evaluate NavigationPolicy::raw_mean on `rows`
// observations (deployment.hpp), as the reference's deployment probe does
// (main.mm:1017-1042). Returns 1, or 0 when the file or a row is rejected.
int refd_navpol_eval(const char* path, const float* obs, uint32_t rows, float* mean_out) {
    auto p = std::make_unique<nav_deployment::NavigationPolicy>();
    if (!p->load(path)) return 0;
    for (uint32_t r = 0; r < rows; r++)
        if (!p->raw_mean(obs + size_t(r) * 184, mean_out + size_t(r) * 4)) return 0;
    return 1;
}

}  // extern "C"
