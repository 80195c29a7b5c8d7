/*
 * TEST INFRASTRUCTURE ONLY - never linked into, or called by, the product.
 *
 * The reference's fixed-shape PPO operators (ppo.hpp, unmodified) compiled at
 * the wide actor's shape by oracle/Makefile: FIXED_PPO_ACTOR_OBS_DIM=184 and
 * FIXED_PPO_HIDDEN_DIM=5120, the 967,688-parameter actor of
 * navigation_wide_deployment.hpp:54-66. ppo.hpp couples the actor's and the
 * critic's hidden widths in one macro (ppo.hpp:17-19,36-45); only the actor
 * operators are exported here. Pins oracle/mdn_oracle.c's o_wide_* functions.
 */
#include <cstdint>
#include <cstring>
#include <memory>

#include "ppo.hpp"

static_assert(fixed_ppo::hidden_dim == 5120 && fixed_ppo::actor_obs_dim == 184, "wide actor shape");
static_assert(fixed_ppo::actor_param_count == 967688, "967,688-parameter actor");

extern "C" {

uint32_t refw_hidden(void) { return uint32_t(fixed_ppo::hidden_dim); }
uint32_t refw_actor_param_count(void) { return uint32_t(fixed_ppo::actor_param_count); }

// fixed_ppo::actor_forward (ppo.hpp:65-80) on `rows` observation rows.
void refw_actor_forward(const float* obs, const float* actor, uint32_t rows, float* hidden, float* mean) {
    auto p = std::make_unique<fixed_ppo::ActorParams>();
    std::memcpy(p->values.data(), actor, sizeof(float) * fixed_ppo::actor_param_count);
    for (uint32_t r = 0; r < rows; r++)
        fixed_ppo::actor_forward(obs + size_t(r) * fixed_ppo::actor_obs_dim, *p, hidden + size_t(r) * fixed_ppo::hidden_dim,
                                 mean + size_t(r) * fixed_ppo::action_dim);
}

}  // extern "C"
