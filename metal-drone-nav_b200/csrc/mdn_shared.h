// Constants and kernel-argument layouts shared by the host (g++) and device
// (nvcc) sides of libmdn. No device code here.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "mdn.h"

namespace mdn {

constexpr int kPixels = 320;
constexpr int kFrames = 8;
constexpr int kActorObs = 184;
constexpr int kCriticObs = 32;
// The control-state critic's inputs (FIXED_PPO_CRITIC_OBS_DIM=64 with
// NAV_CRITIC_CONTROL_STATE, sim.metal:166-180): the 32 above, then 32
// training-only inputs (RAPTOR hidden state, rotor speeds, yaw error, last
// command, desired velocity, goal-closing speed, goal distance, speed).
constexpr int kCriticObsControl = 64;
constexpr int kHidden = 64;
constexpr int kActions = 4;
constexpr int kActorB1 = kHidden * kActorObs;
constexpr int kActorW2 = kActorB1 + kHidden;
constexpr int kActorB2 = kActorW2 + kActions * kHidden;
constexpr int kActorLogStd = kActorB2 + kActions;
constexpr int kActorParams = kActorLogStd + kActions;
constexpr int kCriticB1 = kHidden * kCriticObs;
constexpr int kCriticW2 = kCriticB1 + kHidden;
constexpr int kCriticB2 = kCriticW2 + kHidden;
constexpr int kCriticParams = kCriticB2 + 1;
constexpr float kLogTwoPi = 1.8378770664093453f;
constexpr float kTanV = 0.75f;  // legacy camera, sensor_profile.hpp:44-45
constexpr int kWorldSoaWords = 161;
// Flat actor parameter count at hidden width h (ppo.hpp:35-40).
constexpr uint32_t actor_param_count(uint32_t h) { return h * kActorObs + h + kActions * h + 2 * kActions; }

// Launch shapes of one policy step (rollout.cu plan_step).
struct StepPlan {
    int act_grid = 1;       // persistent k_act CTAs (wide actor)
    int act_rows_grid = 1;  // persistent k_act_rows / k_act_quads CTAs (64-unit actor)
    int act_quads = 0;      // 1: four threads per environment (small shards)
    int advance_group = 1;  // lanes per environment in k_advance (1 or 2)
    int advance_grid = 1;   // k_advance CTAs (grid-stride over environments)
    int reset_grid = 1;     // k_reset_list CTAs (grid-stride over the step's reset list)
    int sense_reset_blocks = 1;  // k_reset_sense blocks (the previous step's listed resets)
};

// Side stream and events of the forked sensing step inside a collected
// rollout (k_reset_sense beside k_sense), and the launch priority of its
// reset kernel.
struct StepFork {
    cudaStream_t side;
    cudaEvent_t fork, join;
    int priority;
};

// Everything one launch of a rollout kernel needs (passed by value).
struct SimArgs {
    mdn_sim_config cfg;
    uint32_t n;          // local environments on this GPU
    uint32_t env_base;   // global id of local env 0 (seeds, clean-env parity)
    // Delay rehearsal (NAV_DELAY_REHEARSAL of the reference's delay-training
    // build): under mode 22, every other group of four environments trains
    // without delays, wind or depth noise.
    uint32_t delay_rehearsal;
    uint32_t tick;       // row block tick*n .. tick*n+n-1
    float room_lo[3], room_hi[3], room_c[3], room_e[3];
    mdn_physics_state* states;
    mdn_sim_run* runs;
    mdn_world* worlds;
    // Structure-of-arrays mirror of `worlds` for thread-per-environment
    // readers: word w of env i's obstacle block at world_soa[w * n + i],
    // w = obstacle * 10 + field (kind bits, centre xyz, size xyz, velocity xyz),
    // w = 160 the obstacle count. Written wherever a world is written.
    float* world_soa;
    float* sensors;
    float* poses;
    float* commands;
    const float* actor;
    const float* critic;
    const mdn_raptor_weights* raptor;
    const mdn_physics_params* physics;
    float* obs;
    float* co;
    float* actions;
    float* logp;
    float* values;
    float* rewards;
    float* next_values;
    uint8_t* terminated;
    uint8_t* truncated;
    int32_t* contact;
    mdn_task_control task_ctl;  // goal-arrival tasks (enabled = 0: legacy episodes)
    mdn_task_state* tasks;
    uint32_t task_config_ok;  // host-side navigation_generate_task config checks (:347-379) passed
    // Actor shape: hidden width and the offsets of b2 / log_std in the flat
    // parameter vector (ppo.hpp:35-40). Wide actors (hidden > 64) are evaluated
    // by the tensor-core forward, which leaves per-slice output sums in
    // wide_partials[wide_slices][n][4]; k_act adds them up.
    uint32_t actor_hidden, actor_b2, actor_log_std;
    const float* wide_partials;
    uint32_t wide_slices;
    // Layered networks (mlp.cu): the step's critic values come from
    // critic_values[n], and k_advance stores the post-step critic observation
    // in next_co[n][32] for the layered critic instead of evaluating the
    // 64-unit one (both null otherwise).
    const float* critic_values;
    float* next_co;
    // Width of a critic observation row in co: kCriticObs, or
    // kCriticObsControl for the control-state critic (layered networks only),
    // whose bootstrap rows k_control_state assembles in next_co_full[n][64]
    // (next_co stays [n][32]; null for the 32-input critic).
    uint32_t co_dim;
    float* next_co_full;
    // Mechanical contact audit (null = off): results[tick][n], safety margin.
    mdn_contact_audit* audit;
    float audit_margin;
    // Frozen challenge bank (ChallengeBankControl, sim.metal:13): level worlds,
    // the env-major schedule [n][bank_stride] of level ids, the level each env
    // plays (0xffffffff: none / rehearsal) and, per row, the level that the
    // transition belongs to (null until a bank is configured).
    uint32_t bank_enabled, bank_count, bank_stride;
    const mdn_world* bank_worlds;
    const uint32_t* bank_schedule;
    uint32_t* bank_active;
    uint32_t* bank_transition;
    // Per-episode plant (NavigationRuntimeConfig, navigation_runtime.hpp:9-14):
    // while runtime.enabled, each env's plant lives in env_physics[n].
    mdn_runtime_config runtime;
    mdn_physics_params* env_physics;
    // Episodes that ended in a step: k_advance appends them to the list and
    // counts them in reset_count[phase], and sets reset_pending[i] of every
    // environment it advances (1 = listed). Inside a collected rollout the
    // next step's k_reset_sense resets and senses the listed environments
    // (reading reset_count[phase ^ 1]) while k_sense senses the others and
    // zeroes reset_count[phase] for its own advance; a step whose state the
    // host may read ends with the k_reset_list flush, which resets them at
    // once and clears their flags.
    uint32_t* reset_list;  // [n]
    uint32_t* reset_count;  // [2]
    uint8_t* reset_pending;  // [n]
    uint32_t phase;  // 0 / 1, alternating over the steps of a collected rollout
};

}  // namespace mdn
