/*
 * TEST INFRASTRUCTURE ONLY - never linked into, or called by, the product.
 *
 * Step-level C entry points over the reference's own CPU path, compiled from
 * the unmodified reference headers where they lie (cpu_reference.hpp,
 * world.hpp, sensor_profile.hpp, guidance.hpp, raptor.hpp, physics.hpp,
 * ppo.hpp) by oracle/Makefile into oracle/_ref/libref_oracle.so. The tests use
 * it to pin the C restatement in oracle/mdn_oracle.c, and bench.py's reference
 * arm times it as the CPU baseline.
 *
 * cpu_reference::Trainer keeps its step functions private
 * (cpu_reference.hpp:210). They are reached by compiling the header with
 * `private` mapped to `public` after every standard header it needs has been
 * included, so no reference file is edited or copied.
 *
 * Where the reference's loop body is inline in collect_rollout
 * (cpu_reference.hpp:396-435) the act/advance halves below call the same
 * Trainer members and header functions in the same order, so a single policy
 * step can be run with teacher forcing.
 */
#include <algorithm>
#include <array>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <iostream>
#include <numeric>
#include <random>
#include <string>
#include <vector>
#include <omp.h>
#include <math.h>  // ::isfinite for physics_domain.hpp, as Apple libc++ provides it

#include "mdn.h"

// The reference header expects these two types to be declared by its includer
// (main.mm:454-465); the C layouts in mdn.h are byte-identical.
using SimConfig = mdn_sim_config;
using SimRun = mdn_sim_run;
static_assert(sizeof(SimConfig) == 84 && sizeof(SimRun) == 184, "sim layout");

#define private public
#include "cpu_reference.hpp"
#undef private
#include "navigation_runtime.hpp"
#include "navigation_tasks.hpp"
#include "vehicle_geometry.hpp"
static_assert(sizeof(VGResult) == sizeof(mdn_contact_audit), "contact audit layout");
static_assert(sizeof(NavigationTaskConfig) == sizeof(mdn_task_config), "task config layout");
static_assert(sizeof(NavigationTaskState) == sizeof(mdn_task_state), "task state layout");

using Trainer = cpu_reference::Trainer;
static_assert(sizeof(RLPhysicsState) == sizeof(mdn_physics_state), "state layout");
static_assert(sizeof(RLPhysicsParams) == sizeof(mdn_physics_params), "params layout");
static_assert(sizeof(WWorld) == sizeof(mdn_world), "world layout");
static_assert(sizeof(RaptorWeights) == sizeof(mdn_raptor_weights), "raptor layout");

extern "C" {

/* vg_world_contact (vehicle_geometry.hpp:311-376): the mechanical contact audit of one pose. */
void ref_vg_world_contact(const float* position, const float* orientation_wxyz, const mdn_world* world, float time,
                          float margin, mdn_contact_audit* out) {
    VGResult r{};
    vg_world_contact(position, orientation_wxyz, *reinterpret_cast<const WWorld*>(world), time, margin, r);
    std::memcpy(out, &r, sizeof(r));
}

/* rl_physics_sample_domain (physics_domain.hpp:100-157): the varied plant and
 * the 17 floats of RLPhysicsDomainSample; rl_physics_domain_stress_range. */
int ref_physics_sample_domain(const mdn_physics_params* nominal, uint32_t* rng, float amplitude,
                              const mdn_domain_range* range, mdn_physics_params* varied, float* sample) {
    RLPhysicsParams n, v{};
    std::memcpy(&n, nominal, sizeof(n));
    RLPhysicsDomainRange r;
    std::memcpy(&r, range, sizeof(r));
    RLPhysicsDomainSample out{};
    const bool ok = rl_physics_sample_domain(n, *rng, amplitude, r, v, out);
    std::memcpy(varied, &v, sizeof(v));
    std::memcpy(sample, &out, sizeof(out));
    return ok ? 1 : 0;
}
void ref_domain_stress_range(mdn_domain_range* out) {
    const RLPhysicsDomainRange r = rl_physics_domain_stress_range();
    std::memcpy(out, &r, sizeof(r));
}
static_assert(sizeof(RLPhysicsDomainRange) == sizeof(mdn_domain_range), "domain range layout");
static_assert(sizeof(NavigationRuntimeConfig) == sizeof(mdn_runtime_config), "runtime config layout");
static_assert(sizeof(RLPhysicsDomainSample) == 17 * sizeof(float), "domain sample layout");

/* ---------------- whole-trainer handle ---------------- */
void* ref_trainer_create(const mdn_sim_config* cfg, uint32_t horizon, const void* raptor, const void* physics) {
    RaptorWeights w;
    std::memcpy(&w, raptor, sizeof(w));
    RLPhysicsParams p;
    std::memcpy(&p, physics, sizeof(p));
    return new Trainer(*cfg, horizon, w, p);
}
void ref_trainer_destroy(void* h) { delete static_cast<Trainer*>(h); }
void ref_set_threads(int n) { omp_set_num_threads(n > 0 ? n : 1); }
int ref_max_threads(void) { return omp_get_max_threads(); }

/* Host views of the trainer's buffers. ids follow MDN_BUF_*; extra ids:
 * 100..103 actor m, actor v, critic m, critic v. */
void* ref_trainer_buffer(void* handle, int id, size_t* bytes) {
    Trainer& t = *static_cast<Trainer*>(handle);
    auto view = [&](auto& vec) -> void* {
        *bytes = vec.size() * sizeof(vec[0]);
        return (void*)vec.data();
    };
    switch (id) {
        case MDN_BUF_STATES: return view(t.states);
        case MDN_BUF_RUNS: return view(t.runs);
        case MDN_BUF_WORLDS: return view(t.worlds);
        case MDN_BUF_SENSORS: return view(t.sensors);
        case MDN_BUF_POSES: return view(t.poses);
        case MDN_BUF_COMMANDS: return view(t.commands);
        case MDN_BUF_ACTOR: return view(t.actor.values);
        case MDN_BUF_CRITIC: return view(t.critic.values);
        case MDN_BUF_OBS: return view(t.observations);
        case MDN_BUF_CO: return view(t.critic_observations);
        case MDN_BUF_ACTIONS: return view(t.actions);
        case MDN_BUF_LOGP: return view(t.old_logp);
        case MDN_BUF_VALUES: return view(t.values);
        case MDN_BUF_REWARDS: return view(t.rewards);
        case MDN_BUF_NEXT_VALUES: return view(t.next_values);
        case MDN_BUF_TERMINATED: return view(t.terminated);
        case MDN_BUF_TRUNCATED: return view(t.truncated);
        case MDN_BUF_ADVANTAGES: return view(t.advantages);
        case MDN_BUF_RETURNS: return view(t.returns);
        case 100: return view(t.actor_m);
        case 101: return view(t.actor_v);
        case 102: return view(t.critic_m);
        case 103: return view(t.critic_v);
        default: *bytes = 0; return nullptr;
    }
}
uint64_t* ref_trainer_optimizer_step(void* h) { return &static_cast<Trainer*>(h)->optimizer_step; }
void ref_trainer_reset_env(void* h, uint32_t n, int first) { static_cast<Trainer*>(h)->reset_env(n, first != 0); }

/* Depth + observation for every environment at tick t (cpu_reference.hpp:399). */
void ref_step_observe(void* handle, uint32_t t) {
    Trainer& tr = *static_cast<Trainer*>(handle);
    cpu_reference::parallel_for(tr.cfg.n, [&](size_t n) { tr.collect_depth_and_obs(t, uint32_t(n)); });
}

/* Batched actor/critic forward and the serial sampling loop (cpu_reference.hpp:400-429). */
void ref_step_act(void* handle, uint32_t t) {
    Trainer& tr = *static_cast<Trainer*>(handle);
    const size_t envs = tr.cfg.n;
    const float* obs = tr.observations.data() + size_t(t) * envs * cpu_reference::actor_dim;
    const float* co = tr.critic_observations.data() + size_t(t) * envs * cpu_reference::critic_dim;
    tr.actor_forward_batch(obs, uint32_t(envs), tr.current_actor_hidden.data(), tr.current_actor_means.data());
    tr.critic_forward_batch(co, uint32_t(envs), tr.current_critic_hidden.data(), tr.current_critic_values.data());
    constexpr uint32_t A = cpu_reference::action_dim, F = cpu_reference::sensor_frames;
    for (uint32_t n = 0; n < tr.cfg.n; n++) {
        const size_t row = size_t(t) * envs + n;
        tr.values[row] = tr.current_critic_values[n];
        uint32_t rng = tr.runs[n].rng;
        for (uint32_t a = 0; a < A; a++) {
            const float action = tr.current_actor_means[n * A + a] +
                std::exp(tr.actor.values[fixed_ppo::actor_log_std_offset + a]) * cpu_reference::sim_normal(rng);
            tr.actions[row * A + a] = action;
            tr.commands[(size_t(n) * F + tr.runs[n].steps % F) * A + a] = std::tanh(action);
        }
        tr.old_logp[row] = fixed_ppo::gaussian_log_prob(tr.actions.data() + row * A, tr.current_actor_means.data() + n * A,
                                                        tr.actor.values.data() + fixed_ppo::actor_log_std_offset);
        tr.runs[n].rng = rng;
        const uint32_t delay = tr.effective_command_delay(n);
        const uint32_t applied = tr.runs[n].steps > delay ? tr.runs[n].steps - delay : 0;
        for (uint32_t a = 0; a < A; a++)
            tr.runs[n].previous_nav[a] = tr.runs[n].steps < delay ? 0.0f : tr.commands[(size_t(n) * F + applied % F) * A + a];
        float r[9];
        cpu_reference::rotation(tr.states[n].orientation_wxyz, r);
        float v[3] = {tr.runs[n].previous_nav[0] * tr.cfg.speed, tr.runs[n].previous_nav[1] * tr.cfg.speed,
                      tr.runs[n].previous_nav[2] * tr.cfg.speed * (tr.cfg.velocity_contract == 0 ? 0.5f : 1.0f)};
        if (tr.cfg.velocity_contract == 1) {
            const float scale = std::min(1.0f, tr.cfg.speed / std::max(wl(wv(v[0], v[1], v[2])), 1e-8f));
            for (float& c : v) c *= scale;
        }
        for (int j = 0; j < 3; j++) tr.runs[n].desired_velocity[j] = r[j * 3] * v[0] + r[j * 3 + 1] * v[1] + r[j * 3 + 2] * v[2];
        tr.runs[n].yaw += tr.runs[n].previous_nav[3] * tr.physics.dt * tr.cfg.substeps * 0.5f;
    }
}

/* Advance, next value, resets (cpu_reference.hpp:430-433). */
void ref_step_advance(void* handle, uint32_t t) {
    Trainer& tr = *static_cast<Trainer*>(handle);
    const size_t envs = tr.cfg.n;
    cpu_reference::parallel_for(envs, [&](size_t n) { tr.advance_env(t, uint32_t(n)); });
    tr.critic_forward_batch(tr.next_critic_observations.data(), uint32_t(envs), tr.next_critic_hidden.data(),
                            tr.next_critic_values.data());
    for (uint32_t n = 0; n < tr.cfg.n; n++) tr.next_values[size_t(t) * envs + n] = tr.next_critic_values[n];
    cpu_reference::parallel_for(envs, [&](size_t n) {
        if (tr.reset_after_bootstrap[n]) tr.reset_env(uint32_t(n), false);
    });
}

void ref_step(void* h, uint32_t t) {
    ref_step_observe(h, t);
    ref_step_act(h, t);
    ref_step_advance(h, t);
}

/* The reference's own loops, unmodified. */
void ref_collect_rollout(void* h) { static_cast<Trainer*>(h)->collect_rollout(); }
void ref_gae_normalize(void* handle) {
    Trainer& tr = *static_cast<Trainer*>(handle);
    fixed_ppo::compute_gae(tr.horizon, tr.cfg.n, tr.rewards.data(), tr.values.data(), tr.next_values.data(),
                           tr.terminated.data(), tr.truncated.data(), cpu_reference::gamma, cpu_reference::gae_lambda,
                           tr.advantages.data(), tr.returns.data());
    fixed_ppo::normalize_advantages(tr.advantages.data(), tr.advantages.size());
}
void ref_gae_only(void* handle) {
    Trainer& tr = *static_cast<Trainer*>(handle);
    fixed_ppo::compute_gae(tr.horizon, tr.cfg.n, tr.rewards.data(), tr.values.data(), tr.next_values.data(),
                           tr.terminated.data(), tr.truncated.data(), cpu_reference::gamma, cpu_reference::gae_lambda,
                           tr.advantages.data(), tr.returns.data());
}
void ref_train_rollout(void* h, uint32_t rollout, float out[4]) {
    static_cast<Trainer*>(h)->train_rollout(rollout, out[0], out[1], out[2], out[3]);
}
/* Trainer::run (cpu_reference.hpp:163-185). out: wall_s, updates, episodes,
 * successes, collisions, timeouts, final_progress, total_path, total_elapsed,
 * success_time, policy, value, entropy, ratio. */
void ref_run(void* h, uint32_t rollouts, double out[14]) {
    const auto m = static_cast<Trainer*>(h)->run(rollouts);
    const double v[14] = {m.wall_seconds, double(m.updates), double(m.episodes), double(m.successes),
                          double(m.collisions), double(m.timeouts), m.final_progress, m.total_path,
                          m.total_elapsed, m.success_time, m.policy_loss, m.value_loss, m.entropy_loss, m.ratio};
    std::memcpy(out, v, sizeof(v));
}
int ref_validate_batched_forward(void* h) { return static_cast<Trainer*>(h)->validate_batched_forward() ? 1 : 0; }

/* Minibatch chunk order of one rollout: epochs x chunk-starts, as
 * train_rollout / PPOTrainer::rollout_update draw it (cpu_reference.hpp:571-578,
 * main.mm:1331-1337). */
void ref_minibatch_order(uint32_t rows, uint32_t minibatch, uint32_t rollout, uint32_t epochs, uint32_t* out) {
    std::vector<uint32_t> starts;
    for (uint32_t i = 0; i < rows; i += minibatch) starts.push_back(i);
    std::mt19937 rng(0x9e3779b9u + rollout * 0x85ebca6bu);
    std::shuffle(starts.begin(), starts.end(), rng);
    for (uint32_t e = 0; e < epochs; e++) {
        if (e == 1) std::shuffle(starts.begin(), starts.end(), rng);
        std::memcpy(out + size_t(e) * starts.size(), starts.data(), starts.size() * sizeof(uint32_t));
    }
}

/* ---------------- operator-level entry points ---------------- */
int ref_raptor_load(const char* path, void* weights) { return raptor_load_weights(path, (RaptorWeights*)weights) ? 1 : 0; }
void ref_raptor_forward(const void* w, const float obs[22], float hidden[16], float action[4]) {
    raptor_forward(*(const RaptorWeights*)w, obs, hidden, action);
}
void ref_physics_step(const void* state, const float action[4], const float wind[3], const void* params, void* out) {
    rl_physics_step(*(const RLPhysicsState*)state, action, wind, *(const RLPhysicsParams*)params, *(RLPhysicsState*)out);
}
void ref_physics_default(void* out) {
    const RLPhysicsParams p = rl_physics_crazyflie_default();
    std::memcpy(out, &p, sizeof(p));
}
float ref_wray(const void* world, const float p[3], const float d[3], float time) {
    return wray(*(const WWorld*)world, wv(p[0], p[1], p[2]), wv(d[0], d[1], d[2]), time);
}
float ref_wray_box(const float p[3], const float d[3], const float c[3], const float e[3]) {
    return wray_box(wv(p[0], p[1], p[2]), wv(d[0], d[1], d[2]), wv(c[0], c[1], c[2]), wv(e[0], e[1], e[2]));
}
float ref_wray_sphere(const float p[3], const float d[3], const float c[3], float r) {
    return wray_sphere(wv(p[0], p[1], p[2]), wv(d[0], d[1], d[2]), wv(c[0], c[1], c[2]), r);
}
float ref_wray_cylinder(const float p[3], const float d[3], const float c[3], float r, float h) {
    return wray_cylinder(wv(p[0], p[1], p[2]), wv(d[0], d[1], d[2]), wv(c[0], c[1], c[2]), r, h);
}
float ref_wclearance(const void* world, const float p[3], float time) {
    return wclearance(*(const WWorld*)world, wv(p[0], p[1], p[2]), time);
}
void ref_wc(const void* obstacle, float time, float out[3]) {
    const WVec c = wc(*(const WObstacle*)obstacle, time);
    out[0] = c.x; out[1] = c.y; out[2] = c.z;
}
void ref_wgenerate(void* world, uint32_t seed, uint32_t family, float distance) {
    wgenerate(*(WWorld*)world, seed, family, distance);
}
uint32_t ref_wtraining_family(uint32_t family, uint32_t* rng) { return wtraining_family(family, *rng); }
void ref_pixel_ray(float tan_h, float tan_v, uint32_t pixel, float out[3]) {
    const WVec r = nav_sensor_pixel_ray(tan_h, tan_v, pixel);
    out[0] = r.x; out[1] = r.y; out[2] = r.z;
}
void ref_nav_guidance(const float* cur, const float* prev, const float* goal, float distance, const float* vel,
                      float sensor_dt, float tan_v, float* hint) {
    nav_guidance(cur, prev, goal, distance, vel, sensor_dt, tan_v, hint);
}
void ref_nav_guidance_memory(const float* cur, const float* prev, const float* goal, float distance, const float* vel,
                             float sensor_dt, float tan_v, const float* range_ring, const float* pose_ring,
                             const float* current_pose, uint32_t latest_frame, uint32_t valid_frames, float* hint,
                             float latest_capture_age) {
    nav_guidance_memory(cur, prev, goal, distance, vel, sensor_dt, tan_v, range_ring, pose_ring, current_pose,
                        latest_frame, valid_frames, hint, nullptr, latest_capture_age);
}
void ref_compute_gae(uint32_t horizon, uint32_t envs, const float* r, const float* v, const float* nv, const uint8_t* term,
                     const uint8_t* trunc, float gamma, float lambda, float* adv, float* ret) {
    fixed_ppo::compute_gae(horizon, envs, r, v, nv, term, trunc, gamma, lambda, adv, ret);
}
void ref_normalize_advantages(float* adv, size_t count) { fixed_ppo::normalize_advantages(adv, count); }
void ref_sample_loss_and_grad(const float* action, const float* mean, const float* log_std, float old_logp, float value,
                              float adv, float ret, float batch, float clip, float vcoef, float ecoef, float* d_mean,
                              float* d_log_std, float* d_value, float losses[4]) {
    const auto l = fixed_ppo::sample_loss_and_grad(action, mean, log_std, old_logp, 0.0f, value, adv, ret, batch, clip,
                                                   vcoef, ecoef, d_mean, d_log_std, d_value);
    losses[0] = l.policy; losses[1] = l.value; losses[2] = l.entropy; losses[3] = l.ratio;
}
void ref_actor_forward(const float* obs, const float* params, float* hidden, float* mean) {
    fixed_ppo::ActorParams p;
    std::memcpy(p.values.data(), params, sizeof(p.values));
    fixed_ppo::actor_forward(obs, p, hidden, mean);
}
float ref_critic_forward(const float* obs, const float* params, float* hidden) {
    fixed_ppo::CriticParams p;
    std::memcpy(p.values.data(), params, sizeof(p.values));
    return fixed_ppo::critic_forward(obs, p, hidden);
}
void ref_adam_update(float* params, const float* grad, float* m, float* v, size_t count, uint64_t step, float lr) {
    fixed_ppo::adam_update(params, grad, m, v, count, step, lr, 0.9f, 0.999f, 1.0e-8f, 0.0f);
}
int ref_run_cpu_self_tests(void) { return fixed_ppo::run_cpu_self_tests() ? 1 : 0; }

/* ---------------- goal-arrival task contract (navigation_tasks.hpp) ---------------- */
int ref_task_default_config(uint32_t stage, uint32_t family, float difficulty, void* cfg) {
    return navigation_task_default_config(*(NavigationTaskConfig*)cfg, stage, family, difficulty) ? 1 : 0;
}
uint32_t ref_generate_task(void* world, void* task, uint32_t* rng, const void* cfg) {
    return navigation_generate_task(*(WWorld*)world, *(NavigationTaskState*)task, *rng, *(const NavigationTaskConfig*)cfg);
}
void ref_task_apply_start(const void* task, void* state) {
    navigation_task_apply_start(*(const NavigationTaskState*)task, *(RLPhysicsState*)state);
}
/* out: reward, goal_distance, actual_speed, then 5 uint flags (waypoint, stable, collision, timeout, done) */
void ref_task_step(void* task, const void* cfg, const float* pos, const float* vel, const float* cmd, uint32_t contact,
                   uint32_t timeout, void* out) {
    const NavigationTaskStep r = navigation_task_step(*(NavigationTaskState*)task, *(const NavigationTaskConfig*)cfg,
                                                      pos, vel, cmd, contact, timeout);
    std::memcpy(out, &r, sizeof(r));
}
float ref_task_segment_clearance(const void* world, const float a[3], const float b[3]) {
    return navigation_task_segment_clearance(*(const WWorld*)world, wv(a[0], a[1], a[2]), wv(b[0], b[1], b[2]));
}
uint32_t ref_actor_param_count(void) { return uint32_t(fixed_ppo::actor_param_count); }
uint32_t ref_critic_param_count(void) { return uint32_t(fixed_ppo::critic_param_count); }

}  // extern "C"
