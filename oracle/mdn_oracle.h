/*
 * TEST INFRASTRUCTURE ONLY. CPU restatement of the metal-drone-nav rollout/PPO
 * path, used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg
 * as the checker. The product never links, loads or calls it.
 *
 * Parity pin: tests/test_oracle_pin.py checks every function here against the
 * reference's own CPU path compiled unmodified (oracle/_ref, built from
 * cpu_reference.hpp and the shared headers) and against the reference golden
 * fixtures (assets/raptor.bin official RAPTOR sequence, assets/physics.bin L2F
 * fixtures, the analytic ray cases of main.mm:108-123, the GAE/normalisation/
 * Adam cases of main.mm:286-375 and ppo.hpp:204-267).
 */
#ifndef MDN_ORACLE_H
#define MDN_ORACLE_H
#include <stddef.h>
#include <stdint.h>
#include "mdn.h"

#ifdef __cplusplus
extern "C" {
#endif

/* world.hpp */
float o_wray_sphere(const float p[3], const float d[3], const float c[3], float r);
float o_wray_box(const float p[3], const float d[3], const float c[3], const float e[3]);
float o_wray_cylinder(const float p[3], const float d[3], const float c[3], float r, float h);
void o_wc(const mdn_obstacle* o, float t, float out[3]);
/* room = {xmin,ymin,zmin,xmax,ymax,zmax}; NULL = reference room. */
float o_wray(const mdn_world* w, const float* room, const float p[3], const float d[3], float t);
float o_wclearance(const mdn_world* w, const float* room, const float p[3], float t, int32_t* argmin);
void o_wgenerate(mdn_world* w, uint32_t seed, uint32_t family, float distance);
uint32_t o_wtraining_family(uint32_t family, uint32_t* rng);
/* family 18 (mixed capability): the generator family of global env `gid` */
uint32_t o_mixed_lane_family(uint32_t gid);
void o_set_argument_order(int right_to_left);
uint32_t o_wrng(uint32_t* s);
float o_wurand(uint32_t* s);
/* sensor_profile.hpp */
void o_pixel_ray(float tan_h, float tan_v, uint32_t pixel, float out[3]);
/* guidance.hpp */
void o_nav_guidance(const float* cur, const float* prev, const float* goal, float distance, const float* vel,
                    float sensor_dt, float tan_v, float* hint);
void o_nav_guidance_memory(const float* cur, const float* prev, const float* goal, float distance, const float* vel,
                           float sensor_dt, float tan_v, const float* range_ring, const float* pose_ring,
                           const float* current_pose, uint32_t latest_frame, uint32_t valid_frames, float* hint,
                           float latest_capture_age);
/* physics.hpp / raptor.hpp */
void o_physics_step(const mdn_physics_state* s, const float action[4], const float wind[3],
                    const mdn_physics_params* p, mdn_physics_state* out);
void o_physics_default(mdn_physics_params* p);
void o_raptor_forward(const mdn_raptor_weights* w, const float obs[22], float hidden[16], float action[4]);
/* ppo.hpp */
void o_compute_gae(uint32_t horizon, uint32_t envs, const float* r, const float* v, const float* nv,
                   const uint8_t* term, const uint8_t* trunc, float gamma, float lambda, float* adv, float* ret);
void o_normalize_advantages(float* adv, size_t count);
void o_sample_loss_and_grad(const float* action, const float* mean, const float* log_std, float old_logp,
                            float value, float adv, float ret, float batch, float clip, float vcoef, float ecoef,
                            float* d_mean, float* d_log_std, float* d_value, float losses[4]);
void o_adam_update(float* params, const float* grad, float* m, float* v, size_t count, float b1corr, float b2corr,
                   float lr);
float o_pow_correction(float beta, uint64_t step);

/* Whole-simulator oracle with reference layouts (buffer ids = MDN_BUF_*, plus
 * 100..103 for the Adam moments). */
typedef struct o_sim o_sim;
o_sim* o_sim_create(const mdn_sim_config* cfg, uint32_t horizon, const mdn_raptor_weights* raptor,
                    const mdn_physics_params* physics, const float* room);
/* A rank's shard: local env i is global env env_base + i (seeds, clean-env parity). */
o_sim* o_sim_create_shard(const mdn_sim_config* cfg, uint32_t horizon, const mdn_raptor_weights* raptor,
                          const mdn_physics_params* physics, const float* room, uint32_t env_base);
void o_sim_rows_grad(o_sim* s, const uint32_t* rows, uint32_t count, float batch, float* grad);
void o_sim_set_task_control(o_sim* s, const mdn_task_control* ctl);
void o_sim_set_challenge_bank(o_sim* s, const mdn_world* worlds, const mdn_bank_control* ctl);
void o_sim_set_runtime(o_sim* s, const mdn_runtime_config* rt);
/* NAV_DELAY_REHEARSAL (sim.metal:14-24) as a switch; off after create. */
void o_sim_set_delay_rehearsal(o_sim* s, int enabled);
int o_physics_sample_domain(const mdn_physics_params* nominal, uint32_t* rng, float amplitude,
                            const mdn_domain_range* r, mdn_physics_params* varied, float* sample_out);
uint32_t o_domain_episode_seed(const mdn_runtime_config* rt, uint32_t cfg_seed, uint32_t env, uint32_t episode);
/* navigation_tasks.hpp */
uint32_t o_generate_task(mdn_world* w, mdn_task_state* task, uint32_t* rng, const mdn_task_config* c, const float* room);
void o_task_apply_start(const mdn_task_state* task, mdn_physics_state* s);
void o_task_step(mdn_task_state* task, const mdn_task_config* c, const float* pos, const float* vel, const float* cmd,
                 uint32_t contact, uint32_t forced_timeout, void* out);
float o_task_segment_clearance(const mdn_world* w, const float* room, const float a[3], const float b[3]);
void o_sim_destroy(o_sim* s);
void* o_sim_buffer(o_sim* s, int id, size_t* bytes);
void o_sim_reset(o_sim* s);
void o_sim_set_config(o_sim* s, const mdn_sim_config* cfg);
void o_sim_observe(o_sim* s, uint32_t tick);
void o_sim_act(o_sim* s, uint32_t tick);
void o_sim_advance(o_sim* s, uint32_t tick);
void o_sim_step(o_sim* s, uint32_t tick);
void o_sim_gae_normalize(o_sim* s, int normalize);
/* sim_critic_obs (sim.metal:159-180) of `count` environments from their state:
 * dim = 32, or 64 with the control-state inputs of the delay-training build. */
void o_critic_obs_rows(const o_sim* s, const mdn_physics_state* states, const mdn_world* worlds,
                       const mdn_sim_run* runs, uint32_t count, uint32_t dim, float* out);
/* One PPO rollout update with the given chunk order (epochs x chunks) and the
 * per-update Adam bias corrections; out[4] = policy, value, entropy, ratio means.
 * grad_norms (optional) receives actor/critic pre-clip norms per update. */
void o_sim_train_rollout(o_sim* s, uint32_t minibatch, uint32_t epochs, const uint32_t* order, uint32_t chunks,
                         const float* b1corr, const float* b2corr, float* out, float* grad_norms);
uint32_t o_actor_param_count(void);
uint32_t o_critic_param_count(void);
/* wide actor (ppo.hpp:65-80 at hidden width `hidden`) */
uint32_t o_wide_param_count(uint32_t hidden);
void o_wide_init(uint32_t hidden, float* actor, float* critic);
void o_wide_actor_forward(uint32_t hidden, const float* obs, const float* actor, float* hid, float* mean);
void o_set_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
