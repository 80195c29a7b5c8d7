/*
 * mdn.h - C-ABI of the B200-native metal-drone-nav rollout/PPO hot path.
 *
 * The reference exposes this path as an Objective-C++ class API:
 *   Metal   (main.mm:44-72)    device, buffers, dispatch, finish()
 *   Sim     (main.mm:516-603)  batched environment: reset/set_config/collect/report
 *   PPOTrainer (main.mm:1110-1476) GAE, clipped PPO, clip+Adam, checkpoints
 * consumed by navigation_training.hpp:7-170 and train_navigation (main.mm:1805-1862).
 * Each entry point below replaces one method of those classes; the comment names
 * the reference member it stands in for. Plain pointers and sizes only: no CUDA,
 * torch or C++ types cross this boundary.
 *
 * Conventions
 *  - Every call returns an int status (MDN_OK == 0). On failure a message is kept
 *    per thread and returned by mdn_last_error().
 *  - Host memory passed in is owned by the caller; device memory is owned by the
 *    library (mdn_sim owns every per-environment buffer, mdn_ppo its optimizer
 *    state), mirroring Sim/PPOTrainer ownership in main.mm.
 *  - One CUDA stream per mdn_sim. Calls are stream-ordered; mdn_sync() is the
 *    reference's Metal::finish (commit + wait + error check).
 *  - Handles are not thread-safe; one host thread drives one handle.
 */
#ifndef MDN_H
#define MDN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MDN_ABI_VERSION 1u

/* ---- status codes ------------------------------------------------------ */
enum {
    MDN_OK = 0,
    MDN_ERR_INVALID = 1,   /* bad argument or unsupported configuration      */
    MDN_ERR_CUDA = 2,      /* CUDA runtime error (message has the cause)      */
    MDN_ERR_NOMEM = 3,     /* device or host allocation failed                */
    MDN_ERR_TIMEOUT = 4,   /* a bounded device or host wait gave up           */
    MDN_ERR_IO = 5,        /* file read/write failed                          */
    MDN_ERR_MISMATCH = 6,  /* checkpoint/config mismatch on resume            */
    MDN_ERR_NCCL = 7,      /* NCCL communicator error                         */
    MDN_ERR_STATE = 8      /* call out of order (e.g. update before collect)  */
};

/* ---- byte-identical POD layouts (the on-disk and device ABI) ----------- */

/* RLPhysicsState, physics.hpp:12-18 (68 bytes). */
typedef struct mdn_physics_state {
    float position[3];
    float orientation_wxyz[4];
    float linear_velocity[3];
    float angular_velocity_body[3];
    float rpm[4];
} mdn_physics_state;

/* RLPhysicsParams, physics.hpp:20-38 (352 bytes). */
typedef struct mdn_physics_params {
    float rotor_positions[12];
    float rotor_thrust_directions[12];
    float rotor_torque_directions[12];
    float rotor_thrust_coefficients[12];
    float rotor_torque_constants[4];
    float rotor_time_constants_rising[4];
    float rotor_time_constants_falling[4];
    float inertia[9];
    float inertia_inverse[9];
    float gravity_world[3];
    float mass;
    float action_min;
    float action_max;
    float dt;
    float position_limit;
    float velocity_limit;
    float angular_velocity_limit;
} mdn_physics_params;

/* WObstacle / WWorld, world.hpp:28-29 (40 and 676 bytes). kind: 0 box,
 * 1 sphere, 2 vertical cylinder, 3 bounded moving sphere. */
typedef struct mdn_obstacle {
    uint32_t kind;
    float center[3], size[3], velocity[3];
} mdn_obstacle;
typedef struct mdn_world {
    mdn_obstacle obstacles[16];
    uint32_t count, seed, family;
    float goal[3], wind[3];
} mdn_world;

/* SimRun, sim.metal:2-8 / main.mm:454-459 (184 bytes). */
typedef struct mdn_sim_run {
    float hidden[16], motors[4], previous_nav[4], desired_velocity[3], yaw;
    uint32_t rng, steps;
    float path, elapsed, peak_speed, min_clearance, initial_distance;
    uint32_t successes, collisions, timeouts, episodes;
    float success_time, total_path, total_elapsed, final_progress, reference_position[3];
} mdn_sim_run;

/* SimConfig, main.mm:461-464 (84 bytes). Defaults in mdn_sim_config_default. */
typedef struct mdn_sim_config {
    uint32_t n, tick, mode, family, substeps, sensor_period, sensor_delay, command_delay, max_steps, seed, eval;
    float speed, distance, wind, depth_noise, dropout, risk_coef, entropy_coef, learning_rate;
    uint32_t velocity_contract, geometry_memory;
} mdn_sim_config;

/* RaptorWeights, raptor.hpp:11-21 (2,084 floats, 8,336 bytes). */
typedef struct mdn_raptor_weights {
    float input_weights[16 * 22];
    float input_bias[16];
    float gru_input_weights[48 * 16];
    float gru_hidden_weights[48 * 16];
    float gru_input_bias[48];
    float gru_hidden_bias[48];
    float initial_hidden_state[16];
    float output_weights[4 * 16];
    float output_bias[4];
} mdn_raptor_weights;

/* Shape of one rollout that the reference fixes at compile time or hard-codes.
 * Zero-initialised fields take the reference value (listed). */
typedef struct mdn_rollout_shape {
    uint32_t actor_obs_dim;     /* 184: 2x80 pooled depth + 21 context + 3 hint (ppo.hpp:26-34) */
    uint32_t critic_obs_dim;    /* 32 (ppo.hpp:14-16), or 64: the control-state critic of the
                                   delay-training build (FIXED_PPO_CRITIC_OBS_DIM=64 with
                                   NAV_CRITIC_CONTROL_STATE, sim.metal:166-180): inputs
                                   32..63 are the RAPTOR hidden state, rotor speeds, yaw
                                   error sine/cosine, last command, desired velocity / 2,
                                   goal-closing speed / 4, goal distance / 10, speed / 4.
                                   64 selects the layered networks (below), here a 64 x 64 x 1
                                   tanh critic unless the layered fields say otherwise     */
    uint32_t actor_hidden;      /* 64 (ppo.hpp:17-19); or a multiple of 256 up to 8192: the
                                   one-hidden-layer tanh actor at that width (5120 = the
                                   967,688-parameter actor of FIXED_PPO_HIDDEN_DIM=5120,
                                   navigation_wide_deployment.hpp:54-66), evaluated and
                                   trained on the tensor cores (TF32 products, fp32
                                   accumulation)                                          */
    uint32_t critic_hidden;     /* 64 (ppo.hpp:41-45)                                        */
    uint32_t flags;             /* MDN_SHAPE_* bits                                          */
    float room_min[3];          /* wray/wclearance room, world.hpp:73-74,85: (-2,-5,0)       */
    float room_max[3];          /*                                        (14, 5,5)          */
    /* Layered networks (no counterpart in the reference, whose actor and
     * critic have one hidden layer of tanh units): hidden layers of the
     * actor / critic (0 = 1) and their activation (MDN_ACT_*, 0 = tanh).
     * Any of them, or a critic other than 64 units, selects the layered
     * path for both networks: dense fp32 kernels, layer by layer, with the
     * parameters flat per layer (W [out][in] then b), the actor's log_std[4]
     * last; one tanh layer gives the reference's layout. actor_hidden and
     * critic_hidden are then 1..2048 (0 = 64). */
    uint32_t actor_layers, critic_layers;
    uint32_t actor_activation, critic_activation;
} mdn_rollout_shape;
#define MDN_SHAPE_CUSTOM_ROOM 1u /* use room_min/room_max instead of the reference room */
#define MDN_ACT_TANH 0u
#define MDN_ACT_GELU 1u /* 0.5 z (1 + erf(z / sqrt 2)) */

/* PpoCheckpointHeader prefix layout, main.mm:984-991 (136 bytes). */
typedef struct mdn_checkpoint_header {
    char magic[8];
    uint32_t version, actor_count, critic_count, horizon, n, family;
    uint32_t base_seed, completed_rollouts;
    uint64_t optimizer_step;
    mdn_sim_config config;
} mdn_checkpoint_header;

/* NavigationTaskConfig (navigation_tasks.hpp:61-89, 144 bytes): goal-arrival
 * task curriculum. NavigationTaskControl (:91-94, 148 bytes). */
typedef struct mdn_task_config {
    uint32_t family, stage, objective, require_detour, max_generation_attempts, max_nav_steps;
    float scene_distance_m, difficulty, goal_distance_min_m, goal_distance_max_m;
    float minimum_endpoint_clearance_m, minimum_witness_clearance_m, goal_radius_m, stable_speed_mps;
    float stable_hold_s, nav_period_s, initial_speed_min_mps, initial_speed_max_mps;
    float progress_reward_per_m, time_cost_per_s, contact_penalty, stable_arrival_bonus, command_smoothness_weight;
    float start_min_xyz[3], start_max_xyz[3], goal_min_xyz[3], goal_max_xyz[3];
    uint32_t generation_version;
} mdn_task_config;
typedef struct mdn_task_control {
    uint32_t enabled;
    mdn_task_config config;
} mdn_task_control;

/* RLPhysicsDomainRange (physics_domain.hpp:17-24) and NavigationRuntimeConfig
 * (navigation_runtime.hpp:9-14): per-episode plant stress variation. */
typedef struct mdn_domain_range {
    float mass_scale_min, mass_scale_max;
    float inertia_axis_scale_min, inertia_axis_scale_max;
    float thrust_gain_min, thrust_gain_max;
    float rising_lag_scale_min, rising_lag_scale_max;
    float falling_lag_scale_min, falling_lag_scale_max;
    float minimum_thrust_to_weight;
} mdn_domain_range;
typedef struct mdn_runtime_config {
    uint32_t enabled;
    float domain_amplitude;  /* 0..1; 0 keeps the nominal plant */
    uint32_t domain_seed;
    mdn_domain_range domain_range;
} mdn_runtime_config;

/* NavigationTaskState (navigation_tasks.hpp:147-177, 192 bytes), one per env. */
typedef struct mdn_task_state {
    uint32_t generation_status, valid, generation_attempts, family, stage, objective, max_nav_steps, step_count;
    uint32_t stable_ticks, was_inside_goal, waypoint_event_latched, terminal;
    float start_position[3], start_yaw_rad, start_velocity_world[3], goal_position[3];
    float initial_distance_m, previous_distance_m, difficulty, start_clearance_m, goal_clearance_m;
    float direct_segment_clearance_m, witness_min_clearance_m, witness_length_m, stable_time_s;
    float last_executed_world_command[4];
    uint32_t witness_point_count;
    float witness_points[4][3];
} mdn_task_state;

/* VGResult (vehicle_geometry.hpp:43-48, 16 bytes): one mechanical contact
 * audit of the declared vehicle geometry against the room and the obstacles. */
typedef struct mdn_contact_audit {
    float physical_clearance_m; /* nonnegative gap; 0 at contact or overlap   */
    float safety_clearance_m;   /* physical clearance minus the safety margin */
    uint32_t contact;           /* declared mechanical contact                 */
    uint32_t ambiguous;         /* unsupported or non-converged case, treated
                                   conservatively (moving spheres, kind 3,
                                   are unsupported by the reference audit)     */
} mdn_contact_audit;

/* Buffer ids for mdn_sim_buffer / download / upload. They name the public
 * members of the reference Sim (main.mm:517-518). */
enum {
    MDN_BUF_STATES = 0,       /* mdn_physics_state[n]                         */
    MDN_BUF_RUNS = 1,         /* mdn_sim_run[n]                               */
    MDN_BUF_WORLDS = 2,       /* mdn_world[n]                                 */
    MDN_BUF_SENSORS = 3,      /* float[n][8][320] range ring (metres)         */
    MDN_BUF_POSES = 4,        /* float[n][8][12] camera pose ring             */
    MDN_BUF_COMMANDS = 5,     /* float[n][8][4] command ring                  */
    MDN_BUF_ACTOR = 6,        /* float[actor_param_count]                     */
    MDN_BUF_CRITIC = 7,       /* float[critic_param_count]                    */
    MDN_BUF_OBS = 8,          /* float[T][n][actor_obs_dim]                   */
    MDN_BUF_CO = 9,           /* float[T][n][critic_obs_dim]                  */
    MDN_BUF_ACTIONS = 10,     /* float[T][n][4]                               */
    MDN_BUF_LOGP = 11,        /* float[T][n]                                  */
    MDN_BUF_VALUES = 12,      /* float[T][n]                                  */
    MDN_BUF_REWARDS = 13,     /* float[T][n]                                  */
    MDN_BUF_NEXT_VALUES = 14, /* float[T][n]                                  */
    MDN_BUF_TERMINATED = 15,  /* uint8[T][n]                                  */
    MDN_BUF_TRUNCATED = 16,   /* uint8[T][n]                                  */
    MDN_BUF_ADVANTAGES = 17,  /* float[T][n]                                  */
    MDN_BUF_RETURNS = 18,     /* float[T][n]                                  */
    MDN_BUF_RAPTOR = 19,      /* mdn_raptor_weights                           */
    MDN_BUF_PHYSICS = 20,     /* mdn_physics_params                           */
    MDN_BUF_CONTACT_ID = 21,  /* int32[T][n] nearest-obstacle id at the step's
                                 closest approach (-1 = room walls)           */
    MDN_BUF_TASK_STATES = 22, /* mdn_task_state[n] (task_states, main.mm:535) */
    MDN_BUF_CONTACT_AUDIT = 23, /* mdn_contact_audit[T][n], written while the
                                   mechanical contact audit is enabled     */
    /* Frozen challenge bank (main.mm:522, 2388); allocated by
     * mdn_sim_set_challenge_bank, except the active ids, which always exist. */
    MDN_BUF_BANK_WORLDS = 24,         /* mdn_world[bank_count] frozen levels      */
    MDN_BUF_BANK_SCHEDULE = 25,       /* uint32[n][schedule_stride] level ids     */
    MDN_BUF_BANK_ACTIVE_IDS = 26,     /* uint32[n] level each env plays           */
    MDN_BUF_BANK_TRANSITION_IDS = 27, /* uint32[T][n] level of each transition    */
    MDN_BUF_RAW_ADVANTAGES = 28,      /* float[T][n] GAE before normalisation     */
    MDN_BUF_ENV_PHYSICS = 29,         /* mdn_physics_params[n] each env's episode
                                         plant (environment_physics, main.mm:537);
                                         allocated while a runtime config is on  */
    MDN_BUF_COUNT = 30
};

/* ---- library / device --------------------------------------------------- */
const char* mdn_last_error(void);
uint32_t mdn_abi_version(void);
void mdn_sim_config_default(mdn_sim_config* out);              /* SimConfig{} defaults, main.mm:462-463 */
void mdn_rollout_shape_default(mdn_rollout_shape* out);
void mdn_physics_crazyflie_default(mdn_physics_params* out);   /* rl_physics_crazyflie_default, physics.hpp:184-219 */
/* Parse a RAPTOR1 file (raptor.hpp:25-40). Returns MDN_ERR_IO on a bad file. */
int mdn_raptor_load(const char* path, mdn_raptor_weights* out);

typedef struct mdn_device mdn_device;
typedef struct mdn_sim mdn_sim;
typedef struct mdn_ppo mdn_ppo;

int mdn_device_open(int gpu, mdn_device** out);                 /* Metal::Metal, main.mm:50-52 */
int mdn_device_close(mdn_device* dev);
/* Metal::finish (main.mm:71): wait for all work queued on the device's sims and
 * trainers, raise any device error, return the GPU time since the last sync.
 * MDN_ERR_TIMEOUT when a wide-actor kernel's bounded barrier wait gave up. */
int mdn_sync(mdn_device* dev, double* gpu_seconds);

/* ---- simulator: Sim (main.mm:516-603) ----------------------------------- */
/* Sim::Sim(Metal&, SimConfig, horizon) main.mm:529-566. raptor/physics may be
 * NULL (then: weights from mdn_raptor_load of the packaged RAPTOR1 file is
 * required, so NULL raptor is MDN_ERR_INVALID; physics NULL = Crazyflie). The
 * actor and critic are initialised exactly as main.mm:548-555 (seed 1789). */
int mdn_sim_create(mdn_device* dev, const mdn_sim_config* cfg, const mdn_rollout_shape* shape,
                   uint32_t horizon, const mdn_raptor_weights* raptor,
                   const mdn_physics_params* physics, mdn_sim** out);
int mdn_sim_destroy(mdn_sim* sim);
int mdn_sim_reset(mdn_sim* sim);                                 /* Sim::reset, main.mm:568 */
int mdn_sim_set_config(mdn_sim* sim, const mdn_sim_config* cfg); /* Sim::set_config, main.mm:567 */
int mdn_sim_get_config(mdn_sim* sim, mdn_sim_config* out);       /* Sim::cfg */
/* Sim::collect(cb, count), main.mm:576-598: `steps` policy steps (0 = horizon)
 * starting at tick 0, rows written at tick % horizon. */
int mdn_sim_collect(mdn_sim* sim, uint32_t steps);
/* One policy step at an explicit tick (teacher-forced parity runs). */
int mdn_sim_step(mdn_sim* sim, uint32_t tick);
/* Device pointer and size of a buffer. A caller that writes MDN_BUF_WORLDS
 * through this pointer must then call mdn_sim_upload(sim, MDN_BUF_WORLDS,
 * NULL, 0, 0), which refreshes the simulator's internal copy of the worlds. */
int mdn_sim_buffer(mdn_sim* sim, int id, void** dev_ptr, size_t* bytes);
/* Replacements for host access to MTLBuffer.contents (navigation_training.hpp:23-24). */
int mdn_sim_download(mdn_sim* sim, int id, void* host, size_t offset, size_t bytes);
int mdn_sim_upload(mdn_sim* sim, int id, const void* host, size_t offset, size_t bytes);
/* Sim::report aggregates (main.mm:599-602): out[0..9] = episodes, successes,
 * collisions, timeouts, success_time, total_path, total_elapsed, final_progress,
 * min_clearance, peak_speed. */
int mdn_sim_report(mdn_sim* sim, double out[10]);
int mdn_sim_dims(mdn_sim* sim, uint32_t* n, uint32_t* horizon, uint32_t* actor_params, uint32_t* critic_params);
/* rl_physics_domain_stress_range (physics_domain.hpp:37-40). */
void mdn_domain_stress_range(mdn_domain_range* out);
/* Sim.runtime_control (main.mm:532-537): with runtime->enabled != 0 every
 * episode reset draws the env's plant (rl_physics_sample_domain,
 * physics_domain.hpp:99-157, seeded per env and episode as
 * sim_domain_episode_seed, sim.metal:50-54), stores it in MDN_BUF_ENV_PHYSICS
 * and hovers each rotor at that plant's thrust (sim.metal:62-82); the advance
 * integrates each env with its own plant (sim.metal:287). A rejected draw
 * stores the nominal plant with a NaN mass, which mdn_sim_validate_tasks
 * reports. Takes effect at the next reset. NULL or enabled == 0: the shared
 * nominal plant. */
int mdn_sim_set_runtime(mdn_sim* sim, const mdn_runtime_config* runtime);
/* navigation_task_default_config (navigation_tasks.hpp:97-142) followed by the
 * overrides of navigation_training::task_settings (navigation_training.hpp:7-14).
 * Returns MDN_ERR_INVALID for an unsupported stage/family/difficulty. */
int mdn_task_settings(uint32_t stage, uint32_t family, float difficulty, mdn_task_config* out);
/* navigation_training::configure (navigation_training.hpp:16-25): enable the
 * goal-arrival task generator and reward for every env, switch the runtime
 * config on with domain_amplitude (0..1), seed 0x3f84d5b5 and the stress range,
 * and reset the sim. The task's nav period must equal substeps x 10 ms and no
 * challenge bank may be enabled. Passing control->enabled == 0 returns to legacy
 * episodes (tasks and runtime config off). */
int mdn_sim_configure_tasks(mdn_sim* sim, const mdn_task_control* control, float domain_amplitude);
/* navigation_training::validate_rollout (navigation_training.hpp:27-35):
 * MDN_ERR_STATE naming the first env whose task generation was rejected, or
 * whose episode plant draw was rejected while the runtime config is on. */
int mdn_sim_validate_tasks(mdn_sim* sim);
/* Pose-aware mechanical contact audit (vehicle_geometry.hpp:241-376, run as
 * navigation_contact.metal:3-25 runs it), enabled per simulator: every policy
 * step then audits each environment's post-integration pose (before an
 * in-step episode reset) at its episode time against the room and its
 * obstacles and writes MDN_BUF_CONTACT_AUDIT[tick][env]. It changes no
 * observation, reward or termination (those keep the 0.18 m sphere contact).
 * safety_margin_m: 0.04 = VG_DEFAULT_SAFETY_MARGIN_M. enabled = 0 turns it off. */
int mdn_sim_set_contact_audit(mdn_sim* sim, int enabled, float safety_margin_m);
/* Delay rehearsal: the reference's NAV_DELAY_REHEARSAL build switch of its
 * delay-training target (sim.metal:14-24, cpu_reference.hpp:1-3,219-223,
 * CMakeLists.txt:72-76), here a run-time switch per simulator. While it is on
 * and cfg.mode == 22 (not evaluation), environments with (global id / 4) even
 * train "clean": no sensor or command delay, wind, depth noise or dropout.
 * Off by default, as in every other reference build. */
int mdn_sim_set_delay_rehearsal(mdn_sim* sim, int enabled);
/* ChallengeBankControl (sim.metal:13, challenge_training.hpp:33-38). */
typedef struct mdn_bank_control {
    uint32_t enabled, bank_count, schedule_stride, horizon;
} mdn_bank_control;
/* Frozen challenge-bank training for a simulator (main.mm:2351-2353,
 * sim_apply_challenge_world sim.metal:95-122). With control->enabled != 0 the
 * bank's bank_count worlds are copied to the device and every episode reset
 * replaces the procedural world by the level that MDN_BUF_BANK_SCHEDULE names
 * for the env: slot 0 at mdn_sim_reset, slot tick + 1 for a reset inside the
 * step at `tick`. Level id 0xffffffff selects a rehearsal world (training
 * family 12 on even, 13 on odd environments, 4 m goals). MDN_BUF_BANK_ACTIVE_IDS
 * holds each env's level and MDN_BUF_BANK_TRANSITION_IDS[tick][env] the level of
 * each transition; MDN_BUF_RAW_ADVANTAGES receives the GAE of each rollout update
 * before normalisation (main.mm:1325-1328). The schedule (uint32[n][stride],
 * zero-filled) is written with mdn_sim_upload, before mdn_sim_reset for the
 * first rollout. control == NULL or enabled == 0 switches banks off (active ids
 * read 0xffffffff after the next reset). schedule_stride must be 1..65536 and
 * bank_worlds hold valid worlds (count <= 16, kinds 0..3). Under several ranks
 * each rank passes the schedule rows of its own environments. */
int mdn_sim_set_challenge_bank(mdn_sim* sim, const mdn_world* bank_worlds, const mdn_bank_control* control);
/* Device time of the last mdn_sim_collect (CUDA events on the sim stream). */
int mdn_sim_last_collect_ms(mdn_sim* sim, float* ms);

/* Per-kernel device time of one policy step at `tick` (sense, act, advance),
 * CUDA events on the sim stream between the launches. Stands in for the
 * reference's per-encoder timestamp profiler (profile.hpp:13-126). */
int mdn_sim_profile_step(mdn_sim* sim, uint32_t tick, float ms[3]);
/* Kernel launches one collect() step and one rollout update enqueue. */
int mdn_launch_counts(mdn_sim* sim, mdn_ppo* ppo, uint32_t* per_policy_step, uint32_t* per_update);
/* Measured dense FP32 FMA throughput of this device (TFLOP/s), a pure-FMA
 * kernel over every SM: the denominator of the CUDA-core roofline. */
int mdn_device_fp32_peak(mdn_device* dev, double* tflops);
/* Self-test of the depth kernel's divide-free quotient (a * RN(1/d) with two
 * fused residual corrections) against IEEE division over `samples` random
 * operand pairs of the ray tests' ranges; *mismatches counts differing bit
 * patterns (0 expected). */
int mdn_selftest_division(mdn_device* dev, uint64_t samples, uint64_t seed, uint64_t* mismatches);
/* The bounded shared-memory barrier wait of the tensor-core kernels, alone in
 * a one-thread kernel: with arrive = 0 nothing arrives, the wait gives up after
 * limit_cycles and the call returns MDN_ERR_TIMEOUT (the status a kernel's
 * timed-out wait surfaces as); with arrive = 1 it returns MDN_OK. No reference
 * counterpart (the reference's Metal waits are unbounded). */
int mdn_selftest_barrier_timeout(mdn_device* dev, uint64_t limit_cycles, int arrive);

/* ---- trainer: PPOTrainer (main.mm:1110-1476) ----------------------------- */
/* PPOTrainer(Sim&, epochs) main.mm:1159-1208; epochs 1..4; minibatch_rows 0 =
 * the reference's 256 rows (main.mm:1115). */
int mdn_ppo_create(mdn_sim* sim, uint32_t epochs, uint32_t minibatch_rows, mdn_ppo** out);
int mdn_ppo_destroy(mdn_ppo* ppo);
/* PPOTrainer::rollout_update(cb, rollout_index), main.mm:1321-1384. */
int mdn_ppo_rollout_update(mdn_ppo* ppo, uint32_t rollout_index);
/* PPOTrainer::metric_mean: policy, value, entropy, ratio means (main.mm:1383). */
int mdn_ppo_metrics(mdn_ppo* ppo, float out[4]);
int mdn_ppo_state(mdn_ppo* ppo, uint64_t* optimizer_step, uint32_t* completed_rollouts);
int mdn_ppo_set_state(mdn_ppo* ppo, uint64_t optimizer_step, uint32_t completed_rollouts);
/* Adam moments: which = 0 actor m, 1 actor v, 2 critic m, 3 critic v. */
int mdn_ppo_moments(mdn_ppo* ppo, int which, float* host, size_t count, int upload);
/* Pre-clip gradient norms of the last update (actor, critic), grad_norm_rows. */
int mdn_ppo_grad_norms(mdn_ppo* ppo, float* host_rows, size_t count);
/* Host-only form of the same order (no device needed): `rows` rollout rows
 * split into `minibatch`-row chunks. `count` must be epochs*ceil(rows/minibatch). */
int mdn_minibatch_order(uint32_t rows, uint32_t minibatch, uint32_t epochs, uint32_t rollout_index, uint32_t* out,
                        size_t count);
/* Minibatch chunk order the trainer uses for `rollout_index`: epochs x chunks
 * first-row indices, drawn as main.mm:1331-1337 draws them (std::mt19937 +
 * std::shuffle, reshuffled at epoch 1). `count` must be epochs*chunks. */
int mdn_ppo_minibatch_order(mdn_ppo* ppo, uint32_t rollout_index, uint32_t* out, size_t count);
/* Device time of the last rollout update (CUDA events). */
int mdn_ppo_last_update_ms(mdn_ppo* ppo, float* ms);
/* Minibatch arithmetic of the 64-unit actor and critic (ppo_actor_forward /
 * ppo_sample_loss_grad / ppo_actor_grad_direct and the critic kernels,
 * ppo.metal:193-657; cpu_reference.hpp:515-551): enabled = 0 (default) runs
 * the fp32 CUDA-core kernel whose sums follow the reference's order (the
 * parity path); enabled = 1 runs the tcgen05 tensor-core kernel, TF32
 * products with fp32 accumulation (gradients within ~1e-2 relative of fp32),
 * for large minibatches. Clip, Adam and the GAE stay fp32 either way. Not for
 * the wide actor, whose products already run on the tensor cores. */
int mdn_ppo_set_tensor_cores(mdn_ppo* ppo, int enabled);
/* Device time of one launch of the minibatch gradient kernels (the gradient
 * partials and their sum, no clip/Adam) for minibatch `update` of the last
 * rollout update, CUDA events on the sim stream: the roofline numerator of
 * the update. Writes only trainer scratch; parameters and moments are
 * untouched. 64-unit actor only. */
int mdn_ppo_profile_minibatch(mdn_ppo* ppo, uint32_t update, float* ms);
/* PPOTrainer::save_checkpoint / load_checkpoint (main.mm:1209-1320): PPOFIX1.
 * Save writes version 6, or version 8 while the runtime config or the task
 * generator is on (plus the runtime/task configuration, per-env episode plants
 * and task states, nominal plant and RAPTOR weights). Load reads versions 3-8;
 * a version 7-8 file's runtime and task configuration must equal the
 * simulator's (set them first: mdn_sim_configure_tasks / mdn_sim_set_runtime);
 * versions 9-10 (reward shaping, calibrated camera) return MDN_ERR_MISMATCH. */
int mdn_ppo_checkpoint_save(mdn_ppo* ppo, const char* path, uint32_t family, uint32_t seed,
                            uint32_t completed_rollouts);
int mdn_ppo_checkpoint_load(mdn_ppo* ppo, const char* path, uint32_t family, uint32_t horizon,
                            uint32_t n, uint32_t seed);
/* Read a checkpoint's header and, for versions 7-8, its runtime and task
 * configuration (zeroed below version 7) on the host, without a device. */
int mdn_checkpoint_inspect(const char* path, mdn_checkpoint_header* header, mdn_runtime_config* runtime,
                           mdn_task_control* tasks);

/* GAE + advantage normalisation of one rollout that allocates no memory.
 * No counterpart in the reference. For callers that cannot call cudaMalloc:
 * code whose device memory is all owned by its own pool (a framework's caching
 * allocator), or code that must not allocate on its hot path (a fixed-latency
 * training/evaluation loop). It computes what the
 * first phase of mdn_ppo_rollout_update computes, from device pointers in the
 * reference's T-major [horizon][envs] layout: rewards, values, next_values
 * (float), terminated, truncated (uint8) in; advantages (normalised) and
 * returns (float) out. gamma/lambda as ppo.hpp:108-126 (0.99/0.95 in the
 * trainer). `stream` is a cudaStream_t or NULL for the default stream.
 * Its scratch is a fixed device array inside libmdn (33 KB on every GPU that
 * loads the library, held until exit): envs <= 1,048,576 (4,096 blocks of
 * 256); larger sizes return MDN_ERR_INVALID. The first call on a device looks
 * up that array's address, so make it before any stream capture; the address
 * is kept for the life of the device's primary context, so after a
 * cudaDeviceReset unload and reload libmdn before calling again. All calls
 * share the array: calls that overlap on the GPU (different streams, or
 * different host threads) race and must be serialised by the caller. */
int mdn_gae_normalize_static(const float* rewards, const float* values, const float* next_values,
                             const uint8_t* terminated, const uint8_t* truncated, float* advantages,
                             float* returns, uint32_t horizon, uint32_t envs, float gamma, float lambda,
                             void* stream);

/* ---- deployment export ----------------------------------------------- */
/* Write a trained actor in the reference's deployable format: NAVPOL1 for the
 * 64-unit actor (nav_deployment::NavigationPolicy::write_file,
 * deployment.hpp:166-201), NAVWID4 for wider ones (the format
 * nav_deployment::WideNavigationPolicy::load reads,
 * navigation_wide_deployment.hpp:15-40). `actor` is the flat parameter vector
 * (ppo.hpp:35-40) of an actor `hidden` units wide, in host memory;
 * `source_checkpoint` is hashed (FNV-1a 64) into the provenance trailer;
 * max_speed_mps is the command scale of NavigationPolicy::infer. */
int mdn_policy_write(const char* path, const float* actor, uint32_t hidden, const char* source_checkpoint,
                     float max_speed_mps);
/* The same for the simulator's current actor (downloaded from the device). */
int mdn_sim_export_policy(mdn_sim* sim, const char* path, const char* source_checkpoint, float max_speed_mps);
/* NavigationPolicy::raw_mean (deployment.hpp; the deployment probe of
 * main.mm:1017-1042) batched on the GPU: the means of the simulator's current
 * actor for `rows` observation rows (host [rows][184] in, host [rows][4] out:
 * the output layer, its bias, then the geometry prior on means 0..2). fp32
 * dense kernels, any actor shape. Allocates its own device scratch. */
int mdn_sim_actor_means(mdn_sim* sim, const float* obs, uint32_t rows, float* means);

/* ---- frozen challenge banks (challenge_evaluation.hpp, challenge_training.hpp) */
/* SHA-256 of a file as 64 lowercase hex digits + NUL (challenge_evaluation::
 * sha256_file, challenge_evaluation.hpp:71-89). */
int mdn_sha256_file(const char* path, char out[65]);

/* One split of a challenge-bank JSONL file, every record validated as
 * challenge_evaluation::parse_level does (challenge_evaluation.hpp:163-280) and
 * the file as load_split does (:282-313): schema 1, families 14/15/16 with their
 * names and geometry contracts (identity or mirror_y transform), the simulator
 * seed derivation, the fixed room, at most 16 AABB/sphere/cylinder obstacles
 * inside it, safe start and goal for the 0.18 m sphere, the obstructed-route /
 * witness contract, unique failure ids, and world_source_sha256 equal to
 * `expected_world_sha256`. Errors are MDN_ERR_INVALID ("challenge bank: ..."
 * with the JSONL line) or MDN_ERR_IO. */
typedef struct mdn_bank mdn_bank;
typedef struct mdn_bank_level {  /* challenge_evaluation::Level, numeric fields */
    uint32_t family, seed, base_seed, environment_index;
    float distance, difficulty, direct_route_clearance_m, witness_min_clearance_m;
    uint32_t witness_sample_count, witness_point_count, mirrored, line_number;
} mdn_bank_level;
enum mdn_bank_text {
    MDN_BANK_FAILURE_ID = 0, MDN_BANK_SPLIT = 1, MDN_BANK_FAMILY_NAME = 2, MDN_BANK_GEOMETRY_CONTRACT = 3,
    MDN_BANK_DIFFICULTY_BAND = 4, MDN_BANK_SCENE_SHA256 = 5, MDN_BANK_WORLD_SOURCE_SHA256 = 6
};
int mdn_bank_load(const char* jsonl_path, const char* split, const char* expected_world_sha256, mdn_bank** out);
int mdn_bank_free(mdn_bank* bank);
/* Level count and the SHA-256 of the whole JSONL file (bank_hash). */
int mdn_bank_info(const mdn_bank* bank, uint32_t* level_count, char bank_sha256[65]);
/* Level `index` (file order within the split): numeric fields and its world
 * (family, seed, goal, wind, obstacles as stored; either pointer may be NULL). */
int mdn_bank_level_get(const mdn_bank* bank, uint32_t index, mdn_bank_level* level, mdn_world* world);
/* All worlds of the split, in level order (capacity >= level count). */
int mdn_bank_worlds(const mdn_bank* bank, mdn_world* out, uint32_t capacity);
/* A text field of a level; valid until mdn_bank_free. NULL on a bad index. */
const char* mdn_bank_level_text(const mdn_bank* bank, uint32_t index, int field);
/* The witness route of a level as float[count][3] (capacity in points). */
int mdn_bank_witness_route(const mdn_bank* bank, uint32_t index, float* xyz, uint32_t capacity, uint32_t* count);

/* challenge_training::Settings (challenge_training.hpp:40-49). */
typedef struct mdn_challenge_settings {
    uint32_t environment_count;      /* all environments of the run (every rank) */
    uint32_t horizon;                /* rollout length; schedules have horizon+1 slots */
    uint32_t sampler_seed;
    uint32_t rehearsal_environments; /* the first R envs play rehearsal worlds */
    uint32_t selection;              /* 0 uniform over the family, 1 failure-weighted */
    float uniform_floor;             /* [0.5, 1] */
    float score_staleness_mix;       /* [0, 1] */
    uint32_t focus_family;           /* 0 balanced 14/15/16, or one family for all */
} mdn_challenge_settings;
void mdn_challenge_settings_default(mdn_challenge_settings* out);
/* The train-split level sampler with per-level failure scores
 * (challenge_training::ChallengeTraining, challenge_training.hpp:53-427). All
 * arrays are env-major over settings.environment_count environments; a
 * schedule is uint32[env][horizon+1]; rollout evidence is [tick][env]. */
typedef struct mdn_challenge mdn_challenge;
int mdn_challenge_create(const char* bank_jsonl, const char* expected_world_sha256,
                         const mdn_challenge_settings* settings, mdn_challenge** out);
int mdn_challenge_destroy(mdn_challenge* sampler);
/* The loaded train split (owned by the sampler). */
int mdn_challenge_bank(mdn_challenge* sampler, const mdn_bank** out);
int mdn_challenge_control(const mdn_challenge* sampler, mdn_bank_control* out);
/* initial_schedule (:106-124): a fresh run's schedule; sets the active ids. */
int mdn_challenge_initial_schedule(mdn_challenge* sampler, uint32_t* schedule);
/* next_schedule (:128-154): slot 0 keeps each env's active level, slots
 * 1..horizon are sampled for resets within the next rollout. */
int mdn_challenge_next_schedule(mdn_challenge* sampler, const uint32_t* active_ids, uint64_t rollout_index,
                                uint32_t* schedule);
int mdn_challenge_active_ids(const mdn_challenge* sampler, uint32_t* out);
/* observe_raw_gae (:160-199): accumulate per-episode mean |GAE| into level
 * scores from one rollout's raw GAE, terminal flags and transition level ids. */
int mdn_challenge_observe_raw_gae(mdn_challenge* sampler, const float* raw_gae, const uint8_t* terminated,
                                  const uint8_t* truncated, const uint32_t* transition_ids, uint64_t rollout_index);
int mdn_challenge_level_stats(const mdn_challenge* sampler, uint32_t level, float* score,
                              uint64_t* completed_episodes, uint64_t* last_visit_rollout);
/* The CHTRN1 version-3 sidecar (save_state/load_state, :204-277), byte for
 * byte the reference's format; checkpoint_sha256 = 64 hex digits. load_state
 * writes the restored active ids (environment_count values) to active_ids. */
int mdn_challenge_save_state(mdn_challenge* sampler, const char* path, const char* checkpoint_sha256,
                             uint64_t completed_rollouts, const uint32_t* active_ids);
int mdn_challenge_load_state(mdn_challenge* sampler, const char* path, const char* checkpoint_sha256,
                             uint64_t completed_rollouts, uint32_t* active_ids);

/* challenge_evaluation::BankScore (challenge_evaluation.hpp:53-66); family
 * slots are families 14, 15, 16. */
typedef struct mdn_bank_score {
    uint64_t episodes, successes, collisions, timeouts;
    uint64_t family_episodes[3], family_successes[3];
    double successful_time_s;
} mdn_bank_score;
/* challenge_evaluation::run (challenge_evaluation.hpp:352-497): evaluate a
 * PPOFIX1 checkpoint's actor and critic (versions 3-9) on every level of one
 * split. Levels run in batches of 128 on an evaluation-mode simulator (one
 * episode per env; no delays, noise or dropout; each level's stored wind), with
 * the level's world, its simulator policy seed and a fresh start, for
 * `max_steps` policy steps. One CSV row per level (the reference's 38 columns),
 * written to a temporary file and renamed into place, and the aggregate score.
 * mode 2, 13 or 17; speed in (0, 3]; max_steps 1..400; raptor as for
 * mdn_sim_create. */
int mdn_bank_evaluate(mdn_device* dev, const mdn_raptor_weights* raptor, const char* checkpoint_path,
                      const char* bank_jsonl, const char* split, const char* world_sha256, const char* output_csv,
                      uint32_t mode, float speed, uint32_t max_steps, mdn_bank_score* score);

/* ---- multi-GPU (no reference counterpart: the reference is one Apple GPU) */
/* Fill a 128-byte NCCL unique id (rank 0) to share through any host channel. */
int mdn_comm_unique_id(uint8_t id[128]);
/* Attach a communicator to the device. Sims created afterwards on this device
 * hold global env ids [rank*n, (rank+1)*n) and their PPO updates allreduce
 * gradients and advantage statistics across `world` ranks. */
int mdn_comm_init(mdn_device* dev, int rank, int world, const uint8_t id[128]);
int mdn_comm_destroy(mdn_device* dev);

#ifdef __cplusplus
}
#endif
#endif /* MDN_H */
