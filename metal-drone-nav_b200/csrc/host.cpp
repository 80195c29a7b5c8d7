// C-ABI implementation: device, simulator and the shared helpers.
// Stands in for the reference's Metal (main.mm:44-72) and Sim
// (main.mm:516-603) host classes; see include/mdn.h for the mapping.
//
// Compiled with -ffp-contract=off: the policy initialisation and camera
// tables below must round exactly like the reference's host code.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <memory>
#include <string>

#include "host_common.h"
#include "ppo_tc.h"

namespace mdn {
static thread_local std::string g_last_error;
void set_last_error(const std::string& msg) { g_last_error = msg; }
}  // namespace mdn

using namespace mdn;

extern "C" const char* mdn_last_error(void) { return g_last_error.c_str(); }
extern "C" uint32_t mdn_abi_version(void) { return MDN_ABI_VERSION; }

extern "C" void mdn_sim_config_default(mdn_sim_config* c) {
    // SimConfig member initialisers, main.mm:462-463
    *c = mdn_sim_config{};
    c->n = 128; c->tick = 0; c->mode = 0; c->family = 0; c->substeps = 5; c->sensor_period = 1;
    c->sensor_delay = 0; c->command_delay = 0; c->max_steps = 200; c->seed = 42; c->eval = 0;
    c->speed = 2; c->distance = 4; c->wind = 0; c->depth_noise = 0; c->dropout = 0; c->risk_coef = 0;
    c->entropy_coef = .005f; c->learning_rate = .0003f; c->velocity_contract = 1; c->geometry_memory = 0;
}

extern "C" void mdn_rollout_shape_default(mdn_rollout_shape* s) {
    *s = mdn_rollout_shape{};
    s->actor_obs_dim = kActorObs;
    s->critic_obs_dim = kCriticObs;
    s->actor_hidden = kHidden;
    s->critic_hidden = kHidden;
    s->flags = 0;
    const float lo[3] = {-2.0f, -5.0f, 0.0f}, hi[3] = {14.0f, 5.0f, 5.0f};  // world.hpp:73-74,85
    for (int j = 0; j < 3; j++) {
        s->room_min[j] = lo[j];
        s->room_max[j] = hi[j];
    }
}

extern "C" void mdn_physics_crazyflie_default(mdn_physics_params* p) {
    // Crazyflie profile of rl-tools L2F as transcribed at physics.hpp:184-219.
    *p = mdn_physics_params{};
    const float positions[12] = {.028f, -.028f, 0, -.028f, -.028f, 0, -.028f, .028f, 0, .028f, .028f, 0};
    const float torque_z[4] = {-1, 1, -1, 1};
    const float inertia_diag[3] = {9.416556729130406e-6f, 9.644051701582312e-6f, 1.745951732253285e-5f};
    const float inertia_inv_diag[3] = {106195.93007988465f, 103690.85846314249f, 57275.35197719487f};
    for (int r = 0; r < 4; ++r) {
        const int i = 3 * r;
        p->rotor_positions[i] = positions[i];
        p->rotor_positions[i + 1] = positions[i + 1];
        p->rotor_thrust_directions[i + 2] = 1.0f;
        p->rotor_torque_directions[i + 2] = torque_z[r];
        p->rotor_thrust_coefficients[i] = 0.00352526f;
        p->rotor_thrust_coefficients[i + 1] = 0.01437313f;
        p->rotor_thrust_coefficients[i + 2] = 0.09223048f;
        p->rotor_torque_constants[r] = 4.665e-3f;
        p->rotor_time_constants_rising[r] = 0.05545454545454546f;
        p->rotor_time_constants_falling[r] = 0.24939393939393945f;
    }
    for (int i = 0; i < 3; ++i) {
        p->inertia[4 * i] = inertia_diag[i];
        p->inertia_inverse[4 * i] = inertia_inv_diag[i];
    }
    p->gravity_world[2] = -9.81f;
    p->mass = 0.027f + 0.0017f + 0.0003f + 0.0016f;
    p->action_min = 0.0f;
    p->action_max = 1.0f;
    p->dt = 0.01f;
    p->position_limit = 100000.0f;
    p->velocity_limit = 100000.0f;
    p->angular_velocity_limit = 100000.0f;
}

extern "C" int mdn_raptor_load(const char* path, mdn_raptor_weights* out) {
    return guarded([&] {
        require(path && out, MDN_ERR_INVALID, "mdn_raptor_load: null argument");
        std::ifstream f(path, std::ios::binary);
        require(bool(f), MDN_ERR_IO, std::string("cannot open RAPTOR file ") + path);
        unsigned char header[16];
        f.read(reinterpret_cast<char*>(header), 16);
        static const unsigned char magic[8] = {'R', 'A', 'P', 'T', 'O', 'R', '1', 0};
        require(bool(f) && std::memcmp(header, magic, 8) == 0, MDN_ERR_IO, "not a RAPTOR1 file");
        uint32_t version, count;
        std::memcpy(&version, header + 8, 4);
        std::memcpy(&count, header + 12, 4);
        require(version == 1 && count == 2084, MDN_ERR_IO, "RAPTOR1 version/count mismatch");
        f.read(reinterpret_cast<char*>(out), sizeof(*out));
        require(bool(f), MDN_ERR_IO, "RAPTOR1 file truncated");
    });
}

// ---------------------------------------------------------------- device
namespace {
uint32_t xorshift(uint32_t& s) {
    s ^= s << 13;
    s ^= s >> 17;
    s ^= s << 5;
    return s;
}
float unit(uint32_t& s) { return float(xorshift(s) >> 8) * (1.0f / 16777216.0f); }

// Camera tables: nav_sensor_pixel_ray (sensor_profile.hpp:81-91 with the
// legacy profile tan_h=1, tan_v=0.75) and the pooled guidance rays
// (guidance.hpp:22-26).
void camera_tables(std::vector<float>& pixel, std::vector<float>& pool) {
    pixel.resize(kPixels * 3);
    pool.resize(80 * 3);
    for (uint32_t k = 0; k < uint32_t(kPixels); k++) {
        const uint32_t row = k / 20u, col = k % 20u;
        const float y = ((float(col) + 0.5f) / 20.0f * 2.0f - 1.0f) * 1.0f;
        const float z = ((float(row) + 0.5f) / 16.0f * 2.0f - 1.0f) * kTanV;
        const float d[3] = {1.0f, -y, -z};
        const float inv = 1.0f / std::fmax(std::sqrt(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]), 1e-8f);
        for (int j = 0; j < 3; j++) pixel[3 * k + j] = d[j] * inv;
    }
    for (uint32_t row = 0; row < 8; row++)
        for (uint32_t col = 0; col < 10; col++) {
            const float y = 0.9f - 0.2f * float(col), z = (0.875f - 0.25f * float(row)) * kTanV;
            const float inv = 1.0f / std::sqrt(1.0f + y * y + z * z);
            const uint32_t k = row * 10 + col;
            pool[3 * k] = inv;
            pool[3 * k + 1] = y * inv;
            pool[3 * k + 2] = z * inv;
        }
}

void use_device(mdn_device* dev) { cuda_check(cudaSetDevice(dev->gpu), "cudaSetDevice"); }
}  // namespace

extern "C" int mdn_device_open(int gpu, mdn_device** out) {
    return guarded([&] {
        require(out != nullptr, MDN_ERR_INVALID, "mdn_device_open: null out");
        int count = 0;
        cuda_check(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
        require(gpu >= 0 && gpu < count, MDN_ERR_INVALID, "mdn_device_open: no such GPU");
        auto dev = std::make_unique<mdn_device>();
        dev->gpu = gpu;
        use_device(dev.get());
        cudaDeviceProp prop{};
        cuda_check(cudaGetDeviceProperties(&prop, gpu), "cudaGetDeviceProperties");
        require(prop.major >= 10, MDN_ERR_INVALID,
                std::string("libmdn is built for sm_100a (B200); device is ") + prop.name);
        dev->sm_count = prop.multiProcessorCount;
        std::vector<float> pixel, pool;
        camera_tables(pixel, pool);
        cuda_check(upload_camera_tables(pixel.data(), pool.data()), "camera tables");
        cuda_check(configure_kernels(), "kernel attributes");
        cuda_check(configure_wide_kernels(), "wide kernel attributes");
        dev->tables_ready = true;
        *out = dev.release();
    });
}

extern "C" int mdn_device_close(mdn_device* dev) {
    return guarded([&] {
        if (!dev) return;
        require(dev->sims.empty() && dev->trainers.empty(), MDN_ERR_STATE,
                "mdn_device_close: destroy trainers and sims first");
        delete dev;
    });
}

extern "C" int mdn_sync(mdn_device* dev, double* gpu_seconds) {
    return guarded([&] {
        require(dev != nullptr, MDN_ERR_INVALID, "mdn_sync: null device");
        use_device(dev);
        double total = 0.0;
        for (mdn_sim* s : dev->sims) {
            sync_stream(dev, s->stream, "stream synchronize");
            total += s->last_collect_ms * 1e-3;
            if (s->wide_error) {
                uint32_t flag = 0;
                cuda_check(cudaMemcpy(&flag, s->wide_error, sizeof(flag), cudaMemcpyDeviceToHost), "wide error flag");
                require(flag == 0, MDN_ERR_TIMEOUT,
                        "wide actor kernel: a barrier wait gave up (flag " + std::to_string(flag) + ")");
            }
        }
        check_trainer_errors(dev);
        cuda_check(cudaGetLastError(), "device error");
        if (gpu_seconds) *gpu_seconds = total;
    });
}

// ------------------------------------------------------------- simulator
mdn::SimArgs mdn_sim::args(uint32_t tick) const {
    SimArgs a{};
    a.cfg = cfg;
    a.cfg.tick = tick;
    a.n = n;
    a.env_base = env_base;
    a.tick = tick;
    for (int j = 0; j < 3; j++) {
        a.room_lo[j] = room_lo[j];
        a.room_hi[j] = room_hi[j];
        a.room_c[j] = room_c[j];
        a.room_e[j] = room_e[j];
    }
    a.states = static_cast<mdn_physics_state*>(buf[MDN_BUF_STATES]);
    a.runs = static_cast<mdn_sim_run*>(buf[MDN_BUF_RUNS]);
    a.worlds = static_cast<mdn_world*>(buf[MDN_BUF_WORLDS]);
    a.world_soa = world_soa;
    a.sensors = static_cast<float*>(buf[MDN_BUF_SENSORS]);
    a.poses = static_cast<float*>(buf[MDN_BUF_POSES]);
    a.commands = static_cast<float*>(buf[MDN_BUF_COMMANDS]);
    a.actor = static_cast<const float*>(buf[MDN_BUF_ACTOR]);
    a.critic = static_cast<const float*>(buf[MDN_BUF_CRITIC]);
    a.raptor = static_cast<const mdn_raptor_weights*>(buf[MDN_BUF_RAPTOR]);
    a.physics = static_cast<const mdn_physics_params*>(buf[MDN_BUF_PHYSICS]);
    a.obs = static_cast<float*>(buf[MDN_BUF_OBS]);
    a.co = static_cast<float*>(buf[MDN_BUF_CO]);
    a.actions = static_cast<float*>(buf[MDN_BUF_ACTIONS]);
    a.logp = static_cast<float*>(buf[MDN_BUF_LOGP]);
    a.values = static_cast<float*>(buf[MDN_BUF_VALUES]);
    a.rewards = static_cast<float*>(buf[MDN_BUF_REWARDS]);
    a.next_values = static_cast<float*>(buf[MDN_BUF_NEXT_VALUES]);
    a.terminated = static_cast<uint8_t*>(buf[MDN_BUF_TERMINATED]);
    a.truncated = static_cast<uint8_t*>(buf[MDN_BUF_TRUNCATED]);
    a.contact = static_cast<int32_t*>(buf[MDN_BUF_CONTACT_ID]);
    a.task_ctl = task_ctl;
    a.tasks = static_cast<mdn_task_state*>(buf[MDN_BUF_TASK_STATES]);
    a.task_config_ok = task_config_ok;
    a.actor_hidden = actor_hidden;
    a.actor_b2 = actor_hidden * (kActorObs + 1 + kActions);
    a.actor_log_std = a.actor_b2 + kActions;
    a.wide_partials = wide_partials;
    a.wide_slices = wide ? actor_hidden / 128 : 0;
    a.critic_values = nullptr;
    a.next_co = nullptr;
    a.co_dim = co_dim;
    a.next_co_full = nullptr;
    if (lay) {  // layered networks: k_act adds b2 and the prior to the actor outputs, as for the wide actor
        a.wide_partials = lay->out_a;
        a.wide_slices = 1;
        a.critic_values = lay->values;
        a.next_co = lay->next_co;
        if (co_dim != kCriticObs) a.next_co_full = lay->next_critic_in;
        a.actor_b2 = lay->actor.bias_offset(lay->actor.layers);
        a.actor_log_std = lay->actor.param_count() - kActions;
    }
    a.audit = audit_enabled ? static_cast<mdn_contact_audit*>(buf[MDN_BUF_CONTACT_AUDIT]) : nullptr;
    a.audit_margin = audit_margin;
    a.delay_rehearsal = delay_rehearsal ? 1u : 0u;
    a.bank_enabled = bank.enabled;
    a.bank_count = bank.enabled ? bank.bank_count : 0;
    a.bank_stride = bank.schedule_stride;
    a.bank_worlds = static_cast<const mdn_world*>(buf[MDN_BUF_BANK_WORLDS]);
    a.bank_schedule = static_cast<const uint32_t*>(buf[MDN_BUF_BANK_SCHEDULE]);
    a.bank_active = static_cast<uint32_t*>(buf[MDN_BUF_BANK_ACTIVE_IDS]);
    a.bank_transition = bytes[MDN_BUF_BANK_TRANSITION_IDS] ? static_cast<uint32_t*>(buf[MDN_BUF_BANK_TRANSITION_IDS])
                                                           : nullptr;
    a.runtime = runtime;
    a.env_physics = static_cast<mdn_physics_params*>(buf[MDN_BUF_ENV_PHYSICS]);
    a.reset_list = reset_mem;
    a.reset_count = reset_mem ? reset_mem + n : nullptr;
    a.reset_pending = reset_mem ? reinterpret_cast<uint8_t*>(reset_mem + n + 32) : nullptr;
    a.phase = tick & 1u;
    return a;
}

void mdn_sim::release_graphs() {
    for (auto& g : graphs) cudaGraphExecDestroy(g.second);
    graphs.clear();
}

namespace {
void validate_config(const mdn_sim_config& c) {
    require(c.n >= 1, MDN_ERR_INVALID, "SimConfig.n must be positive");
    require(c.substeps >= 1 && c.substeps <= 64, MDN_ERR_INVALID, "SimConfig.substeps must be 1..64");
    require(c.sensor_period >= 1, MDN_ERR_INVALID, "SimConfig.sensor_period must be positive");
    // main.mm:727 (sim_evaluate): the 8-deep rings hold <=6 sensor frames and <=7 command steps.
    require(c.sensor_delay <= 6 && c.command_delay <= 7, MDN_ERR_INVALID,
            "delay rings support <=6 sensor frames and <=7 command steps");
    require(c.mode <= 22, MDN_ERR_INVALID, "SimConfig.mode: sim_act defines modes 0..22");
    require(c.geometry_memory <= 1, MDN_ERR_INVALID, "SimConfig.geometry_memory must be 0 or 1");
    require(std::isfinite(c.speed) && std::isfinite(c.distance), MDN_ERR_INVALID, "SimConfig speed/distance");
}

void init_policy(std::vector<float>& actor, std::vector<float>& critic, uint32_t hidden) {
    // main.mm:548-555 / cpu_reference.hpp:89-103: seed 1789 Box-Muller draws,
    // with the parameter offsets of an actor `hidden` units wide (ppo.hpp:35-40).
    const size_t b1 = size_t(hidden) * kActorObs, w2 = b1 + hidden, b2 = w2 + size_t(kActions) * hidden, ls = b2 + kActions;
    actor.assign(actor_param_count(hidden), 0.0f);
    critic.assign(kCriticParams, 0.0f);
    uint32_t seed = 1789;
    auto normal = [&]() {
        const float u = std::max(unit(seed), 1e-7f);
        const float a = std::sqrt(-2.0f * std::log(u));
        return a * std::cos(6.2831853f * unit(seed));
    };
    for (size_t i = 0; i < b1; i++) actor[i] = normal() * 0.04f;
    for (size_t i = w2; i < b2; i++) actor[i] = normal() * 0.01f;
    for (int i = 0; i < kActions; i++) actor[ls + i] = -1.0f;
    for (int i = 0; i < kCriticB1; i++) critic[i] = normal() * 0.15f;
    for (int i = kCriticW2; i < kCriticB2; i++) critic[i] = normal() * 0.1f;
}

mdn_sim* checked(mdn_sim* s) {
    require(s != nullptr, MDN_ERR_INVALID, "null mdn_sim");
    use_device(s->dev);
    return s;
}
}  // namespace

extern "C" int mdn_sim_create(mdn_device* dev, const mdn_sim_config* cfg, const mdn_rollout_shape* shape,
                              uint32_t horizon, const mdn_raptor_weights* raptor, const mdn_physics_params* physics,
                              mdn_sim** out) {
    return guarded([&] {
        require(dev && cfg && out, MDN_ERR_INVALID, "mdn_sim_create: null argument");
        require(raptor != nullptr, MDN_ERR_INVALID, "mdn_sim_create: RAPTOR weights are required (mdn_raptor_load)");
        require(horizon >= 1, MDN_ERR_INVALID, "mdn_sim_create: horizon must be positive");
        validate_config(*cfg);
        use_device(dev);
        auto sim = std::make_unique<mdn_sim>();
        sim->dev = dev;
        sim->cfg = *cfg;
        sim->cfg.tick = 0;
        sim->horizon = horizon;
        sim->n = cfg->n;
        sim->env_base = uint32_t(dev->rank) * cfg->n;
        mdn_rollout_shape_default(&sim->shape);
        if (shape) {
            require(shape->actor_obs_dim == 0 || shape->actor_obs_dim == kActorObs, MDN_ERR_INVALID,
                    "actor_obs_dim: this build implements the 184-input guided actor");
            require(shape->critic_obs_dim == 0 || shape->critic_obs_dim == kCriticObs ||
                        shape->critic_obs_dim == kCriticObsControl,
                    MDN_ERR_INVALID, "critic_obs_dim: 32, or 64 for the control-state critic");
            const uint32_t ah = shape->actor_hidden, ch = shape->critic_hidden;
            require(shape->actor_activation <= MDN_ACT_GELU && shape->critic_activation <= MDN_ACT_GELU,
                    MDN_ERR_INVALID, "activation: MDN_ACT_TANH or MDN_ACT_GELU");
            require(shape->actor_layers <= 8 && shape->critic_layers <= 8, MDN_ERR_INVALID,
                    "layers: at most 8 hidden layers per network");
            // The control-state critic (64 inputs, sim.metal:166-180) runs on the
            // layered kernels: the fused ones are built for 32 critic inputs.
            const bool control_state = shape->critic_obs_dim == kCriticObsControl;
            const bool layered = shape->actor_layers > 1 || shape->critic_layers > 1 || shape->actor_activation != 0 ||
                                 shape->critic_activation != 0 || (ch != 0 && ch != uint32_t(kHidden)) ||
                                 control_state;
            if (layered) {
                require(ah <= 2048 && ch <= 2048, MDN_ERR_INVALID,
                        "layered networks: actor_hidden and critic_hidden 1..2048 (0 = 64)");
            } else {
                require(ah == 0 || ah == uint32_t(kHidden) || (ah % 256 == 0 && ah >= 256 && ah <= 8192), MDN_ERR_INVALID,
                        "actor_hidden: 64, or a multiple of 256 up to 8192 (tensor-core wide actor)");
            }
            if (ah != 0) sim->shape.actor_hidden = ah;
            if (ch != 0) sim->shape.critic_hidden = ch;
            sim->shape.actor_layers = shape->actor_layers ? shape->actor_layers : 1;
            sim->shape.critic_layers = shape->critic_layers ? shape->critic_layers : 1;
            sim->shape.actor_activation = shape->actor_activation;
            sim->shape.critic_activation = shape->critic_activation;
            sim->layered = layered;
            sim->co_dim = control_state ? kCriticObsControl : kCriticObs;
            sim->shape.critic_obs_dim = sim->co_dim;
            if (shape->flags & MDN_SHAPE_CUSTOM_ROOM) {
                for (int j = 0; j < 3; j++) {
                    require(shape->room_max[j] > shape->room_min[j], MDN_ERR_INVALID, "room bounds");
                    sim->shape.room_min[j] = shape->room_min[j];
                    sim->shape.room_max[j] = shape->room_max[j];
                }
                sim->shape.flags |= MDN_SHAPE_CUSTOM_ROOM;
            }
        }
        for (int j = 0; j < 3; j++) {
            sim->room_lo[j] = sim->shape.room_min[j];
            sim->room_hi[j] = sim->shape.room_max[j];
            sim->room_c[j] = (sim->room_lo[j] + sim->room_hi[j]) * 0.5f;
            sim->room_e[j] = (sim->room_hi[j] - sim->room_lo[j]) * 0.5f;
        }
        const size_t n = sim->n, rows = n * horizon;
        sim->actor_hidden = sim->shape.actor_hidden;
        sim->actor_params = actor_param_count(sim->actor_hidden);
        MlpShape mlp_actor, mlp_critic;
        if (sim->layered) {
            mlp_actor.in = kActorObs;
            mlp_actor.hidden = sim->shape.actor_hidden;
            mlp_actor.layers = sim->shape.actor_layers;
            mlp_actor.out = kActions;
            mlp_actor.activation = sim->shape.actor_activation;
            mlp_actor.log_std = true;
            mlp_critic.in = sim->co_dim;
            mlp_critic.hidden = sim->shape.critic_hidden;
            mlp_critic.layers = sim->shape.critic_layers;
            mlp_critic.out = 1;
            mlp_critic.activation = sim->shape.critic_activation;
            sim->actor_params = mlp_actor.param_count();
            sim->critic_params = mlp_critic.param_count();
        }
        const bool wide = !sim->layered && sim->actor_hidden != uint32_t(kHidden);
        require(!wide || rows < (size_t(1) << 31), MDN_ERR_INVALID, "wide actor: horizon x n must stay below 2^31 rows");
        size_t* b = sim->bytes;
        b[MDN_BUF_STATES] = n * sizeof(mdn_physics_state);
        b[MDN_BUF_RUNS] = n * sizeof(mdn_sim_run);
        b[MDN_BUF_WORLDS] = n * sizeof(mdn_world);
        b[MDN_BUF_SENSORS] = n * kFrames * kPixels * sizeof(float);
        b[MDN_BUF_POSES] = n * kFrames * 12 * sizeof(float);
        b[MDN_BUF_COMMANDS] = n * kFrames * kActions * sizeof(float);
        b[MDN_BUF_ACTOR] = size_t(sim->actor_params) * sizeof(float);
        b[MDN_BUF_CRITIC] = size_t(sim->critic_params) * sizeof(float);
        b[MDN_BUF_OBS] = rows * kActorObs * sizeof(float);
        b[MDN_BUF_CO] = rows * sim->co_dim * sizeof(float);
        b[MDN_BUF_ACTIONS] = rows * kActions * sizeof(float);
        for (int id : {MDN_BUF_LOGP, MDN_BUF_VALUES, MDN_BUF_REWARDS, MDN_BUF_NEXT_VALUES, MDN_BUF_ADVANTAGES,
                       MDN_BUF_RETURNS, MDN_BUF_CONTACT_ID})
            b[id] = rows * sizeof(float);
        b[MDN_BUF_TERMINATED] = rows;
        b[MDN_BUF_TRUNCATED] = rows;
        b[MDN_BUF_RAPTOR] = sizeof(mdn_raptor_weights);
        b[MDN_BUF_PHYSICS] = sizeof(mdn_physics_params);
        b[MDN_BUF_TASK_STATES] = n * sizeof(mdn_task_state);
        b[MDN_BUF_CONTACT_AUDIT] = 0;  // allocated when the audit is enabled
        b[MDN_BUF_BANK_ACTIVE_IDS] = n * sizeof(uint32_t);
        // Bank worlds, schedule, transition ids and raw advantages are
        // allocated by mdn_sim_set_challenge_bank.
        for (int id : {MDN_BUF_BANK_WORLDS, MDN_BUF_BANK_SCHEDULE, MDN_BUF_BANK_TRANSITION_IDS, MDN_BUF_RAW_ADVANTAGES,
                       MDN_BUF_ENV_PHYSICS})
            b[id] = 0;  // MDN_BUF_ENV_PHYSICS: allocated by mdn_sim_set_runtime
        for (int id = 0; id < MDN_BUF_COUNT; id++) {
            const cudaError_t e = cudaMalloc(&sim->buf[id], std::max<size_t>(b[id], 16));
            if (e != cudaSuccess) {
                for (int k = 0; k < id; k++) cudaFree(sim->buf[k]);
                throw Error(MDN_ERR_NOMEM, std::string("cudaMalloc failed: ") + cudaGetErrorString(e));
            }
        }
        {
            cudaError_t e = cudaMalloc(&sim->world_soa, n * kWorldSoaWords * sizeof(float));
            const size_t reset_bytes = (n + 32) * sizeof(uint32_t) + ((size_t(n) + 15) & ~size_t(15));
            if (e == cudaSuccess) e = cudaMalloc(&sim->reset_mem, reset_bytes);
            if (e == cudaSuccess) e = cudaMemset(sim->reset_mem, 0, reset_bytes);
            if (e != cudaSuccess) {
                for (int k = 0; k < MDN_BUF_COUNT; k++) cudaFree(sim->buf[k]);
                cudaFree(sim->world_soa);
                cudaFree(sim->reset_mem);
                throw Error(MDN_ERR_NOMEM, std::string("cudaMalloc failed: ") + cudaGetErrorString(e));
            }
        }
        if (wide) {
            const size_t slices = sim->actor_hidden / 128;
            cudaError_t e = cudaMalloc(&sim->wide_partials, slices * n * 4 * sizeof(float));
            if (e == cudaSuccess) e = cudaMalloc(&sim->wide_error, sizeof(uint32_t));
            if (e != cudaSuccess) {
                for (int k = 0; k < MDN_BUF_COUNT; k++) cudaFree(sim->buf[k]);
                cudaFree(sim->world_soa);
                cudaFree(sim->reset_mem);
                cudaFree(sim->wide_partials);
                throw Error(MDN_ERR_NOMEM, std::string("cudaMalloc failed: ") + cudaGetErrorString(e));
            }
            cuda_check(cudaMemset(sim->wide_error, 0, sizeof(uint32_t)), "clear wide error flag");
            sim->wide = new WideStep{};
            const float* obs = static_cast<const float*>(sim->buf[MDN_BUF_OBS]);
            const float* actor = static_cast<const float*>(sim->buf[MDN_BUF_ACTOR]);
            const uint32_t h = sim->actor_hidden;
            cuda_check(wide_make_map(&sim->wide->obs_map, obs, kActorObs, rows, kActorObs * sizeof(float), 128),
                       "observation tensor map");
            cuda_check(wide_make_map(&sim->wide->w1_map, actor, kActorObs, h, kActorObs * sizeof(float), 256),
                       "actor W1 tensor map");
            WideRowsArgs& wa = sim->wide->args;
            wa.rows = uint32_t(n);
            wa.row0 = 0;
            wa.hidden = h;
            wa.b1 = actor + size_t(h) * kActorObs;
            wa.w2 = wa.b1 + h;
            wa.partials = sim->wide_partials;
            wa.error = sim->wide_error;
            sim->wide->sm_count = dev->sm_count;
        }
        if (sim->layered) {
            // Per-step scratch of the layered networks: two activation
            // buffers of the wider network, the actor outputs, the values, the
            // post-step critic observations and, for the control-state critic,
            // its 64-input bootstrap rows.
            const size_t widest = std::max(mlp_actor.hidden, mlp_critic.hidden);
            const size_t act_floats = n * widest;
            const size_t full_rows = sim->co_dim != kCriticObs ? n * sim->co_dim : 0;
            const size_t bytes = (2 * act_floats + n * 4 + n + n * kCriticObs + full_rows) * sizeof(float);
            const cudaError_t e = cudaMalloc(&sim->lay_mem, bytes);
            if (e != cudaSuccess) {
                for (int k = 0; k < MDN_BUF_COUNT; k++) cudaFree(sim->buf[k]);
                cudaFree(sim->world_soa);
                cudaFree(sim->reset_mem);
                throw Error(MDN_ERR_NOMEM, std::string("cudaMalloc failed: ") + cudaGetErrorString(e));
            }
            float* f = static_cast<float*>(sim->lay_mem);
            sim->lay = new LayeredStep{};
            LayeredStep& L = *sim->lay;
            L.actor = mlp_actor;
            L.critic = mlp_critic;
            L.actor_params = static_cast<const float*>(sim->buf[MDN_BUF_ACTOR]);
            L.critic_params = static_cast<const float*>(sim->buf[MDN_BUF_CRITIC]);
            L.obs = static_cast<const float*>(sim->buf[MDN_BUF_OBS]);
            L.co = static_cast<const float*>(sim->buf[MDN_BUF_CO]);
            L.act[0] = f;
            L.act[1] = f + act_floats;
            L.out_a = f + 2 * act_floats;
            L.values = L.out_a + n * 4;
            L.next_co = L.values + n;
            L.next_critic_in = sim->co_dim != kCriticObs ? L.next_co + n * kCriticObs : L.next_co;
            L.next_values = static_cast<float*>(sim->buf[MDN_BUF_NEXT_VALUES]);
        }
        cuda_check(cudaStreamCreateWithFlags(&sim->stream, cudaStreamNonBlocking), "cudaStreamCreate");
        {
            int least = 0, greatest = 0;
            cuda_check(cudaDeviceGetStreamPriorityRange(&least, &greatest), "stream priority range");
            sim->fork.priority = greatest;
            cuda_check(cudaStreamCreateWithPriority(&sim->fork.side, cudaStreamNonBlocking, greatest),
                       "cudaStreamCreate (reset branch)");
            cuda_check(cudaEventCreateWithFlags(&sim->fork.fork, cudaEventDisableTiming), "cudaEventCreate");
            cuda_check(cudaEventCreateWithFlags(&sim->fork.join, cudaEventDisableTiming), "cudaEventCreate");
        }
        cuda_check(cudaEventCreate(&sim->ev_start), "cudaEventCreate");
        cuda_check(cudaEventCreate(&sim->ev_stop), "cudaEventCreate");
        std::vector<float> actor, critic;
        if (sim->layered) init_layered(mlp_actor, mlp_critic, actor, critic);
        else init_policy(actor, critic, sim->actor_hidden);
        mdn_physics_params params;
        if (physics) params = *physics;
        else mdn_physics_crazyflie_default(&params);
        sim->nominal = params;
        cuda_check(cudaMemcpyAsync(sim->buf[MDN_BUF_ACTOR], actor.data(), b[MDN_BUF_ACTOR], cudaMemcpyHostToDevice,
                                   sim->stream), "upload actor");
        cuda_check(cudaMemcpyAsync(sim->buf[MDN_BUF_CRITIC], critic.data(), b[MDN_BUF_CRITIC], cudaMemcpyHostToDevice,
                                   sim->stream), "upload critic");
        cuda_check(cudaMemcpyAsync(sim->buf[MDN_BUF_RAPTOR], raptor, sizeof(*raptor), cudaMemcpyHostToDevice, sim->stream),
                   "upload raptor");
        cuda_check(cudaMemcpyAsync(sim->buf[MDN_BUF_PHYSICS], &params, sizeof(params), cudaMemcpyHostToDevice, sim->stream),
                   "upload physics");
        for (int id : {MDN_BUF_OBS, MDN_BUF_CO, MDN_BUF_ACTIONS, MDN_BUF_LOGP, MDN_BUF_VALUES, MDN_BUF_REWARDS,
                       MDN_BUF_NEXT_VALUES, MDN_BUF_TERMINATED, MDN_BUF_TRUNCATED, MDN_BUF_ADVANTAGES, MDN_BUF_RETURNS,
                       MDN_BUF_CONTACT_ID, MDN_BUF_TASK_STATES})
            cuda_check(cudaMemsetAsync(sim->buf[id], 0, b[id], sim->stream), "clear rollout buffers");
        cuda_check(cudaMemsetAsync(sim->buf[MDN_BUF_BANK_ACTIVE_IDS], 0xff, b[MDN_BUF_BANK_ACTIVE_IDS], sim->stream),
                   "clear bank ids");
        // Launch shapes; MDN_ADVANCE_GROUP (1 or 2) overrides the advance
        // kernel's lanes per environment and MDN_ACT_THREADS (1 or 4) the
        // actor's threads per environment, for tuning.
        const char* group_env = std::getenv("MDN_ADVANCE_GROUP");
        const char* act_env = std::getenv("MDN_ACT_THREADS");
        sim->plan = plan_step(n, dev->sm_count, group_env ? std::atoi(group_env) : 0, act_env ? std::atoi(act_env) : 0);
        mdn_domain_stress_range(&sim->runtime.domain_range);  // runtime config off (main.mm:532)
        cuda_check(launch_reset(sim->args(0), true, sim->stream), "reset");
        cuda_check(cudaStreamSynchronize(sim->stream), "mdn_sim_create");
        dev->sims.push_back(sim.get());
        *out = sim.release();
    });
}

extern "C" int mdn_sim_destroy(mdn_sim* sim) {
    return guarded([&] {
        if (!sim) return;
        use_device(sim->dev);
        cudaStreamSynchronize(sim->stream);
        sim->release_graphs();
        for (int id = 0; id < MDN_BUF_COUNT; id++) cudaFree(sim->buf[id]);
        cudaFree(sim->world_soa);
        cudaFree(sim->reset_mem);
        cudaFree(sim->wide_partials);
        cudaFree(sim->wide_error);
        delete sim->wide;
        cudaFree(sim->lay_mem);
        delete sim->lay;
        cudaFree(sim->report_dev);
        cudaEventDestroy(sim->ev_start);
        cudaEventDestroy(sim->ev_stop);
        if (sim->fork.fork) cudaEventDestroy(sim->fork.fork);
        if (sim->fork.join) cudaEventDestroy(sim->fork.join);
        if (sim->fork.side) cudaStreamDestroy(sim->fork.side);
        cudaStreamDestroy(sim->stream);
        auto& v = sim->dev->sims;
        v.erase(std::remove(v.begin(), v.end(), sim), v.end());
        delete sim;
    });
}

extern "C" int mdn_sim_reset(mdn_sim* sim) {
    return guarded([&] {
        checked(sim);
        cuda_check(launch_reset(sim->args(0), true, sim->stream), "reset");
    });
}

extern "C" int mdn_sim_set_config(mdn_sim* sim, const mdn_sim_config* cfg) {
    return guarded([&] {
        checked(sim);
        require(cfg != nullptr, MDN_ERR_INVALID, "null config");
        require(cfg->n == sim->cfg.n, MDN_ERR_INVALID, "cannot resize simulator");  // main.mm:567
        validate_config(*cfg);
        cuda_check(cudaStreamSynchronize(sim->stream), "set_config");
        sim->cfg = *cfg;
        sim->cfg.tick = 0;
        sim->release_graphs();  // kernel arguments captured by value
    });
}

extern "C" int mdn_sim_get_config(mdn_sim* sim, mdn_sim_config* out) {
    return guarded([&] {
        checked(sim);
        require(out != nullptr, MDN_ERR_INVALID, "null out");
        *out = sim->cfg;
    });
}

extern "C" int mdn_sim_step(mdn_sim* sim, uint32_t tick) {
    return guarded([&] {
        checked(sim);
        require(tick < sim->horizon, MDN_ERR_INVALID, "tick must be below the horizon");
        cuda_check(launch_step(sim->args(tick), sim->plan, sim->nominal, sim->stream, sim->wide, true, nullptr, sim->lay),
                   "step");
    });
}

extern "C" int mdn_sim_collect(mdn_sim* sim, uint32_t steps) {
    return guarded([&] {
        checked(sim);
        if (steps == 0) steps = sim->horizon;
        cudaGraphExec_t exec = nullptr;
        for (auto& g : sim->graphs)
            if (g.first == steps) exec = g.second;
        if (!exec) {
            // Sim::collect (main.mm:576-598): one command stream of `steps`
            // policy steps, rows at tick % horizon. Captured once per length.
            cudaGraph_t graph;
            cuda_check(cudaStreamBeginCapture(sim->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
            cudaError_t launch = cudaSuccess;
            // Inside the rollout each step's ended episodes are reset by the
            // next step's k_reset_sense, beside its k_sense; the last step
            // flushes them, so the state after a collect is the same as after
            // single steps.
            for (uint32_t t = 0; t < steps && launch == cudaSuccess; t++) {
                SimArgs a = sim->args(t % sim->horizon);
                a.phase = t & 1u;
                launch = launch_step(a, sim->plan, sim->nominal, sim->stream, sim->wide, t + 1 == steps,
                                     t > 0 ? &sim->fork : nullptr, sim->lay);
            }
            const cudaError_t end = cudaStreamEndCapture(sim->stream, &graph);
            cuda_check(launch, "capture step");
            cuda_check(end, "end capture");
            const cudaError_t inst = cudaGraphInstantiate(&exec, graph, 0);
            cudaGraphDestroy(graph);
            cuda_check(inst, "graph instantiate");
            sim->graphs.emplace_back(steps, exec);
        }
        cuda_check(cudaEventRecord(sim->ev_start, sim->stream), "event");
        cuda_check(cudaGraphLaunch(exec, sim->stream), "graph launch");
        cuda_check(cudaEventRecord(sim->ev_stop, sim->stream), "event");
    });
}

extern "C" int mdn_sim_set_contact_audit(mdn_sim* sim, int enabled, float safety_margin_m) {
    return guarded([&] {
        checked(sim);
        require(std::isfinite(safety_margin_m), MDN_ERR_INVALID, "contact audit: margin must be finite");
        cuda_check(cudaStreamSynchronize(sim->stream), "contact audit");
        if (enabled && sim->bytes[MDN_BUF_CONTACT_AUDIT] == 0) {
            const size_t bytes = size_t(sim->n) * sim->horizon * sizeof(mdn_contact_audit);
            void* p = nullptr;
            const cudaError_t e = cudaMalloc(&p, bytes);
            require(e == cudaSuccess, MDN_ERR_NOMEM, std::string("contact audit buffer: ") + cudaGetErrorString(e));
            cudaFree(sim->buf[MDN_BUF_CONTACT_AUDIT]);
            sim->buf[MDN_BUF_CONTACT_AUDIT] = p;
            sim->bytes[MDN_BUF_CONTACT_AUDIT] = bytes;
            cuda_check(cudaMemset(p, 0, bytes), "clear contact audit");
        }
        sim->audit_enabled = enabled != 0;
        sim->audit_margin = safety_margin_m;
        sim->release_graphs();  // kernel arguments are captured by value
    });
}

extern "C" int mdn_sim_set_delay_rehearsal(mdn_sim* sim, int enabled) {
    return guarded([&] {
        checked(sim);
        cuda_check(cudaStreamSynchronize(sim->stream), "delay rehearsal");
        sim->delay_rehearsal = enabled != 0;
        sim->release_graphs();  // kernel arguments are captured by value
    });
}

namespace {
// (Re)allocate a simulator buffer of `bytes` filled with byte `fill`.
void sim_realloc(mdn_sim* sim, int id, size_t bytes, int fill) {
    void* p = nullptr;
    const cudaError_t e = cudaMalloc(&p, std::max<size_t>(bytes, 16));
    require(e == cudaSuccess, MDN_ERR_NOMEM, std::string("challenge bank buffer: ") + cudaGetErrorString(e));
    const cudaError_t m = cudaMemset(p, fill, std::max<size_t>(bytes, 16));
    if (m != cudaSuccess) {
        cudaFree(p);
        cuda_check(m, "clear challenge bank buffer");
    }
    cudaFree(sim->buf[id]);
    sim->buf[id] = p;
    sim->bytes[id] = bytes;
}
}  // namespace

extern "C" int mdn_sim_set_challenge_bank(mdn_sim* sim, const mdn_world* bank_worlds, const mdn_bank_control* control) {
    return guarded([&] {
        checked(sim);
        cuda_check(cudaStreamSynchronize(sim->stream), "challenge bank");
        if (!control || control->enabled == 0) {
            sim->bank = mdn_bank_control{};
            sim->release_graphs();
            return;
        }
        const mdn_bank_control c = *control;
        require(c.schedule_stride >= 1 && c.schedule_stride <= 65536, MDN_ERR_INVALID,
                "challenge bank: schedule_stride must be 1..65536");
        require(c.bank_count <= (1u << 20), MDN_ERR_INVALID, "challenge bank: at most 2^20 levels");
        require(c.bank_count == 0 || bank_worlds != nullptr, MDN_ERR_INVALID, "challenge bank: null worlds");
        for (uint32_t k = 0; k < c.bank_count; k++) {
            const mdn_world& w = bank_worlds[k];
            require(w.count <= 16, MDN_ERR_INVALID, "challenge bank: a world holds more than 16 obstacles");
            for (uint32_t o = 0; o < w.count; o++)
                require(w.obstacles[o].kind <= 3, MDN_ERR_INVALID, "challenge bank: unknown obstacle kind");
        }
        const size_t n = sim->n;
        sim_realloc(sim, MDN_BUF_BANK_WORLDS, size_t(c.bank_count) * sizeof(mdn_world), 0);
        if (c.bank_count)
            cuda_check(cudaMemcpy(sim->buf[MDN_BUF_BANK_WORLDS], bank_worlds, size_t(c.bank_count) * sizeof(mdn_world),
                                  cudaMemcpyHostToDevice),
                       "upload challenge bank");
        if (sim->bytes[MDN_BUF_BANK_SCHEDULE] != n * c.schedule_stride * sizeof(uint32_t))
            sim_realloc(sim, MDN_BUF_BANK_SCHEDULE, n * c.schedule_stride * sizeof(uint32_t), 0);
        const size_t rows = n * sim->horizon;
        if (sim->bytes[MDN_BUF_BANK_TRANSITION_IDS] == 0)
            sim_realloc(sim, MDN_BUF_BANK_TRANSITION_IDS, rows * sizeof(uint32_t), 0xff);
        if (sim->bytes[MDN_BUF_RAW_ADVANTAGES] == 0) sim_realloc(sim, MDN_BUF_RAW_ADVANTAGES, rows * sizeof(float), 0);
        sim->bank = c;
        sim->release_graphs();  // kernel arguments are captured by value
    });
}

extern "C" void mdn_domain_stress_range(mdn_domain_range* out) {
    if (out) *out = mdn_domain_range{0.90f, 1.10f, 0.90f, 1.10f, 0.90f, 1.10f, 0.75f, 1.35f, 0.75f, 1.35f, 1.15f};
}

namespace mdn {
// Sim.runtime_control (main.mm:532-537); the per-env plant buffer is
// allocated the first time the config is switched on.
// The reference's initial runtime buffer (main.mm:532): off, with the stress
// range filled in. Checkpoints store these bytes and compare them on resume.
mdn_runtime_config default_runtime() {
    mdn_runtime_config r{};
    mdn_domain_stress_range(&r.domain_range);
    return r;
}

void set_runtime(mdn_sim* sim, const mdn_runtime_config* runtime) {
    cuda_check(cudaStreamSynchronize(sim->stream), "runtime config");
    if (runtime && runtime->enabled && sim->bytes[MDN_BUF_ENV_PHYSICS] == 0)
        sim_realloc(sim, MDN_BUF_ENV_PHYSICS, size_t(sim->n) * sizeof(mdn_physics_params), 0);
    sim->runtime = runtime ? *runtime : default_runtime();
    sim->release_graphs();  // kernel arguments are captured by value
}
}  // namespace mdn

extern "C" int mdn_sim_set_runtime(mdn_sim* sim, const mdn_runtime_config* runtime) {
    return guarded([&] {
        checked(sim);
        set_runtime(sim, runtime);
    });
}

extern "C" int mdn_sim_last_collect_ms(mdn_sim* sim, float* ms) {
    return guarded([&] {
        checked(sim);
        sync_event(sim->dev, sim->ev_stop, "event sync");
        cuda_check(cudaEventElapsedTime(&sim->last_collect_ms, sim->ev_start, sim->ev_stop), "elapsed");
        if (ms) *ms = sim->last_collect_ms;
    });
}

namespace mdn {
// Callers that wrote the worlds buffer directly (checkpoint load) refresh the mirror.
void refresh_world_mirror(mdn_sim* sim) { cuda_check(launch_world_mirror(sim->args(0), sim->stream), "world mirror"); }
}  // namespace mdn

extern "C" int mdn_sim_buffer(mdn_sim* sim, int id, void** dev_ptr, size_t* bytes) {
    return guarded([&] {
        checked(sim);
        require(id >= 0 && id < MDN_BUF_COUNT, MDN_ERR_INVALID, "unknown buffer id");
        if (dev_ptr) *dev_ptr = sim->buf[id];
        if (bytes) *bytes = sim->bytes[id];
    });
}

extern "C" int mdn_sim_download(mdn_sim* sim, int id, void* host, size_t offset, size_t bytes) {
    return guarded([&] {
        checked(sim);
        require(id >= 0 && id < MDN_BUF_COUNT, MDN_ERR_INVALID, "unknown buffer id");
        require(host != nullptr || bytes == 0, MDN_ERR_INVALID, "null host pointer");
        require(offset <= sim->bytes[id] && bytes <= sim->bytes[id] - offset, MDN_ERR_INVALID, "download out of range");
        cuda_check(cudaMemcpyAsync(host, static_cast<char*>(sim->buf[id]) + offset, bytes, cudaMemcpyDeviceToHost,
                                   sim->stream), "download");
        sync_stream(sim->dev, sim->stream, "download");
    });
}

extern "C" int mdn_sim_upload(mdn_sim* sim, int id, const void* host, size_t offset, size_t bytes) {
    return guarded([&] {
        checked(sim);
        require(id >= 0 && id < MDN_BUF_COUNT, MDN_ERR_INVALID, "unknown buffer id");
        require(host != nullptr || bytes == 0, MDN_ERR_INVALID, "null host pointer");
        require(offset <= sim->bytes[id] && bytes <= sim->bytes[id] - offset, MDN_ERR_INVALID, "upload out of range");
        cuda_check(cudaMemcpyAsync(static_cast<char*>(sim->buf[id]) + offset, host, bytes, cudaMemcpyHostToDevice,
                                   sim->stream), "upload");
        if (id == MDN_BUF_WORLDS) cuda_check(launch_world_mirror(sim->args(0), sim->stream), "world mirror");
        cuda_check(cudaStreamSynchronize(sim->stream), "upload");
        if (id == MDN_BUF_PHYSICS) {  // k_advance takes the nominal plant by value
            std::memcpy(reinterpret_cast<char*>(&sim->nominal) + offset, host, bytes);
            sim->release_graphs();
        }
    });
}

extern "C" int mdn_sim_report(mdn_sim* sim, double out[10]) {
    return guarded([&] {
        checked(sim);
        require(out != nullptr, MDN_ERR_INVALID, "null out");
        // Sim::report (main.mm:599-602), reduced on the GPU (k_report): the
        // host reads back ten doubles instead of every run record.
        if (!sim->report_dev)
            cuda_check(cudaMalloc(&sim->report_dev, 10 * sizeof(double)), "report buffer");
        cuda_check(launch_report(sim->args(0), sim->report_dev, sim->stream), "report");
        double v[10];
        cuda_check(cudaMemcpyAsync(v, sim->report_dev, sizeof(v), cudaMemcpyDeviceToHost, sim->stream), "report");
        sync_stream(sim->dev, sim->stream, "report");
        std::memcpy(out, v, sizeof(v));
    });
}

extern "C" int mdn_sim_dims(mdn_sim* sim, uint32_t* n, uint32_t* horizon, uint32_t* actor_params,
                            uint32_t* critic_params) {
    return guarded([&] {
        checked(sim);
        if (n) *n = sim->n;
        if (horizon) *horizon = sim->horizon;
        if (actor_params) *actor_params = sim->actor_params;
        if (critic_params) *critic_params = sim->critic_params;
    });
}

extern "C" int mdn_sim_actor_means(mdn_sim* sim, const float* obs, uint32_t rows, float* means) {
    return guarded([&] {
        checked(sim);
        require(obs != nullptr && means != nullptr && rows > 0, MDN_ERR_INVALID, "actor means: bad argument");
        MlpShape net;
        if (sim->layered) {
            net = sim->lay->actor;
        } else {
            net.in = kActorObs;
            net.hidden = sim->actor_hidden;
            net.layers = 1;
            net.out = kActions;
            net.activation = kActTanh;
            net.log_std = true;
        }
        const size_t x_floats = size_t(rows) * kActorObs, h_floats = size_t(rows) * net.hidden;
        float* mem = nullptr;
        const cudaError_t e = cudaMalloc(&mem, (x_floats + 2 * h_floats + size_t(rows) * kActions) * sizeof(float));
        require(e == cudaSuccess, MDN_ERR_NOMEM, std::string("actor means: cudaMalloc failed: ") + cudaGetErrorString(e));
        struct Free {
            float* p;
            ~Free() { cudaFree(p); }
        } guard{mem};
        float* out = mem + x_floats + 2 * h_floats;
        cuda_check(cudaMemcpyAsync(mem, obs, x_floats * sizeof(float), cudaMemcpyHostToDevice, sim->stream),
                   "actor means: upload");
        cuda_check(launch_network_forward(net, static_cast<const float*>(sim->buf[MDN_BUF_ACTOR]), mem, rows,
                                          mem + x_floats, mem + x_floats + h_floats, out, true, sim->stream),
                   "actor means: forward");
        cuda_check(cudaMemcpyAsync(means, out, size_t(rows) * kActions * sizeof(float), cudaMemcpyDeviceToHost,
                                   sim->stream),
                   "actor means: download");
        sync_stream(sim->dev, sim->stream, "actor means");
        // The geometry prior (ppo.hpp:77) after the output layer and its bias.
        for (uint32_t r = 0; r < rows; r++)
            for (int a = 0; a < 3; a++) means[size_t(r) * kActions + a] += obs[size_t(r) * kActorObs + kActorObs - 3 + a];
    });
}

extern "C" int mdn_sim_profile_step(mdn_sim* sim, uint32_t tick, float ms[3]) {
    return guarded([&] {
        checked(sim);
        require(ms != nullptr && tick < sim->horizon, MDN_ERR_INVALID, "profile_step: bad argument");
        cudaEvent_t ev[4];
        for (auto& e : ev) cuda_check(cudaEventCreate(&e), "event");
        const cudaError_t launch =
            launch_step_profiled(sim->args(tick), sim->plan, sim->nominal, sim->stream, ev, sim->wide, sim->lay);
        const cudaError_t wait = cudaEventSynchronize(ev[3]);
        for (int k = 0; k < 3 && launch == cudaSuccess && wait == cudaSuccess; k++) cudaEventElapsedTime(&ms[k], ev[k], ev[k + 1]);
        for (auto& e : ev) cudaEventDestroy(e);
        cuda_check(launch, "profiled step");
        cuda_check(wait, "profiled step");
    });
}

extern "C" int mdn_selftest_division(mdn_device* dev, uint64_t samples, uint64_t seed, uint64_t* mismatches) {
    return guarded([&] {
        require(dev != nullptr && mismatches != nullptr, MDN_ERR_INVALID, "division self-test: null argument");
        use_device(dev);
        cuda_check(division_check(samples, seed, mismatches, dev->sm_count), "division self-test");
    });
}

extern "C" int mdn_selftest_barrier_timeout(mdn_device* dev, uint64_t limit_cycles, int arrive) {
    return guarded([&] {
        require(dev != nullptr && limit_cycles > 0 && limit_cycles < (uint64_t(1) << 40), MDN_ERR_INVALID,
                "barrier self-test: bad argument");
        use_device(dev);
        uint32_t timed_out = 0;
        cuda_check(barrier_selftest((long long)limit_cycles, arrive, &timed_out), "barrier self-test");
        require(timed_out == 0, MDN_ERR_TIMEOUT,
                "barrier self-test: the bounded wait gave up after " + std::to_string(limit_cycles) + " cycles");
    });
}

extern "C" int mdn_device_fp32_peak(mdn_device* dev, double* tflops) {
    return guarded([&] {
        require(dev && tflops, MDN_ERR_INVALID, "null argument");
        use_device(dev);
        cuda_check(fp32_peak(dev->sm_count, tflops), "fp32 peak");
    });
}

// navigation_task_default_config (navigation_tasks.hpp:97-142) with the
// overrides of navigation_training::task_settings (navigation_training.hpp:7-14).
extern "C" int mdn_task_settings(uint32_t stage, uint32_t family, float difficulty, mdn_task_config* out) {
    return guarded([&] {
        require(out != nullptr, MDN_ERR_INVALID, "null out");
        require(stage <= 2u && std::isfinite(difficulty) && difficulty >= 0.0f && difficulty <= 1.0f, MDN_ERR_INVALID,
                "unsupported task stage/difficulty");
        if (stage == 0u || stage == 1u) require(family == 0u, MDN_ERR_INVALID, "open/hold stages use family 0");
        else
            require(family == 1u || family == 2u || family == 4u || family == 5u || family == 12u, MDN_ERR_INVALID,
                    "clutter stage supports families 1, 2, 4, 5, 12");
        mdn_task_config c{};
        c.generation_version = 1u;
        c.family = family;
        c.stage = stage;
        c.objective = 1u;  // final hold
        c.require_detour = 0u;
        c.max_generation_attempts = 64u;
        c.max_nav_steps = 400u;
        c.scene_distance_m = 8.0f;
        c.difficulty = difficulty;
        c.minimum_endpoint_clearance_m = 0.30f;
        c.minimum_witness_clearance_m = 0.02f;
        c.goal_radius_m = 0.35f;
        c.stable_speed_mps = 0.50f;
        c.stable_hold_s = 0.20f;
        c.nav_period_s = 0.05f;
        c.initial_speed_min_mps = 0.0f;
        c.initial_speed_max_mps = 0.0f;
        c.progress_reward_per_m = 2.0f;
        c.time_cost_per_s = 0.20f;
        c.contact_penalty = 10.0f;
        c.stable_arrival_bonus = 10.0f;
        c.command_smoothness_weight = 0.05f;
        const float start_low[3] = {-1.0f, -2.0f, 0.8f}, start_high[3] = {1.0f, 2.0f, 2.4f};
        const float goal_low[3] = {-1.2f, -4.0f, 0.5f}, goal_high[3] = {13.2f, 4.0f, 4.5f};
        for (int a = 0; a < 3; a++) {
            c.start_min_xyz[a] = start_low[a];
            c.start_max_xyz[a] = start_high[a];
            c.goal_min_xyz[a] = goal_low[a];
            c.goal_max_xyz[a] = goal_high[a];
        }
        if (stage == 1u) {
            c.goal_distance_min_m = 0.8f;
            c.goal_distance_max_m = 2.0f;
            for (int a = 0; a < 3; a++) {
                c.start_min_xyz[a] = goal_low[a];
                c.start_max_xyz[a] = goal_high[a];
            }
        } else if (stage == 2u) {
            c.goal_distance_min_m = 2.0f;
            c.goal_distance_max_m = 7.0f;
        } else {
            c.goal_distance_min_m = 2.0f;
            c.goal_distance_max_m = 6.0f;
        }
        // navigation_training::task_settings overrides
        c.time_cost_per_s = .2f;
        c.command_smoothness_weight = .05f;
        c.initial_speed_max_mps = stage == 1u ? .5f : 1.0f;
        *out = c;
    });
}

namespace {
// The configuration checks of navigation_generate_task
// (navigation_tasks.hpp:347-379): validity of every field, family 0 for the
// open/hold stages, the clutter families, and start/goal boxes inside the
// room by the endpoint clearance.
bool task_config_ok(const mdn_task_config& c) {
    using std::isfinite;
    if (c.generation_version != 1u || c.stage > 2u || c.objective > 1u || c.family > 16u || c.require_detour > 1u ||
        !isfinite(c.scene_distance_m) || c.scene_distance_m < 3.0f || c.scene_distance_m > 10.0f ||
        !isfinite(c.difficulty) || c.difficulty < 0.0f || c.difficulty > 1.0f || !isfinite(c.goal_distance_min_m) ||
        !isfinite(c.goal_distance_max_m) || c.goal_distance_min_m <= c.goal_radius_m ||
        c.goal_distance_max_m < c.goal_distance_min_m || !isfinite(c.minimum_endpoint_clearance_m) ||
        c.minimum_endpoint_clearance_m < 0.30f || !isfinite(c.minimum_witness_clearance_m) ||
        c.minimum_witness_clearance_m < 0.02f || !isfinite(c.goal_radius_m) || c.goal_radius_m <= 0.0f ||
        !isfinite(c.stable_speed_mps) || c.stable_speed_mps < 0.0f || !isfinite(c.stable_hold_s) ||
        c.stable_hold_s < 0.0f || !isfinite(c.nav_period_s) || c.nav_period_s <= 0.0f ||
        !isfinite(c.initial_speed_min_mps) || !isfinite(c.initial_speed_max_mps) || c.initial_speed_min_mps < 0.0f ||
        c.initial_speed_max_mps < c.initial_speed_min_mps || !isfinite(c.progress_reward_per_m) ||
        c.progress_reward_per_m < 0.0f || !isfinite(c.time_cost_per_s) || c.time_cost_per_s < 0.0f ||
        !isfinite(c.contact_penalty) || c.contact_penalty < 0.0f || !isfinite(c.stable_arrival_bonus) ||
        c.stable_arrival_bonus < 0.0f || !isfinite(c.command_smoothness_weight) || c.command_smoothness_weight < 0.0f ||
        c.max_nav_steps == 0u || c.max_generation_attempts == 0u)
        return false;
    if ((c.stage == 0u || c.stage == 1u) && c.family != 0u) return false;
    if (c.stage == 2u && !(c.family == 1u || c.family == 2u || c.family == 4u || c.family == 5u || c.family == 12u))
        return false;
    for (int axis = 0; axis < 3; axis++) {
        const float room_min = axis == 0 ? -2.0f : (axis == 1 ? -5.0f : 0.0f);
        const float room_max = axis == 0 ? 14.0f : 5.0f;
        const float m = c.minimum_endpoint_clearance_m;
        if (!isfinite(c.start_min_xyz[axis]) || !isfinite(c.start_max_xyz[axis]) || !isfinite(c.goal_min_xyz[axis]) ||
            !isfinite(c.goal_max_xyz[axis]) || c.start_min_xyz[axis] >= c.start_max_xyz[axis] ||
            c.goal_min_xyz[axis] >= c.goal_max_xyz[axis] || c.start_min_xyz[axis] < room_min + m ||
            c.start_max_xyz[axis] > room_max - m || c.goal_min_xyz[axis] < room_min + m ||
            c.goal_max_xyz[axis] > room_max - m)
            return false;
    }
    return true;
}
}  // namespace

// navigation_training::configure (navigation_training.hpp:16-25): install the
// task control and reset every environment.
extern "C" int mdn_sim_configure_tasks(mdn_sim* sim, const mdn_task_control* control, float domain_amplitude) {
    return guarded([&] {
        checked(sim);
        require(control != nullptr, MDN_ERR_INVALID, "null task control");
        require(std::isfinite(domain_amplitude) && domain_amplitude >= 0.0f && domain_amplitude <= 1.0f,
                MDN_ERR_INVALID, "domain amplitude must be0..1");
        if (control->enabled) {
            require(std::fabs(control->config.nav_period_s - float(sim->cfg.substeps) * 0.01f) < 1e-6f,
                    MDN_ERR_INVALID, "task/simulator clock mismatch");
            require(sim->bank.enabled == 0, MDN_ERR_INVALID, "task generator and frozen bank cannot both own the world");
        }
        cuda_check(cudaStreamSynchronize(sim->stream), "configure tasks");
        mdn_runtime_config runtime = default_runtime();
        if (control->enabled) {
            runtime.enabled = 1;
            runtime.domain_amplitude = domain_amplitude;
            runtime.domain_seed = 0x3f84d5b5u;
        }
        set_runtime(sim, &runtime);
        sim->task_ctl = *control;
        sim->task_config_ok = task_config_ok(control->config) ? 1u : 0u;
        sim->release_graphs();  // kernel arguments captured by value
        cuda_check(launch_reset(sim->args(0), true, sim->stream), "reset");
    });
}

// navigation_training::validate_rollout (navigation_training.hpp:27-35).
extern "C" int mdn_sim_validate_tasks(mdn_sim* sim) {
    return guarded([&] {
        checked(sim);
        std::vector<mdn_task_state> tasks(sim->n);
        cuda_check(cudaMemcpyAsync(tasks.data(), sim->buf[MDN_BUF_TASK_STATES], sim->bytes[MDN_BUF_TASK_STATES],
                                   cudaMemcpyDeviceToHost, sim->stream), "download task states");
        cuda_check(cudaStreamSynchronize(sim->stream), "validate tasks");
        std::vector<mdn_physics_params> plants;
        if (sim->runtime.enabled) {
            plants.resize(sim->n);
            cuda_check(cudaMemcpyAsync(plants.data(), sim->buf[MDN_BUF_ENV_PHYSICS], sim->bytes[MDN_BUF_ENV_PHYSICS],
                                       cudaMemcpyDeviceToHost, sim->stream), "download episode plants");
            cuda_check(cudaStreamSynchronize(sim->stream), "validate tasks");
        }
        for (uint32_t env = 0; env < sim->n; env++) {
            require(tasks[env].valid && tasks[env].generation_status == 4u, MDN_ERR_STATE,
                    "task generation rejected env=" + std::to_string(env) +
                        " status=" + std::to_string(tasks[env].generation_status));
            if (!plants.empty())
                require(std::isfinite(plants[env].mass) && plants[env].mass > 0, MDN_ERR_STATE,
                        "episode dynamics sample rejected");
        }
    });
}
