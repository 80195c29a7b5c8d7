/* C++ host veneer over the C-ABI of mdn.h: the reference's host classes and
 * the navigation_training helpers, so a port of the reference's C++/ObjC++
 * trainers (navigation_training.hpp:7-170, train_navigation main.mm:1805-1862)
 * keeps its class and function names. Header-only; link libmdn.so.
 *
 *   Metal (main.mm:44-72)        -> mdn::host::Device  (finish() = Metal::finish)
 *   Sim (main.mm:516-603)        -> mdn::host::Sim     (buffers: download/upload
 *                                                        instead of MTLBuffer.contents)
 *   PPOTrainer (main.mm:1110-1476) -> mdn::host::PPOTrainer
 *   navigation_training::*       -> mdn::host::navigation_training::*
 *
 * Errors: every failing call throws mdn::host::Error (a std::runtime_error,
 * as the reference's require() does, main.mm:27) carrying the MDN_ERR_* code. */
#pragma once

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <iostream>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "mdn.h"

namespace mdn {
namespace host {

static_assert(sizeof(mdn_checkpoint_header) == 136, "PPOFIX1 header (main.mm:978-984)");

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& what) : std::runtime_error(what), code(c) {}
};

inline void check(int status) {
    if (status != MDN_OK) throw Error(status, mdn_last_error());
}

inline void require(bool ok, const std::string& what) {
    if (!ok) throw Error(MDN_ERR_INVALID, what);
}

// The reference's Metal object: one device (main.mm:44-72).
class Device {
public:
    explicit Device(int gpu = 0) { check(mdn_device_open(gpu, &h_)); }
    ~Device() {
        if (h_) {
            mdn_comm_destroy(h_);
            mdn_device_close(h_);
        }
    }
    Device(const Device&) = delete;
    Device& operator=(const Device&) = delete;
    // Metal::finish: wait for the queued work, raise device errors, return GPU seconds.
    double finish() {
        double s = 0.0;
        check(mdn_sync(h_, &s));
        return s;
    }
    mdn_device* get() const { return h_; }

private:
    mdn_device* h_ = nullptr;
};

// The reference's Sim (main.mm:516-603).
class Sim {
public:
    Sim(Device& device, const mdn_sim_config& config, uint32_t horizon, const mdn_raptor_weights* raptor = nullptr,
        const mdn_physics_params* physics = nullptr, const mdn_rollout_shape* shape = nullptr)
        : device_(&device), cfg(config), horizon(horizon) {
        mdn_raptor_weights packaged;
        if (!raptor) {
            check(mdn_raptor_load(default_raptor_path().c_str(), &packaged));
            raptor = &packaged;
        }
        check(mdn_sim_create(device.get(), &config, shape, horizon, raptor, physics, &h_));
        uint32_t n = 0, t = 0;
        check(mdn_sim_dims(h_, &n, &t, &actor_params, &critic_params));
    }
    ~Sim() {
        if (h_) mdn_sim_destroy(h_);
    }
    Sim(const Sim&) = delete;
    Sim& operator=(const Sim&) = delete;

    void reset() { check(mdn_sim_reset(h_)); }
    void set_config(const mdn_sim_config& c) {
        check(mdn_sim_set_config(h_, &c));
        cfg = c;
    }
    // Sim::collect(cb, count): `count` policy steps (0 = the horizon).
    void collect(uint32_t count = 0) { check(mdn_sim_collect(h_, count)); }
    void step(uint32_t tick) { check(mdn_sim_step(h_, tick)); }
    // Host copies of a public buffer (MDN_BUF_*), the reference's .contents.
    template <class T>
    std::vector<T> download(int id) const {
        void* p = nullptr;
        size_t bytes = 0;
        check(mdn_sim_buffer(h_, id, &p, &bytes));
        std::vector<T> out(bytes / sizeof(T));
        check(mdn_sim_download(h_, id, out.data(), 0, out.size() * sizeof(T)));
        return out;
    }
    template <class T>
    void upload(int id, const std::vector<T>& values, size_t offset_bytes = 0) {
        check(mdn_sim_upload(h_, id, values.data(), offset_bytes, values.size() * sizeof(T)));
    }
    void upload(int id, const void* host, size_t bytes, size_t offset_bytes = 0) {
        check(mdn_sim_upload(h_, id, host, offset_bytes, bytes));
    }
    // Sim::report aggregates (main.mm:599-602), printed like the reference.
    std::array<double, 10> report(const std::string& label = "", double wall = 0.0) {
        std::array<double, 10> r{};
        check(mdn_sim_report(h_, r.data()));
        if (!label.empty())
            std::cout << label << " episodes=" << r[0] << " success=" << r[1] << " collision=" << r[2]
                      << " timeout=" << r[3] << " wall_s=" << wall << "\n";
        return r;
    }
    // NavigationPolicy::raw_mean (deployment.hpp) of the current actor for
    // observation rows [rows][184], evaluated on the GPU: [rows][4] means.
    std::vector<float> actor_means(const std::vector<float>& obs) const {
        const uint32_t rows = uint32_t(obs.size() / 184);
        std::vector<float> means(size_t(rows) * 4);
        check(mdn_sim_actor_means(h_, obs.data(), rows, means.data()));
        return means;
    }
    float last_collect_ms() const {
        float ms = 0.0f;
        check(mdn_sim_last_collect_ms(h_, &ms));
        return ms;
    }
    void set_runtime(const mdn_runtime_config* runtime) { check(mdn_sim_set_runtime(h_, runtime)); }
    void set_delay_rehearsal(bool on) { check(mdn_sim_set_delay_rehearsal(h_, on ? 1 : 0)); }

    mdn_sim* get() const { return h_; }
    Device& device() const { return *device_; }

    mdn_sim_config cfg;
    uint32_t horizon;
    uint32_t actor_params = 0, critic_params = 0;

    static std::string default_raptor_path() {
        const char* env = std::getenv("MDN_RAPTOR");
        return env && *env ? env : std::string("metal-drone-nav_b200/assets/raptor.bin");
    }

private:
    Device* device_;
    mdn_sim* h_ = nullptr;
};

// The reference's PPOTrainer (main.mm:1110-1476).
class PPOTrainer {
public:
    explicit PPOTrainer(Sim& sim, uint32_t epochs = 2, uint32_t minibatch_rows = 0) : sim_(&sim) {
        check(mdn_ppo_create(sim.get(), epochs, minibatch_rows, &h_));
    }
    ~PPOTrainer() {
        if (h_) mdn_ppo_destroy(h_);
    }
    PPOTrainer(const PPOTrainer&) = delete;
    PPOTrainer& operator=(const PPOTrainer&) = delete;

    void rollout_update(uint32_t rollout_index) { check(mdn_ppo_rollout_update(h_, rollout_index)); }
    std::array<float, 4> metric_mean() const {
        std::array<float, 4> m{};
        check(mdn_ppo_metrics(h_, m.data()));
        return m;
    }
    uint64_t optimizer_step() const { return state().first; }
    uint32_t completed_rollouts() const { return state().second; }
    void set_completed_rollouts(uint32_t done) { check(mdn_ppo_set_state(h_, optimizer_step(), done)); }
    float last_update_ms() const {
        float ms = 0.0f;
        check(mdn_ppo_last_update_ms(h_, &ms));
        return ms;
    }
    void set_tensor_cores(bool on) { check(mdn_ppo_set_tensor_cores(h_, on ? 1 : 0)); }
    void load_checkpoint(const std::string& path, uint32_t family, uint32_t horizon, uint32_t n, uint32_t seed) {
        check(mdn_ppo_checkpoint_load(h_, path.c_str(), family, horizon, n, seed));
    }
    void save_checkpoint(const std::string& path, uint32_t family, uint32_t seed, uint32_t completed) {
        check(mdn_ppo_checkpoint_save(h_, path.c_str(), family, seed, completed));
    }
    mdn_ppo* get() const { return h_; }

private:
    std::pair<uint64_t, uint32_t> state() const {
        uint64_t step = 0;
        uint32_t done = 0;
        check(mdn_ppo_state(h_, &step, &done));
        return {step, done};
    }
    Sim* sim_;
    mdn_ppo* h_ = nullptr;
};

// ---------------------------------------------------------------------------
// navigation_training (navigation_training.hpp:7-170): goal-arrival task
// settings, configuration and validation, actor loading, evaluation and the
// training loop, over the classes above.
namespace navigation_training {

// task_settings (navigation_training.hpp:7-14): navigation_task_default_config
// plus the trainer's overrides, as an enabled task control.
inline mdn_task_control task_settings(uint32_t stage, uint32_t family) {
    mdn_task_control control{};
    control.enabled = 1;
    check(mdn_task_settings(stage, family, 0.5f, &control.config));
    return control;
}

// configure (:16-25): per-episode plant variation at `amplitude` and the task
// control, then a reset of every environment.
inline void configure(Sim& sim, const mdn_task_control& tasks, float amplitude) {
    check(mdn_sim_configure_tasks(sim.get(), &tasks, amplitude));
}

// validate_rollout (:27-35): every task generated and every plant valid.
inline void validate_rollout(Sim& sim) { check(mdn_sim_validate_tasks(sim.get())); }

// load_actor (:37-61): the actor (and optionally the critic) of a PPOFIX1
// checkpoint into `sim`, without its optimiser or simulator state. A critic of
// another size is an incompatible warm start (this build's critic has the
// reference's 32 inputs, so the 32 -> 64-input migration never applies).
inline void load_actor(Sim& sim, const std::string& path, bool critic = false) {
    mdn_checkpoint_header h{};
    check(mdn_checkpoint_inspect(path.c_str(), &h, nullptr, nullptr));
    require(h.actor_count == sim.actor_params, "task actor dimensions");
    std::ifstream file(path, std::ios::binary);
    require(bool(file), "cannot open " + path);
    file.seekg(sizeof(mdn_checkpoint_header));  // the parameters follow the header
    std::vector<float> actor(h.actor_count);
    file.read(reinterpret_cast<char*>(actor.data()), std::streamsize(actor.size() * sizeof(float)));
    require(bool(file), "task parameter load failed");
    sim.upload(MDN_BUF_ACTOR, actor);
    if (critic) {
        require(h.critic_count == sim.critic_params, "task critic dimensions: incompatible warmstart");
        std::vector<float> values(h.critic_count);
        file.read(reinterpret_cast<char*>(values.data()), std::streamsize(values.size() * sizeof(float)));
        require(bool(file), "task parameter load failed");
        sim.upload(MDN_BUF_CRITIC, values);
    }
}

struct Score {
    double success = 0, collision = 0, timeout = 0, successful_time_s = 0;
};

// evaluate (:63-113): 128 evaluation environments of the task stage, one
// 400-step episode each with the given actor, the per-environment CSV
// (when `output` is set) and the success / collision / timeout fractions.
inline Score evaluate(Device& device, const float* actor, uint32_t stage, uint32_t family, float amplitude,
                      uint32_t seed, const std::string& output = "", uint32_t mode = 17) {
    mdn_sim_config config;
    mdn_sim_config_default(&config);
    config.n = 128;
    config.eval = 1;
    config.mode = mode;
    config.seed = seed;
    config.family = family;
    config.speed = 1.5f;
    config.distance = 8;
    config.max_steps = 400;
    config.geometry_memory = 1;
    Sim sim(device, config, 32);
    const mdn_task_control settings = task_settings(stage, family);
    configure(sim, settings, amplitude);
    sim.upload(MDN_BUF_ACTOR, actor, sim.actor_params * sizeof(float));
    validate_rollout(sim);
    const auto tasks0 = sim.download<mdn_task_state>(MDN_BUF_TASK_STATES);
    sim.collect(400);
    device.finish();
    validate_rollout(sim);
    std::ofstream file;
    if (!output.empty()) {
        const std::filesystem::path destination(output);
        if (destination.has_parent_path()) std::filesystem::create_directories(destination.parent_path());
        file.open(output);
        require(bool(file), "cannot write task evaluation");
        file << "seed,env,stage,family,mode,domain_amplitude,start_x,start_y,start_z,start_yaw,initial_vx,initial_vy,"
                "initial_vz,goal_x,goal_y,goal_z,initial_distance_m,direct_clearance_m,witness_length_m,mass_kg,"
                "success,collision,timeout,time_s,path_m,goal_error_m,final_speed_mps,hold_s,peak_speed_mps,"
                "min_sphere_clearance_m,success_rule\n";
    }
    const auto runs = sim.download<mdn_sim_run>(MDN_BUF_RUNS);
    const auto states = sim.download<mdn_physics_state>(MDN_BUF_STATES);
    const auto tasks = sim.download<mdn_task_state>(MDN_BUF_TASK_STATES);
    const auto plants = sim.download<mdn_physics_params>(MDN_BUF_ENV_PHYSICS);
    const auto nominal = sim.download<mdn_physics_params>(MDN_BUF_PHYSICS);
    Score result;
    for (uint32_t env = 0; env < config.n; env++) {
        const mdn_sim_run& run = runs[env];
        const mdn_task_state& task = tasks0[env];
        const mdn_physics_state& state = states[env];
        require(run.episodes == 1, "evaluation must complete exactly one task per environment");
        result.success += run.successes;
        result.collision += run.collisions;
        result.timeout += run.timeouts;
        result.successful_time_s += run.success_time;
        const float dx = task.goal_position[0] - state.position[0], dy = task.goal_position[1] - state.position[1],
                    dz = task.goal_position[2] - state.position[2];
        const float error = std::sqrt(dx * dx + dy * dy + dz * dz);
        const float speed = std::sqrt(state.linear_velocity[0] * state.linear_velocity[0] +
                                      state.linear_velocity[1] * state.linear_velocity[1] +
                                      state.linear_velocity[2] * state.linear_velocity[2]);
        if (run.successes)
            require(error <= settings.config.goal_radius_m + 1e-5f &&
                        speed <= settings.config.stable_speed_mps + 1e-5f && tasks[env].stable_time_s >= .2f - 1e-6f,
                    "stable-arrival invariant failed");
        if (file.is_open()) {
            const float mass = plants.size() == config.n ? plants[env].mass : nominal[0].mass;
            file << seed << ',' << env << ',' << stage << ',' << task.family << ',' << mode << ',' << amplitude;
            for (float v : task.start_position) file << ',' << v;
            file << ',' << task.start_yaw_rad;
            for (float v : task.start_velocity_world) file << ',' << v;
            for (float v : task.goal_position) file << ',' << v;
            file << ',' << task.initial_distance_m << ',' << task.direct_segment_clearance_m << ','
                 << task.witness_length_m << ',' << mass << ',' << run.successes << ',' << run.collisions << ','
                 << run.timeouts << ',' << run.elapsed << ',' << run.path << ',' << error << ',' << speed << ','
                 << tasks[env].stable_time_s << ',' << run.peak_speed << ',' << run.min_clearance
                 << ",radius0.35_speed0.5_hold0.2\n";
        }
    }
    result.success /= config.n;
    result.collision /= config.n;
    result.timeout /= config.n;
    if (result.success > 0) result.successful_time_s /= result.success * config.n;
    std::cout << "task_eval stage=" << stage << " family=" << family << " seed=" << seed << " amplitude=" << amplitude
              << " mode=" << mode << " success=" << result.success << " collision=" << result.collision
              << " timeout=" << result.timeout << " mean_arrival_s=" << result.successful_time_s << "\n";
    return result;
}

// train (:115-170): task PPO with periodic checkpoints, evaluation and a
// kept best checkpoint (success first, then fewer collisions, then faster
// arrival), resuming from `checkpoint` when it exists.
inline void train(Device& device, uint32_t rollouts, const std::string& checkpoint, const std::string& warmstart,
                  uint32_t stage, uint32_t family, float amplitude, uint32_t seed, uint32_t every = 50) {
    require(rollouts > 0, "task training requires positive rollouts");
    mdn_sim_config config;
    mdn_sim_config_default(&config);
    config.n = 128;
    config.mode = 22;
    config.family = family;
    config.seed = seed;
    config.speed = 1.5f;
    config.distance = 8;
    config.max_steps = 400;
    config.geometry_memory = 1;
    config.entropy_coef = .001f;
    config.learning_rate = .0001f;
    Sim sim(device, config, 32);
    configure(sim, task_settings(stage, family), amplitude);
    PPOTrainer trainer(sim);
    const bool resume = std::filesystem::exists(checkpoint);
    if (resume) {
        trainer.load_checkpoint(checkpoint, family, 32, config.n, seed);
    } else {
        load_actor(sim, warmstart, true);
        auto actor = sim.download<float>(MDN_BUF_ACTOR);
        for (uint32_t a = 0; a < 4; a++) actor[actor.size() - 4 + a] = -1.0f;  // log_std
        sim.upload(MDN_BUF_ACTOR, actor);
    }
    validate_rollout(sim);
    const std::filesystem::path path(checkpoint);
    if (path.has_parent_path()) std::filesystem::create_directories(path.parent_path());
    std::ofstream history(checkpoint + ".history.csv", std::ios::app);
    require(bool(history), "task history write");
    if (!resume)
        history << "rollout,total_transitions,wall_s,collect_gpu_s,update_gpu_s,policy_loss,value_loss,ratio,success,"
                   "collision,timeout,mean_arrival_s\n";
    const uint32_t finish = trainer.completed_rollouts() + rollouts;
    auto evaluate_current = [&](const std::string& output) {
        const auto actor = sim.download<float>(MDN_BUF_ACTOR);
        return evaluate(device, actor.data(), stage, family, amplitude, 800001, output);
    };
    Score best;
    if (resume && std::filesystem::exists(checkpoint + ".best")) {
        Sim selected(device, config, 32);
        load_actor(selected, checkpoint + ".best");
        const auto actor = selected.download<float>(MDN_BUF_ACTOR);
        best = evaluate(device, actor.data(), stage, family, amplitude, 800001);
    }
    if (!resume) {
        best = evaluate_current(checkpoint + ".initial-dev.csv");
        trainer.save_checkpoint(checkpoint + ".best", family, seed, trainer.completed_rollouts());
        history << 0 << ",0,0,0,0,0,0,1," << best.success << ',' << best.collision << ',' << best.timeout << ','
                << best.successful_time_s << '\n';
        history.flush();
    }
    for (uint32_t rollout = trainer.completed_rollouts(); rollout < finish; rollout++) {
        // generation or dynamics errors are rejected before their transitions reach PPO
        sim.collect();
        const double collect_s = device.finish();
        validate_rollout(sim);
        trainer.rollout_update(rollout);
        device.finish();
        const double update_s = trainer.last_update_ms() * 1e-3;
        trainer.set_completed_rollouts(rollout + 1);
        if ((rollout + 1) % every == 0 || rollout + 1 == finish) {
            trainer.save_checkpoint(checkpoint, family, seed, rollout + 1);
            const Score score = evaluate_current(checkpoint + ".dev.csv");
            if (score.success > best.success || (score.success == best.success && score.collision < best.collision) ||
                (score.success == best.success && score.collision == best.collision &&
                 score.successful_time_s < best.successful_time_s)) {
                best = score;
                trainer.save_checkpoint(checkpoint + ".best", family, seed, rollout + 1);
                std::filesystem::copy_file(checkpoint + ".dev.csv", checkpoint + ".best-dev.csv",
                                           std::filesystem::copy_options::overwrite_existing);
            }
            const auto metrics = trainer.metric_mean();
            history << rollout + 1 << ',' << uint64_t(rollout + 1) * config.n * 32 << ",0," << collect_s << ','
                    << update_s << ',' << metrics[0] << ',' << metrics[1] << ',' << metrics[3] << ',' << score.success
                    << ',' << score.collision << ',' << score.timeout << ',' << score.successful_time_s << '\n';
            history.flush();
            sim.report("train-arrival", 0);
        }
    }
}

}  // namespace navigation_training
}  // namespace host
}  // namespace mdn
