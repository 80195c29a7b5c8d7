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
