// Internal host-side declarations shared by the C-ABI implementation files.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <fstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "mdn.h"
#include "mdn_shared.h"
#include "mlp.h"
#include "wide.h"

namespace mdn {

// Errors are raised as exceptions inside the library and converted to status
// codes at the C boundary (the reference's require(), main.mm:27).
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};
inline void require(bool ok, int code, const std::string& msg) {
    if (!ok) throw Error(code, msg);
}
inline void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw Error(MDN_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}
void set_last_error(const std::string& msg);

template <class F>
int guarded(F&& fn) {
    try {
        fn();
        return MDN_OK;
    } catch (const Error& e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::bad_alloc&) {
        set_last_error("host allocation failed");
        return MDN_ERR_NOMEM;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return MDN_ERR_INVALID;
    }
}

// Kernel launchers (rollout.cu, ppo.cu).
cudaError_t upload_camera_tables(const float* pixel_rays, const float* pool_rays);
cudaError_t configure_kernels();
cudaError_t launch_reset(const SimArgs& a, bool first, cudaStream_t s);
cudaError_t launch_world_mirror(const SimArgs& a, cudaStream_t s);
// Sim::report's ten aggregates of the run records into out[10] (device).
cudaError_t launch_report(const SimArgs& a, double* out, cudaStream_t s);
StepPlan plan_step(uint32_t n, int sm_count, int group_override, int act_override);
// flush = false leaves the step's ended episodes to the next step, which
// must then pass `fork` (only inside a collected rollout, whose last step
// flushes): its listed resets run in k_reset_sense on the fork's side stream.
cudaError_t launch_step(const SimArgs& a, const StepPlan& plan, const mdn_physics_params& nominal, cudaStream_t s,
                        const WideStep* wide, bool flush = true, const StepFork* fork = nullptr,
                        const LayeredStep* layered = nullptr);
size_t act_smem_bytes();
cudaError_t launch_step_profiled(const SimArgs& a, const StepPlan& plan, const mdn_physics_params& nominal, cudaStream_t s,
                                 cudaEvent_t ev[4], const WideStep* wide, const LayeredStep* layered = nullptr);
cudaError_t fp32_peak(int sm_count, double* tflops);
cudaError_t division_check(uint64_t samples, uint64_t seed, uint64_t* mismatches, int sm_count);
int kernels_per_step(const mdn_sim_config& c, bool wide);

// read_checkpoint_header (main.mm:993-1000) for PPOFIX1 versions 3..10
// (ppo_host.cpp); throws on a bad prefix, version or truncation.
void read_checkpoint_header(std::ifstream& f, mdn_checkpoint_header& h);
// Raises MDN_ERR_TIMEOUT when a trainer's tensor-core minibatch kernel gave up
// on a barrier wait (ppo_host.cpp); the device's streams must be idle.
void check_trainer_errors(struct ::mdn_device* dev);
// Host waits of a device's work (comm.cpp). On one GPU they are
// cudaStreamSynchronize / cudaEventSynchronize. Under NCCL they poll, so a
// collective stuck on a lost peer cannot block the host forever: a
// communicator error, or no completion within the device's deadline, aborts
// the communicator and raises MDN_ERR_NCCL.
void sync_stream(struct ::mdn_device* dev, cudaStream_t s, const char* what);
void sync_event(struct ::mdn_device* dev, cudaEvent_t e, const char* what);

}  // namespace mdn

struct mdn_device {
    int gpu = 0;
    int sm_count = 0;
    bool tables_ready = false;
    // multi-GPU
    int rank = 0, world = 1;
    void* nccl_comm = nullptr;
    bool comm_failed = false;     // the communicator was aborted (a peer failed or timed out)
    double nccl_timeout_s = 600;  // host deadline of a collective (MDN_NCCL_TIMEOUT_S)
    std::vector<struct mdn_sim*> sims;
    std::vector<struct mdn_ppo*> trainers;
};

struct mdn_sim {
    mdn_device* dev = nullptr;
    mdn_sim_config cfg{};
    mdn_rollout_shape shape{};
    uint32_t horizon = 0, n = 0, env_base = 0;
    cudaStream_t stream = nullptr;
    mdn::StepFork fork{};  // side stream + events of the collected rollout's forked sensing
    void* buf[MDN_BUF_COUNT] = {};
    float* world_soa = nullptr;  // device mirror of the worlds, structure of arrays
    uint32_t* reset_mem = nullptr;  // [n] reset list, its two counts, then [n] pending bytes (k_advance -> k_sense / k_reset_list)
    uint32_t actor_hidden = mdn::kHidden;                   // 64, or a wide actor (multiple of 256)
    uint32_t actor_params = mdn::actor_param_count(mdn::kHidden);
    uint32_t critic_params = mdn::kCriticParams;
    // Layered networks (mlp.cu): shapes, step launch arguments, scratch.
    bool layered = false;
    uint32_t co_dim = mdn::kCriticObs;  // critic observation width: 32, or 64 (control-state critic)
    mdn::LayeredStep* lay = nullptr;
    void* lay_mem = nullptr;
    float* wide_partials = nullptr;                         // [hidden/128][n][4] slice sums of the wide forward
    double* report_dev = nullptr;                           // [10] Sim::report aggregates (k_report)
    uint32_t* wide_error = nullptr;                         // barrier-timeout flag of the wide kernels
    mdn::WideStep* wide = nullptr;                          // tensor maps + launch arguments (wide actors)
    bool delay_rehearsal = false;                           // mdn_sim_set_delay_rehearsal
    bool audit_enabled = false;                             // mechanical contact audit (mdn_sim_set_contact_audit)
    float audit_margin = 0.04f;
    mdn_bank_control bank{};                                // frozen challenge bank (mdn_sim_set_challenge_bank)
    mdn_physics_params nominal{};  // host mirror of MDN_BUF_PHYSICS (k_advance takes it by value)
    mdn_runtime_config runtime{};                           // per-episode plant variation (mdn_sim_set_runtime)
    size_t bytes[MDN_BUF_COUNT] = {};
    float room_lo[3], room_hi[3], room_c[3], room_e[3];
    mdn::StepPlan plan;
    // collect() graphs cached by step count
    std::vector<std::pair<uint32_t, cudaGraphExec_t>> graphs;
    cudaEvent_t ev_start = nullptr, ev_stop = nullptr;
    float last_collect_ms = 0.0f;
    mdn_task_control task_ctl{};  // goal-arrival tasks, set by mdn_sim_configure_tasks
    uint32_t task_config_ok = 0;
    mdn::SimArgs args(uint32_t tick) const;
    void release_graphs();
};
