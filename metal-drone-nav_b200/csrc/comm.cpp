// Multi-GPU plumbing: one process per GPU, environments sharded by rank, and an
// NCCL allreduce over NVLink for the PPO gradients (per minibatch) and the
// global advantage statistics (per rollout). The reference has no counterpart
// (it runs on one Apple GPU); semantics follow its single-device update:
// advantage normalisation over all rows (ppo.hpp:128-140) and loss scale 1/B
// with B the global minibatch (ppo.hpp:159).
#include <dlfcn.h>
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <cstdlib>
#include <memory>
#include <mutex>
#include <thread>

#include <algorithm>
#include <cstring>

#include "host_common.h"

namespace mdn {

// NCCL is resolved at run time: a process that already loaded an NCCL (torch
// bundles one) keeps using it, so two different libnccl.so.2 never meet in
// one process. MDN_NCCL_LIB names a library to load otherwise.
namespace {
struct Nccl {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
    decltype(&ncclCommGetAsyncError) async_error = nullptr;
    decltype(&ncclCommAbort) abort = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    bool ok = false;
    std::string why;
};
const Nccl& nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) {
            const char* path = std::getenv("MDN_NCCL_LIB");
            h = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        }
        if (!h) {
            n.why = std::string("cannot load NCCL: ") + dlerror();
            return;
        }
        n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        n.init_rank_config = reinterpret_cast<decltype(n.init_rank_config)>(dlsym(h, "ncclCommInitRankConfig"));
        n.async_error = reinterpret_cast<decltype(n.async_error)>(dlsym(h, "ncclCommGetAsyncError"));
        n.abort = reinterpret_cast<decltype(n.abort)>(dlsym(h, "ncclCommAbort"));
        n.all_reduce = reinterpret_cast<decltype(n.all_reduce)>(dlsym(h, "ncclAllReduce"));
        n.destroy = reinterpret_cast<decltype(n.destroy)>(dlsym(h, "ncclCommDestroy"));
        n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
        n.ok = n.get_unique_id && n.init_rank_config && n.async_error && n.abort && n.all_reduce && n.destroy &&
               n.error_string;
        if (!n.ok) n.why = "NCCL library lacks required symbols";
    });
    return n;
}
const Nccl& need_nccl() {
    const Nccl& n = nccl();
    require(n.ok, MDN_ERR_NCCL, n.why);
    return n;
}
}  // namespace

namespace {
using Clock = std::chrono::steady_clock;
double seconds_since(Clock::time_point t0) { return std::chrono::duration<double>(Clock::now() - t0).count(); }

// Poll `ready` until it reports something other than cudaErrorNotReady or
// `limit_s` passes; true when the work completed (with any status).
template <class Ready>
bool drained_within(Ready ready, double limit_s) {
    const auto t0 = Clock::now();
    for (;;) {
        if (ready() != cudaErrorNotReady) return true;
        if (seconds_since(t0) > limit_s) return false;
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
}

// Abort the communicator (NCCL kernels waiting on a peer return), let the
// stream drain and mark the device so no later update enqueues a collective.
// Both steps are bounded: ncclCommAbort runs on a helper thread that is left
// behind if it does not return in time, and the stream is polled, not
// synchronised. The error names what did not finish.
[[noreturn]] void abort_comm(mdn_device* dev, cudaStream_t s, const std::string& why) {
    const double limit = std::min(dev->nccl_timeout_s, 30.0);
    bool aborted = true;
    if (dev->nccl_comm && nccl().ok) {
        auto done = std::make_shared<std::atomic<bool>>(false);
        ncclComm_t comm = static_cast<ncclComm_t>(dev->nccl_comm);
        const int gpu = dev->gpu;
        std::thread([comm, done, gpu] {
            cudaSetDevice(gpu);
            nccl().abort(comm);
            done->store(true);
        }).detach();
        const auto t0 = Clock::now();
        while (!done->load() && seconds_since(t0) < limit) std::this_thread::sleep_for(std::chrono::milliseconds(1));
        aborted = done->load();
    }
    dev->nccl_comm = nullptr;
    dev->comm_failed = true;
    const bool drained = !s || drained_within([&] { return cudaStreamQuery(s); }, limit);
    cudaGetLastError();
    std::string msg = why;
    if (!aborted) msg += "; ncclCommAbort did not return within " + std::to_string(limit) + " s";
    if (!drained) msg += "; the stream did not drain within " + std::to_string(limit) + " s";
    throw Error(MDN_ERR_NCCL, msg);
}

// Poll `ready` (a stream or an event) and the communicator's asynchronous
// error until the work is done, the communicator reports an error, or the
// device's deadline passes.
template <class Ready>
void poll_until(mdn_device* dev, cudaStream_t s, const char* what, Ready ready) {
    const auto t0 = Clock::now();
    for (;;) {
        const cudaError_t q = ready();
        if (q != cudaErrorNotReady) {
            cuda_check(q, what);
            return;
        }
        ncclResult_t state = ncclSuccess;
        nccl().async_error(static_cast<ncclComm_t>(dev->nccl_comm), &state);
        if (state != ncclSuccess && state != ncclInProgress)
            abort_comm(dev, s, std::string(what) + ": NCCL communicator error: " + nccl().error_string(state));
        if (seconds_since(t0) > dev->nccl_timeout_s)
            abort_comm(dev, s, std::string(what) + ": collective did not complete within " +
                                   std::to_string(dev->nccl_timeout_s) + " s (a peer rank is gone or stalled)");
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

// A non-blocking communicator may answer a call with ncclInProgress; wait
// (bounded) until it has taken the call.
ncclResult_t settle(mdn_device* dev, ncclResult_t r) {
    const auto t0 = Clock::now();
    while (r == ncclInProgress) {
        nccl().async_error(static_cast<ncclComm_t>(dev->nccl_comm), &r);
        if (r == ncclInProgress && seconds_since(t0) > dev->nccl_timeout_s) return ncclInternalError;
        if (r == ncclInProgress) std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
    return r;
}

cudaError_t allreduce(mdn_device* dev, void* buf, size_t count, ncclDataType_t type, cudaStream_t s, std::string& err) {
    if (dev->world <= 1) return cudaSuccess;
    if (!dev->nccl_comm) {
        err = dev->comm_failed ? "NCCL communicator was aborted after a failure" : "no NCCL communicator";
        return cudaErrorUnknown;
    }
    const ncclResult_t r = settle(
        dev, nccl().all_reduce(buf, buf, count, type, ncclSum, static_cast<ncclComm_t>(dev->nccl_comm), s));
    if (r != ncclSuccess) {
        err = std::string("ncclAllReduce: ") + nccl().error_string(r);
        return cudaErrorUnknown;
    }
    return cudaSuccess;
}
}  // namespace

cudaError_t comm_allreduce_double(mdn_device* dev, double* buf, size_t count, cudaStream_t s, std::string& err) {
    return allreduce(dev, buf, count, ncclFloat64, s, err);
}

cudaError_t comm_allreduce_float(mdn_device* dev, float* buf, size_t count, cudaStream_t s, std::string& err) {
    return allreduce(dev, buf, count, ncclFloat32, s, err);
}

// After an abort, work queued behind a collective that never finished may
// stay blocked: waits on such a device are bounded and raise MDN_ERR_NCCL.
template <class Ready>
void wait_after_abort(mdn_device* dev, const char* what, Ready ready) {
    if (!drained_within(ready, std::min(dev->nccl_timeout_s, 30.0)))
        throw Error(MDN_ERR_NCCL, std::string(what) + ": work is still blocked behind an aborted NCCL collective");
    cuda_check(ready(), what);
}

void sync_stream(mdn_device* dev, cudaStream_t s, const char* what) {
    if (dev->comm_failed) return wait_after_abort(dev, what, [&] { return cudaStreamQuery(s); });
    if (dev->world <= 1 || !dev->nccl_comm) {
        cuda_check(cudaStreamSynchronize(s), what);
        return;
    }
    poll_until(dev, s, what, [&] { return cudaStreamQuery(s); });
}

void sync_event(mdn_device* dev, cudaEvent_t e, const char* what) {
    if (dev->comm_failed) return wait_after_abort(dev, what, [&] { return cudaEventQuery(e); });
    if (dev->world <= 1 || !dev->nccl_comm) {
        cuda_check(cudaEventSynchronize(e), what);
        return;
    }
    poll_until(dev, nullptr, what, [&] { return cudaEventQuery(e); });
}

}  // namespace mdn

using namespace mdn;

extern "C" int mdn_comm_unique_id(uint8_t id[128]) {
    return guarded([&] {
        require(id != nullptr, MDN_ERR_INVALID, "null id");
        static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
        const Nccl& nc = need_nccl();
        ncclUniqueId uid;
        const ncclResult_t r = nc.get_unique_id(&uid);
        require(r == ncclSuccess, MDN_ERR_NCCL, std::string("ncclGetUniqueId: ") + nc.error_string(r));
        std::memcpy(id, &uid, 128);
    });
}

extern "C" int mdn_comm_init(mdn_device* dev, int rank, int world, const uint8_t id[128]) {
    return guarded([&] {
        require(dev && id, MDN_ERR_INVALID, "mdn_comm_init: null argument");
        require(world >= 1 && rank >= 0 && rank < world, MDN_ERR_INVALID, "mdn_comm_init: bad rank/world");
        require(dev->sims.empty(), MDN_ERR_STATE, "mdn_comm_init must precede mdn_sim_create on this device");
        cuda_check(cudaSetDevice(dev->gpu), "cudaSetDevice");
        dev->rank = rank;
        dev->world = world;
        if (world == 1) return;
        const Nccl& nc = need_nccl();
        ncclUniqueId uid;
        std::memcpy(&uid, id, 128);
        const char* limit = std::getenv("MDN_NCCL_TIMEOUT_S");
        if (limit && *limit) dev->nccl_timeout_s = std::max(1.0, std::atof(limit));
        // Non-blocking communicator: the host polls its state against the
        // deadline instead of blocking inside NCCL.
        ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
        config.blocking = 0;
        ncclComm_t comm = nullptr;
        ncclResult_t r = nc.init_rank_config(&comm, world, uid, rank, &config);
        const auto t0 = Clock::now();
        while (r == ncclInProgress && comm) {
            nc.async_error(comm, &r);
            if (r == ncclInProgress && seconds_since(t0) > dev->nccl_timeout_s) {
                nc.abort(comm);
                throw Error(MDN_ERR_NCCL, "ncclCommInitRankConfig: the ranks did not all join within " +
                                              std::to_string(dev->nccl_timeout_s) + " s");
            }
            if (r == ncclInProgress) std::this_thread::sleep_for(std::chrono::milliseconds(1));
        }
        if (r != ncclSuccess && comm) nc.abort(comm);
        require(r == ncclSuccess, MDN_ERR_NCCL, std::string("ncclCommInitRankConfig: ") + nc.error_string(r));
        dev->comm_failed = false;
        dev->nccl_comm = comm;
    });
}

extern "C" int mdn_comm_destroy(mdn_device* dev) {
    return guarded([&] {
        require(dev != nullptr, MDN_ERR_INVALID, "null device");
        if (dev->nccl_comm) {
            cuda_check(cudaSetDevice(dev->gpu), "cudaSetDevice");
            if (nccl().ok) nccl().destroy(static_cast<ncclComm_t>(dev->nccl_comm));
            dev->nccl_comm = nullptr;
        }
        dev->comm_failed = false;
        dev->rank = 0;
        dev->world = 1;
    });
}
