// Multi-GPU plumbing: one process per GPU, environments sharded by rank, and an
// NCCL allreduce over NVLink for the PPO gradients (per minibatch) and the
// global advantage statistics (per rollout). The reference has no counterpart
// (it runs on one Apple GPU); semantics follow its single-device update:
// advantage normalisation over all rows (ppo.hpp:128-140) and loss scale 1/B
// with B the global minibatch (ppo.hpp:159).
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <mutex>

#include "host_common.h"

namespace mdn {

// NCCL is resolved at run time: a process that already loaded an NCCL (torch
// bundles one) keeps using it, so two different libnccl.so.2 never meet in
// one process. MDN_NCCL_LIB names a library to load otherwise.
namespace {
struct Nccl {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) init_rank = nullptr;
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
        n.init_rank = reinterpret_cast<decltype(n.init_rank)>(dlsym(h, "ncclCommInitRank"));
        n.all_reduce = reinterpret_cast<decltype(n.all_reduce)>(dlsym(h, "ncclAllReduce"));
        n.destroy = reinterpret_cast<decltype(n.destroy)>(dlsym(h, "ncclCommDestroy"));
        n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
        n.ok = n.get_unique_id && n.init_rank && n.all_reduce && n.destroy && n.error_string;
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

cudaError_t comm_allreduce_double(mdn_device* dev, double* buf, size_t count, cudaStream_t s, std::string& err) {
    if (dev->world <= 1 || !dev->nccl_comm) return cudaSuccess;
    const ncclResult_t r = nccl().all_reduce(buf, buf, count, ncclFloat64, ncclSum, static_cast<ncclComm_t>(dev->nccl_comm), s);
    if (r != ncclSuccess) {
        err = std::string("ncclAllReduce: ") + nccl().error_string(r);
        return cudaErrorUnknown;
    }
    return cudaSuccess;
}

cudaError_t comm_allreduce_float(mdn_device* dev, float* buf, size_t count, cudaStream_t s, std::string& err) {
    if (dev->world <= 1 || !dev->nccl_comm) return cudaSuccess;
    const ncclResult_t r = nccl().all_reduce(buf, buf, count, ncclFloat32, ncclSum, static_cast<ncclComm_t>(dev->nccl_comm), s);
    if (r != ncclSuccess) {
        err = std::string("ncclAllReduce: ") + nccl().error_string(r);
        return cudaErrorUnknown;
    }
    return cudaSuccess;
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
        ncclComm_t comm;
        const ncclResult_t r = nc.init_rank(&comm, world, uid, rank);
        require(r == ncclSuccess, MDN_ERR_NCCL, std::string("ncclCommInitRank: ") + nc.error_string(r));
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
        dev->rank = 0;
        dev->world = 1;
    });
}
