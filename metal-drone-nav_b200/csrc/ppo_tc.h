// Host-side interface of the tensor-core PPO minibatch kernel (ppo_tc.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "ppo_args.h"
#include "wide.h"

namespace mdn {

// TMA maps of one trainer: the rollout's observations [rows][184] and critic
// observations [rows][32] in boxes of 128 rows, K-major (128-byte swizzle) and
// MN-major (128-byte swizzle, 32-byte atoms); actor W1 [64][184] and critic W1
// [64][32] in boxes of 64 rows, K-major.
struct TcMaps {
    WideMap obs_k, obs_mn, co_k, co_mn, w1, cw1;
};

cudaError_t tc_make_maps(TcMaps* m, const float* obs, const float* co, uint64_t rows, const float* actor,
                         const float* critic);
cudaError_t configure_tc_kernels();
// CTAs of the tensor-core minibatch kernel: one per 128-row tile, at most one per SM.
uint32_t tc_grid(uint32_t minibatch, int sm_count);
// Gradient partials of minibatch `update` (grid CTAs, one partial each, in the
// layout of the fp32 kernel) and their fixed-order sum into p.grad when grid > 1.
// One bounded mbarrier wait on the device (k_barrier_selftest): *timed_out = 1
// when it gave up after `limit` clock cycles.
cudaError_t barrier_selftest(long long limit, int arrive, uint32_t* timed_out);
cudaError_t launch_minibatch_tc(const PpoArgs& p, const TcMaps& m, uint32_t update, uint32_t grid, cudaStream_t s);

}  // namespace mdn
