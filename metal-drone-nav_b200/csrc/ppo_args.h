// Arguments of the PPO update kernels (ppo.cu), passed by value.
#pragma once
#include <cstdint>

#include "mdn_shared.h"

namespace mdn {

constexpr int kPpoParams = kActorParams + kCriticParams;  // flat [actor | critic] gradient

struct PpoArgs {
    uint32_t n, horizon;          // local envs, rollout horizon
    uint64_t global_rows;         // rows over all ranks (advantage statistics)
    float gamma, lambda, clip, value_coef, entropy_coef, learning_rate, max_norm;
    const float* rewards;
    const float* values;
    const float* next_values;
    const uint8_t* terminated;
    const uint8_t* truncated;
    float* advantages;
    float* returns;
    float* raw_advantages;        // [rows] GAE before normalisation, or null (challenge banks)
    double* stat_partials;        // [gae blocks]
    double* stats;                // [2] sum, sum of squares (allreduced under NCCL)
    float* stat_values;           // [2] mean, inverse std
    const float* obs;
    const float* co;
    const float* actions;
    const float* logp;
    float* actor;
    float* critic;
    float* actor_m;
    float* actor_v;
    float* critic_m;
    float* critic_v;
    const uint32_t* starts;       // [updates] first row of each minibatch chunk
    const uint32_t* batch;        // [updates] local rows in the chunk
    const uint32_t* global_batch; // [updates] rows over all ranks (loss scale 1/B)
    const float* bias_corr;       // [updates][2] 1 - beta^step
    float* mb_ah;                 // [minibatch][64] actor hidden
    float* mb_ch;                 // [minibatch][64] critic hidden
    float* mb_adelta;             // [minibatch][64]
    float* mb_cdelta;             // [minibatch][64]
    float* mb_dm;                 // [minibatch][4]
    float* mb_dls;                // [minibatch][4]
    float* mb_dv;                 // [minibatch]
    float* grad_partials;         // [chunks][kPpoParams]
    float* grad;                  // [kPpoParams]
    float* loss_partials;         // [updates][fwd_grid][4]
    float* metric_rows;           // [updates][4]
    float* metric_mean;           // [4]
    float* grad_norms;            // [updates][2]
    uint32_t fwd_grid, grad_chunk;
    // Actor shape (ppo.hpp:35-40): offsets of b2 and log_std. A wide actor
    // (wide_slices != 0) takes its means from the tensor-core forward's slice
    // sums wide_partials[wide_slices][wide_rows_cap][4]; the loss and gradient
    // kernels then handle only the critic, b2 and log_std.
    uint32_t actor_b2, actor_log_std;
    const float* wide_partials;
    uint32_t wide_slices, wide_rows_cap;
    // barrier-timeout flag of the tensor-core minibatch kernel (ppo_tc.cu)
    uint32_t* tc_error;
};

cudaError_t configure_ppo_kernels();
uint32_t gae_blocks(uint32_t n);
cudaError_t launch_gae_sum(const PpoArgs& p, cudaStream_t s);
cudaError_t launch_adv_stats(const PpoArgs& p, int mode, cudaStream_t s);
cudaError_t launch_adv_finalize(const PpoArgs& p, int mode, cudaStream_t s);
cudaError_t launch_adv_sq(const PpoArgs& p, cudaStream_t s);
cudaError_t launch_adv_apply(const PpoArgs& p, int sm_count, cudaStream_t s);
cudaError_t launch_minibatch(const PpoArgs& p, uint32_t update, uint32_t chunks, cudaStream_t s);
cudaError_t launch_clip_adam(const PpoArgs& p, uint32_t update, uint32_t chunks, cudaStream_t s);
// Fixed-order sum of `chunks` gradient partials into p.grad.
cudaError_t launch_grad_reduce(const PpoArgs& p, uint32_t chunks, cudaStream_t s);
// Critic-only clip + Adam (plus the update's metric row) reading the critic
// gradient at grad_critic; the wide actor's step runs in wide.cu.
cudaError_t launch_clip_adam_critic(const PpoArgs& p, uint32_t update, const float* grad_critic, cudaStream_t s);
cudaError_t launch_metrics_mean(const PpoArgs& p, uint32_t updates, cudaStream_t s);

}  // namespace mdn
