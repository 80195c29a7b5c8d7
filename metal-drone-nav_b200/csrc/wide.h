// Host-side interface of the wide-actor tensor-core kernels (wide.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace mdn {

// Opaque storage for one TMA tensor map (CUtensorMap is 128 bytes, 64-byte
// aligned); kept opaque so host files need no driver-API header.
struct alignas(64) WideMap {
    unsigned char bytes[128];
};

// Observation rows x hidden units (k_wide_forward, k_wide_backward). The row count and first row
// are either the fixed `rows`/`row0` or read on the device from
// rows_dev[index] / row0_dev[index] (the PPO update's per-minibatch arrays,
// so a captured graph replays unchanged); `rows` is then the capacity.
struct WideRowsArgs {
    uint32_t rows;              // rows (or capacity, with rows_dev)
    uint32_t row0;              // first row in the observation tensor map
    const uint32_t* rows_dev;   // optional
    const uint32_t* row0_dev;   // optional
    uint32_t index;
    uint32_t hidden;            // a multiple of 256
    const float* b1;            // [hidden]
    const float* w2;            // [4][hidden]
    // forward
    float* partials;            // [hidden/128][rows][4] per-slice output sums
    // backward
    const float* d_mean;        // [rows][4] loss derivatives w.r.t. the means
    float* delta;               // [ceil256(rows)][hidden] hidden deltas (zero past the rows)
    float* colsum_out;          // [groups][5][hidden]: sum delta, sum d_mean[a] * tanh
    uint32_t* error;            // device flag: nonzero when a barrier wait gave up
};

// dW1 partials (k_wide_wgrad): out[split][h][k] over `splits` row ranges.
struct WideGradArgs {
    uint32_t rows, row0;
    const uint32_t* rows_dev;
    const uint32_t* row0_dev;
    uint32_t index;
    uint32_t hidden;
    uint32_t splits;
    float* out;                 // [splits][hidden][184]
    uint32_t* error;
};

// Flat gradient of the wide actor followed by the critic's.
struct WideAssembleArgs {
    uint32_t hidden, splits, groups;
    const float* w1_parts;      // [splits][hidden * 184]
    const float* colsums;       // [groups][5][hidden]
    const float* small_grad;    // the loss kernels' gradient in the 64-unit layout (b2, log_std, critic)
    float* grad;                // [actor_param_count(hidden) + critic params]
};

struct WideAdamArgs {
    const float* grad;
    float* params;
    float* m;
    float* v;
    size_t count;               // actor parameters (log_std = the last four)
    const float* bias_corr;     // this update's 1 - beta1^t, 1 - beta2^t
    float learning_rate, max_norm;
    const float* partials;      // set by the launcher
    uint32_t partial_count;
    float* norm_out;            // pre-clip norm (optional)
    uint32_t no_clamp;          // 1: no log-std clamp on the last four (a critic)
};

// Everything a rollout step needs to run the wide forward (host side).
struct WideStep {
    WideMap obs_map;            // observations [horizon * n][184], boxes of 128 rows
    WideMap w1_map;             // actor W1 [hidden][184], boxes of 256 rows
    WideRowsArgs args;          // row0 is set per tick
    int sm_count;
};

// Tensor map of an fp32 matrix [rows][inner] (row pitch in bytes, a multiple of
// 16; base 16-byte aligned) read in boxes of 32 columns x box_rows rows, in
// the 128-byte swizzle for a K-major MMA operand, or (mn_major) the 128-byte
// swizzle with 32-byte atoms that MN-major tf32 operands need.
cudaError_t wide_make_map(WideMap* out, const float* base, uint64_t inner, uint64_t rows, uint64_t pitch_bytes,
                          uint32_t box_rows, bool mn_major = false);
cudaError_t configure_wide_kernels();
// obs_map: boxes of 128 rows; w1_map: W1 [hidden][184], boxes of 256 rows.
cudaError_t launch_wide_forward(const WideMap& obs_map, const WideMap& w1_map, const WideRowsArgs& p, int sm_count,
                                cudaStream_t s);
uint32_t wide_backward_groups(uint32_t hidden, int sm_count);
// obs_map: boxes of 256 rows; w1_map: boxes of 128 rows (the backward tile is
// 128 hidden units x 256 rows).
cudaError_t launch_wide_backward(const WideMap& obs_map, const WideMap& w1_map, const WideRowsArgs& p, int sm_count,
                                 cudaStream_t s);
// delta_map: deltas [ceil256(rows)][hidden], boxes of 32 rows; obs_map: boxes of 32 rows.
cudaError_t launch_wide_wgrad(const WideMap& delta_map, const WideMap& obs_map, const WideGradArgs& p, int sm_count,
                              cudaStream_t s);
cudaError_t launch_wide_assemble(const WideAssembleArgs& p, int sm_count, cudaStream_t s);
cudaError_t launch_wide_clip_adam(const WideAdamArgs& p, float* partials_scratch, int sm_count, cudaStream_t s);

}  // namespace mdn
