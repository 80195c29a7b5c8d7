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

struct WideForwardArgs {
    uint32_t rows;       // observation rows in this launch
    uint32_t row0;       // first row (row coordinate inside the observation tensor map)
    uint32_t hidden;     // hidden width, a multiple of 256
    const float* b1;     // [hidden]
    const float* w2;     // [4][hidden]
    float* partials;     // [hidden / 128][rows][4] per-slice output sums
    uint32_t* error;     // device flag: nonzero when a barrier wait gave up
};

// Everything a rollout step needs to run the wide forward (host side).
struct WideStep {
    WideMap obs_map;        // observations [horizon * n][184], boxes of 128 rows
    WideMap w1_map;         // actor W1 [hidden][184], boxes of 256 rows
    WideForwardArgs args;   // row0 is set per tick
    int sm_count;
};

// Tensor map of an fp32 matrix [rows][inner] (row pitch in bytes, a multiple of
// 16; base 16-byte aligned) read in boxes of 32 columns x box_rows rows.
cudaError_t wide_make_map(WideMap* out, const float* base, uint64_t inner, uint64_t rows, uint64_t pitch_bytes,
                          uint32_t box_rows);
cudaError_t configure_wide_kernels();
// obs_map: boxes of 128 rows; w1_map: W1 [hidden][184], boxes of 256 rows.
cudaError_t launch_wide_forward(const WideMap& obs_map, const WideMap& w1_map, const WideForwardArgs& p, int sm_count,
                                cudaStream_t s);

}  // namespace mdn
