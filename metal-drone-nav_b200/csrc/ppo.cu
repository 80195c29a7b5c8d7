// PPO update kernels for sm_100a (reference: ppo.metal, ppo.hpp,
// cpu_reference.hpp:515-608, PPOTrainer::rollout_update main.mm:1321-1384).
//
//   k_gae_sum      GAE reverse scan per env (ppo.hpp:108-126) + fp64 partial sums
//   k_adv_stats    fixed-order fp64 reduction -> mean / inverse std (ppo.hpp:128-140)
//   k_adv_sq       fp64 partial sums of squared deviations
//   k_adv_apply    (a - mean) * inv_std
//   k_mb_forward   minibatch actor+critic forward, clipped-PPO loss and its
//                  derivatives (ppo.hpp:144-181), hidden deltas
//   k_mb_grad      per-chunk gradient partials (cpu_reference.hpp:515-551)
//   k_grad_reduce  fixed-order sum of the chunk partials
//   k_clip_adam    global-norm clip to 0.5 + Adam + log-std clamp, one CTA per
//                  network (cpu_reference.hpp:553-567, main.mm:1369-1378)
// All reductions use a fixed tree/order: results do not depend on scheduling.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "host_common.h"
#include "mdn_device.cuh"
#include "ppo_args.h"

namespace mdn {

// ------------------------------------------------------------- advantages
constexpr int kGaeThreads = 256;

__device__ __forceinline__ double block_sum_double(double v, double* scratch) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0) scratch[wid] = v;
    __syncthreads();
    double total = 0.0;
    if (threadIdx.x == 0) {
        for (int w = 0; w < int(blockDim.x >> 5); w++) total += scratch[w];
    }
    __syncthreads();
    return total;  // valid in thread 0
}

__global__ void __launch_bounds__(kGaeThreads) k_gae_sum(PpoArgs p) {
    __shared__ double scratch[32];
    const uint32_t env = blockIdx.x * blockDim.x + threadIdx.x;
    double local = 0.0;
    if (env < p.n) {
        float carry = 0.0f;
        for (uint32_t rev = 0; rev < p.horizon; ++rev) {
            const uint32_t t = p.horizon - 1 - rev;
            const size_t k = size_t(t) * p.n + env;
            const bool term = p.terminated[k] != 0;
            const bool boundary = term || p.truncated[k] != 0;
            const float bootstrap = term ? 0.0f : p.next_values[k];
            const float value = p.values[k];
            const float delta = p.rewards[k] + p.gamma * bootstrap - value;
            carry = delta + (boundary ? 0.0f : p.gamma * p.lambda * carry);
            p.advantages[k] = carry;
            if (p.raw_advantages) p.raw_advantages[k] = carry;
            p.returns[k] = carry + value;
            local += double(carry);
        }
    }
    const double total = block_sum_double(local, scratch);
    if (threadIdx.x == 0) p.stat_partials[blockIdx.x] = total;
}

// Sum the per-block partials in block order; mode 0 -> mean, mode 1 -> inv std.
__global__ void k_adv_stats(PpoArgs p, uint32_t blocks, int mode) {
    __shared__ double scratch[32];
    double local = 0.0;
    for (uint32_t b = threadIdx.x; b < blocks; b += blockDim.x) local += p.stat_partials[b];
    const double total = block_sum_double(local, scratch);
    if (threadIdx.x == 0) {
        // Under NCCL the host allreduces stats[] between the two passes; the
        // count is the global row count.
        if (mode == 0) {
            p.stats[0] = total;
        } else {
            p.stats[1] = total;
        }
    }
}

__global__ void k_adv_finalize(PpoArgs p, int mode) {
    // ppo.hpp:132 and :138, evaluated exactly as the reference does.
    if (threadIdx.x != 0) return;
    const double count = double(p.global_rows);
    if (mode == 0) {
        p.stat_values[0] = float(p.stats[0] / count);
    } else {
        p.stat_values[1] = 1.0f / sqrtf(float(p.stats[1] / count) + 1.0e-8f);
    }
}

__global__ void __launch_bounds__(kGaeThreads) k_adv_sq(PpoArgs p) {
    __shared__ double scratch[32];
    const float mean = p.stat_values[0];
    double local = 0.0;
    const size_t rows = size_t(p.n) * p.horizon;
    // Same env-major partition as k_gae_sum: block b covers envs [b*256, b*256+256).
    const uint32_t env = blockIdx.x * blockDim.x + threadIdx.x;
    if (env < p.n)
        for (uint32_t t = 0; t < p.horizon; t++) {
            const double d = double(p.advantages[size_t(t) * p.n + env] - mean);
            local += d * d;
        }
    (void)rows;
    const double total = block_sum_double(local, scratch);
    if (threadIdx.x == 0) p.stat_partials[blockIdx.x] = total;
}

__global__ void k_adv_apply(PpoArgs p) {
    const float mean = p.stat_values[0], inv = p.stat_values[1];
    const size_t rows = size_t(p.n) * p.horizon;
    for (size_t k = blockIdx.x * size_t(blockDim.x) + threadIdx.x; k < rows; k += size_t(gridDim.x) * blockDim.x)
        p.advantages[k] = (p.advantages[k] - mean) * inv;
}

// ------------------------------------------------------------ minibatch
// CTA tile: 64 rows x 64 hidden, 256 threads, each thread 4 rows x 4 hidden.
// Thread t: row group rg = t / 16 (rows 4*rg..4*rg+3), hidden group hg = t % 16
// (hidden 4*hg..4*hg+3); the 16 threads of a row group are one half-warp.
constexpr int kMbThreads = 256;
constexpr int kMbRows = 64;
constexpr int kObsPitch = kActorObs + 1;
constexpr int kCoPitch = kCriticObs + 1;
constexpr size_t kMbSmemFloats = size_t(kActorObs) * kHidden + size_t(kCriticObs) * kHidden +
                                 size_t(kMbRows) * kObsPitch + size_t(kMbRows) * kCoPitch + 4 * kHidden + 4 * kHidden + 64;

__device__ __forceinline__ float half_warp_sum(float v) {
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// kWide: the actor means come from the tensor-core forward's slice sums
// (p.wide_partials); only the critic, b2 and log_std are handled here.
template <bool kWide>
__global__ void __launch_bounds__(kMbThreads) k_mb_forward(PpoArgs p, uint32_t update) {
    extern __shared__ float sm[];
    float* w1t = sm;                                   // [184][64]
    float* cw1t = w1t + kActorObs * kHidden;           // [32][64]
    float* obs_t = cw1t + kCriticObs * kHidden;        // [64][185]
    float* co_t = obs_t + kMbRows * kObsPitch;         // [64][33]
    float* w2 = co_t + kMbRows * kCoPitch;             // [4][64]
    float* b1 = w2 + 4 * kHidden;                      // [64]
    float* cb1 = b1 + kHidden;                         // [64]
    float* cw2 = cb1 + kHidden;                        // [64]
    float* cb2 = cw2 + kHidden;                        // [1]
    float* b2 = cb2 + 1;                               // [4]
    float* log_std = b2 + 4;                           // [4]
    float* sums = log_std + 4;                         // [4] loss sums of this CTA
    const int tid = threadIdx.x;
    const float* actor = p.actor;
    const float* critic = p.critic;
    constexpr bool wide = kWide;
    if (!wide)
        for (int k = tid; k < kActorObs * kHidden; k += kMbThreads) {
            const int h = k / kActorObs, c = k % kActorObs;
            w1t[c * kHidden + h] = actor[k];
        }
    for (int k = tid; k < kCriticObs * kHidden; k += kMbThreads) {
        const int h = k / kCriticObs, c = k % kCriticObs;
        cw1t[c * kHidden + h] = critic[k];
    }
    if (!wide)
        for (int k = tid; k < 4 * kHidden; k += kMbThreads) w2[k] = actor[kActorW2 + k];
    if (tid < kHidden) {
        if (!wide) b1[tid] = actor[kActorB1 + tid];
        cb1[tid] = critic[kCriticB1 + tid];
        cw2[tid] = critic[kCriticW2 + tid];
    }
    if (tid < 4) {
        b2[tid] = actor[p.actor_b2 + tid];
        log_std[tid] = actor[p.actor_log_std + tid];
        sums[tid] = 0.0f;
    }
    if (tid == 0) cb2[0] = critic[kCriticB2];
    const uint32_t begin = p.starts[update];
    const uint32_t b = p.batch[update];
    const float scale = 1.0f / fmaxf(float(p.global_batch[update]), 1.0f);
    const int rg = tid >> 4, hg = tid & 15;
    float csum[4] = {0, 0, 0, 0};
    for (uint32_t tile = blockIdx.x * kMbRows; tile < b; tile += gridDim.x * kMbRows) {
        __syncthreads();
        const uint32_t rows = min(uint32_t(kMbRows), b - tile);
        const float* og = p.obs + (size_t(begin) + tile) * kActorObs;
        if (wide) {  // the wide actor's means come from the tensor cores: only the geometry prior is read
            for (int k = tid; k < kMbRows * 3; k += kMbThreads) {
                const int r = k / 3, c = kActorObs - 3 + k % 3;
                obs_t[r * kObsPitch + c] = r < int(rows) ? og[r * kActorObs + c] : 0.0f;
            }
        } else {
            for (int k = tid; k < kMbRows * kActorObs; k += kMbThreads) {
                const int r = k / kActorObs, c = k % kActorObs;
                obs_t[r * kObsPitch + c] = r < int(rows) ? og[k] : 0.0f;
            }
        }
        const float* cg = p.co + (size_t(begin) + tile) * kCriticObs;
        for (int k = tid; k < kMbRows * kCriticObs; k += kMbThreads) {
            const int r = k / kCriticObs, c = k % kCriticObs;
            co_t[r * kCoPitch + c] = r < int(rows) ? cg[k] : 0.0f;
        }
        __syncthreads();
        // actor pre-activations: in-order dot from zero, bias after (cpu_reference.hpp:439-442)
        float acc[4][4];
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
            for (int h = 0; h < 4; h++) acc[r][h] = 0.0f;
        for (int k = 0; k < (wide ? 0 : kActorObs); k++) {
            const float4 w = *reinterpret_cast<const float4*>(&w1t[k * kHidden + 4 * hg]);
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const float o = obs_t[(4 * rg + r) * kObsPitch + k];
                acc[r][0] = fmaf(o, w.x, acc[r][0]);
                acc[r][1] = fmaf(o, w.y, acc[r][1]);
                acc[r][2] = fmaf(o, w.z, acc[r][2]);
                acc[r][3] = fmaf(o, w.w, acc[r][3]);
            }
        }
        float cacc[4][4];
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
            for (int h = 0; h < 4; h++) cacc[r][h] = 0.0f;
        for (int k = 0; k < kCriticObs; k++) {
            const float4 w = *reinterpret_cast<const float4*>(&cw1t[k * kHidden + 4 * hg]);
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const float o = co_t[(4 * rg + r) * kCoPitch + k];
                cacc[r][0] = fmaf(o, w.x, cacc[r][0]);
                cacc[r][1] = fmaf(o, w.y, cacc[r][1]);
                cacc[r][2] = fmaf(o, w.z, cacc[r][2]);
                cacc[r][3] = fmaf(o, w.w, cacc[r][3]);
            }
        }
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int lr = 4 * rg + r;
            const bool valid = lr < int(rows);
            const size_t grow = size_t(tile) + lr;  // row within the minibatch
            float hid[4], chid[4];
#pragma unroll
            for (int h = 0; h < 4; h++) {
                hid[h] = tanhf(acc[r][h] + b1[4 * hg + h]);
                chid[h] = tanhf(cacc[r][h] + cb1[4 * hg + h]);
            }
            float mean[4];
            if (wide) {
                // slice sums of the tensor-core forward: slices hg, hg+16, ... on
                // lane hg of the half-warp, then the fixed half-warp tree
                float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (valid)
                    for (uint32_t sl = hg; sl < p.wide_slices; sl += 16) {
                        const float4 v = *reinterpret_cast<const float4*>(
                            p.wide_partials + (size_t(sl) * p.wide_rows_cap + grow) * 4);
                        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
                    }
                const float sm4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
                for (int a = 0; a < 4; a++) {
                    mean[a] = half_warp_sum(sm4[a]) + b2[a];
                    if (a < 3) mean[a] += obs_t[lr * kObsPitch + kActorObs - 3 + a];
                }
            } else {
#pragma unroll
                for (int a = 0; a < 4; a++) {
                    float part = 0.0f;
#pragma unroll
                    for (int h = 0; h < 4; h++) part = fmaf(hid[h], w2[a * kHidden + 4 * hg + h], part);
                    mean[a] = half_warp_sum(part) + b2[a];
                    if (a < 3) mean[a] += obs_t[lr * kObsPitch + kActorObs - 3 + a];
                }
            }
            float vpart = 0.0f;
#pragma unroll
            for (int h = 0; h < 4; h++) vpart = fmaf(chid[h], cw2[4 * hg + h], vpart);
            const float value = half_warp_sum(vpart) + cb2[0];
            // clipped-PPO loss and derivatives, ppo.hpp:144-181 (every lane of the
            // half-warp evaluates it; lanes are identical)
            float dm[4], dls[4], dvalue = 0.0f, loss[4] = {0, 0, 0, 0};
            if (valid) {
                const size_t src = size_t(begin) + grow;
                const float* act = p.actions + src * kActions;
                float logp = 0.0f;
#pragma unroll
                for (int a = 0; a < 4; a++) {
                    const float inv_std = expf(-log_std[a]);
                    const float d = (act[a] - mean[a]) * inv_std;
                    logp += -0.5f * (d * d + 2.0f * log_std[a] + kLogTwoPi);
                }
                const float adv = p.advantages[src], ret = p.returns[src];
                const float raw = logp - p.logp[src];
                const float lr_ = clampf(raw, -20.0f, 20.0f);
                const float ratio = expf(lr_);
                const float clip = p.clip;
                const float clipped = clampf(ratio, 1.0f - clip, 1.0f + clip);
                const float chosen = smin(ratio * adv, clipped * adv);
                const bool in_range = raw >= -20.0f && raw <= 20.0f;
                const bool active = in_range && (adv >= 0.0f ? ratio <= 1.0f + clip : ratio >= 1.0f - clip);
                float entropy = 0.0f;
#pragma unroll
                for (int a = 0; a < 4; a++) {
                    const float inv_var = expf(-2.0f * log_std[a]);
                    const float diff = act[a] - mean[a];
                    if (active) {
                        const float dlogp = -ratio * adv * scale;
                        dm[a] = dlogp * diff * inv_var;
                        dls[a] = dlogp * (diff * diff * inv_var - 1.0f);
                    } else {
                        dm[a] = 0.0f;
                        dls[a] = 0.0f;
                    }
                    dls[a] -= p.entropy_coef * scale;
                    entropy += -p.entropy_coef * (log_std[a] + 0.5f * (1.0f + kLogTwoPi)) * scale;
                }
                dvalue = p.value_coef * (value - ret) * scale;
                loss[0] = -chosen * scale;
                loss[1] = 0.5f * p.value_coef * (value - ret) * (value - ret) * scale;
                loss[2] = entropy;
                loss[3] = ratio;
                if (hg == 0) {
                    float* o = p.mb_dm + grow * 4;
                    float* l = p.mb_dls + grow * 4;
#pragma unroll
                    for (int a = 0; a < 4; a++) {
                        o[a] = dm[a];
                        l[a] = dls[a];
                    }
                    p.mb_dv[grow] = dvalue;
#pragma unroll
                    for (int k = 0; k < 4; k++) csum[k] += loss[k];
                }
            } else {
#pragma unroll
                for (int a = 0; a < 4; a++) dm[a] = dls[a] = 0.0f;
            }
            if (valid) {
                // hidden deltas: (W2^T d_mean) * (1 - h^2), d_value * w2c * (1 - hc^2)
                float4 hv, dh, chv, cdh;
                float* hvp = &hv.x;
                float* dhp = &dh.x;
                float* chp = &chv.x;
                float* cdp = &cdh.x;
#pragma unroll
                for (int h = 0; h < 4; h++) {
                    float s = 0.0f;
#pragma unroll
                    for (int a = 0; a < 4; a++) s = fmaf(dm[a], w2[a * kHidden + 4 * hg + h], s);
                    hvp[h] = hid[h];
                    dhp[h] = s * (1.0f - hid[h] * hid[h]);
                    chp[h] = chid[h];
                    cdp[h] = dvalue * cw2[4 * hg + h] * (1.0f - chid[h] * chid[h]);
                }
                if (!wide) {
                    *reinterpret_cast<float4*>(p.mb_ah + grow * kHidden + 4 * hg) = hv;
                    *reinterpret_cast<float4*>(p.mb_adelta + grow * kHidden + 4 * hg) = dh;
                }
                *reinterpret_cast<float4*>(p.mb_ch + grow * kHidden + 4 * hg) = chv;
                *reinterpret_cast<float4*>(p.mb_cdelta + grow * kHidden + 4 * hg) = cdh;
            }
        }
    }
    // CTA loss sums (ppo_metrics_batch, main.mm:941-951), fixed order: row-group
    // leaders add in row order via shared atomics would be order-dependent, so
    // stage per-thread sums and add them sequentially.
    __syncthreads();
    float* stage = obs_t;  // reuse
    for (int k = 0; k < 4; k++) stage[tid * 4 + k] = csum[k];
    __syncthreads();
    if (tid < 4) {
        float s = 0.0f;
        for (int t = 0; t < kMbThreads; t += 16) s += stage[t * 4 + tid];
        p.loss_partials[(size_t(update) * p.fwd_grid + blockIdx.x) * 4 + tid] = s;
    }
}

// Gradient partials of one row chunk. Thread t owns actor W1 entries (h, i)
// for i = t % 184 ... (strided) and all 64 hidden via 4 passes, plus the small
// blocks. Chunk c covers minibatch rows [c*chunk, min(b, (c+1)*chunk)).
constexpr int kGradThreads = 256;
constexpr int kGradTile = 16;

template <bool kWide>
__global__ void __launch_bounds__(kGradThreads) k_mb_grad(PpoArgs p, uint32_t update) {
    __shared__ float dtile[kGradTile][kHidden];      // actor deltas
    __shared__ float otile[kGradTile][kActorObs];    // observations
    __shared__ float cdtile[kGradTile][kHidden];     // critic deltas
    __shared__ float cotile[kGradTile][kCriticObs];  // critic observations
    __shared__ float htile[kGradTile][kHidden];      // actor hidden
    __shared__ float chtile[kGradTile][kHidden];     // critic hidden
    __shared__ float dmt[kGradTile][4], dlst[kGradTile][4], dvt[kGradTile];
    const uint32_t begin = p.starts[update];
    const uint32_t b = p.batch[update];
    const uint32_t c0 = blockIdx.x * p.grad_chunk;
    const uint32_t c1 = min(b, c0 + p.grad_chunk);
    const int tid = threadIdx.x;
    // Actor W1: 64 x 184 outputs. Thread t handles column i = t (t < 184) for
    // all 64 hidden in registers... 64 accumulators per thread.
    float aw1[kHidden];
#pragma unroll
    for (int h = 0; h < kHidden; h++) aw1[h] = 0.0f;
    // Other outputs: W2 (256) + critic W1 (2048) + critic w2 (64) + biases.
    // Thread t accumulates: W2 entry t (a = t/64, h = t%64); critic W1 entries
    // t + 256*j (j < 8); b1 (t<64), cb1 (64<=t<128), cw2 (128<=t<192), b2/ls (192..199), cb2 (200).
    float w2acc = 0.0f, cw1acc[8] = {0, 0, 0, 0, 0, 0, 0, 0}, misc = 0.0f;
    // Wide actor: its W1, b1 and W2 come from the tensor-core backward, so the
    // actor's deltas, hidden activations and observations are not read here.
    constexpr bool wide = kWide;
    for (uint32_t r0 = c0; r0 < c1; r0 += kGradTile) {
        const uint32_t nr = min(uint32_t(kGradTile), c1 - r0);
        __syncthreads();
        for (int k = tid; k < kGradTile * kHidden; k += kGradThreads) {
            const int r = k / kHidden, h = k % kHidden;
            const bool v = r < int(nr);
            const size_t row = size_t(r0) + r;
            if (!wide) {
                dtile[r][h] = v ? p.mb_adelta[row * kHidden + h] : 0.0f;
                htile[r][h] = v ? p.mb_ah[row * kHidden + h] : 0.0f;
            }
            cdtile[r][h] = v ? p.mb_cdelta[row * kHidden + h] : 0.0f;
            chtile[r][h] = v ? p.mb_ch[row * kHidden + h] : 0.0f;
        }
        if (!wide)
            for (int k = tid; k < kGradTile * kActorObs; k += kGradThreads) {
                const int r = k / kActorObs, c = k % kActorObs;
                otile[r][c] = r < int(nr) ? p.obs[(size_t(begin) + r0 + r) * kActorObs + c] : 0.0f;
            }
        for (int k = tid; k < kGradTile * kCriticObs; k += kGradThreads) {
            const int r = k / kCriticObs, c = k % kCriticObs;
            cotile[r][c] = r < int(nr) ? p.co[(size_t(begin) + r0 + r) * kCriticObs + c] : 0.0f;
        }
        for (int k = tid; k < kGradTile * 4; k += kGradThreads) {
            const int r = k / 4, a = k % 4;
            dmt[r][a] = r < int(nr) ? p.mb_dm[(size_t(r0) + r) * 4 + a] : 0.0f;
            dlst[r][a] = r < int(nr) ? p.mb_dls[(size_t(r0) + r) * 4 + a] : 0.0f;
        }
        if (tid < kGradTile) dvt[tid] = tid < int(nr) ? p.mb_dv[size_t(r0) + tid] : 0.0f;
        __syncthreads();
        for (int r = 0; r < int(nr); r++) {
            if (tid < kActorObs && !wide) {
                const float o = otile[r][tid];
#pragma unroll
                for (int h = 0; h < kHidden; h++) aw1[h] = fmaf(dtile[r][h], o, aw1[h]);
            }
            if (!wide) {
                const int a = tid >> 6, h = tid & 63;  // actor W2[a][h] = sum dm * hidden
                w2acc = fmaf(dmt[r][a], htile[r][h], w2acc);
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int e = tid + kGradThreads * j;  // critic W1 [64][32]
                const int h = e / kCriticObs, c = e % kCriticObs;
                cw1acc[j] = fmaf(cdtile[r][h], cotile[r][c], cw1acc[j]);
            }
            if (tid < 64) misc += wide ? 0.0f : dtile[r][tid];
            else if (tid < 128) misc += cdtile[r][tid - 64];
            else if (tid < 192) misc = fmaf(dvt[r], chtile[r][tid - 128], misc);
            else if (tid < 196) misc += dmt[r][tid - 192];
            else if (tid < 200) misc += dlst[r][tid - 196];
            else if (tid == 200) misc += dvt[r];
        }
    }
    float* out = p.grad_partials + size_t(blockIdx.x) * kPpoParams;
    if (tid < kActorObs)
#pragma unroll
        for (int h = 0; h < kHidden; h++) out[h * kActorObs + tid] = aw1[h];
    out[kActorW2 + tid] = w2acc;
#pragma unroll
    for (int j = 0; j < 8; j++) out[kActorParams + tid + kGradThreads * j] = cw1acc[j];
    if (tid < 64) out[kActorB1 + tid] = misc;
    else if (tid < 128) out[kActorParams + kCriticB1 + tid - 64] = misc;
    else if (tid < 192) out[kActorParams + kCriticW2 + tid - 128] = misc;
    else if (tid < 196) out[kActorB2 + tid - 192] = misc;
    else if (tid < 200) out[kActorLogStd + tid - 196] = misc;
    else if (tid == 200) out[kActorParams + kCriticB2] = misc;
}

__global__ void k_grad_reduce(PpoArgs p, uint32_t chunks) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < uint32_t(kPpoParams); i += gridDim.x * blockDim.x) {
        float s = 0.0f;
        for (uint32_t c = 0; c < chunks; c++) s += p.grad_partials[size_t(c) * kPpoParams + i];
        p.grad[i] = s;
    }
}

// One CTA per network: norm of the (reduced) gradient, clip to max_norm, Adam
// with the host-supplied bias corrections, log-std clamp; CTA 0 also reduces
// the loss partials into the update's metric row.
constexpr int kAdamThreads = 1024;
constexpr int kAdamPerThread = (kActorParams + kAdamThreads - 1) / kAdamThreads;  // 12

__global__ void __launch_bounds__(kAdamThreads) k_clip_adam(PpoArgs p, uint32_t update, const float* grad_src,
                                                             int first_net) {
    __shared__ float red[32];
    const int net = blockIdx.x + first_net;  // 0 actor, 1 critic
    const int count = net == 0 ? kActorParams : kCriticParams;
    const int base = net == 0 ? 0 : kActorParams;
    float* params = net == 0 ? p.actor : p.critic;
    float* m = net == 0 ? p.actor_m : p.critic_m;
    float* v = net == 0 ? p.actor_v : p.critic_v;
    const int tid = threadIdx.x;
    float g[kAdamPerThread];
    float sq = 0.0f;
#pragma unroll
    for (int j = 0; j < kAdamPerThread; j++) {
        const int i = tid + j * kAdamThreads;
        g[j] = i < count ? grad_src[base + i] : 0.0f;
        sq = fmaf(g[j], g[j], sq);
    }
    // fixed-order block reduction
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
    if ((tid & 31) == 0) red[tid >> 5] = sq;
    __syncthreads();
    if (tid < 32) {
        float s = red[tid];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (tid == 0) red[0] = s;
    }
    __syncthreads();
    const float norm = sqrtf(red[0] + 1.0e-20f);
    const float scale = smin(1.0f, p.max_norm / norm);
    if (tid == 0) p.grad_norms[update * 2 + net] = norm;
    const float b1c = p.bias_corr[update * 2], b2c = p.bias_corr[update * 2 + 1];
    const float lr = p.learning_rate;
#pragma unroll
    for (int j = 0; j < kAdamPerThread; j++) {
        const int i = tid + j * kAdamThreads;
        if (i >= count) continue;
        const float gs = g[j] * scale;
        const float mi = 0.9f * m[i] + (1.0f - 0.9f) * gs;
        const float vi = 0.999f * v[i] + (1.0f - 0.999f) * gs * gs;
        m[i] = mi;
        v[i] = vi;
        const float mh = mi / b1c, vh = vi / b2c;
        float pi = params[i] - lr * mh / (sqrtf(vh) + 1.0e-8f);
        if (net == 0 && i >= kActorLogStd) pi = clampf(pi, -2.0f, 0.5f);  // ppo_clip_log_std, main.mm:934-940
        params[i] = pi;
    }
    if (blockIdx.x == 0 && tid < 4) {
        float s = 0.0f;
        for (uint32_t c = 0; c < p.fwd_grid; c++) s += p.loss_partials[(size_t(update) * p.fwd_grid + c) * 4 + tid];
        if (tid == 3) s /= float(p.batch[update]);  // mean ratio, main.mm:949
        p.metric_rows[update * 4 + tid] = s;
    }
}

__global__ void k_metrics_mean(PpoArgs p, uint32_t updates) {
    // ppo_metrics_mean, main.mm:952-962
    if (threadIdx.x >= 4) return;
    float s = 0.0f;
    for (uint32_t u = 0; u < updates; u++) s += p.metric_rows[u * 4 + threadIdx.x];
    p.metric_mean[threadIdx.x] = updates ? s / float(updates) : 0.0f;
}

// Fused minibatch kernel of the 64-unit actor and critic: forward, clipped-PPO
// loss and derivatives (ppo.hpp:144-181), hidden deltas and the gradient
// partial of one contiguous run of minibatch rows (cpu_reference.hpp:515-551),
// without writing the hidden activations or deltas to HBM. CTA c owns rows
// [c * grad_chunk, (c+1) * grad_chunk) of the minibatch and walks them in
// 16-row tiles (two CTAs fit an SM and overlap each other's phases); every
// accumulator adds its rows in row order, and the forward
// keeps the in-order k chain of the batched reference, so the results equal
// the unfused kernels' bit for bit.
//   forward: thread (row = t / 16, hg = t % 16) computes hidden 4hg..4hg+3 of
//            both networks for its row; inputs are read 4 at a time.
//   gradient: thread (ty = t / 16, tx = t % 16) accumulates actor W1[4ty+i][12tx+j]
//            (48 values), critic W1[4ty+i][2tx+j] (8), one W2 entry and one of
//            the small blocks (b1, critic b1 / w2, b2, log_std, critic b2).
constexpr int kFuseRows = 16;
constexpr int kFuseObsPitch = 192;  // 184 inputs + zero padding (12 per gradient thread)
constexpr size_t kFuseSmemFloats = size_t(kActorObs) * kHidden + size_t(kCriticObs) * kHidden + 4 * kHidden +
                                   3 * kHidden + 12 + size_t(kFuseRows) * kFuseObsPitch +
                                   size_t(kFuseRows) * kCriticObs + 4 * size_t(kFuseRows) * kHidden +
                                   size_t(kFuseRows) * 9 + 4 * kMbThreads;

__global__ void __launch_bounds__(kMbThreads, 2) k_mb_fused(PpoArgs p, uint32_t update) {
    extern __shared__ __align__(16) float fsm[];
    float* w1t = fsm;                                   // [184][64]
    float* cw1t = w1t + kActorObs * kHidden;            // [32][64]
    float* w2 = cw1t + kCriticObs * kHidden;            // [4][64]
    float* b1 = w2 + 4 * kHidden;                       // [64]
    float* cb1 = b1 + kHidden;                          // [64]
    float* cw2 = cb1 + kHidden;                         // [64]
    float* small = cw2 + kHidden;                       // b2[4], log_std[4], cb2, pad
    float* obs = small + 12;                            // [32][192]
    float* co = obs + kFuseRows * kFuseObsPitch;        // [32][32]
    float* hid = co + kFuseRows * kCriticObs;           // [32][64]
    float* chid = hid + kFuseRows * kHidden;            // [32][64]
    float* dl = chid + kFuseRows * kHidden;             // [32][64] actor hidden deltas
    float* cdl = dl + kFuseRows * kHidden;              // [32][64] critic hidden deltas
    float* rowv = cdl + kFuseRows * kHidden;            // [32][9]: d_mean[4], d_log_std[4], d_value
    float* stage = rowv + kFuseRows * 9;                // [256][4] loss sums
    float* b2 = small;
    float* log_std = small + 4;
    const int tid = threadIdx.x;
    const float* actor = p.actor;
    const float* critic = p.critic;
    for (int k = tid; k < kActorObs * kHidden; k += kMbThreads) {
        const int h = k / kActorObs, c = k % kActorObs;
        w1t[c * kHidden + h] = actor[k];
    }
    for (int k = tid; k < kCriticObs * kHidden; k += kMbThreads) {
        const int h = k / kCriticObs, c = k % kCriticObs;
        cw1t[c * kHidden + h] = critic[k];
    }
    for (int k = tid; k < 4 * kHidden; k += kMbThreads) w2[k] = actor[kActorW2 + k];
    if (tid < kHidden) {
        b1[tid] = actor[kActorB1 + tid];
        cb1[tid] = critic[kCriticB1 + tid];
        cw2[tid] = critic[kCriticW2 + tid];
    }
    if (tid < 4) {
        b2[tid] = actor[p.actor_b2 + tid];
        log_std[tid] = actor[p.actor_log_std + tid];
    }
    if (tid == 0) small[8] = critic[kCriticB2];
    for (int k = tid; k < kFuseRows * kFuseObsPitch; k += kMbThreads) obs[k] = 0.0f;  // padding stays zero
    const float cb2 = critic[kCriticB2];

    const uint32_t begin = p.starts[update];
    const uint32_t b = p.batch[update];
    const float scale = 1.0f / fmaxf(float(p.global_batch[update]), 1.0f);
    const uint32_t c0 = blockIdx.x * p.grad_chunk;
    const uint32_t c1 = min(b, c0 + p.grad_chunk);
    const int rg = tid >> 4, hg = tid & 15;   // forward mapping
    const int ty = tid >> 4, tx = tid & 15;   // gradient mapping
    float acc[4][12];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 12; j++) acc[i][j] = 0.0f;
    float cacc[4][2] = {{0, 0}, {0, 0}, {0, 0}, {0, 0}};
    float w2acc = 0.0f, misc = 0.0f;
    float csum[4] = {0, 0, 0, 0};
    for (uint32_t r0 = c0; r0 < c1; r0 += kFuseRows) {
        const int nr = int(min(uint32_t(kFuseRows), c1 - r0));
        __syncthreads();  // the previous tile's gradient loop is done with the tiles
        {
            const float4* og = reinterpret_cast<const float4*>(p.obs + (size_t(begin) + r0) * kActorObs);
            for (int k = tid; k < nr * (kActorObs / 4); k += kMbThreads) {
                const int r = k / (kActorObs / 4), c = k % (kActorObs / 4);
                *reinterpret_cast<float4*>(obs + r * kFuseObsPitch + 4 * c) = og[k];
            }
            const float4* cg = reinterpret_cast<const float4*>(p.co + (size_t(begin) + r0) * kCriticObs);
            for (int k = tid; k < nr * (kCriticObs / 4); k += kMbThreads)
                reinterpret_cast<float4*>(co)[k] = cg[k];
        }
        __syncthreads();
        // ---- forward: row rg x hidden 4hg..4hg+3 (in-order k chains from zero)
        float za[4] = {0, 0, 0, 0}, zc[4] = {0, 0, 0, 0};
        {
            const float* o0 = obs + rg * kFuseObsPitch;
#pragma unroll 2
            for (int k = 0; k < kActorObs; k += 4) {
                const float4 a = *reinterpret_cast<const float4*>(o0 + k);
                const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const float4 w = *reinterpret_cast<const float4*>(w1t + (k + kk) * kHidden + 4 * hg);
                    za[0] = fmaf(av[kk], w.x, za[0]);
                    za[1] = fmaf(av[kk], w.y, za[1]);
                    za[2] = fmaf(av[kk], w.z, za[2]);
                    za[3] = fmaf(av[kk], w.w, za[3]);
                }
            }
            const float* q0 = co + rg * kCriticObs;
#pragma unroll
            for (int k = 0; k < kCriticObs; k += 4) {
                const float4 a = *reinterpret_cast<const float4*>(q0 + k);
                const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const float4 w = *reinterpret_cast<const float4*>(cw1t + (k + kk) * kHidden + 4 * hg);
                    zc[0] = fmaf(av[kk], w.x, zc[0]);
                    zc[1] = fmaf(av[kk], w.y, zc[1]);
                    zc[2] = fmaf(av[kk], w.z, zc[2]);
                    zc[3] = fmaf(av[kk], w.w, zc[3]);
                }
            }
        }
        // ---- activations, loss, derivatives and deltas, one row per half-warp
        {
            const int lr = rg;
            const bool valid = lr < nr;
            float hv[4], chv[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                hv[j] = tanhf(za[j] + b1[4 * hg + j]);
                chv[j] = tanhf(zc[j] + cb1[4 * hg + j]);
            }
            float mean[4];
#pragma unroll
            for (int a = 0; a < 4; a++) {
                float part = 0.0f;
#pragma unroll
                for (int j = 0; j < 4; j++) part = fmaf(hv[j], w2[a * kHidden + 4 * hg + j], part);
                mean[a] = half_warp_sum(part) + b2[a];
                if (a < 3) mean[a] += obs[lr * kFuseObsPitch + kActorObs - 3 + a];
            }
            float vpart = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; j++) vpart = fmaf(chv[j], cw2[4 * hg + j], vpart);
            const float value = half_warp_sum(vpart) + cb2;
            float dm[4] = {0, 0, 0, 0}, dls[4] = {0, 0, 0, 0}, dvalue = 0.0f;
            if (valid) {
                const size_t src = size_t(begin) + r0 + lr;
                const float* act = p.actions + src * kActions;
                float logp = 0.0f;
#pragma unroll
                for (int a = 0; a < 4; a++) {
                    const float inv_std = expf(-log_std[a]);
                    const float d = (act[a] - mean[a]) * inv_std;
                    logp += -0.5f * (d * d + 2.0f * log_std[a] + kLogTwoPi);
                }
                const float adv = p.advantages[src], ret = p.returns[src];
                const float raw = logp - p.logp[src];
                const float lr_ = clampf(raw, -20.0f, 20.0f);
                const float ratio = expf(lr_);
                const float clip = p.clip;
                const float clipped = clampf(ratio, 1.0f - clip, 1.0f + clip);
                const float chosen = smin(ratio * adv, clipped * adv);
                const bool in_range = raw >= -20.0f && raw <= 20.0f;
                const bool active = in_range && (adv >= 0.0f ? ratio <= 1.0f + clip : ratio >= 1.0f - clip);
                float entropy = 0.0f;
#pragma unroll
                for (int a = 0; a < 4; a++) {
                    const float inv_var = expf(-2.0f * log_std[a]);
                    const float diff = act[a] - mean[a];
                    if (active) {
                        const float dlogp = -ratio * adv * scale;
                        dm[a] = dlogp * diff * inv_var;
                        dls[a] = dlogp * (diff * diff * inv_var - 1.0f);
                    }
                    dls[a] -= p.entropy_coef * scale;
                    entropy += -p.entropy_coef * (log_std[a] + 0.5f * (1.0f + kLogTwoPi)) * scale;
                }
                dvalue = p.value_coef * (value - ret) * scale;
                if (hg == 0) {
                    csum[0] += -chosen * scale;
                    csum[1] += 0.5f * p.value_coef * (value - ret) * (value - ret) * scale;
                    csum[2] += entropy;
                    csum[3] += ratio;
                }
            }
            if (hg == 0) {
                float* rv = rowv + lr * 9;
#pragma unroll
                for (int a = 0; a < 4; a++) {
                    rv[a] = dm[a];
                    rv[4 + a] = dls[a];
                }
                rv[8] = dvalue;
            }
            float4 hv4, dh4, chv4, cdh4;
            float* hp = &hv4.x;
            float* dp = &dh4.x;
            float* chp = &chv4.x;
            float* cdp = &cdh4.x;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                float s = 0.0f;
#pragma unroll
                for (int a = 0; a < 4; a++) s = fmaf(dm[a], w2[a * kHidden + 4 * hg + j], s);
                hp[j] = hv[j];
                dp[j] = valid ? s * (1.0f - hv[j] * hv[j]) : 0.0f;
                chp[j] = chv[j];
                cdp[j] = valid ? dvalue * cw2[4 * hg + j] * (1.0f - chv[j] * chv[j]) : 0.0f;
            }
            *reinterpret_cast<float4*>(hid + lr * kHidden + 4 * hg) = hv4;
            *reinterpret_cast<float4*>(dl + lr * kHidden + 4 * hg) = dh4;
            *reinterpret_cast<float4*>(chid + lr * kHidden + 4 * hg) = chv4;
            *reinterpret_cast<float4*>(cdl + lr * kHidden + 4 * hg) = cdh4;
        }
        __syncthreads();
        // ---- gradient accumulation over the tile's rows, in row order
        for (int r = 0; r < nr; r++) {
            const float4 d = *reinterpret_cast<const float4*>(dl + r * kHidden + 4 * ty);
            const float* orow = obs + r * kFuseObsPitch + 12 * tx;
            const float4 oa = *reinterpret_cast<const float4*>(orow);
            const float4 ob = *reinterpret_cast<const float4*>(orow + 4);
            const float4 oc = *reinterpret_cast<const float4*>(orow + 8);
            const float ov[12] = {oa.x, oa.y, oa.z, oa.w, ob.x, ob.y, ob.z, ob.w, oc.x, oc.y, oc.z, oc.w};
            const float dv4[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 12; j++) acc[i][j] = fmaf(dv4[i], ov[j], acc[i][j]);
            const float4 cd = *reinterpret_cast<const float4*>(cdl + r * kHidden + 4 * ty);
            const float2 cv = *reinterpret_cast<const float2*>(co + r * kCriticObs + 2 * tx);
            const float cdv[4] = {cd.x, cd.y, cd.z, cd.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                cacc[i][0] = fmaf(cdv[i], cv.x, cacc[i][0]);
                cacc[i][1] = fmaf(cdv[i], cv.y, cacc[i][1]);
            }
            const float* rv = rowv + r * 9;
            w2acc = fmaf(rv[tid >> 6], hid[r * kHidden + (tid & 63)], w2acc);  // W2[a][h] = sum d_mean[a] h
            if (tid < 64) misc += dl[r * kHidden + tid];
            else if (tid < 128) misc += cdl[r * kHidden + tid - 64];
            else if (tid < 192) misc = fmaf(rv[8], chid[r * kHidden + tid - 128], misc);
            else if (tid < 196) misc += rv[tid - 192];
            else if (tid < 200) misc += rv[4 + tid - 196];
            else if (tid == 200) misc += rv[8];
        }
    }
    // gradient partial of this CTA (the same layout as k_mb_grad)
    float* out = p.grad_partials + size_t(blockIdx.x) * kPpoParams;
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 12; j++) {
            const int c = 12 * tx + j;
            if (c < kActorObs) out[(4 * ty + i) * kActorObs + c] = acc[i][j];
        }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        out[kActorParams + (4 * ty + i) * kCriticObs + 2 * tx] = cacc[i][0];
        out[kActorParams + (4 * ty + i) * kCriticObs + 2 * tx + 1] = cacc[i][1];
    }
    out[kActorW2 + tid] = w2acc;
    if (tid < 64) out[kActorB1 + tid] = misc;
    else if (tid < 128) out[kActorParams + kCriticB1 + tid - 64] = misc;
    else if (tid < 192) out[kActorParams + kCriticW2 + tid - 128] = misc;
    else if (tid < 196) out[kActorB2 + tid - 192] = misc;
    else if (tid < 200) out[kActorLogStd + tid - 196] = misc;
    else if (tid == 200) out[kActorParams + kCriticB2] = misc;
    // loss sums of this CTA: per-thread row sums (half-warp leaders), added in thread order
    __syncthreads();
    for (int k = 0; k < 4; k++) stage[tid * 4 + k] = csum[k];
    __syncthreads();
    if (tid < 4) {
        float s = 0.0f;
        for (int t = 0; t < kMbThreads; t += 16) s += stage[t * 4 + tid];
        p.loss_partials[(size_t(update) * p.fwd_grid + blockIdx.x) * 4 + tid] = s;
    }
}

// ------------------------------------------------------------- launchers
size_t mb_forward_smem_bytes() { return kMbSmemFloats * sizeof(float); }

cudaError_t configure_ppo_kernels() {
    cudaError_t e = cudaFuncSetAttribute(k_mb_fused, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(kFuseSmemFloats * sizeof(float)));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_mb_forward<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(mb_forward_smem_bytes()));
}

uint32_t gae_blocks(uint32_t n) { return (n + kGaeThreads - 1) / kGaeThreads; }

cudaError_t launch_gae_sum(const PpoArgs& p, cudaStream_t s) {
    k_gae_sum<<<gae_blocks(p.n), kGaeThreads, 0, s>>>(p);
    return cudaGetLastError();
}
cudaError_t launch_adv_stats(const PpoArgs& p, int mode, cudaStream_t s) {
    k_adv_stats<<<1, 256, 0, s>>>(p, gae_blocks(p.n), mode);
    return cudaGetLastError();
}
cudaError_t launch_adv_finalize(const PpoArgs& p, int mode, cudaStream_t s) {
    k_adv_finalize<<<1, 32, 0, s>>>(p, mode);
    return cudaGetLastError();
}
cudaError_t launch_adv_sq(const PpoArgs& p, cudaStream_t s) {
    k_adv_sq<<<gae_blocks(p.n), kGaeThreads, 0, s>>>(p);
    return cudaGetLastError();
}
cudaError_t launch_adv_apply(const PpoArgs& p, int sm_count, cudaStream_t s) {
    const size_t rows = size_t(p.n) * p.horizon;
    const unsigned grid = unsigned(std::min<size_t>((rows + 255) / 256, size_t(sm_count) * 8));
    k_adv_apply<<<grid, 256, 0, s>>>(p);
    return cudaGetLastError();
}
cudaError_t launch_minibatch(const PpoArgs& p, uint32_t update, uint32_t chunks, cudaStream_t s) {
    if (p.wide_slices) {
        k_mb_forward<true><<<p.fwd_grid, kMbThreads, mb_forward_smem_bytes(), s>>>(p, update);
        k_mb_grad<true><<<chunks, kGradThreads, 0, s>>>(p, update);
    } else {
        // one kernel per minibatch: p.fwd_grid == chunks CTAs of p.grad_chunk rows
        k_mb_fused<<<chunks, kMbThreads, kFuseSmemFloats * sizeof(float), s>>>(p, update);
    }
    if (chunks > 1) k_grad_reduce<<<(kPpoParams + 255) / 256, 256, 0, s>>>(p, chunks);
    return cudaGetLastError();
}
cudaError_t launch_grad_reduce(const PpoArgs& p, uint32_t chunks, cudaStream_t s) {
    k_grad_reduce<<<(kPpoParams + 255) / 256, 256, 0, s>>>(p, chunks);
    return cudaGetLastError();
}
cudaError_t launch_clip_adam(const PpoArgs& p, uint32_t update, uint32_t chunks, cudaStream_t s) {
    k_clip_adam<<<2, kAdamThreads, 0, s>>>(p, update, chunks > 1 ? p.grad : p.grad_partials, 0);
    return cudaGetLastError();
}
cudaError_t launch_clip_adam_critic(const PpoArgs& p, uint32_t update, const float* grad_critic, cudaStream_t s) {
    // k_clip_adam reads the critic at grad_src[kActorParams + i].
    k_clip_adam<<<1, kAdamThreads, 0, s>>>(p, update, grad_critic - kActorParams, 1);
    return cudaGetLastError();
}
cudaError_t launch_metrics_mean(const PpoArgs& p, uint32_t updates, cudaStream_t s) {
    k_metrics_mean<<<1, 32, 0, s>>>(p, updates);
    return cudaGetLastError();
}

// ------------------------------------------------- allocation-free entry
// Scratch of mdn_gae_normalize_static: one fp64 partial sum per 256-env block,
// the two fp64 totals and the two float statistics. A fixed file-scope device
// array, so the entry point never allocates. Every kernel writes the slots it
// later reads before reading them (partials by block, totals, statistics), so
// nothing has to start at zero; leftovers of an earlier call are overwritten.
constexpr uint32_t kStaticGaeMaxBlocks = 4096;  // envs <= 4096 * 256
struct StaticGaeScratch {
    double partials[kStaticGaeMaxBlocks];
    double stats[2];
    float values[2];
};
static __device__ __align__(256) StaticGaeScratch g_static_gae_scratch;

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
StaticGaeScratch* g_static_ptr[kMaxDevices] = {};
int g_static_sms[kMaxDevices] = {};

}  // namespace
}  // namespace mdn

extern "C" int mdn_gae_normalize_static(const float* rewards, const float* values, const float* next_values,
                                        const uint8_t* terminated, const uint8_t* truncated, float* advantages,
                                        float* returns, uint32_t horizon, uint32_t envs, float gamma, float lambda,
                                        void* stream) {
    using namespace mdn;
    return guarded([&] {
        require(rewards && values && next_values && terminated && truncated && advantages && returns, MDN_ERR_INVALID,
                "mdn_gae_normalize_static: null pointer");
        require(horizon >= 1 && envs >= 1, MDN_ERR_INVALID, "mdn_gae_normalize_static: empty rollout");
        require(gae_blocks(envs) <= kStaticGaeMaxBlocks, MDN_ERR_INVALID,
                "mdn_gae_normalize_static: envs exceeds the fixed scratch limit of 1,048,576 (4,096 blocks of 256)");
        int dev = 0;
        cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
        require(dev >= 0 && dev < kMaxDevices, MDN_ERR_INVALID, "mdn_gae_normalize_static: device index too large");
        StaticGaeScratch* scratch;
        int sms;
        {
            // Set-up, once per device with that device current: the host-side
            // name of the array is not a device address; ask the runtime.
            std::lock_guard<std::mutex> lock(g_static_mu);
            if (!g_static_ptr[dev]) {
                void* ptr = nullptr;
                cuda_check(cudaGetSymbolAddress(&ptr, g_static_gae_scratch), "cudaGetSymbolAddress(scratch)");
                int count = 0;
                cuda_check(cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev), "SM count");
                g_static_sms[dev] = count;
                g_static_ptr[dev] = static_cast<StaticGaeScratch*>(ptr);
            }
            scratch = g_static_ptr[dev];
            sms = g_static_sms[dev];
        }
        PpoArgs p{};
        p.n = envs;
        p.horizon = horizon;
        p.global_rows = uint64_t(envs) * horizon;
        p.gamma = gamma;
        p.lambda = lambda;
        p.rewards = rewards;
        p.values = values;
        p.next_values = next_values;
        p.terminated = terminated;
        p.truncated = truncated;
        p.advantages = advantages;
        p.returns = returns;
        p.stat_partials = scratch->partials;
        p.stats = scratch->stats;
        p.stat_values = scratch->values;
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        cuda_check(launch_gae_sum(p, s), "gae");
        cuda_check(launch_adv_stats(p, 0, s), "advantage sum");
        cuda_check(launch_adv_finalize(p, 0, s), "advantage mean");
        cuda_check(launch_adv_sq(p, s), "advantage variance");
        cuda_check(launch_adv_stats(p, 1, s), "advantage variance sum");
        cuda_check(launch_adv_finalize(p, 1, s), "advantage scale");
        cuda_check(launch_adv_apply(p, sms, s), "advantage normalise");
    });
}
