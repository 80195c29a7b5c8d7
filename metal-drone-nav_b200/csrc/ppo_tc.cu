// PPO minibatch step of the 64-unit actor and critic on the tcgen05 tensor
// cores (TF32 products, fp32 accumulators): the same quantities as k_mb_fused
// (ppo.cu) -- forward, clipped-PPO loss and derivatives (ppo.hpp:144-181),
// hidden deltas and the gradient partial of every parameter
// (cpu_reference.hpp:515-551) -- for large minibatches.
//
// One persistent CTA per SM walks 128-row tiles of the minibatch:
//   forward   D_a[128 rows x 64] = obs . W1^T and D_c[128 x 64] = co . cW1^T
//             (M = 128 rows; A = the rows, K-major, 128-byte swizzle; B = the
//             weights, resident in shared memory);
//   epilogue  one thread per row (two groups of four warps, tiles alternate
//             between the groups): tanh, means + geometry prior, value, loss and
//             derivatives, hidden deltas. The deltas go to shared memory as the
//             K-major A operand of the weight gradients; the small gradients
//             (dW2, db1, critic b1 / w2, b2, log_std, critic b2, loss sums) are
//             summed over the warp's rows by a fixed shuffle tree and kept per
//             lane across tiles;
//   wgrad     G_a[64 x 192] += delta_a^T . obs and G_c[64 x 32] += delta_c^T .
//             co (M = 64 hidden units; K = the tile's rows). The rows are
//             fetched a second time (from L2) by TMA in the MN-major layout
//             tf32 operands require there (128-byte swizzle, 32-byte atoms):
//             one shared copy cannot be both K-major and MN-major.
// The hidden activations and deltas never reach HBM; a row-epoch reads its
// observation, critic observation, action, log-prob, advantage and return
// once from HBM. At the end each CTA writes its gradient partial in the layout
// of k_mb_fused, so k_grad_reduce / k_clip_adam apply unchanged.
//
// Warp roles: warp 0 issues TMA loads (one ring of 16 KB row panels for
// both layouts), warp 1 owns tensor memory and issues the MMAs, warps 2-9 are
// the epilogue. Every barrier wait is bounded; a wait that gives up sets a
// bit of the error flag and the kernel winds down.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>

#include "mdn_device.cuh"
#include "ppo_args.h"
#include "ppo_tc.h"
#include "tc.cuh"

namespace mdn {

namespace {
constexpr int kTcRows = 128;                  // rows per tile
constexpr int kTcPanel = 32;                  // fp32 columns per 128-byte panel
constexpr int kTcObsPanels = 6;               // 184 inputs padded to 192 (TMA zero-fills)
constexpr int kTcInPanels = kTcObsPanels + 1; // + the critic's 32 inputs
constexpr int kTcStages = 6;
constexpr int kTcStageBytes = kTcRows * 128;  // one 128-row panel
constexpr int kTcWPanelBytes = kHidden * 128; // one 64-row weight panel
constexpr int kTcDeltaBytes = kHidden * 128;  // 64 hidden x 32 rows, K-major
constexpr int kTcEpiWarps = 8;
constexpr int kTcThreads = (2 + kTcEpiWarps) * 32;
constexpr int kTcChunks = 15;                 // per-lane small-gradient columns (see epilogue)
constexpr long long kTcWaitLimit = 2000000000ll;

// tensor-memory columns
constexpr uint32_t kColD = 0;      // D buffers: [128 * buf, +64) actor, [+64, +128) critic
constexpr uint32_t kColGa = 256;   // G_a panel p at 256 + 32 p (p < 6)
constexpr uint32_t kColGc = 448;   // G_c

// shared-memory layout (from a 1024-byte aligned base)
constexpr size_t kOffRing = 0;
constexpr size_t kOffW1 = kOffRing + size_t(kTcStages) * kTcStageBytes;
constexpr size_t kOffCw1 = kOffW1 + size_t(kTcObsPanels) * kTcWPanelBytes;
constexpr size_t kOffDa = kOffCw1 + kTcWPanelBytes;
constexpr size_t kOffDc = kOffDa + 4 * size_t(kTcDeltaBytes);
constexpr size_t kOffPar = kOffDc + 4 * size_t(kTcDeltaBytes);
// b1[64], W2[4][64], cb1[64], cw2[64], b2[4], log_std[4], cb2, pad
constexpr int kParFloats = 64 + 256 + 64 + 64 + 4 + 4 + 4;
constexpr size_t kOffBar = kOffPar + kParFloats * sizeof(float);

struct TcBarriers {
    uint64_t full[kTcStages];
    uint64_t empty[kTcStages];
    uint64_t fwd_full[2];
    uint64_t fwd_empty[2];
    uint64_t delta_full;
    uint64_t delta_empty;
    uint64_t weights;
    uint64_t final_mma;
    uint32_t tmem_base;
};
constexpr size_t kTcSmem = 1024 + kOffBar + sizeof(TcBarriers);
static_assert(kTcSmem <= 227 * 1024, "tensor-core minibatch kernel exceeds the shared-memory budget");
static_assert(size_t(kTcEpiWarps) * kTcChunks * 32 * sizeof(float) <= size_t(kTcStages) * kTcStageBytes,
              "final reduction staging reuses the ring");

// tanh(x) = 1 - 2 / (1 + e^(2x)) on the hardware base-2 exponential and
// reciprocal (ex2.approx / rcp.approx): absolute error ~1e-7, far below the
// TF32 products it follows; saturates to +-1.
__device__ __forceinline__ float tc_tanh(float x) {
    float e, r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x * 2.8853900817779268f));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
    return fmaf(-2.0f, r, 1.0f);
}

// Sum of x[i] over the warp's 32 lanes; lane j receives the total of column
// j. A fixed halving tree (31 exchanges), so the result does not depend on
// scheduling.
__device__ __forceinline__ float lane_column_sum(float (&x)[32], int lane) {
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
        const bool upper = (lane & s) != 0;
#pragma unroll
        for (int i = 0; i < s; i++) {
            const float send = upper ? x[i] : x[i + s];
            const float keep = upper ? x[i + s] : x[i];
            x[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
        }
    }
    return x[0];
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void epilogue_bar_sync() {
    asm volatile("bar.sync 1, %0;" ::"r"(kTcEpiWarps * 32) : "memory");
}
}  // namespace

__global__ void __launch_bounds__(kTcThreads, 1)
    k_mb_tc(const __grid_constant__ CUtensorMap obs_k, const __grid_constant__ CUtensorMap obs_mn,
            const __grid_constant__ CUtensorMap co_k, const __grid_constant__ CUtensorMap co_mn,
            const __grid_constant__ CUtensorMap w1_map, const __grid_constant__ CUtensorMap cw1_map, PpoArgs p,
            uint32_t update) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ring = smem + kOffRing;
    uint8_t* w1s = smem + kOffW1;
    uint8_t* cw1s = smem + kOffCw1;
    uint8_t* da = smem + kOffDa;
    uint8_t* dc = smem + kOffDc;
    float* par = reinterpret_cast<float*>(smem + kOffPar);
    TcBarriers& s = *reinterpret_cast<TcBarriers*>(smem + kOffBar);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const uint32_t begin = p.starts[update];
    const uint32_t b = p.batch[update];
    const uint32_t tiles = (b + kTcRows - 1) / kTcRows;
    const uint32_t count = blockIdx.x < tiles ? (tiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0u;
    auto tile_row0 = [&](uint32_t j) { return int32_t(begin + (blockIdx.x + j * gridDim.x) * kTcRows); };

    if (threadIdx.x == 0) {
        for (int i = 0; i < kTcStages; i++) {
            tc::mbar_init(&s.full[i], 1);
            tc::mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            tc::mbar_init(&s.fwd_full[i], 1);
            tc::mbar_init(&s.fwd_empty[i], 4);
        }
        tc::mbar_init(&s.delta_full, 4);
        tc::mbar_init(&s.delta_empty, 1);
        tc::mbar_init(&s.weights, 1);
        tc::mbar_init(&s.final_mma, 1);
        tc::fence_barrier_init();
        tc::prefetch_tmap(&obs_k);
        tc::prefetch_tmap(&obs_mn);
        tc::prefetch_tmap(&co_k);
        tc::prefetch_tmap(&co_mn);
    }
    if (warp == 1) {
        tc::tmem_alloc(&s.tmem_base, 512);
        tc::tmem_relinquish();
    }
    // small parameters for the epilogue
    for (int k = threadIdx.x; k < kParFloats; k += kTcThreads) {
        float v = 0.0f;
        if (k < 64) v = p.actor[kActorB1 + k];
        else if (k < 320) v = p.actor[kActorW2 + (k - 64)];
        else if (k < 384) v = p.critic[kCriticB1 + (k - 320)];
        else if (k < 448) v = p.critic[kCriticW2 + (k - 384)];
        else if (k < 452) v = p.actor[kActorB2 + (k - 448)];
        else if (k < 456) v = p.actor[kActorLogStd + (k - 452)];
        else if (k == 456) v = p.critic[kCriticB2];
        par[k] = v;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = s.tmem_base;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------ TMA producer
        // order: K(0); then for s >= 1: K(s), MN(s - 1) -- the next tile's
        // forward panels go ahead of this tile's weight-gradient panels.
        bool ok = true;
        if (count > 0) {
            tc::mbar_arrive_expect_tx(&s.weights, (kTcObsPanels + 1) * kTcWPanelBytes);
            for (int q = 0; q < kTcObsPanels; q++)
                tc::tma_load_2d(w1s + q * kTcWPanelBytes, &w1_map, q * kTcPanel, 0, &s.weights);
            tc::tma_load_2d(cw1s, &cw1_map, 0, 0, &s.weights);
        }
        uint32_t it = 0;
        auto load = [&](const CUtensorMap* map, int32_t x, int32_t y) {
            const uint32_t st = it % kTcStages, use = it / kTcStages;
            if (use > 0 && !tc::mbar_wait(&s.empty[st], (use - 1) & 1, kTcWaitLimit)) return false;
            tc::mbar_arrive_expect_tx(&s.full[st], kTcStageBytes);
            tc::tma_load_2d(ring + size_t(st) * kTcStageBytes, map, x, y, &s.full[st]);
            it++;
            return true;
        };
        for (uint32_t t = 0; t <= count && ok && count > 0; t++) {
            if (t < count) {
                const int32_t y = tile_row0(t);
                for (int q = 0; q < kTcObsPanels && ok; q++) ok = load(&obs_k, q * kTcPanel, y);
                if (ok) ok = load(&co_k, 0, y);
            }
            if (t >= 1 && ok) {
                const int32_t y = tile_row0(t - 1);
                for (int q = 0; q < kTcObsPanels && ok; q++) ok = load(&obs_mn, q * kTcPanel, y);
                if (ok) ok = load(&co_mn, 0, y);
            }
        }
        // every copy this CTA issued has landed before it may exit
        for (uint32_t k = it > kTcStages ? it - kTcStages : 0; k < it; k++)
            if (!tc::mbar_wait(&s.full[k % kTcStages], (k / kTcStages) & 1, kTcWaitLimit)) ok = false;
        if (count > 0 && !tc::mbar_wait(&s.weights, 0, kTcWaitLimit)) ok = false;
        if (!ok) atomicOr(p.tc_error, 1u);
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------- MMA issuer
        constexpr uint32_t idesc_fwd = tc::tf32_idesc(kTcRows, kHidden, 0, 0);
        constexpr uint32_t idesc_wg = tc::tf32_idesc(kHidden, kTcPanel, 0, 1);
        bool ok = count == 0 || tc::mbar_wait(&s.weights, 0, kTcWaitLimit);
        uint32_t it = 0;
        auto take = [&](uint32_t& addr) {
            const uint32_t st = it % kTcStages;
            if (!tc::mbar_wait(&s.full[st], (it / kTcStages) & 1, kTcWaitLimit)) return false;
            tc::fence_after_sync();
            addr = tc::smem_u32(ring + size_t(st) * kTcStageBytes);
            return true;
        };
        auto release = [&]() {
            tc::mma_commit(&s.empty[it % kTcStages]);
            it++;
        };
        for (uint32_t t = 0; t <= count && ok && count > 0; t++) {
            if (t < count) {
                // forward of tile t into accumulator buffer t & 1
                const uint32_t buf = t & 1;
                if (t >= 2 && !tc::mbar_wait(&s.fwd_empty[buf], ((t >> 1) - 1) & 1, kTcWaitLimit)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t d_a = tmem + kColD + 128 * buf, d_c = d_a + 64;
                for (int q = 0; q < kTcInPanels && ok; q++) {
                    uint32_t a_addr;
                    if (!take(a_addr)) {
                        ok = false;
                        break;
                    }
                    const bool critic = q == kTcObsPanels;
                    const uint32_t b_addr = tc::smem_u32(critic ? cw1s : w1s + q * kTcWPanelBytes);
#pragma unroll
                    for (int kk = 0; kk < kTcPanel / 8; kk++)
                        tc::mma_tf32(critic ? d_c : d_a, tc::sw128_desc(a_addr + kk * 32, 16, 1024),
                                     tc::sw128_desc(b_addr + kk * 32, 16, 1024), idesc_fwd,
                                     (!critic && q != 0) || kk != 0 ? 1u : 0u);
                    release();
                }
                if (!ok) break;
                tc::mma_commit(&s.fwd_full[buf]);
            }
            if (t >= 1) {
                // weight gradients of tile j = t - 1 once its deltas are in shared memory
                const uint32_t j = t - 1;
                if (!tc::mbar_wait(&s.delta_full, j & 1, kTcWaitLimit)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                for (int q = 0; q < kTcInPanels && ok; q++) {
                    uint32_t b_addr;
                    if (!take(b_addr)) {
                        ok = false;
                        break;
                    }
                    const bool critic = q == kTcObsPanels;
                    const uint32_t a_base = tc::smem_u32(critic ? dc : da);
                    const uint32_t d = tmem + (critic ? kColGc : kColGa + 32 * q);
#pragma unroll
                    for (int w = 0; w < 4; w++)          // the tile's four 32-row groups (K)
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)   // 8 rows per MMA
                            tc::mma_tf32(d, tc::sw128_desc(a_base + w * kTcDeltaBytes + kk * 32, 16, 1024),
                                         tc::sw128b32_desc(b_addr + (32 * w + 8 * kk) * 128, kTcStageBytes, 512),
                                         idesc_wg, (j | w | kk) != 0 ? 1u : 0u);
                    release();
                }
                if (!ok) break;
                tc::mma_commit(&s.delta_empty);
            }
        }
        tc::mma_commit(&s.final_mma);
        if (!ok) atomicOr(p.tc_error, 2u);
    } else if (warp >= 2) {
        // --------------------------------------------------------- epilogue
        const int ew = warp - 2;   // 0..7
        const int g = ew >> 2;     // this group takes the tiles j with j % 2 == g (accumulator buffer g)
        const int q = warp & 3;    // tensor-memory lanes 32q..32q+31 = rows 32q..32q+31 of a tile
        const float* b1 = par;
        const float* w2 = par + 64;
        const float* cb1 = par + 320;
        const float* cw2 = par + 384;
        const float* b2 = par + 448;
        const float* log_std = par + 452;
        const float cb2 = par[456];
        const float scale = 1.0f / fmaxf(float(p.global_batch[update]), 1.0f);
        // Per-lane running sums, lane j holding column j of each chunk:
        // 0-7 dW2[a][32c + j] (chunk 2a + c), 8-9 critic w2, 10-11 b1,
        // 12-13 critic b1, 14 = d_mean[4], d_log_std[4], d_value, loss sums[4].
        float acc[kTcChunks];
#pragma unroll
        for (int k = 0; k < kTcChunks; k++) acc[k] = 0.0f;
        bool ok = true;
        for (uint32_t j = g; j < count; j += 2) {
            if (!tc::mbar_wait(&s.fwd_full[g], (j >> 1) & 1, kTcWaitLimit)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const uint32_t local = (blockIdx.x + j * gridDim.x) * kTcRows + 32 * q + lane;  // row of the minibatch
            const bool valid = local < b;
            const size_t src = size_t(begin) + local;
            const uint32_t lane_addr = tmem + (uint32_t(32 * q) << 16) + kColD + 128 * g;
            float hc[64], hh[64];
            {
                float v[32];
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    tc::tmem_ld32(lane_addr + 64 + 32 * c, v);
#pragma unroll
                    for (int i = 0; i < 32; i++) hc[32 * c + i] = tc_tanh(v[i] + cb1[32 * c + i]);
                }
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    tc::tmem_ld32(lane_addr + 32 * c, v);
#pragma unroll
                    for (int i = 0; i < 32; i++) hh[32 * c + i] = tc_tanh(v[i] + b1[32 * c + i]);
                }
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&s.fwd_empty[g]);  // the accumulator buffer is free again
            float value = cb2;
#pragma unroll
            for (int i = 0; i < 64; i++) value = fmaf(cw2[i], hc[i], value);
            float mean[4];
#pragma unroll
            for (int a = 0; a < 4; a++) {
                float m = b2[a];
#pragma unroll
                for (int i = 0; i < 64; i++) m = fmaf(w2[a * 64 + i], hh[i], m);
                mean[a] = m;
            }
            // clipped-PPO loss and derivatives (ppo.hpp:144-181)
            float dm[4] = {0, 0, 0, 0}, dls[4] = {0, 0, 0, 0}, dvalue = 0.0f, loss[4] = {0, 0, 0, 0};
            if (valid) {
#pragma unroll
                for (int a = 0; a < 3; a++) mean[a] += __ldg(p.obs + src * kActorObs + kActorObs - 3 + a);
                const float* act = p.actions + src * kActions;
                float logp = 0.0f;
#pragma unroll
                for (int a = 0; a < 4; a++) {
                    const float d = (act[a] - mean[a]) * expf(-log_std[a]);
                    logp += -0.5f * (d * d + 2.0f * log_std[a] + kLogTwoPi);
                }
                const float adv = p.advantages[src], ret = p.returns[src];
                const float raw = logp - p.logp[src];
                const float ratio = expf(clampf(raw, -20.0f, 20.0f));
                const float clipped = clampf(ratio, 1.0f - p.clip, 1.0f + p.clip);
                const float chosen = smin(ratio * adv, clipped * adv);
                const bool in_range = raw >= -20.0f && raw <= 20.0f;
                const bool active = in_range && (adv >= 0.0f ? ratio <= 1.0f + p.clip : ratio >= 1.0f - p.clip);
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
                loss[0] = -chosen * scale;
                loss[1] = 0.5f * p.value_coef * (value - ret) * (value - ret) * scale;
                loss[2] = entropy;
                loss[3] = ratio;
            }
            float x[32];
            // dW2[a][h] = sum over rows of d_mean[a] tanh_h; critic w2 = sum d_value tanh_c
#pragma unroll
            for (int a = 0; a < 4; a++)
#pragma unroll
                for (int c = 0; c < 2; c++) {
#pragma unroll
                    for (int i = 0; i < 32; i++) x[i] = dm[a] * hh[32 * c + i];
                    acc[2 * a + c] += lane_column_sum(x, lane);
                }
#pragma unroll
            for (int c = 0; c < 2; c++) {
#pragma unroll
                for (int i = 0; i < 32; i++) x[i] = dvalue * hc[32 * c + i];
                acc[8 + c] += lane_column_sum(x, lane);
            }
            // hidden deltas, in place: (W2^T d_mean)(1 - h^2) and d_value cw2 (1 - hc^2)
#pragma unroll
            for (int i = 0; i < 64; i++) {
                float sv = dm[0] * w2[i];
                sv = fmaf(dm[1], w2[64 + i], sv);
                sv = fmaf(dm[2], w2[128 + i], sv);
                sv = fmaf(dm[3], w2[192 + i], sv);
                hh[i] = sv * (1.0f - hh[i] * hh[i]);
                hc[i] = dvalue * cw2[i] * (1.0f - hc[i] * hc[i]);
            }
            // The previous tile's weight-gradient MMAs must be done reading the
            // delta operands before they are overwritten.
            if (j >= 1 && !tc::mbar_wait(&s.delta_empty, (j - 1) & 1, kTcWaitLimit)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            {
                // K-major 128-byte swizzle: hidden unit h is a 128-byte row of the
                // [64 x 32 rows] operand, this thread's row is column `lane`.
                uint8_t* pa = da + q * kTcDeltaBytes;
                uint8_t* pc = dc + q * kTcDeltaBytes;
                const uint32_t in_granule = (lane & 3) * 4;
#pragma unroll
                for (int h = 0; h < 64; h++) {
                    const uint32_t off = (h >> 3) * 1024 + (h & 7) * 128 + ((((lane >> 2) ^ (h & 7))) << 4) + in_granule;
                    *reinterpret_cast<float*>(pa + off) = hh[h];
                    *reinterpret_cast<float*>(pc + off) = hc[h];
                }
            }
            fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor cores
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&s.delta_full);
            // b1 and critic b1: sums of the deltas
#pragma unroll
            for (int c = 0; c < 2; c++) {
#pragma unroll
                for (int i = 0; i < 32; i++) x[i] = hh[32 * c + i];
                acc[10 + c] += lane_column_sum(x, lane);
#pragma unroll
                for (int i = 0; i < 32; i++) x[i] = hc[32 * c + i];
                acc[12 + c] += lane_column_sum(x, lane);
            }
#pragma unroll
            for (int i = 0; i < 32; i++) x[i] = 0.0f;
#pragma unroll
            for (int a = 0; a < 4; a++) {
                x[a] = dm[a];
                x[4 + a] = dls[a];
                x[9 + a] = loss[a];
            }
            x[8] = dvalue;
            acc[14] += lane_column_sum(x, lane);
        }
        if (!ok) atomicOr(p.tc_error, 4u);
        // every MMA is done: the weight-gradient accumulators are final and the ring is free
        const bool mma_done = count == 0 || tc::mbar_wait(&s.final_mma, 0, kTcWaitLimit);
        tc::fence_after_sync();
        float* red = reinterpret_cast<float*>(ring);
#pragma unroll
        for (int k = 0; k < kTcChunks; k++) red[(ew * kTcChunks + k) * 32 + lane] = acc[k];
        epilogue_bar_sync();
        float* out = p.grad_partials + size_t(blockIdx.x) * kPpoParams;
        if (g == 0) {
            // dW1 and critic dW1: lanes 32q..32q+15 of the M = 64 accumulators
            // hold hidden units 16q..16q+15
            const uint32_t gaddr = tmem + (uint32_t(32 * q) << 16);
            const int hid = 16 * q + lane;
            float v[32];
            for (int pp = 0; pp < kTcObsPanels; pp++) {
                tc::tmem_ld32(gaddr + kColGa + 32 * pp, v);
                if (lane < 16)
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        if (32 * pp + i < kActorObs) out[hid * kActorObs + 32 * pp + i] = count ? v[i] : 0.0f;
            }
            tc::tmem_ld32(gaddr + kColGc, v);
            if (lane < 16)
#pragma unroll
                for (int i = 0; i < 32; i++) out[kActorParams + hid * kCriticObs + i] = count ? v[i] : 0.0f;
            // small gradients: the eight warps' columns added in warp order
            for (int idx = ew * 32 + lane; idx < kTcChunks * 32; idx += 128) {
                const int k = idx >> 5, col = idx & 31;
                float sum = 0.0f;
                for (int w = 0; w < kTcEpiWarps; w++) sum += red[(w * kTcChunks + k) * 32 + col];
                if (k < 8) out[kActorW2 + (k >> 1) * 64 + (k & 1) * 32 + col] = sum;
                else if (k < 10) out[kActorParams + kCriticW2 + (k - 8) * 32 + col] = sum;
                else if (k < 12) out[kActorB1 + (k - 10) * 32 + col] = sum;
                else if (k < 14) out[kActorParams + kCriticB1 + (k - 12) * 32 + col] = sum;
                else if (col < 4) out[kActorB2 + col] = sum;
                else if (col < 8) out[kActorLogStd + col - 4] = sum;
                else if (col == 8) out[kActorParams + kCriticB2] = sum;
                else if (col < 13) p.loss_partials[(size_t(update) * p.fwd_grid + blockIdx.x) * 4 + col - 9] = sum;
            }
        }
        if (!mma_done) atomicOr(p.tc_error, 8u);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 512);
    }
}

// ------------------------------------------------------------- launchers
namespace {
CUtensorMap as_map(const WideMap& m) {
    CUtensorMap out;
    static_assert(sizeof(CUtensorMap) <= sizeof(m.bytes), "tensor map storage");
    std::memcpy(&out, m.bytes, sizeof(out));
    return out;
}
}  // namespace

cudaError_t tc_make_maps(TcMaps* m, const float* obs, const float* co, uint64_t rows, const float* actor,
                         const float* critic) {
    cudaError_t e = wide_make_map(&m->obs_k, obs, kActorObs, rows, kActorObs * sizeof(float), kTcRows, false);
    if (e == cudaSuccess) e = wide_make_map(&m->obs_mn, obs, kActorObs, rows, kActorObs * sizeof(float), kTcRows, true);
    if (e == cudaSuccess) e = wide_make_map(&m->co_k, co, kCriticObs, rows, kCriticObs * sizeof(float), kTcRows, false);
    if (e == cudaSuccess) e = wide_make_map(&m->co_mn, co, kCriticObs, rows, kCriticObs * sizeof(float), kTcRows, true);
    // W1 [64][184] and critic W1 [64][32] (the first blocks of the flat parameter vectors, ppo.hpp:35-45)
    if (e == cudaSuccess) e = wide_make_map(&m->w1, actor, kActorObs, kHidden, kActorObs * sizeof(float), kHidden, false);
    if (e == cudaSuccess) e = wide_make_map(&m->cw1, critic, kCriticObs, kHidden, kCriticObs * sizeof(float), kHidden, false);
    return e;
}

cudaError_t configure_tc_kernels() {
    return cudaFuncSetAttribute(k_mb_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kTcSmem));
}

uint32_t tc_grid(uint32_t minibatch, int sm_count) {
    const uint32_t tiles = (minibatch + kTcRows - 1) / kTcRows;
    return tiles < uint32_t(sm_count) ? (tiles ? tiles : 1u) : uint32_t(sm_count);
}

cudaError_t launch_minibatch_tc(const PpoArgs& p, const TcMaps& m, uint32_t update, uint32_t grid, cudaStream_t s) {
    k_mb_tc<<<grid, kTcThreads, kTcSmem, s>>>(as_map(m.obs_k), as_map(m.obs_mn), as_map(m.co_k), as_map(m.co_mn),
                                              as_map(m.w1), as_map(m.cw1), p, update);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || grid <= 1) return e;
    return launch_grad_reduce(p, grid, s);
}

}  // namespace mdn
