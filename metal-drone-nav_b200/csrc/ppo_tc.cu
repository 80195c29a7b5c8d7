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
// Warp roles: warp 0 loads the forward panels, warp 10 the weight-gradient
// panels (two rings of 16 KB row panels), warp 1 owns tensor memory and
// issues the MMAs, warps 2-9 are the epilogue. Every barrier wait is bounded; a wait that gives up sets a
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
// Two rings of 128-row panels: the K-major panels of the forward (read from
// HBM) and the MN-major panels of the weight gradients (re-read from L2),
// each with its own producer warp, so forward loads keep streaming while
// weight-gradient panels wait for a tile's deltas.
constexpr int kKStages = 4;
constexpr int kMStages = 2;
constexpr int kTcStageBytes = kTcRows * 128;  // one 128-row panel
constexpr int kTcWPanelBytes = kHidden * 128; // one 64-row weight panel
constexpr int kTcDeltaBytes = kHidden * 128;  // 64 hidden x 32 rows, K-major
constexpr int kTcEpiWarps = 8;
constexpr int kWarpKProducer = 0, kWarpMma = 1, kWarpEpi0 = 2, kWarpMProducer = 2 + kTcEpiWarps;
constexpr int kTcThreads = (kWarpMProducer + 1) * 32;
constexpr int kTcChunks = 15;                 // per-lane small-gradient columns (see epilogue)
constexpr long long kTcWaitLimit = 2000000000ll;

// tensor-memory columns
constexpr uint32_t kColD = 0;      // D buffers: [128 * buf, +64) actor, [+64, +128) critic
constexpr uint32_t kColGa = 256;   // G_a panel p at 256 + 32 p (p < 6)
constexpr uint32_t kColGc = 448;   // G_c

// shared-memory layout (from a 1024-byte aligned base)
constexpr size_t kOffKRing = 0;
constexpr size_t kOffMRing = kOffKRing + size_t(kKStages) * kTcStageBytes;
constexpr size_t kOffW1 = kOffMRing + size_t(kMStages) * kTcStageBytes;
constexpr size_t kOffCw1 = kOffW1 + size_t(kTcObsPanels) * kTcWPanelBytes;
constexpr size_t kOffDa = kOffCw1 + kTcWPanelBytes;
constexpr size_t kOffDc = kOffDa + 4 * size_t(kTcDeltaBytes);
constexpr size_t kOffPar = kOffDc + 4 * size_t(kTcDeltaBytes);
// b1[64], W2[4][64], cb1[64], cw2[64], b2[4], log_std[4], cb2, pad,
// then W2 transposed [64][4] (one 128-bit load per hidden unit)
constexpr int kParW2t = 64 + 256 + 64 + 64 + 4 + 4 + 4;
constexpr int kParFloats = kParW2t + 256;
constexpr size_t kOffBar = kOffPar + kParFloats * sizeof(float);

struct TcBarriers {
    uint64_t kfull[kKStages];
    uint64_t kempty[kKStages];
    uint64_t mfull[kMStages];
    uint64_t mempty[kMStages];
    uint64_t fwd_full[2];     // per accumulator buffer: forward of its tile done
    uint64_t fwd_empty[2];    // per accumulator buffer: the epilogue has read it
    uint64_t delta_full;      // a tile's deltas are in shared memory (4 warps)
    uint64_t delta_empty[2];  // the weight gradients of an even / odd tile are done
    uint64_t weights;
    uint64_t final_mma;
    uint32_t tmem_base;
};
constexpr size_t kTcSmem = 1024 + kOffBar + sizeof(TcBarriers);
static_assert(kTcSmem <= 227 * 1024, "tensor-core minibatch kernel exceeds the shared-memory budget");
static_assert(size_t(kTcEpiWarps) * kTcChunks * 32 * sizeof(float) <= size_t(kKStages) * kTcStageBytes,
              "final reduction staging reuses the K ring");

// tanh(x) = 1 - 2 / (1 + e^(2x)) on the hardware base-2 exponential and
// reciprocal (ex2.approx / rcp.approx): absolute error ~1e-7, far below the
// TF32 products it follows; saturates to +-1.
__device__ __forceinline__ float tc_tanh(float x) {
    float e, r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x * 2.8853900817779268f));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
    return fmaf(-2.0f, r, 1.0f);
}

// One step of the halving tree: lanes with bit S set keep the upper half of
// x[0..2S) (added to the partner's copy of it), the others the lower half.
template <int S>
__device__ __forceinline__ void column_sum_step(float (&x)[32], int lane) {
    const bool upper = (lane & S) != 0;
#pragma unroll
    for (int i = 0; i < S; i++) {
        const float send = upper ? x[i] : x[i + S];
        const float keep = upper ? x[i + S] : x[i];
        x[i] = keep + __shfl_xor_sync(0xffffffffu, send, S);
    }
}
// Sum of x[i] over the warp's 32 lanes; lane j receives the total of column
// j. A fixed halving tree (31 exchanges), so the result does not depend on
// scheduling.
__device__ __forceinline__ float lane_column_sum(float (&x)[32], int lane) {
    column_sum_step<16>(x, lane);
    column_sum_step<8>(x, lane);
    column_sum_step<4>(x, lane);
    column_sum_step<2>(x, lane);
    column_sum_step<1>(x, lane);
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
    uint8_t* kring = smem + kOffKRing;
    uint8_t* mring = smem + kOffMRing;
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
        for (int i = 0; i < kKStages; i++) {
            tc::mbar_init(&s.kfull[i], 1);
            tc::mbar_init(&s.kempty[i], 1);
        }
        for (int i = 0; i < kMStages; i++) {
            tc::mbar_init(&s.mfull[i], 1);
            tc::mbar_init(&s.mempty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            tc::mbar_init(&s.fwd_full[i], 1);
            tc::mbar_init(&s.fwd_empty[i], 4);
            tc::mbar_init(&s.delta_empty[i], 1);
        }
        tc::mbar_init(&s.delta_full, 4);
        tc::mbar_init(&s.weights, 1);
        tc::mbar_init(&s.final_mma, 1);
        tc::fence_barrier_init();
        tc::prefetch_tmap(&obs_k);
        tc::prefetch_tmap(&obs_mn);
        tc::prefetch_tmap(&co_k);
        tc::prefetch_tmap(&co_mn);
    }
    if (warp == kWarpMma) {
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
        else if (k >= kParW2t) v = p.actor[kActorW2 + ((k - kParW2t) & 3) * 64 + ((k - kParW2t) >> 2)];
        par[k] = v;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = s.tmem_base;

    // One ring of 16 KB panels: `it` counts the panels through it.
    auto ring_load = [&](uint8_t* ring, uint64_t* full, uint64_t* empty, int stages, uint32_t& it,
                         const CUtensorMap* map, int32_t x, int32_t y) {
        const uint32_t st = it % stages, use = it / stages;
        if (use > 0 && !tc::mbar_wait(&empty[st], (use - 1) & 1, kTcWaitLimit)) return false;
        tc::mbar_arrive_expect_tx(&full[st], kTcStageBytes);
        tc::tma_load_2d(ring + size_t(st) * kTcStageBytes, map, x, y, &full[st]);
        it++;
        return true;
    };
    auto ring_drain = [&](uint64_t* full, int stages, uint32_t it) {
        // every copy this warp issued has landed before the CTA may exit
        bool ok = true;
        for (uint32_t k = it > uint32_t(stages) ? it - stages : 0; k < it; k++)
            if (!tc::mbar_wait(&full[k % stages], (k / stages) & 1, kTcWaitLimit)) ok = false;
        return ok;
    };

    if (warp == kWarpKProducer && lane == 0) {
        // ------------------------------------- forward panels (K-major, HBM)
        bool ok = true;
        uint32_t it = 0;
        if (count > 0) {
            tc::mbar_arrive_expect_tx(&s.weights, (kTcObsPanels + 1) * kTcWPanelBytes);
            for (int q = 0; q < kTcObsPanels; q++)
                tc::tma_load_2d(w1s + q * kTcWPanelBytes, &w1_map, q * kTcPanel, 0, &s.weights);
            tc::tma_load_2d(cw1s, &cw1_map, 0, 0, &s.weights);
        }
        for (uint32_t t = 0; t < count && ok; t++) {
            const int32_t y = tile_row0(t);
            for (int q = 0; q < kTcObsPanels && ok; q++)
                ok = ring_load(kring, s.kfull, s.kempty, kKStages, it, &obs_k, q * kTcPanel, y);
            if (ok) ok = ring_load(kring, s.kfull, s.kempty, kKStages, it, &co_k, 0, y);
        }
        if (!ring_drain(s.kfull, kKStages, it)) ok = false;
        if (count > 0 && !tc::mbar_wait(&s.weights, 0, kTcWaitLimit)) ok = false;
        if (!ok) atomicOr(p.tc_error, 1u);
    } else if (warp == kWarpMProducer && lane == 0) {
        // -------------------------------- weight-gradient panels (MN-major, L2)
        bool ok = true;
        uint32_t it = 0;
        for (uint32_t t = 0; t < count && ok; t++) {
            const int32_t y = tile_row0(t);
            for (int q = 0; q < kTcObsPanels && ok; q++)
                ok = ring_load(mring, s.mfull, s.mempty, kMStages, it, &obs_mn, q * kTcPanel, y);
            if (ok) ok = ring_load(mring, s.mfull, s.mempty, kMStages, it, &co_mn, 0, y);
        }
        if (!ring_drain(s.mfull, kMStages, it)) ok = false;
        if (!ok) atomicOr(p.tc_error, 16u);
    } else if (warp == kWarpMma && lane == 0) {
        // ------------------------------------------------------- MMA issuer
        // Event loop over two streams of work, each advanced one panel at a
        // time when its inputs are ready: forwards (tile f, panel fp) run up to
        // two tiles ahead of the epilogue (two accumulator buffers); weight
        // gradients (tile w, panel wp) follow each tile's deltas.
        constexpr uint32_t idesc_fwd = tc::tf32_idesc(kTcRows, kHidden, 0, 0);
        constexpr uint32_t idesc_wg = tc::tf32_idesc(kHidden, kTcPanel, 0, 1);
        bool ok = count == 0 || tc::mbar_wait(&s.weights, 0, kTcWaitLimit);
        uint32_t f = 0, fp = 0, w = 0, wp = 0, kit = 0, mit = 0;
        bool f_ready = false, w_ready = false;
        long long idle_since = clock64();
        while (ok && w < count) {
            bool progressed = false;
            if (f < count) {
                if (!f_ready) {
                    f_ready = f < 2 || tc::mbar_test_wait(&s.fwd_empty[f & 1], ((f >> 1) - 1) & 1);
                    if (f_ready) tc::fence_after_sync();
                }
                if (f_ready && tc::mbar_test_wait(&s.kfull[kit % kKStages], (kit / kKStages) & 1)) {
                    tc::fence_after_sync();
                    const uint32_t a_addr = tc::smem_u32(kring + size_t(kit % kKStages) * kTcStageBytes);
                    const bool critic = fp == kTcObsPanels;
                    const uint32_t b_addr = tc::smem_u32(critic ? cw1s : w1s + fp * kTcWPanelBytes);
                    const uint32_t d = tmem + kColD + 128 * (f & 1) + (critic ? 64 : 0);
#pragma unroll
                    for (int kk = 0; kk < kTcPanel / 8; kk++)
                        tc::mma_tf32(d, tc::sw128_desc(a_addr + kk * 32, 16, 1024),
                                     tc::sw128_desc(b_addr + kk * 32, 16, 1024), idesc_fwd,
                                     (!critic && fp != 0) || kk != 0 ? 1u : 0u);
                    tc::mma_commit(&s.kempty[kit % kKStages]);
                    kit++;
                    progressed = true;
                    if (++fp == kTcInPanels) {
                        tc::mma_commit(&s.fwd_full[f & 1]);
                        f++;
                        fp = 0;
                        f_ready = false;
                    }
                }
            }
            if (w < f) {  // a tile's deltas exist only after its forward
                if (!w_ready) {
                    w_ready = tc::mbar_test_wait(&s.delta_full, w & 1);
                    if (w_ready) tc::fence_after_sync();
                }
                if (w_ready && tc::mbar_test_wait(&s.mfull[mit % kMStages], (mit / kMStages) & 1)) {
                    tc::fence_after_sync();
                    const uint32_t b_addr = tc::smem_u32(mring + size_t(mit % kMStages) * kTcStageBytes);
                    const bool critic = wp == kTcObsPanels;
                    const uint32_t a_base = tc::smem_u32(critic ? dc : da);
                    const uint32_t d = tmem + (critic ? kColGc : kColGa + 32 * wp);
#pragma unroll
                    for (int g = 0; g < 4; g++)          // the tile's four 32-row groups (K)
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)   // 8 rows per MMA
                            tc::mma_tf32(d, tc::sw128_desc(a_base + g * kTcDeltaBytes + kk * 32, 16, 1024),
                                         tc::sw128b32_desc(b_addr + (32 * g + 8 * kk) * 128, kTcStageBytes, 512),
                                         idesc_wg, (w | g | kk) != 0 ? 1u : 0u);
                    tc::mma_commit(&s.mempty[mit % kMStages]);
                    mit++;
                    progressed = true;
                    if (++wp == kTcInPanels) {
                        tc::mma_commit(&s.delta_empty[w & 1]);
                        w++;
                        wp = 0;
                        w_ready = false;
                    }
                }
            }
            if (progressed) {
                idle_since = clock64();
            } else {
                if (clock64() - idle_since > kTcWaitLimit) ok = false;
                __nanosleep(32);  // leave the issue slots to the epilogue warps
            }
        }
        tc::mma_commit(&s.final_mma);
        if (!ok) atomicOr(p.tc_error, 2u);
    } else if (warp >= kWarpEpi0 && warp < kWarpEpi0 + kTcEpiWarps) {
        // --------------------------------------------------------- epilogue
        const int ew = warp - kWarpEpi0;  // 0..7
        const int g = ew >> 2;            // this group takes the tiles j with j % 2 == g (accumulator buffer g)
        const int q = warp & 3;           // tensor-memory lanes 32q..32q+31 = rows 32q..32q+31 of a tile
        const float scale = 1.0f / fmaxf(float(p.global_batch[update]), 1.0f);
        // Per-lane running sums, lane j holding column j of each chunk:
        // 0-7 dW2[a][32c + j] (chunk 2a + c), 8-9 critic w2, 10-11 b1,
        // 12-13 critic b1, 14 = d_mean[4], d_log_std[4], d_value, loss sums[4].
        float acc[kTcChunks];
#pragma unroll
        for (int k = 0; k < kTcChunks; k++) acc[k] = 0.0f;
        bool ok = true;
        for (uint32_t j = g; j < count; j += 2) {
            const uint32_t local = (blockIdx.x + j * gridDim.x) * kTcRows + 32 * q + lane;  // row of the minibatch
            const bool valid = local < b;
            const size_t src = size_t(begin) + local;
            // The row's own inputs of the loss, requested before waiting for the
            // forward so their memory latency overlaps it.
            float4 act4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            float hint[3] = {0.0f, 0.0f, 0.0f}, adv = 0.0f, ret = 0.0f, old_logp = 0.0f;
            if (valid) {
                act4 = __ldg(reinterpret_cast<const float4*>(p.actions + src * kActions));
#pragma unroll
                for (int a = 0; a < 3; a++) hint[a] = __ldg(p.obs + src * kActorObs + kActorObs - 3 + a);
                adv = __ldg(p.advantages + src);
                ret = __ldg(p.returns + src);
                old_logp = __ldg(p.logp + src);
            }
            if (!tc::mbar_wait(&s.fwd_full[g], (j >> 1) & 1, kTcWaitLimit)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            // The parameters are re-read from shared memory every tile: the
            // opaque pointer keeps the compiler from hoisting ~450 loop-invariant
            // loads into registers (and spilling them).
            const float* pr = par;
            asm volatile("" : "+l"(pr));
            const float* b1 = pr;
            const float* w2 = pr + 64;
            const float* cb1 = pr + 320;
            const float* cw2 = pr + 384;
            const float* b2 = pr + 448;
            const float* log_std = pr + 452;
            const float cb2 = pr[456];
            const uint32_t lane_addr = tmem + (uint32_t(32 * q) << 16) + kColD + 128 * g;
            // Activations: the value and means are formed in fp32 as the tanh
            // values are produced, and the tanh values replace the
            // pre-activations in tensor memory, where the backward reads them
            // 32 at a time (the buffer is released at the end of the tile).
            float value = cb2, mean[4];
#pragma unroll
            for (int a = 0; a < 4; a++) mean[a] = b2[a];
            {
                float v[32];
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    tc::tmem_ld32(lane_addr + 64 + 32 * c, v);
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        v[i] = tc_tanh(v[i] + cb1[32 * c + i]);
                        value = fmaf(cw2[32 * c + i], v[i], value);
                    }
                    tc::tmem_st32(lane_addr + 64 + 32 * c, v);
                }
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    tc::tmem_ld32(lane_addr + 32 * c, v);
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        v[i] = tc_tanh(v[i] + b1[32 * c + i]);
#pragma unroll
                        for (int a = 0; a < 4; a++) mean[a] = fmaf(w2[a * 64 + 32 * c + i], v[i], mean[a]);
                    }
                    tc::tmem_st32(lane_addr + 32 * c, v);
                }
                tc::tmem_wait_st();
            }
            // clipped-PPO loss and derivatives (ppo.hpp:144-181)
            float dm[4] = {0, 0, 0, 0}, dls[4] = {0, 0, 0, 0}, dvalue = 0.0f, loss[4] = {0, 0, 0, 0};
            if (valid) {
#pragma unroll
                for (int a = 0; a < 3; a++) mean[a] += hint[a];
                const float act[4] = {act4.x, act4.y, act4.z, act4.w};
                float logp = 0.0f;
#pragma unroll
                for (int a = 0; a < 4; a++) {
                    const float d = (act[a] - mean[a]) * expf(-log_std[a]);
                    logp += -0.5f * (d * d + 2.0f * log_std[a] + kLogTwoPi);
                }
                const float raw = logp - old_logp;
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
            // dW2[a][h] = sum over rows of d_mean[a] tanh_h, critic w2 = sum
            // d_value tanh_c: before the delta handover, off its critical path
#pragma unroll
            for (int c = 0; c < 2; c++) {
                float v[32];
                tc::tmem_ld32(lane_addr + 64 + 32 * c, v);
#pragma unroll
                for (int i = 0; i < 32; i++) x[i] = dvalue * v[i];
                acc[8 + c] += lane_column_sum(x, lane);
                tc::tmem_ld32(lane_addr + 32 * c, v);
#pragma unroll
                for (int a = 0; a < 4; a++) {
#pragma unroll
                    for (int i = 0; i < 32; i++) x[i] = dm[a] * v[i];
                    acc[2 * a + c] += lane_column_sum(x, lane);
                }
            }
            // The previous tile's weight-gradient MMAs (tile j - 1, the other
            // group's) must be done reading the delta operands first.
            if (j >= 1 && !tc::mbar_wait(&s.delta_empty[(j - 1) & 1], ((j - 1) >> 1) & 1, kTcWaitLimit)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            {
                // hidden deltas (W2^T d_mean)(1 - h^2) and d_value cw2 (1 - hc^2)
                // into the K-major 128-byte-swizzled operands: hidden unit h is a
                // 128-byte row of the [64 x 32 rows] operand, this thread's row is
                // column `lane`; the row's 16-byte granule is (lane / 4) ^ (h % 8).
                uint8_t* pa = da + q * kTcDeltaBytes + (lane & 3) * 4;
                uint8_t* pc = dc + q * kTcDeltaBytes + (lane & 3) * 4;
                uint32_t gran[8];
#pragma unroll
                for (int r8 = 0; r8 < 8; r8++) gran[r8] = r8 * 128 + (((lane >> 2) ^ r8) << 4);
                const float4* w2t = reinterpret_cast<const float4*>(pr + kParW2t);
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    float ha[32], hv[32];
                    tc::tmem_ld32(lane_addr + 32 * c, ha);
                    tc::tmem_ld32(lane_addr + 64 + 32 * c, hv);
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        const int h = 32 * c + i;
                        const float4 wc = w2t[h];
                        const float sv = fmaf(dm[3], wc.w, fmaf(dm[2], wc.z, fmaf(dm[1], wc.y, dm[0] * wc.x)));
                        ha[i] = sv * (1.0f - ha[i] * ha[i]);
                        hv[i] = dvalue * cw2[h] * (1.0f - hv[i] * hv[i]);
                        const uint32_t off = (h >> 3) * 1024 + gran[h & 7];
                        *reinterpret_cast<float*>(pa + off) = ha[i];
                        *reinterpret_cast<float*>(pc + off) = hv[i];
                    }
                    // b1 and critic b1: sums of the deltas, from the registers
                    acc[10 + c] += lane_column_sum(ha, lane);
                    acc[12 + c] += lane_column_sum(hv, lane);
                }
            }
            fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor cores
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive(&s.delta_full);
                tc::mbar_arrive(&s.fwd_empty[g]);  // the accumulator buffer is free again
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
        // every MMA is done: the weight-gradient accumulators are final and the rings are free
        const bool mma_done = count == 0 || tc::mbar_wait(&s.final_mma, 0, kTcWaitLimit);
        tc::fence_after_sync();
        float* red = reinterpret_cast<float*>(kring);
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
    if (warp == kWarpMma) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 512);
    }
}

// Bounded-wait self-test: one thread waits on a shared-memory mbarrier with
// the same bounded wait the tensor-core kernels use. With arrive = 0 nothing
// ever arrives, the wait gives up after `limit` cycles and the kernel records
// it in *flag (no TMA, no MMA, no tensor memory); with arrive = 1 the thread
// arrives first and the wait succeeds.
__global__ void k_barrier_selftest(uint32_t* flag, long long limit, int arrive) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    tc::mbar_init(&bar, 1);
    tc::fence_barrier_init();
    if (arrive) tc::mbar_arrive(&bar);
    *flag = tc::mbar_wait(&bar, 0, limit) ? 0u : 1u;
}

cudaError_t barrier_selftest(long long limit, int arrive, uint32_t* timed_out) {
    uint32_t* d = nullptr;
    cudaError_t e = cudaMalloc(&d, sizeof(uint32_t));
    if (e != cudaSuccess) return e;
    k_barrier_selftest<<<1, 32>>>(d, limit, arrive);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpy(timed_out, d, sizeof(uint32_t), cudaMemcpyDeviceToHost);
    cudaFree(d);
    return e;
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
