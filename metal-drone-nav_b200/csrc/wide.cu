// Wide actor on the tcgen05 tensor cores (sm_100a): the one-hidden-layer tanh
// actor of ppo.hpp:65-80 at hidden widths of 256..8192 units (the reference's
// 967,688-parameter actor is hidden = 5120, navigation_wide_deployment.hpp:54-66),
// forward in the rollout and forward + backward in the PPO update.
//
// k_wide_forward computes, for a block of observation rows,
//     partial[s][row][a] = sum_{h in slice s} tanh(obs[row] . W1[h] + b1[h]) * W2[a][h]
// for 128-unit hidden slices s (the consumer adds the slices in a fixed
// order, then b2 and the geometry prior). k_wide_backward recomputes
// the same pre-activations and, from the per-row mean derivatives d_mean of
// ppo.hpp:144-181, writes the hidden deltas
//     delta[row][h] = (sum_a d_mean[row][a] W2[a][h]) (1 - tanh^2)
// and the column sums of delta (-> db1) and of d_mean[a] * tanh (-> dW2),
// i.e. actor_backward_sample (ppo.hpp:269-287) summed over the rows.
// k_wide_wgrad then forms dW1 = delta^T . obs on the tensor cores.
//
// Operands arrive by TMA in the 128-byte swizzled layout; matrix products are
// tcgen05.mma.kind::tf32 with fp32 accumulators in tensor memory. The
// [rows x hidden] activation never reaches HBM in the forward pass; in the
// backward pass only the deltas do (they are the A operand of dW1).
//
// Warp roles (persistent CTA, one per SM): warp 0 issues TMA loads, warp 1
// owns tensor memory and issues the MMAs, the remaining warps are the
// epilogue. Accumulators are double-buffered in tensor memory so an epilogue
// overlaps the next tile's MMAs. Every barrier wait is bounded; a wait that
// gives up sets the error flag, the kernel drains its copies and exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>

#include "mdn_shared.h"
#include "tc.cuh"
#include "wide.h"

namespace mdn {

namespace {
constexpr int kRowsBM = 128;          // rows per tile (tensor-memory lanes)
constexpr int kRowsBN = 256;          // hidden units per tile (accumulator columns)
constexpr int kPanel = 32;            // fp32 columns per 128-byte swizzled panel
constexpr int kObsPanels = 6;         // 184 inputs padded to 192 (TMA zero-fills 184..191)
constexpr int kRowsStages = 4;
constexpr int kRowsABytes = kRowsBM * 128;  // one K panel of the row tile
constexpr int kRowsBBytes = kRowsBN * 128;  // one K panel of the weight tile
constexpr int kRowsStageBytes = kRowsABytes + kRowsBBytes;
constexpr int kRowsEpiWarps = 8;
constexpr int kRowsThreads = (2 + kRowsEpiWarps) * 32;
constexpr int kColSums = 5;           // delta, d_mean[0..3] * tanh
constexpr int kBackHidden = 128;      // backward tile: hidden units (tensor-memory lanes)
constexpr int kBackRows = 256;        // backward tile: rows (accumulator columns)
static_assert(kBackHidden * 128 == kRowsABytes && kBackRows * 128 == kRowsBBytes, "backward reuses the stage sizes");
constexpr long long kWaitLimit = 2000000000ll;  // clock cycles (~1 s) before a wait gives up

// k_wide_wgrad: 128 hidden units x 192 inputs per item, 32 rows per stage.
constexpr int kGradBM = 128;
constexpr int kGradBN = 192;
constexpr int kGradRows = 32;
constexpr int kGradStages = 5;
constexpr int kGradAPanelBytes = kGradRows * 128;  // 32 rows x 32 hidden units
constexpr int kGradABytes = 4 * kGradAPanelBytes;
constexpr int kGradBBytes = kObsPanels * kGradAPanelBytes;
constexpr int kGradStageBytes = kGradABytes + kGradBBytes;
constexpr int kGradThreads = 6 * 32;

constexpr int kMaxStages = kRowsStages > kGradStages ? kRowsStages : kGradStages;
struct Barriers {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t done;
    uint32_t tmem_base;
};
constexpr size_t kRowsSmemFwd = 1024 + size_t(kRowsStages) * kRowsStageBytes + sizeof(Barriers);
constexpr size_t kRowsSmemBwd = kRowsSmemFwd + size_t(kBackHidden) * kColSums * sizeof(float);
constexpr size_t kGradSmem = 1024 + size_t(kGradStages) * kGradStageBytes + sizeof(Barriers);

// tanh from the logistic identity tanh(x) = 1 - 2 / (1 + e^(2x)), with
// e^(2x) = 2^(x * 2 log2 e) on the hardware base-2 exponential and the
// hardware reciprocal (ex2.approx / rcp.approx, a few ulp each): absolute
// error ~1e-7, far below the tf32 products it follows. Saturates to +-1 for
// large |x| (e^(2x) -> inf or 0).
constexpr float kTwoLog2e = 2.8853900817779268f;
// tanh(z) given y = z * 2 log2 e (callers fold the bias into one FMA)
__device__ __forceinline__ float wide_tanh_scaled(float y) {
    float e, r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(y));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
    return fmaf(-2.0f, r, 1.0f);
}
__device__ __forceinline__ float wide_tanh(float x) { return wide_tanh_scaled(x * kTwoLog2e); }
}  // namespace

__global__ void __launch_bounds__(kRowsThreads, 1)
    k_wide_forward(const __grid_constant__ CUtensorMap obs_map, const __grid_constant__ CUtensorMap w1_map,
                   WideRowsArgs p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stage_base = smem;
    Barriers& s = *reinterpret_cast<Barriers*>(smem + size_t(kRowsStages) * kRowsStageBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const uint32_t rows = p.rows_dev ? p.rows_dev[p.index] : p.rows;
    const uint32_t row0 = p.row0_dev ? p.row0_dev[p.index] : p.row0;
    const uint32_t m_tiles = (rows + kRowsBM - 1) / kRowsBM;
    const uint32_t n_tiles = p.hidden / kRowsBN;
    const uint32_t tiles = m_tiles * n_tiles;  // t = m * n_tiles + n, strided over the grid

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRowsStages; i++) {
            tc::mbar_init(&s.full[i], 1);
            tc::mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            tc::mbar_init(&s.tfull[i], 1);
            tc::mbar_init(&s.tempty[i], kRowsEpiWarps);
        }
        tc::mbar_init(&s.done, 1);
        tc::fence_barrier_init();
        tc::prefetch_tmap(&obs_map);
        tc::prefetch_tmap(&w1_map);
    }
    if (warp == 1) {
        tc::tmem_alloc(&s.tmem_base, 512);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = s.tmem_base;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------ TMA producer
        uint32_t it = 0;
        bool ok = true;
        for (uint32_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            const uint32_t m = t / n_tiles, n = t % n_tiles;
            for (int kp = 0; kp < kObsPanels; kp++, it++) {
                const uint32_t st = it % kRowsStages, use = it / kRowsStages;
                if (use > 0 && !tc::mbar_wait(&s.empty[st], (use - 1) & 1, kWaitLimit)) {
                    ok = false;
                    break;
                }
                uint8_t* a_dst = stage_base + size_t(st) * kRowsStageBytes;
                tc::mbar_arrive_expect_tx(&s.full[st], kRowsStageBytes);
                tc::tma_load_2d(a_dst, &obs_map, kp * kPanel, int32_t(row0 + m * kRowsBM), &s.full[st]);
                tc::tma_load_2d(a_dst + kRowsABytes, &w1_map, kp * kPanel, int32_t(n * kRowsBN), &s.full[st]);
            }
        }
        for (uint32_t k = it > kRowsStages ? it - kRowsStages : 0; k < it; k++)
            if (!tc::mbar_wait(&s.full[k % kRowsStages], (k / kRowsStages) & 1, kWaitLimit)) ok = false;
        if (!ok) atomicOr(p.error, 1u);
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------- MMA issuer
        constexpr uint32_t idesc = tc::tf32_idesc(kRowsBM, kRowsBN, 0, 0);
        uint32_t it = 0, j = 0;
        bool ok = true;
        for (uint32_t t = blockIdx.x; t < tiles && ok; t += gridDim.x, j++) {
            const uint32_t buf = j & 1, use = j >> 1;
            if (use > 0 && !tc::mbar_wait(&s.tempty[buf], (use - 1) & 1, kWaitLimit)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const uint32_t d = tmem + buf * kRowsBN;
            for (int kp = 0; kp < kObsPanels; kp++, it++) {
                const uint32_t st = it % kRowsStages;
                if (!tc::mbar_wait(&s.full[st], (it / kRowsStages) & 1, kWaitLimit)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t a_addr = tc::smem_u32(stage_base + size_t(st) * kRowsStageBytes);
                const uint32_t b_addr = a_addr + kRowsABytes;
#pragma unroll
                for (int kk = 0; kk < kPanel / 8; kk++) {  // K = 8 per tf32 MMA = 32 bytes of a 128-byte row
                    tc::mma_tf32(d, tc::sw128_desc(a_addr + kk * 32, 16, 1024), tc::sw128_desc(b_addr + kk * 32, 16, 1024),
                                 idesc, (kp | kk) != 0);
                }
                tc::mma_commit(&s.empty[st]);
            }
            if (!ok) break;
            tc::mma_commit(&s.tfull[buf]);
        }
        tc::mma_commit(&s.done);
        if (!tc::mbar_wait(&s.done, 0, kWaitLimit)) ok = false;
        if (!ok) atomicOr(p.error, 2u);
    } else if (warp >= 2) {
        // --------------------------------------------------------- epilogue
        const int ew = warp - 2;
        const int quarter = warp & 3;   // tensor-memory lanes 32*quarter .. +31
        const int half = ew >> 2;       // columns [128*half, 128*half+128) of the tile
        bool ok = true;
        uint32_t j = 0;
        for (uint32_t t = blockIdx.x; t < tiles; t += gridDim.x, j++) {
            const uint32_t m = t / n_tiles, n = t % n_tiles;
            const uint32_t buf = j & 1, use = j >> 1;
            if (!tc::mbar_wait(&s.tfull[buf], use & 1, kWaitLimit)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const uint32_t row = m * kRowsBM + quarter * 32 + lane;
            const uint32_t col0 = n * kRowsBN + half * 128;
            float pm0 = 0.0f, pm1 = 0.0f, pm2 = 0.0f, pm3 = 0.0f;
#pragma unroll 1
            for (int c = 0; c < 4; c++) {
                float v[32];
                tc::tmem_ld32(tmem + (uint32_t(quarter * 32) << 16) + buf * kRowsBN + half * 128 + c * 32, v);
#pragma unroll
                for (int q = 0; q < 32; q += 4) {
                    const uint32_t h = col0 + c * 32 + q;
                    const float4 b = __ldg(reinterpret_cast<const float4*>(p.b1 + h));
                    const float4 w0 = __ldg(reinterpret_cast<const float4*>(p.w2 + h));
                    const float4 w1 = __ldg(reinterpret_cast<const float4*>(p.w2 + p.hidden + h));
                    const float4 w2 = __ldg(reinterpret_cast<const float4*>(p.w2 + 2 * p.hidden + h));
                    const float4 w3 = __ldg(reinterpret_cast<const float4*>(p.w2 + 3 * p.hidden + h));
                    const float a0 = wide_tanh(v[q] + b.x), a1 = wide_tanh(v[q + 1] + b.y);
                    const float a2 = wide_tanh(v[q + 2] + b.z), a3 = wide_tanh(v[q + 3] + b.w);
                    pm0 = fmaf(a3, w0.w, fmaf(a2, w0.z, fmaf(a1, w0.y, fmaf(a0, w0.x, pm0))));
                    pm1 = fmaf(a3, w1.w, fmaf(a2, w1.z, fmaf(a1, w1.y, fmaf(a0, w1.x, pm1))));
                    pm2 = fmaf(a3, w2.w, fmaf(a2, w2.z, fmaf(a1, w2.y, fmaf(a0, w2.x, pm2))));
                    pm3 = fmaf(a3, w3.w, fmaf(a2, w3.z, fmaf(a1, w3.y, fmaf(a0, w3.x, pm3))));
                }
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&s.tempty[buf]);
            if (row < rows) {
                const uint32_t slice = n * 2 + half;
                *reinterpret_cast<float4*>(p.partials + (size_t(slice) * p.rows + row) * 4) =
                    make_float4(pm0, pm1, pm2, pm3);
            }
        }
        if (!ok) atomicOr(p.error, 4u);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 512);
    }
}

// Backward over one minibatch, transposed: tile = 128 hidden units (tensor-
// memory lanes) x 256 rows (accumulator columns), D = W1 . obs^T, both
// operands K-major. A thread owns one hidden unit h, so b1[h] and W2[.][h] sit
// in registers and the column sums over rows (db1, dW2) are per-thread running
// sums. CTA c keeps hidden tile c % h_tiles and walks row tiles
// c / h_tiles, + groups, ...; its sums go to colsum_out[group][5][hidden].
__global__ void __launch_bounds__(kRowsThreads, 1)
    k_wide_backward(const __grid_constant__ CUtensorMap obs_map, const __grid_constant__ CUtensorMap w1_map,
                    WideRowsArgs p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stage_base = smem;
    Barriers& s = *reinterpret_cast<Barriers*>(smem + size_t(kRowsStages) * kRowsStageBytes);
    float* halves = reinterpret_cast<float*>(smem + size_t(kRowsStages) * kRowsStageBytes + sizeof(Barriers));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const uint32_t rows = p.rows_dev ? p.rows_dev[p.index] : p.rows;
    const uint32_t row0 = p.row0_dev ? p.row0_dev[p.index] : p.row0;
    const uint32_t r_tiles = (rows + kBackRows - 1) / kBackRows;
    const uint32_t h_tiles = p.hidden / kBackHidden;
    const uint32_t groups = gridDim.x / h_tiles;
    const uint32_t my_h = blockIdx.x % h_tiles, my_g = blockIdx.x / h_tiles;
    const uint32_t count = my_g < r_tiles ? (r_tiles - my_g + groups - 1) / groups : 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRowsStages; i++) {
            tc::mbar_init(&s.full[i], 1);
            tc::mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            tc::mbar_init(&s.tfull[i], 1);
            tc::mbar_init(&s.tempty[i], kRowsEpiWarps);
        }
        tc::mbar_init(&s.done, 1);
        tc::fence_barrier_init();
        tc::prefetch_tmap(&obs_map);
        tc::prefetch_tmap(&w1_map);
    }
    if (warp == 1) {
        tc::tmem_alloc(&s.tmem_base, 512);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = s.tmem_base;

    if (warp == 0 && lane == 0) {
        uint32_t it = 0;
        bool ok = true;
        for (uint32_t j = 0; j < count && ok; j++) {
            const uint32_t rt = my_g + j * groups;
            for (int kp = 0; kp < kObsPanels; kp++, it++) {
                const uint32_t st = it % kRowsStages, use = it / kRowsStages;
                if (use > 0 && !tc::mbar_wait(&s.empty[st], (use - 1) & 1, kWaitLimit)) {
                    ok = false;
                    break;
                }
                uint8_t* a_dst = stage_base + size_t(st) * kRowsStageBytes;
                tc::mbar_arrive_expect_tx(&s.full[st], kRowsStageBytes);
                tc::tma_load_2d(a_dst, &w1_map, kp * kPanel, int32_t(my_h * kBackHidden), &s.full[st]);
                tc::tma_load_2d(a_dst + kRowsABytes, &obs_map, kp * kPanel, int32_t(row0 + rt * kBackRows), &s.full[st]);
            }
        }
        for (uint32_t k = it > kRowsStages ? it - kRowsStages : 0; k < it; k++)
            if (!tc::mbar_wait(&s.full[k % kRowsStages], (k / kRowsStages) & 1, kWaitLimit)) ok = false;
        if (!ok) atomicOr(p.error, 64u);
    } else if (warp == 1 && lane == 0) {
        constexpr uint32_t idesc = tc::tf32_idesc(kBackHidden, kBackRows, 0, 0);
        uint32_t it = 0;
        bool ok = true;
        for (uint32_t j = 0; j < count && ok; j++) {
            const uint32_t buf = j & 1, use = j >> 1;
            if (use > 0 && !tc::mbar_wait(&s.tempty[buf], (use - 1) & 1, kWaitLimit)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const uint32_t d = tmem + buf * kBackRows;
            for (int kp = 0; kp < kObsPanels; kp++, it++) {
                const uint32_t st = it % kRowsStages;
                if (!tc::mbar_wait(&s.full[st], (it / kRowsStages) & 1, kWaitLimit)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t a_addr = tc::smem_u32(stage_base + size_t(st) * kRowsStageBytes);
                const uint32_t b_addr = a_addr + kRowsABytes;
#pragma unroll
                for (int kk = 0; kk < kPanel / 8; kk++)
                    tc::mma_tf32(d, tc::sw128_desc(a_addr + kk * 32, 16, 1024), tc::sw128_desc(b_addr + kk * 32, 16, 1024),
                                 idesc, (kp | kk) != 0);
                tc::mma_commit(&s.empty[st]);
            }
            if (!ok) break;
            tc::mma_commit(&s.tfull[buf]);
        }
        tc::mma_commit(&s.done);
        if (!tc::mbar_wait(&s.done, 0, kWaitLimit)) ok = false;
        if (!ok) atomicOr(p.error, 128u);
    } else if (warp >= 2) {
        const int ew = warp - 2;
        const int quarter = warp & 3;   // hidden units 32*quarter .. +31 of the tile
        const int half = ew >> 2;       // rows [128*half, 128*half+128) of each row tile
        const uint32_t h = my_h * kBackHidden + quarter * 32 + lane;
        const float b1s = p.b1[h] * kTwoLog2e;
        const float w0 = p.w2[h], w1 = p.w2[p.hidden + h], w2 = p.w2[2 * p.hidden + h], w3 = p.w2[3 * p.hidden + h];
        float s_delta = 0.0f, s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
        bool ok = true;
        for (uint32_t j = 0; j < count; j++) {
            const uint32_t rt = my_g + j * groups;
            const uint32_t buf = j & 1, use = j >> 1;
            if (!tc::mbar_wait(&s.tfull[buf], use & 1, kWaitLimit)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const uint32_t r_base = rt * kBackRows + half * 128;
#pragma unroll 1
            for (int c = 0; c < 4; c++) {
                float v[32];
                tc::tmem_ld32(tmem + (uint32_t(quarter * 32) << 16) + buf * kBackRows + half * 128 + c * 32, v);
#pragma unroll
                for (int q = 0; q < 32; q++) {
                    const uint32_t row = r_base + c * 32 + q;
                    // rows past the minibatch get d_mean = 0, hence delta = 0 (the dW1
                    // product reads whole 32-row groups)
                    const float4 dm = row < rows ? __ldg(reinterpret_cast<const float4*>(p.d_mean) + row)
                                                 : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    const float a = wide_tanh_scaled(fmaf(v[q], kTwoLog2e, b1s));
                    const float g = fmaf(dm.x, w0, fmaf(dm.y, w1, fmaf(dm.z, w2, dm.w * w3)));
                    const float delta = g * fmaf(-a, a, 1.0f);
                    p.delta[size_t(row) * p.hidden + h] = delta;
                    s_delta += delta;
                    s0 = fmaf(dm.x, a, s0);
                    s1 = fmaf(dm.y, a, s1);
                    s2 = fmaf(dm.z, a, s2);
                    s3 = fmaf(dm.w, a, s3);
                }
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&s.tempty[buf]);
        }
        if (!ok) atomicOr(p.error, 256u);
        // the two row halves of each hidden unit, half 0 first
        float* mine = halves + (size_t(quarter) * 32 + lane) * kColSums;
        if (half == 1) {
            mine[0] = s_delta; mine[1] = s0; mine[2] = s1; mine[3] = s2; mine[4] = s3;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kRowsEpiWarps * 32) : "memory");
        if (half == 0) {
            const float out[kColSums] = {s_delta + mine[0], s0 + mine[1], s1 + mine[2], s2 + mine[3], s3 + mine[4]};
#pragma unroll
            for (int v = 0; v < kColSums; v++) p.colsum_out[(size_t(my_g) * kColSums + v) * p.hidden + h] = out[v];
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 512);
    }
}

// dW1 partials: out[split][h][k] = sum over the split's rows of delta[row][h] * obs[row0 + row][k].
// Both operands are MN-major (hidden units / inputs contiguous in each row),
// loaded as 32-row x 32-column boxes in the 128-byte / 32-byte-atom swizzle;
// one MMA consumes an 8-row group (two 4-row atoms).
__global__ void __launch_bounds__(kGradThreads, 1)
    k_wide_wgrad(const __grid_constant__ CUtensorMap delta_map, const __grid_constant__ CUtensorMap obs_map,
                 WideGradArgs p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Barriers& s = *reinterpret_cast<Barriers*>(smem + size_t(kGradStages) * kGradStageBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rows = p.rows_dev ? p.rows_dev[p.index] : p.rows;
    const uint32_t row0 = p.row0_dev ? p.row0_dev[p.index] : p.row0;
    const uint32_t groups32 = (rows + kGradRows - 1) / kGradRows;          // 32-row groups in the minibatch
    const uint32_t splits = p.splits < groups32 ? p.splits : groups32;    // every split gets >= 1 group
    const uint32_t per = (groups32 + splits - 1) / splits;
    const uint32_t m_tiles = p.hidden / kGradBM;
    const uint32_t items = m_tiles * p.splits;  // splits past `splits` write zeros
    auto item_range = [&](uint32_t item, uint32_t& mt, uint32_t& sp, uint32_t& g0, uint32_t& g1) {
        mt = item % m_tiles;
        sp = item / m_tiles;
        g0 = sp * per < groups32 ? sp * per : groups32;
        g1 = g0 + per < groups32 ? g0 + per : groups32;
        if (sp >= splits) g0 = g1 = groups32;
    };

    if (threadIdx.x == 0) {
        for (int i = 0; i < kGradStages; i++) {
            tc::mbar_init(&s.full[i], 1);
            tc::mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            tc::mbar_init(&s.tfull[i], 1);
            tc::mbar_init(&s.tempty[i], 4);
        }
        tc::mbar_init(&s.done, 1);
        tc::fence_barrier_init();
        tc::prefetch_tmap(&delta_map);
        tc::prefetch_tmap(&obs_map);
    }
    if (warp == 1) {
        tc::tmem_alloc(&s.tmem_base, 512);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = s.tmem_base;

    if (warp == 0 && lane == 0) {
        uint32_t it = 0;
        bool ok = true;
        for (uint32_t item = blockIdx.x; item < items && ok; item += gridDim.x) {
            uint32_t mt, sp, g0, g1;
            item_range(item, mt, sp, g0, g1);
            for (uint32_t g = g0; g < g1; g++, it++) {
                const uint32_t st = it % kGradStages, use = it / kGradStages;
                if (use > 0 && !tc::mbar_wait(&s.empty[st], (use - 1) & 1, kWaitLimit)) {
                    ok = false;
                    break;
                }
                uint8_t* a_dst = smem + size_t(st) * kGradStageBytes;
                uint8_t* b_dst = a_dst + kGradABytes;
                tc::mbar_arrive_expect_tx(&s.full[st], kGradStageBytes);
                for (int q = 0; q < 4; q++)
                    tc::tma_load_2d(a_dst + q * kGradAPanelBytes, &delta_map, int32_t(mt * kGradBM + q * 32),
                                    int32_t(g * kGradRows), &s.full[st]);
                for (int q = 0; q < kObsPanels; q++)
                    tc::tma_load_2d(b_dst + q * kGradAPanelBytes, &obs_map, q * kPanel, int32_t(row0 + g * kGradRows),
                                    &s.full[st]);
            }
        }
        for (uint32_t k = it > kGradStages ? it - kGradStages : 0; k < it; k++)
            if (!tc::mbar_wait(&s.full[k % kGradStages], (k / kGradStages) & 1, kWaitLimit)) ok = false;
        if (!ok) atomicOr(p.error, 8u);
    } else if (warp == 1 && lane == 0) {
        constexpr uint32_t idesc = tc::tf32_idesc(kGradBM, kGradBN, 1, 1);
        uint32_t it = 0, j = 0;
        bool ok = true;
        for (uint32_t item = blockIdx.x; item < items && ok; item += gridDim.x, j++) {
            uint32_t mt, sp, g0, g1;
            item_range(item, mt, sp, g0, g1);
            const uint32_t buf = j & 1, use = j >> 1;
            if (use > 0 && !tc::mbar_wait(&s.tempty[buf], (use - 1) & 1, kWaitLimit)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const uint32_t d = tmem + buf * 256;
            for (uint32_t g = g0; g < g1; g++, it++) {
                const uint32_t st = it % kGradStages;
                if (!tc::mbar_wait(&s.full[st], (it / kGradStages) & 1, kWaitLimit)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t a_addr = tc::smem_u32(smem + size_t(st) * kGradStageBytes);
                const uint32_t b_addr = a_addr + kGradABytes;
#pragma unroll
                for (int kk = 0; kk < kGradRows / 8; kk++)  // 8 rows (one 1024-byte atom) per MMA
                    tc::mma_tf32(d, tc::sw128b32_desc(a_addr + kk * 1024, kGradAPanelBytes, 512),
                                 tc::sw128b32_desc(b_addr + kk * 1024, kGradAPanelBytes, 512), idesc,
                                 (g != g0 || kk != 0) ? 1u : 0u);
                tc::mma_commit(&s.empty[st]);
            }
            if (!ok) break;
            tc::mma_commit(&s.tfull[buf]);
        }
        tc::mma_commit(&s.done);
        if (!tc::mbar_wait(&s.done, 0, kWaitLimit)) ok = false;
        if (!ok) atomicOr(p.error, 16u);
    } else if (warp >= 2) {
        const int quarter = warp & 3;
        bool ok = true;
        uint32_t j = 0;
        for (uint32_t item = blockIdx.x; item < items; item += gridDim.x, j++) {
            uint32_t mt, sp, g0, g1;
            item_range(item, mt, sp, g0, g1);
            const uint32_t buf = j & 1, use = j >> 1;
            if (!tc::mbar_wait(&s.tfull[buf], use & 1, kWaitLimit)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const uint32_t h = mt * kGradBM + quarter * 32 + lane;
            float* out = p.out + (size_t(sp) * p.hidden + h) * kActorObs;
            const bool empty = g0 == g1;  // no rows: the accumulator was never written
#pragma unroll 1
            for (int c = 0; c < kGradBN / 32; c++) {
                float v[32];
                tc::tmem_ld32(tmem + (uint32_t(quarter * 32) << 16) + buf * 256 + c * 32, v);
#pragma unroll
                for (int q = 0; q < 32; q++)
                    if (c * 32 + q < kActorObs) out[c * 32 + q] = empty ? 0.0f : v[q];
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&s.tempty[buf]);
        }
        if (!ok) atomicOr(p.error, 32u);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 512);
    }
}

// The wide actor's flat gradient (ppo.hpp:35-40 layout at width H) followed by
// the critic's: dW1 (sum of the splits), b1 / W2 (sums of the column-sum
// groups), b2 / log_std and the critic from the small-layout gradient of the
// loss kernels. Fixed summation orders throughout.
__global__ void k_wide_assemble(WideAssembleArgs p) {
    const uint32_t H = p.hidden;
    const size_t o_b1 = size_t(H) * kActorObs, o_w2 = o_b1 + H, o_b2 = o_w2 + size_t(kActions) * H,
                 o_ls = o_b2 + kActions, o_critic = o_ls + kActions, total = o_critic + kCriticParams;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        float g = 0.0f;
        if (i < o_b1) {  // W1: the splits of k_wide_wgrad
            for (uint32_t sp = 0; sp < p.splits; sp++) g += p.w1_parts[sp * o_b1 + i];
        } else if (i < o_w2) {  // b1: column sums of the deltas
            const size_t h = i - o_b1;
            for (uint32_t gr = 0; gr < p.groups; gr++) g += p.colsums[(size_t(gr) * 5 + 0) * H + h];
        } else if (i < o_b2) {  // W2[a][h]: column sums of d_mean[a] * tanh
            const size_t a = (i - o_w2) / H, h = (i - o_w2) % H;
            for (uint32_t gr = 0; gr < p.groups; gr++) g += p.colsums[(size_t(gr) * 5 + 1 + a) * H + h];
        } else if (i < o_ls) {
            g = p.small_grad[kActorB2 + (i - o_b2)];
        } else if (i < o_critic) {
            g = p.small_grad[kActorLogStd + (i - o_ls)];
        } else {
            g = p.small_grad[kActorParams + (i - o_critic)];
        }
        p.grad[i] = g;
    }
}

// Sum of squares of the actor gradient, one partial per block (fixed order).
__global__ void k_wide_sumsq(const float* grad, size_t count, float* partials) {
    __shared__ float red[32];
    float s = 0.0f;
    const size_t per = (count + gridDim.x - 1) / gridDim.x;
    const size_t lo = blockIdx.x * per, hi = lo + per < count ? lo + per : count;
    for (size_t i = lo + threadIdx.x; i < hi; i += blockDim.x) s = fmaf(grad[i], grad[i], s);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < int(blockDim.x >> 5); w++) t += red[w];
        partials[blockIdx.x] = t;
    }
}

// Global-norm clip to max_norm and Adam over the actor (main.mm:1202,1369-1378,
// ppo.hpp:310-324), then the log-std clamp (main.mm:934-940). Every block
// re-adds the norm partials in the same order.
__global__ void k_wide_adam(WideAdamArgs p) {
    __shared__ float scale_s;
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (uint32_t b = 0; b < p.partial_count; b++) t += p.partials[b];
        const float norm = sqrtf(t + 1.0e-20f);
        const float r = p.max_norm / norm;
        scale_s = r < 1.0f ? r : 1.0f;  // std::min(1, max_norm / norm)
        if (blockIdx.x == 0 && p.norm_out) *p.norm_out = norm;
    }
    __syncthreads();
    const float scale = scale_s;
    const float b1c = p.bias_corr[0], b2c = p.bias_corr[1], lr = p.learning_rate;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < p.count; i += size_t(gridDim.x) * blockDim.x) {
        const float gs = p.grad[i] * scale;
        const float mi = 0.9f * p.m[i] + (1.0f - 0.9f) * gs;
        const float vi = 0.999f * p.v[i] + (1.0f - 0.999f) * gs * gs;
        p.m[i] = mi;
        p.v[i] = vi;
        const float mh = mi / b1c, vh = vi / b2c;
        float w = p.params[i] - lr * mh / (sqrtf(vh) + 1.0e-8f);
        if (!p.no_clamp && i >= p.count - kActions) w = fminf(fmaxf(w, -2.0f), 0.5f);
        p.params[i] = w;
    }
}

// ------------------------------------------------------------------- host
namespace {
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_tiled() {
    static EncodeTiled fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(ptr);
    }
    return fn;
}

void to_map(const WideMap& m, CUtensorMap& out) { std::memcpy(&out, m.bytes, sizeof(out)); }
}  // namespace

cudaError_t wide_make_map(WideMap* out, const float* base, uint64_t inner, uint64_t rows, uint64_t pitch_bytes,
                          uint32_t box_rows, bool mn_major) {
    static_assert(sizeof(CUtensorMap) <= sizeof(WideMap::bytes), "tensor map storage");
    EncodeTiled fn = encode_tiled();
    if (!fn) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (pitch_bytes & 15) || box_rows == 0 || box_rows > 256)
        return cudaErrorInvalidValue;
    CUtensorMap map;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {pitch_bytes};
    const cuuint32_t box[2] = {uint32_t(kPanel), box_rows};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, elem,
                          CU_TENSOR_MAP_INTERLEAVE_NONE,
                          mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    std::memcpy(out->bytes, &map, sizeof(map));
    return cudaSuccess;
}

cudaError_t configure_wide_kernels() {
    cudaError_t e = cudaFuncSetAttribute(k_wide_forward, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kRowsSmemFwd));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_wide_backward, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kRowsSmemBwd));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_wide_wgrad, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kGradSmem));
    return e;
}

cudaError_t launch_wide_forward(const WideMap& obs_map, const WideMap& w1_map, const WideRowsArgs& p, int sm_count,
                                cudaStream_t s) {
    if (p.hidden % kRowsBN != 0 || p.rows == 0) return cudaErrorInvalidValue;
    CUtensorMap om, wm;
    to_map(obs_map, om);
    to_map(w1_map, wm);
    const uint32_t tiles = ((p.rows + kRowsBM - 1) / kRowsBM) * (p.hidden / kRowsBN);
    const unsigned grid = unsigned(tiles < uint32_t(sm_count) ? tiles : uint32_t(sm_count));
    k_wide_forward<<<grid, kRowsThreads, kRowsSmemFwd, s>>>(om, wm, p);
    return cudaGetLastError();
}

// Row groups of the backward grid (hidden tiles x groups CTAs, one per SM at
// a time): the smallest count that makes the grid whole waves of the SMs
// (5120 hidden units: 40 tiles x 37 groups = 10 waves of 148), so no SM idles
// while the others work; one wave of floor(SMs / tiles) groups when that
// would take more than 16 waves.
uint32_t wide_backward_groups(uint32_t hidden, int sm_count) {
    const uint32_t n_tiles = hidden / kBackHidden, sms = uint32_t(sm_count);
    uint32_t a = n_tiles, b = sms;
    while (b) {
        const uint32_t t = a % b;
        a = b;
        b = t;
    }
    const uint32_t whole = sms / a;  // n_tiles * whole is a multiple of the SM count
    if (size_t(n_tiles) * whole <= size_t(16) * sms) return whole;
    const uint32_t g = sms / n_tiles;
    return g > 0 ? g : 1;
}

cudaError_t launch_wide_backward(const WideMap& obs_map, const WideMap& w1_map, const WideRowsArgs& p, int sm_count,
                                 cudaStream_t s) {
    if (p.hidden % kRowsBN != 0 || p.rows == 0) return cudaErrorInvalidValue;
    CUtensorMap om, wm;
    to_map(obs_map, om);
    to_map(w1_map, wm);
    const unsigned grid = (p.hidden / kBackHidden) * wide_backward_groups(p.hidden, sm_count);
    k_wide_backward<<<grid, kRowsThreads, kRowsSmemBwd, s>>>(om, wm, p);
    return cudaGetLastError();
}

cudaError_t launch_wide_wgrad(const WideMap& delta_map, const WideMap& obs_map, const WideGradArgs& p, int sm_count,
                              cudaStream_t s) {
    if (p.hidden % kGradBM != 0 || p.splits == 0) return cudaErrorInvalidValue;
    CUtensorMap dm, om;
    to_map(delta_map, dm);
    to_map(obs_map, om);
    const uint32_t items = (p.hidden / kGradBM) * p.splits;
    const unsigned grid = unsigned(items < uint32_t(sm_count) ? items : uint32_t(sm_count));
    k_wide_wgrad<<<grid, kGradThreads, kGradSmem, s>>>(dm, om, p);
    return cudaGetLastError();
}

cudaError_t launch_wide_assemble(const WideAssembleArgs& p, int sm_count, cudaStream_t s) {
    k_wide_assemble<<<sm_count * 4, 256, 0, s>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_wide_clip_adam(const WideAdamArgs& p, float* partials_scratch, int sm_count, cudaStream_t s) {
    const unsigned blocks = unsigned(sm_count) * 2;
    k_wide_sumsq<<<blocks, 256, 0, s>>>(p.grad, p.count, partials_scratch);
    WideAdamArgs q = p;
    q.partials = partials_scratch;
    q.partial_count = blocks;
    k_wide_adam<<<blocks, 256, 0, s>>>(q);
    return cudaGetLastError();
}

}  // namespace mdn
