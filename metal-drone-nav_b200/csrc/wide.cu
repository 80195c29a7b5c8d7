// Wide actor on the tcgen05 tensor cores (sm_100a): the one-hidden-layer tanh
// actor of ppo.hpp:65-80 at hidden widths of 256..8192 units (the reference's
// 967,688-parameter actor is hidden = 5120, navigation_wide_deployment.hpp:54-66).
//
// k_wide_forward computes, for a block of observation rows,
//     partial[s][row][a] = sum_{h in slice s} tanh(obs[row] . W1[h] + b1[h]) * W2[a][h]
// for 128-unit hidden slices s. The matrix product obs . W1^T runs as
// tcgen05.mma.kind::tf32 (fp32 accumulate in tensor memory) on 128-row x
// 256-unit tiles; operands arrive by TMA in the 128-byte swizzled layout, one
// 32-column K panel per pipeline stage. The epilogue warps read the
// accumulator from tensor memory, apply bias + tanh and fold the four output
// rows of W2 in, so the [rows x hidden] activation never reaches HBM. The sum
// over slices (fixed order), the output bias and the geometry prior are added
// by the consumer (the act kernel, or the PPO loss kernel).
//
// Warp roles (persistent CTA, one per SM): warp 0 issues TMA loads, warp 1
// owns tensor memory and issues the MMAs, warps 2-9 are the epilogue (two per
// tensor-memory lane quarter, each taking half of the tile's 256 columns). The
// accumulator is double-buffered (2 x 256 columns) so the epilogue of one tile
// overlaps the MMAs of the next.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>

#include "mdn_shared.h"
#include "tc.cuh"
#include "wide.h"

namespace mdn {

namespace {
constexpr int kWideBM = 128;          // rows per tile (tensor-memory lanes)
constexpr int kWideBN = 256;          // hidden units per tile (accumulator columns)
constexpr int kWidePanel = 32;        // fp32 K columns per 128-byte swizzled panel
constexpr int kWidePanels = 6;        // 184 inputs padded to 192 (TMA zero-fills 184..191)
constexpr int kWideStages = 4;
constexpr int kWideABytes = kWideBM * 128;  // one K panel of the row tile
constexpr int kWideBBytes = kWideBN * 128;  // one K panel of the weight tile
constexpr int kWideStageBytes = kWideABytes + kWideBBytes;
constexpr int kWideEpiWarps = 8;
constexpr int kWideThreads = (2 + kWideEpiWarps) * 32;
constexpr long long kWaitLimit = 2000000000ll;  // clock cycles (~1 s) before a wait gives up

struct WideSmem {
    uint64_t full[kWideStages];
    uint64_t empty[kWideStages];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t done;
    uint32_t tmem_base;
};
constexpr size_t kWideSmemBytes = 1024 /* alignment slack */ + size_t(kWideStages) * kWideStageBytes + sizeof(WideSmem);
}  // namespace

__global__ void __launch_bounds__(kWideThreads, 1)
    k_wide_forward(const __grid_constant__ CUtensorMap obs_map, const __grid_constant__ CUtensorMap w1_map,
                   WideForwardArgs p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stage_base = smem;
    WideSmem& s = *reinterpret_cast<WideSmem*>(smem + size_t(kWideStages) * kWideStageBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const uint32_t m_tiles = (p.rows + kWideBM - 1) / kWideBM;
    const uint32_t n_tiles = p.hidden / kWideBN;
    const uint32_t tiles = m_tiles * n_tiles;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kWideStages; i++) {
            tc::mbar_init(&s.full[i], 1);
            tc::mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            tc::mbar_init(&s.tfull[i], 1);
            tc::mbar_init(&s.tempty[i], kWideEpiWarps);
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
        uint32_t it = 0;  // pipeline slot counter over all tiles of this CTA
        bool ok = true;
        for (uint32_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            const uint32_t m = t / n_tiles, n = t % n_tiles;
            for (int kp = 0; kp < kWidePanels; kp++, it++) {
                const uint32_t st = it % kWideStages, use = it / kWideStages;
                if (use > 0 && !tc::mbar_wait(&s.empty[st], (use - 1) & 1, kWaitLimit)) {
                    ok = false;
                    break;
                }
                uint8_t* a_dst = stage_base + size_t(st) * kWideStageBytes;
                uint8_t* b_dst = a_dst + kWideABytes;
                tc::mbar_arrive_expect_tx(&s.full[st], kWideStageBytes);
                tc::tma_load_2d(a_dst, &obs_map, kp * kWidePanel, int32_t(p.row0 + m * kWideBM), &s.full[st]);
                tc::tma_load_2d(b_dst, &w1_map, kp * kWidePanel, int32_t(n * kWideBN), &s.full[st]);
            }
        }
        // Drain: every load issued must land before the CTA may exit.
        const uint32_t issued = it;
        for (uint32_t k = issued > kWideStages ? issued - kWideStages : 0; k < issued; k++)
            if (!tc::mbar_wait(&s.full[k % kWideStages], (k / kWideStages) & 1, kWaitLimit)) ok = false;
        if (!ok) atomicOr(p.error, 1u);
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------- MMA issuer
        constexpr uint32_t idesc = tc::tf32_idesc(kWideBM, kWideBN, 0, 0);
        uint32_t it = 0, local = 0;
        bool ok = true;
        for (uint32_t t = blockIdx.x; t < tiles && ok; t += gridDim.x, local++) {
            const uint32_t buf = local & 1, use = local >> 1;
            if (use > 0 && !tc::mbar_wait(&s.tempty[buf], (use - 1) & 1, kWaitLimit)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const uint32_t d = tmem + buf * kWideBN;
            for (int kp = 0; kp < kWidePanels; kp++, it++) {
                const uint32_t st = it % kWideStages;
                if (!tc::mbar_wait(&s.full[st], (it / kWideStages) & 1, kWaitLimit)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t a_addr = tc::smem_u32(stage_base + size_t(st) * kWideStageBytes);
                const uint32_t b_addr = a_addr + kWideABytes;
#pragma unroll
                for (int kk = 0; kk < kWidePanel / 8; kk++) {  // K = 8 per tf32 MMA = 32 bytes of the 128-byte row
                    const uint64_t ad = tc::sw128_desc(a_addr + kk * 32, 16, 1024);
                    const uint64_t bd = tc::sw128_desc(b_addr + kk * 32, 16, 1024);
                    tc::mma_tf32(d, ad, bd, idesc, (kp | kk) != 0);
                }
                tc::mma_commit(&s.empty[st]);  // frees the stage once these MMAs have read it
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
        const int quarter = warp & 3;         // tensor-memory lanes 32*quarter .. +31
        const int half = ew >> 2;             // columns [128*half, 128*half+128) of the tile
        const uint32_t row_in_tile = quarter * 32 + lane;
        uint32_t local = 0;
        bool ok = true;
        for (uint32_t t = blockIdx.x; t < tiles; t += gridDim.x, local++) {
            const uint32_t m = t / n_tiles, n = t % n_tiles;
            const uint32_t buf = local & 1, use = local >> 1;
            if (!tc::mbar_wait(&s.tfull[buf], use & 1, kWaitLimit)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const uint32_t col0 = n * kWideBN + half * 128;  // first hidden unit of this warp's slice
            float pm0 = 0.0f, pm1 = 0.0f, pm2 = 0.0f, pm3 = 0.0f;
#pragma unroll 1
            for (int c = 0; c < 4; c++) {
                float v[32];
                tc::tmem_ld32(tmem + (uint32_t(quarter * 32) << 16) + buf * kWideBN + half * 128 + c * 32, v);
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    const uint32_t h = col0 + c * 32 + j;
                    const float4 b = __ldg(reinterpret_cast<const float4*>(p.b1 + h));
                    const float4 w0 = __ldg(reinterpret_cast<const float4*>(p.w2 + h));
                    const float4 w1 = __ldg(reinterpret_cast<const float4*>(p.w2 + p.hidden + h));
                    const float4 w2 = __ldg(reinterpret_cast<const float4*>(p.w2 + 2 * p.hidden + h));
                    const float4 w3 = __ldg(reinterpret_cast<const float4*>(p.w2 + 3 * p.hidden + h));
                    const float a0 = tanhf(v[j] + b.x), a1 = tanhf(v[j + 1] + b.y);
                    const float a2 = tanhf(v[j + 2] + b.z), a3 = tanhf(v[j + 3] + b.w);
                    pm0 = fmaf(a3, w0.w, fmaf(a2, w0.z, fmaf(a1, w0.y, fmaf(a0, w0.x, pm0))));
                    pm1 = fmaf(a3, w1.w, fmaf(a2, w1.z, fmaf(a1, w1.y, fmaf(a0, w1.x, pm1))));
                    pm2 = fmaf(a3, w2.w, fmaf(a2, w2.z, fmaf(a1, w2.y, fmaf(a0, w2.x, pm2))));
                    pm3 = fmaf(a3, w3.w, fmaf(a2, w3.z, fmaf(a1, w3.y, fmaf(a0, w3.x, pm3))));
                }
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&s.tempty[buf]);
            const uint32_t row = m * kWideBM + row_in_tile;
            if (row < p.rows) {
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
}  // namespace

// fp32 matrix [rows][inner] with a row pitch of `pitch_bytes` (a multiple of
// 16), read in boxes of box_rows x 32 columns with 128-byte swizzle.
cudaError_t wide_make_map(WideMap* out, const float* base, uint64_t inner, uint64_t rows, uint64_t pitch_bytes,
                          uint32_t box_rows) {
    static_assert(sizeof(CUtensorMap) <= sizeof(WideMap::bytes), "tensor map storage");
    EncodeTiled fn = encode_tiled();
    if (!fn) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (pitch_bytes & 15)) return cudaErrorInvalidValue;
    CUtensorMap map;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {pitch_bytes};
    const cuuint32_t box[2] = {uint32_t(kWidePanel), box_rows};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, elem,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    std::memcpy(out->bytes, &map, sizeof(map));
    return cudaSuccess;
}

cudaError_t configure_wide_kernels() {
    return cudaFuncSetAttribute(k_wide_forward, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kWideSmemBytes));
}

cudaError_t launch_wide_forward(const WideMap& obs_map, const WideMap& w1_map, const WideForwardArgs& p, int sm_count,
                                cudaStream_t s) {
    if (p.hidden % kWideBN != 0 || p.rows == 0) return cudaErrorInvalidValue;
    CUtensorMap om, wm;
    std::memcpy(&om, obs_map.bytes, sizeof(om));
    std::memcpy(&wm, w1_map.bytes, sizeof(wm));
    const uint32_t tiles = ((p.rows + kWideBM - 1) / kWideBM) * (p.hidden / kWideBN);
    const unsigned grid = unsigned(tiles < uint32_t(sm_count) ? tiles : uint32_t(sm_count));
    k_wide_forward<<<grid, kWideThreads, kWideSmemBytes, s>>>(om, wm, p);
    return cudaGetLastError();
}

}  // namespace mdn
