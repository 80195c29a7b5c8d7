// Layered actor/critic networks on sm_100a CUDA cores (fp32): dense layers
// with a fused bias + activation epilogue, the backward deltas with the
// activation derivative fused, chunked weight-gradient partials summed in a
// fixed order (results are deterministic run to run), and the clipped-PPO loss
// of these networks. Register-tiled products: a 256-thread CTA computes a
// 128 x 64 output tile, 8 x 4 per thread, from 16-deep shared-memory slices,
// the next slice loaded into registers while the current one is multiplied.
#include <cuda_runtime.h>

#include <cmath>

#include "mdn_device.cuh"
#include "mlp.h"

namespace mdn {

uint32_t MlpShape::weight_offset(uint32_t l) const {
    uint32_t off = 0;
    for (uint32_t j = 0; j < l; j++) off += out_dim(j) * in_dim(j) + out_dim(j);
    return off;
}
uint32_t MlpShape::bias_offset(uint32_t l) const { return weight_offset(l) + out_dim(l) * in_dim(l); }
uint32_t MlpShape::param_count() const { return weight_offset(layers + 1) + (log_std ? kActions : 0); }

namespace {

constexpr int kBM = 128, kBN = 64, kBK = 16, kDenseThreads = 256, kPad = 4;
constexpr int kLossThreads = 256;

__device__ __forceinline__ void resolve(const DenseRows& r, uint32_t& rows, uint32_t& row0) {
    rows = r.rows_dev ? r.rows_dev[r.index] : r.rows;
    row0 = r.row0_dev ? r.row0_dev[r.index] : r.row0;
    if (rows > r.rows) rows = r.rows;  // never past the capacity the grid was sized for
}

// tanh, or GELU in its exact erf form 0.5 z (1 + erf(z / sqrt 2)).
__device__ __forceinline__ float act_fwd(int act, float z) {
    if (act == kActTanh) return tanhf(z);
    if (act == kActGelu) return 0.5f * z * (1.0f + erff(z * 0.70710678118654752f));
    return z;
}
// Derivative at the pre-activation z: 1 - tanh(z)^2, or Phi(z) + z phi(z).
__device__ __forceinline__ float act_grad(int act, float z) {
    if (act == kActTanh) {
        const float t = tanhf(z);
        return 1.0f - t * t;
    }
    if (act == kActGelu)
        return 0.5f * (1.0f + erff(z * 0.70710678118654752f)) + z * 0.39894228040143268f * expf(-0.5f * z * z);
    return 1.0f;
}

// One 128 x 64 output tile of C = A B over the reduction dimension kdim, by a
// 256-thread CTA: thread (ty, tx) = (tid / 16, tid % 16) accumulates rows
// 8 ty .. 8 ty + 7 and columns 4 tx .. 4 tx + 3, each sum in reduction order.
// A(k, m) and B(k, n) come from the loaders `ga` / `gb` (which return 0 out
// of bounds); A_KMAJOR / B_KMAJOR say which index is contiguous in memory, so
// that consecutive threads load consecutive addresses. The next 16-deep
// slice is loaded into registers while the current one is multiplied from
// shared memory (two shared buffers, one barrier per slice).
template <bool A_KMAJOR, bool B_KMAJOR, typename GA, typename GB>
__device__ __forceinline__ void gemm_tile(uint32_t kdim, GA ga, GB gb, float (&acc)[8][4]) {
    __shared__ __align__(16) float as[2][kBK][kBM + kPad];
    __shared__ __align__(16) float bs[2][kBK][kBN + kPad];
    const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
    float ra[8], rb[4];
    auto a_index = [&](int j, int& kk, int& mm) {
        const int e = tid + kDenseThreads * j;
        kk = A_KMAJOR ? e % kBK : e / kBM;
        mm = A_KMAJOR ? e / kBK : e % kBM;
    };
    auto b_index = [&](int j, int& kk, int& nn) {
        const int e = tid + kDenseThreads * j;
        kk = B_KMAJOR ? e % kBK : e / kBN;
        nn = B_KMAJOR ? e / kBK : e % kBN;
    };
    auto load = [&](uint32_t k0) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int kk, mm;
            a_index(j, kk, mm);
            ra[j] = ga(k0 + kk, mm);
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int kk, nn;
            b_index(j, kk, nn);
            rb[j] = gb(k0 + kk, nn);
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int kk, mm;
            a_index(j, kk, mm);
            as[buf][kk][mm] = ra[j];
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int kk, nn;
            b_index(j, kk, nn);
            bs[buf][kk][nn] = rb[j];
        }
    };
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
    load(0);
    store(0);
    __syncthreads();
    int buf = 0;
    for (uint32_t k0 = 0; k0 < kdim; k0 += kBK) {
        const bool more = k0 + kBK < kdim;
        if (more) load(k0 + kBK);
#pragma unroll
        for (int kk = 0; kk < kBK; kk++) {
            const float4 a0 = *reinterpret_cast<const float4*>(&as[buf][kk][ty * 8]);
            const float4 a1 = *reinterpret_cast<const float4*>(&as[buf][kk][ty * 8 + 4]);
            const float4 b = *reinterpret_cast<const float4*>(&bs[buf][kk][tx * 4]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        if (more) store(buf ^ 1);
        __syncthreads();
        buf ^= 1;
    }
}

__global__ void __launch_bounds__(kDenseThreads) k_dense_fwd(DenseFwd p, DenseRows r, int x_row0) {
    uint32_t rows, row0;
    resolve(r, rows, row0);
    const uint32_t m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
    if (m0 >= rows) return;  // CTA-uniform
    const float* x = p.x + (x_row0 ? size_t(row0) * p.k : 0);
    float acc[8][4];
    gemm_tile<true, true>(
        p.k,
        [&](uint32_t k, int mm) {
            const uint32_t m = m0 + mm;
            return (m < rows && k < p.k) ? x[size_t(m) * p.k + k] : 0.0f;
        },
        [&](uint32_t k, int nn) {
            const uint32_t n = n0 + nn;
            return (n < p.n && k < p.k) ? p.w[size_t(n) * p.k + k] : 0.0f;
        },
        acc);
    // Dot from zero in k order, then the bias, then the activation.
    const int ty = threadIdx.x / 16, tx = threadIdx.x % 16;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t m = m0 + ty * 8 + i;
        if (m >= rows) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t n = n0 + tx * 4 + j;
            if (n >= p.n) continue;
            const float z = p.b ? acc[i][j] + p.b[n] : acc[i][j];
            if (p.z) p.z[size_t(m) * p.n + n] = z;
            p.y[size_t(m) * p.n + n] = act_fwd(p.act, z);
        }
    }
}

__global__ void __launch_bounds__(kDenseThreads) k_dense_bwd(DenseBwd p, DenseRows r) {
    uint32_t rows, row0;
    resolve(r, rows, row0);
    const uint32_t m0 = blockIdx.y * kBM, c0 = blockIdx.x * kBN;  // output rows, output columns (k)
    if (m0 >= rows) return;
    float acc[8][4];
    gemm_tile<true, false>(
        p.n,
        [&](uint32_t n, int mm) {
            const uint32_t m = m0 + mm;
            return (m < rows && n < p.n) ? p.dy[size_t(m) * p.n + n] : 0.0f;
        },
        [&](uint32_t n, int cc) {
            const uint32_t c = c0 + cc;
            return (n < p.n && c < p.k) ? p.w[size_t(n) * p.k + c] : 0.0f;
        },
        acc);
    const int ty = threadIdx.x / 16, tx = threadIdx.x % 16;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t m = m0 + ty * 8 + i;
        if (m >= rows) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t c = c0 + tx * 4 + j;
            if (c >= p.k) continue;
            const size_t at = size_t(m) * p.k + c;
            p.dx[at] = acc[i][j] * act_grad(p.act, p.zp[at]);
        }
    }
}

// CTA (k tile, n tile, chunk): the chunk's rows in order. The input column
// k == K stands for the bias (X = 1).
__global__ void __launch_bounds__(kDenseThreads) k_dense_wgrad(DenseWgrad p, DenseRows r) {
    uint32_t rows, row0;
    resolve(r, rows, row0);
    const uint32_t k0 = blockIdx.x * kBN, n0 = blockIdx.y * kBM, c = blockIdx.z;
    const uint32_t lo = c * p.chunk_rows, hi = lo + p.chunk_rows < rows ? lo + p.chunk_rows : rows;
    const float* x = p.x + (p.x_row0 ? size_t(row0) * p.k : 0);
    float acc[8][4];
    const uint32_t span = hi > lo ? hi - lo : 0;
    gemm_tile<false, false>(
        span,
        [&](uint32_t dm, int nn) {
            const uint32_t m = lo + dm, n = n0 + nn;
            return (dm < span && n < p.n) ? p.dy[size_t(m) * p.n + n] : 0.0f;
        },
        [&](uint32_t dm, int kk) {
            const uint32_t m = lo + dm, k = k0 + kk;
            if (dm >= span) return 0.0f;
            return k < p.k ? x[size_t(m) * p.k + k] : (k == p.k ? 1.0f : 0.0f);
        },
        acc);
    float* out = p.part + size_t(c) * (size_t(p.n) * p.k + p.n);
    const int ty = threadIdx.x / 16, tx = threadIdx.x % 16;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t n = n0 + ty * 8 + i;
        if (n >= p.n) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t k = k0 + tx * 4 + j;
            if (k < p.k) out[size_t(n) * p.k + k] = acc[i][j];
            else if (k == p.k) out[size_t(p.n) * p.k + n] = acc[i][j];
        }
    }
}

__global__ void k_chunk_sum(const float* part, uint32_t chunks, size_t count, float* grad) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < count; i += size_t(gridDim.x) * blockDim.x) {
        float s = 0.0f;
        for (uint32_t c = 0; c < chunks; c++) s += part[size_t(c) * count + i];
        grad[i] = s;
    }
}

// Fixed-tree sum over the CTA (warp xor tree, then the warps in order).
__device__ __forceinline__ float cta_sum(float v, float* red) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < int(blockDim.x >> 5); w++) t += red[w];
    return t;
}

// ppo.hpp:144-181 per row (the fused kernels' formulas), one thread per row.
__global__ void __launch_bounds__(kLossThreads) k_layered_loss(LayeredLoss p, DenseRows r) {
    __shared__ float red[kLossThreads / 32];
    uint32_t rows, row0;
    resolve(r, rows, row0);
    const uint32_t m = blockIdx.x * kLossThreads + threadIdx.x;
    const float scale = 1.0f / fmaxf(float(p.global_batch[r.index]), 1.0f);
    float dls[4] = {0, 0, 0, 0}, loss[4] = {0, 0, 0, 0};
    if (m < rows) {
        const size_t src = size_t(row0) + m;
        const float* prior = p.obs + src * kActorObs + kActorObs - 3;  // ppo.hpp:77 geometry prior
        float mean[4];
#pragma unroll
        for (int a = 0; a < 4; a++) {
            mean[a] = p.out_a[size_t(m) * 4 + a] + p.b2[a];
            if (a < 3) mean[a] += prior[a];
        }
        const float value = p.out_c[m];
        const float* act = p.actions + src * kActions;
        float log_std[4];
#pragma unroll
        for (int a = 0; a < 4; a++) log_std[a] = p.log_std[a];
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
        const float clipped = clampf(ratio, 1.0f - p.clip, 1.0f + p.clip);
        const float chosen = smin(ratio * adv, clipped * adv);
        const bool in_range = raw >= -20.0f && raw <= 20.0f;
        const bool active = in_range && (adv >= 0.0f ? ratio <= 1.0f + p.clip : ratio >= 1.0f - p.clip);
        float entropy = 0.0f;
#pragma unroll
        for (int a = 0; a < 4; a++) {
            const float inv_var = expf(-2.0f * log_std[a]);
            const float diff = act[a] - mean[a];
            float dm = 0.0f;
            if (active) {
                const float dlogp = -ratio * adv * scale;
                dm = dlogp * diff * inv_var;
                dls[a] = dlogp * (diff * diff * inv_var - 1.0f);
            }
            dls[a] -= p.entropy_coef * scale;
            entropy += -p.entropy_coef * (log_std[a] + 0.5f * (1.0f + kLogTwoPi)) * scale;
            p.d_out_a[size_t(m) * 4 + a] = dm;
        }
        p.d_out_c[m] = p.value_coef * (value - ret) * scale;
        loss[0] = -chosen * scale;
        loss[1] = 0.5f * p.value_coef * (value - ret) * (value - ret) * scale;
        loss[2] = entropy;
        loss[3] = ratio;
    }
    if (blockIdx.x * kLossThreads >= rows) {  // CTA-uniform: a CTA past the rows contributes zeros
        if (threadIdx.x < 8) p.cta_sums[size_t(blockIdx.x) * 8 + threadIdx.x] = 0.0f;
        return;
    }
    float sums[8];
#pragma unroll
    for (int a = 0; a < 4; a++) sums[a] = cta_sum(dls[a], red);
#pragma unroll
    for (int a = 0; a < 4; a++) sums[4 + a] = cta_sum(loss[a], red);
    if (threadIdx.x == 0)
#pragma unroll
        for (int j = 0; j < 8; j++) p.cta_sums[size_t(blockIdx.x) * 8 + j] = sums[j];
}

__global__ void k_layered_finish(const float* cta_sums, uint32_t ctas, float* log_std_grad, float* metric_row,
                                 const uint32_t* rows_dev, uint32_t index) {
    const int j = threadIdx.x;
    if (j >= 8) return;
    float s = 0.0f;
    for (uint32_t c = 0; c < ctas; c++) s += cta_sums[size_t(c) * 8 + j];
    if (j < 4) log_std_grad[j] = s;
    else if (j == 7) metric_row[3] = s / float(rows_dev[index]);  // mean ratio, main.mm:949
    else metric_row[j - 4] = s;
}

inline unsigned cdiv(size_t a, size_t b) { return unsigned((a + b - 1) / b); }

}  // namespace

cudaError_t launch_dense_fwd(const DenseFwd& p, const DenseRows& r, bool x_row0, cudaStream_t s) {
    const dim3 grid(cdiv(p.n, kBN), cdiv(r.rows, kBM));
    k_dense_fwd<<<grid, kDenseThreads, 0, s>>>(p, r, x_row0 ? 1 : 0);
    return cudaGetLastError();
}
cudaError_t launch_dense_bwd(const DenseBwd& p, const DenseRows& r, cudaStream_t s) {
    const dim3 grid(cdiv(p.k, kBN), cdiv(r.rows, kBM));
    k_dense_bwd<<<grid, kDenseThreads, 0, s>>>(p, r);
    return cudaGetLastError();
}
cudaError_t launch_dense_wgrad(const DenseWgrad& p, const DenseRows& r, uint32_t chunks, cudaStream_t s) {
    const dim3 grid(cdiv(size_t(p.k) + 1, kBN), cdiv(p.n, kBM), chunks);
    k_dense_wgrad<<<grid, kDenseThreads, 0, s>>>(p, r);
    return cudaGetLastError();
}
cudaError_t launch_chunk_sum(const float* part, uint32_t chunks, size_t count, float* grad, cudaStream_t s) {
    const unsigned blocks = std::max(1u, std::min(cdiv(count, 256), 1024u));
    k_chunk_sum<<<blocks, 256, 0, s>>>(part, chunks, count, grad);
    return cudaGetLastError();
}
uint32_t layered_loss_ctas(uint32_t rows) { return cdiv(rows, kLossThreads); }
cudaError_t launch_layered_loss(const LayeredLoss& p, const DenseRows& r, cudaStream_t s) {
    k_layered_loss<<<layered_loss_ctas(r.rows), kLossThreads, 0, s>>>(p, r);
    return cudaGetLastError();
}
cudaError_t launch_layered_finish(const float* cta_sums, uint32_t ctas, float* log_std_grad, float* metric_row,
                                  const uint32_t* rows_dev, uint32_t index, cudaStream_t s) {
    k_layered_finish<<<1, 32, 0, s>>>(cta_sums, ctas, log_std_grad, metric_row, rows_dev, index);
    return cudaGetLastError();
}

namespace {
// Layers 0..L-1 of a network over `rows` rows of x (starting at x_row0), the
// hidden activations alternating between act[0] and act[1]; the output layer
// writes `out` (bias when with_bias).
cudaError_t network_forward(const MlpShape& net, const float* params, const float* x, uint32_t rows, uint32_t row0,
                            float* const act[2], float* out, bool with_bias, cudaStream_t s) {
    DenseRows r;
    r.rows = rows;
    r.row0 = row0;
    const float* in = x;
    bool in_row0 = true;
    for (uint32_t l = 0; l <= net.layers; l++) {
        const bool last = l == net.layers;
        DenseFwd f{};
        f.x = in;
        f.w = params + net.weight_offset(l);
        f.b = (!last || with_bias) ? params + net.bias_offset(l) : nullptr;
        f.y = last ? out : act[l & 1];
        f.z = nullptr;
        f.k = net.in_dim(l);
        f.n = net.out_dim(l);
        f.act = last ? -1 : int(net.activation);
        const cudaError_t e = launch_dense_fwd(f, r, in_row0, s);
        if (e != cudaSuccess) return e;
        in = f.y;
        in_row0 = false;
    }
    return cudaSuccess;
}
}  // namespace

cudaError_t launch_network_forward(const MlpShape& net, const float* params, const float* x, uint32_t rows,
                                   float* act0, float* act1, float* out, bool out_bias, cudaStream_t s) {
    float* const act[2] = {act0, act1};
    return network_forward(net, params, x, rows, 0, act, out, out_bias, s);
}

cudaError_t launch_layered_step_forward(const LayeredStep& L, uint32_t n, uint32_t tick, cudaStream_t s) {
    const cudaError_t e = network_forward(L.actor, L.actor_params, L.obs, n, tick * n, L.act, L.out_a, false, s);
    if (e != cudaSuccess) return e;
    return network_forward(L.critic, L.critic_params, L.co, n, tick * n, L.act, L.values, true, s);
}

cudaError_t launch_layered_bootstrap(const LayeredStep& L, uint32_t n, uint32_t tick, cudaStream_t s) {
    return network_forward(L.critic, L.critic_params, L.next_critic_in, n, 0, L.act, L.next_values + size_t(tick) * n, true, s);
}

void init_layered(const MlpShape& actor, const MlpShape& critic, std::vector<float>& a, std::vector<float>& c) {
    uint32_t seed = 1789;
    auto unit = [&]() {
        seed ^= seed << 13;
        seed ^= seed >> 17;
        seed ^= seed << 5;
        return float(seed >> 8) * (1.0f / 16777216.0f);
    };
    auto normal = [&]() {
        const float u = std::max(unit(), 1e-7f);
        const float r = std::sqrt(-2.0f * std::log(u));
        return r * std::cos(6.2831853f * unit());
    };
    auto fill = [&](const MlpShape& s, std::vector<float>& p, float first, float last) {
        p.assign(s.param_count(), 0.0f);
        for (uint32_t l = 0; l <= s.layers; l++) {
            const float scale = l == 0 ? first : (l == s.layers ? last : 1.0f / std::sqrt(float(s.in_dim(l))));
            const uint32_t w = s.weight_offset(l), count = s.out_dim(l) * s.in_dim(l);
            for (uint32_t i = 0; i < count; i++) p[w + i] = normal() * scale;
        }
        if (s.log_std)
            for (int i = 0; i < kActions; i++) p[s.param_count() - kActions + i] = -1.0f;
    };
    fill(actor, a, 0.04f, 0.01f);
    fill(critic, c, 0.15f, 0.1f);
}

}  // namespace mdn
