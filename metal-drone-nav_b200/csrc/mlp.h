// Layered actor and critic networks (mlp.cu): L hidden layers of one width,
// tanh or GELU, for the network shapes that the reference does not compile in
// (its actor and critic have one hidden layer of 64 tanh units, ppo.hpp:35-45).
// Parameters are flat, layer by layer: W_l [out][in] row-major, then b_l [out];
// the actor ends with log_std[4]. With one tanh hidden layer this is exactly
// the reference's layout (ppo.hpp:35-45), so the same offsets hold.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

namespace mdn {

enum Activation : uint32_t { kActTanh = 0, kActGelu = 1 };

// One network: in -> hidden x layers -> out.
struct MlpShape {
    uint32_t in = 0, hidden = 0, layers = 1, out = 0, activation = kActTanh;
    bool log_std = false;  // the actor's 4 trailing log-std parameters
    uint32_t weight_offset(uint32_t l) const;  // W of layer l (l = layers: output layer)
    uint32_t bias_offset(uint32_t l) const;
    uint32_t in_dim(uint32_t l) const { return l == 0 ? in : hidden; }
    uint32_t out_dim(uint32_t l) const { return l == layers ? out : hidden; }
    uint32_t param_count() const;
};

// Row range of a dense launch: `rows` and the first row of the input matrix,
// or, with rows_dev, both read on the device at [index] (the PPO update's
// per-minibatch arrays, so a captured graph replays unchanged; `rows` is then
// the capacity that sizes the grid).
struct DenseRows {
    uint32_t rows = 0, row0 = 0;
    const uint32_t* rows_dev = nullptr;
    const uint32_t* row0_dev = nullptr;
    uint32_t index = 0;
};

// Y[m][n] = act(sum_k X[m][k] W[n][k] + b[n]) for m < rows; X starts at row0
// (the other operands at row 0). Z, if set, receives the pre-activation.
// act = none for the output layers; b may be null (no bias).
struct DenseFwd {
    const float* x;      // [.][k], leading dimension k
    const float* w;      // [n][k]
    const float* b;      // [n] or null
    float* y;            // [rows][n]
    float* z;            // [rows][n] or null
    uint32_t k, n;
    int act;             // -1 none, else Activation
};

// dX[m][k] = (sum_n dY[m][n] W[n][k]) * act'(Zp[m][k]), the delta of the
// layer below (Zp: that layer's pre-activation).
struct DenseBwd {
    const float* dy;     // [rows][n]
    const float* w;      // [n][k]
    const float* zp;     // [rows][k]
    float* dx;           // [rows][k]
    uint32_t k, n;
    int act;
};

// Weight gradient partials: part[c][n][k] = sum over chunk c's rows of
// dY[m][n] X[m][k], and part[c][n][k_dim] = sum dY[m][n] (the bias), written
// in the flat order W then b at part + c * (n * k + n).
struct DenseWgrad {
    const float* dy;     // [rows][n]
    const float* x;      // [.][k] (starts at row0 when x_row0)
    bool x_row0;
    float* part;         // [chunks][n * k + n]
    uint32_t k, n, chunk_rows;
};

cudaError_t launch_dense_fwd(const DenseFwd& p, const DenseRows& r, bool x_row0, cudaStream_t s);
cudaError_t launch_dense_bwd(const DenseBwd& p, const DenseRows& r, cudaStream_t s);
cudaError_t launch_dense_wgrad(const DenseWgrad& p, const DenseRows& r, uint32_t chunks, cudaStream_t s);
// grad[i] = sum over c < chunks of part[c * count + i], in chunk order.
cudaError_t launch_chunk_sum(const float* part, uint32_t chunks, size_t count, float* grad, cudaStream_t s);

// Clipped-PPO loss of the layered networks, one thread per minibatch row
// (the same formulas as the fused kernels, ppo.hpp:144-181): means =
// out_a[m] + b2 + geometry prior, value = out_c[m]. Writes d_out_a (the
// actor output deltas), d_out_c (the critic's), per-CTA sums of the log-std
// derivatives and of the four loss metrics.
struct LayeredLoss {
    const float* out_a;      // [rows][4] actor output layer, no bias
    const float* out_c;      // [rows] critic value (with its bias)
    const float* obs;        // rollout observations (prior = obs[row][181..183])
    const float* actions;
    const float* logp;
    const float* advantages;
    const float* returns;
    const float* b2;         // actor output bias [4]
    const float* log_std;    // [4]
    const uint32_t* global_batch;  // [updates] rows over all ranks (loss scale)
    float clip, value_coef, entropy_coef;
    float* d_out_a;          // [rows][4]
    float* d_out_c;          // [rows]
    float* cta_sums;         // [ctas][8]: 4 log-std derivative sums, 4 loss sums
};
cudaError_t launch_layered_loss(const LayeredLoss& p, const DenseRows& r, cudaStream_t s);
// Folds the loss CTAs' sums into the actor gradient's log-std slots and the
// update's metric row (mean ratio = ratio sum / rows).
cudaError_t launch_layered_finish(const float* cta_sums, uint32_t ctas, float* log_std_grad, float* metric_row,
                                  const uint32_t* rows_dev, uint32_t index, cudaStream_t s);
uint32_t layered_loss_ctas(uint32_t rows);

// What one rollout step of a layered simulator needs (host side): the two
// networks, their parameters, and per-step scratch.
struct LayeredStep {
    MlpShape actor, critic;
    const float* actor_params;
    const float* critic_params;
    const float* obs;        // rollout observations [horizon * n][184]
    const float* co;         // rollout critic observations [horizon * n][32]
    float* act[2];           // [n][max hidden] activations, alternating by layer
    float* out_a;            // [n][4] actor output layer (no bias; k_act adds b2 and the prior)
    float* values;           // [n] critic values of this step's rows
    float* next_co;          // [n][32] post-step critic observations (k_advance)
    float* next_critic_in;   // [n][critic.in] the bootstrap critic's inputs: next_co, or the
                             // control-state critic's 64-input rows (k_control_state)
    float* next_values;      // rollout bootstrap values [horizon * n]
};
// Actor and critic forward over the step's rows (tick * n ...): out_a, values.
cudaError_t launch_layered_step_forward(const LayeredStep& L, uint32_t n, uint32_t tick, cudaStream_t s);
// Critic over next_critic_in into next_values[tick * n ...] (sim.metal:327's bootstrap value).
cudaError_t launch_layered_bootstrap(const LayeredStep& L, uint32_t n, uint32_t tick, cudaStream_t s);

// A network's forward over `rows` rows of x (device memory, from row 0):
// hidden activations alternate between act0 and act1 ([rows][hidden] each),
// the output layer writes out [rows][net.out] (with its bias when out_bias).
cudaError_t launch_network_forward(const MlpShape& net, const float* params, const float* x, uint32_t rows,
                                   float* act0, float* act1, float* out, bool out_bias, cudaStream_t s);

// Initial parameters: the seed-1789 Box-Muller stream of main.mm:548-555,
// actor first, then critic, layer by layer: the first layer's weights at the
// reference's first-layer scale (0.04 actor, 0.15 critic), hidden-to-hidden
// weights at 1/sqrt(fan_in), the output layer at the reference's scale (0.01,
// 0.1); biases 0, log_std -1. One tanh layer of 64 reproduces the reference.
void init_layered(const MlpShape& actor, const MlpShape& critic, std::vector<float>& a, std::vector<float>& c);

}  // namespace mdn
