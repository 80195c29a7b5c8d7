// C-ABI implementation of the trainer: PPOTrainer (main.mm:1110-1476).
//
// One rollout update = GAE + advantage normalisation + epochs x minibatch
// chunks of (forward/loss, gradients, [allreduce], clip+Adam). The kernel
// sequence is captured once into a CUDA graph; what changes between rollouts
// (chunk order, batch sizes, Adam bias corrections) lives in small device
// arrays uploaded before each launch, so the graph is replayed unchanged.
//
// Compiled with -ffp-contract=off: the bias corrections 1 - beta^step are
// computed here with std::pow(float, float), as cpu_reference.hpp:558-559 does.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <filesystem>
#include <fstream>
#include <memory>
#include <random>

#include "host_common.h"
#include "ppo_args.h"
#include "ppo_tc.h"

using namespace mdn;

namespace mdn {
// NCCL hooks (comm.cpp); no-ops on a single GPU.
cudaError_t comm_allreduce_double(mdn_device* dev, double* buf, size_t count, cudaStream_t s, std::string& err);
cudaError_t comm_allreduce_float(mdn_device* dev, float* buf, size_t count, cudaStream_t s, std::string& err);
void refresh_world_mirror(mdn_sim* sim);
}  // namespace mdn

struct mdn_ppo {
    mdn_sim* sim = nullptr;
    uint32_t epochs = 2, minibatch = 256, rows = 0, minibatches = 0, updates = 0;
    uint32_t fwd_grid = 1, grad_chunk = 64, grad_chunks = 1;
    uint64_t optimizer_step = 0;
    uint32_t completed_rollouts = 0;
    std::vector<uint32_t> starts;
    // device memory
    void* mem = nullptr;
    PpoArgs args{};
    uint32_t* d_starts = nullptr;  // [updates*3]: starts, batch, global batch
    float* d_bias = nullptr;       // [updates*2]
    // pinned staging for the per-rollout arrays
    uint32_t* h_idx = nullptr;
    float* h_bias = nullptr;
    cudaEvent_t staged = nullptr, ev_start = nullptr, ev_stop = nullptr;
    cudaGraphExec_t graph = nullptr;
    float last_update_ms = 0.0f;
    uint32_t launches = 0;  // kernel nodes in the update graph
    // wide actor (tensor-core update, wide.cu)
    bool wide = false;
    uint32_t wide_splits = 0, wide_groups = 0;
    void* wide_mem = nullptr;
    float* wide_partials = nullptr;   // [hidden/128][minibatch][4] forward slice sums
    float* wide_delta = nullptr;      // [ceil128(minibatch)][hidden] hidden deltas
    float* wide_w1_parts = nullptr;   // [splits][hidden][184] dW1 partials
    float* wide_colsums = nullptr;    // [groups][5][hidden] db1 / dW2 partials
    float* wide_grad = nullptr;       // [actor params + critic params]
    float* wide_norm_parts = nullptr; // [2 * SMs]
    WideMap obs32_map{}, delta_map{}, obs256_map{}, w1_128_map{};
    // 64-unit actor on the tensor cores (mdn_ppo_set_tensor_cores, ppo_tc.cu)
    bool tensor_cores = false;
    bool tc_maps_ready = false;
    TcMaps tc_maps{};
    uint32_t tc_grid = 1;
    uint32_t* tc_error = nullptr;
    // layered networks (mlp.cu): per hidden layer the activations y and
    // pre-activations z of the minibatch rows, the output layers, two delta
    // buffers, the weight-gradient partials and the flat gradient
    bool layered = false;
    void* lay_mem = nullptr;
    std::vector<float*> lay_ya, lay_za, lay_yc, lay_zc;
    float* lay_out_a = nullptr;   // [minibatch][4]
    float* lay_out_c = nullptr;   // [minibatch]
    float* lay_dout_a = nullptr;  // [minibatch][4]
    float* lay_dout_c = nullptr;  // [minibatch]
    float* lay_d[2] = {nullptr, nullptr};  // [minibatch][widest]
    float* lay_part = nullptr;    // [chunks][largest layer's W + b]
    float* lay_cta = nullptr;     // [loss CTAs][8]
    float* lay_grad = nullptr;    // [actor params + critic params]
    float* lay_norm = nullptr;    // [2 * SMs]
    uint32_t lay_loss_ctas = 1;
};

namespace {
// Row chunks of one layer's weight-gradient launch: enough CTAs (k tiles x
// n tiles x chunks) for two per SM, chunks of at least 64 rows.
void layer_chunks(uint32_t k, uint32_t n, uint32_t rows, uint32_t sms, uint32_t& chunks, uint32_t& chunk_rows) {
    const uint32_t tiles = ((k + 1 + 63) / 64) * ((n + 127) / 128);  // k_dense_wgrad tiles: 128 units x 64 inputs
    const uint32_t want = std::max<uint32_t>(1, (2 * sms + tiles - 1) / tiles);
    chunk_rows = std::max<uint32_t>(64, ((rows + want - 1) / want + 15) / 16 * 16);
    chunks = (rows + chunk_rows - 1) / chunk_rows;
}
}  // namespace

namespace {
size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// The raw-GAE copy that challenge-bank training scores levels with
// (main.mm:1325-1328); null while the simulator has no bank.
float* raw_advantages_of(const mdn_sim* sim) {
    return sim->bytes[MDN_BUF_RAW_ADVANTAGES] ? static_cast<float*>(sim->buf[MDN_BUF_RAW_ADVANTAGES]) : nullptr;
}

mdn_ppo* checked(mdn_ppo* p) {
    require(p != nullptr && p->sim != nullptr, MDN_ERR_INVALID, "null mdn_ppo");
    cuda_check(cudaSetDevice(p->sim->dev->gpu), "cudaSetDevice");
    return p;
}

// Enqueue one whole rollout update on the sim stream (captured into a graph).
// One minibatch of the layered networks: actor and critic forward storing
// each hidden layer's activations and pre-activations, the loss, then layer
// by layer from the top: weight-gradient partials of the layer (summed in
// chunk order into the flat gradient) and the deltas of the layer below;
// [allreduce]; clip + Adam per network (log-std clamp on the actor).
void enqueue_layered_minibatch(mdn_ppo* t, uint32_t u, bool multi) {
    mdn_sim* sim = t->sim;
    mdn_device* dev = sim->dev;
    const LayeredStep& L = *sim->lay;
    const PpoArgs& p = t->args;
    cudaStream_t s = sim->stream;
    std::string err;
    DenseRows R;
    R.rows = t->minibatch;
    R.rows_dev = p.batch;
    R.row0_dev = p.starts;
    R.index = u;
    auto forward = [&](const MlpShape& net, const float* params, const float* x, const std::vector<float*>& ys,
                       const std::vector<float*>& zs, float* out, bool out_bias) {
        const float* in = x;
        bool in_row0 = true;
        for (uint32_t l = 0; l <= net.layers; l++) {
            const bool last = l == net.layers;
            DenseFwd f{};
            f.x = in;
            f.w = params + net.weight_offset(l);
            f.b = (!last || out_bias) ? params + net.bias_offset(l) : nullptr;
            f.y = last ? out : ys[l];
            f.z = last ? nullptr : zs[l];
            f.k = net.in_dim(l);
            f.n = net.out_dim(l);
            f.act = last ? -1 : int(net.activation);
            cuda_check(launch_dense_fwd(f, R, in_row0, s), "layered forward");
            in = f.y;
            in_row0 = false;
        }
    };
    auto backward = [&](const MlpShape& net, const float* params, const float* x0, const std::vector<float*>& ys,
                        const std::vector<float*>& zs, const float* dout, float* grad) {
        const float* dy = dout;
        for (int l = int(net.layers); l >= 0; l--) {
            DenseWgrad w{};
            w.dy = dy;
            w.x = l == 0 ? x0 : ys[l - 1];
            w.x_row0 = l == 0;
            w.part = t->lay_part;
            w.k = net.in_dim(uint32_t(l));
            w.n = net.out_dim(uint32_t(l));
            uint32_t chunks = 1;
            layer_chunks(w.k, w.n, t->minibatch, uint32_t(dev->sm_count), chunks, w.chunk_rows);
            cuda_check(launch_dense_wgrad(w, R, chunks, s), "layered weight gradient");
            cuda_check(launch_chunk_sum(t->lay_part, chunks, size_t(w.n) * w.k + w.n,
                                        grad + net.weight_offset(uint32_t(l)), s),
                       "layered gradient sum");
            if (l == 0) break;
            DenseBwd b{};
            b.dy = dy;
            b.w = params + net.weight_offset(uint32_t(l));
            b.zp = zs[l - 1];
            b.dx = t->lay_d[(net.layers - uint32_t(l)) & 1u];
            b.k = net.in_dim(uint32_t(l));
            b.n = net.out_dim(uint32_t(l));
            b.act = int(net.activation);
            cuda_check(launch_dense_bwd(b, R, s), "layered deltas");
            dy = b.dx;
        }
    };
    const uint32_t actor_n = sim->actor_params;
    float* grad_a = t->lay_grad;
    float* grad_c = t->lay_grad + actor_n;
    forward(L.actor, p.actor, p.obs, t->lay_ya, t->lay_za, t->lay_out_a, false);
    forward(L.critic, p.critic, p.co, t->lay_yc, t->lay_zc, t->lay_out_c, true);
    LayeredLoss lo{};
    lo.out_a = t->lay_out_a;
    lo.out_c = t->lay_out_c;
    lo.obs = p.obs;
    lo.actions = p.actions;
    lo.logp = p.logp;
    lo.advantages = p.advantages;
    lo.returns = p.returns;
    lo.b2 = p.actor + L.actor.bias_offset(L.actor.layers);
    lo.log_std = p.actor + actor_n - kActions;
    lo.global_batch = p.global_batch;
    lo.clip = p.clip;
    lo.value_coef = p.value_coef;
    lo.entropy_coef = p.entropy_coef;
    lo.d_out_a = t->lay_dout_a;
    lo.d_out_c = t->lay_dout_c;
    lo.cta_sums = t->lay_cta;
    cuda_check(launch_layered_loss(lo, R, s), "layered loss");
    backward(L.actor, p.actor, p.obs, t->lay_ya, t->lay_za, t->lay_dout_a, grad_a);
    backward(L.critic, p.critic, p.co, t->lay_yc, t->lay_zc, t->lay_dout_c, grad_c);
    cuda_check(launch_layered_finish(t->lay_cta, t->lay_loss_ctas, grad_a + actor_n - kActions, p.metric_rows + 4 * u,
                                     p.batch, u, s),
               "layered loss sums");
    if (multi)
        cuda_check(comm_allreduce_float(dev, t->lay_grad, size_t(actor_n) + sim->critic_params, s, err), err.c_str());
    WideAdamArgs ad{};
    ad.grad = grad_a;
    ad.params = p.actor;
    ad.m = p.actor_m;
    ad.v = p.actor_v;
    ad.count = actor_n;
    ad.bias_corr = p.bias_corr + 2 * u;
    ad.learning_rate = p.learning_rate;
    ad.max_norm = p.max_norm;
    ad.norm_out = p.grad_norms + 2 * u;
    cuda_check(launch_wide_clip_adam(ad, t->lay_norm, dev->sm_count, s), "layered actor clip+adam");
    WideAdamArgs ac = ad;
    ac.grad = grad_c;
    ac.params = p.critic;
    ac.m = p.critic_m;
    ac.v = p.critic_v;
    ac.count = sim->critic_params;
    ac.no_clamp = 1;
    ac.norm_out = p.grad_norms + 2 * u + 1;
    cuda_check(launch_wide_clip_adam(ac, t->lay_norm, dev->sm_count, s), "layered critic clip+adam");
}

void enqueue_update(mdn_ppo* t) {
    mdn_sim* sim = t->sim;
    mdn_device* dev = sim->dev;
    cudaStream_t s = sim->stream;
    const PpoArgs& p = t->args;
    std::string err;
    cuda_check(launch_gae_sum(p, s), "gae");
    cuda_check(launch_adv_stats(p, 0, s), "advantage sum");
    cuda_check(comm_allreduce_double(dev, p.stats, 1, s, err), err.c_str());
    cuda_check(launch_adv_finalize(p, 0, s), "advantage mean");
    cuda_check(launch_adv_sq(p, s), "advantage variance");
    cuda_check(launch_adv_stats(p, 1, s), "advantage variance sum");
    cuda_check(comm_allreduce_double(dev, p.stats + 1, 1, s, err), err.c_str());
    cuda_check(launch_adv_finalize(p, 1, s), "advantage scale");
    cuda_check(launch_adv_apply(p, dev->sm_count, s), "advantage normalise");
    const bool multi = dev->world > 1;
    const uint32_t chunks = multi ? std::max<uint32_t>(t->grad_chunks, 2) : t->grad_chunks;
    for (uint32_t u = 0; u < t->updates; u++) {
        if (t->layered) {
            enqueue_layered_minibatch(t, u, multi);
            continue;
        }
        if (t->wide) {
            // Wide actor: tensor-core forward -> loss (+ critic, b2, log_std
            // gradients) -> tensor-core backward (deltas, db1/dW2 partials) ->
            // dW1 = delta^T obs -> flat gradient -> [allreduce] -> clip + Adam.
            const uint32_t H = sim->actor_hidden;
            const int sms = dev->sm_count;
            const float* actor = static_cast<const float*>(sim->buf[MDN_BUF_ACTOR]);
            WideRowsArgs fa{};
            fa.rows = t->minibatch;
            fa.rows_dev = p.batch;
            fa.row0_dev = p.starts;
            fa.index = u;
            fa.hidden = H;
            fa.b1 = actor + size_t(H) * kActorObs;
            fa.w2 = fa.b1 + H;
            fa.partials = t->wide_partials;
            fa.error = sim->wide_error;
            cuda_check(launch_wide_forward(sim->wide->obs_map, sim->wide->w1_map, fa, sms, s), "wide forward");
            cuda_check(launch_minibatch(p, u, chunks, s), "minibatch");
            WideRowsArgs ba = fa;
            ba.partials = nullptr;
            ba.d_mean = p.mb_dm;
            ba.delta = t->wide_delta;
            ba.colsum_out = t->wide_colsums;
            cuda_check(launch_wide_backward(t->obs256_map, t->w1_128_map, ba, sms, s), "wide backward");
            WideGradArgs ga{};
            ga.rows = t->minibatch;
            ga.rows_dev = p.batch;
            ga.row0_dev = p.starts;
            ga.index = u;
            ga.hidden = H;
            ga.splits = t->wide_splits;
            ga.out = t->wide_w1_parts;
            ga.error = sim->wide_error;
            cuda_check(launch_wide_wgrad(t->delta_map, t->obs32_map, ga, sms, s), "wide weight gradient");
            WideAssembleArgs aa{};
            aa.hidden = H;
            aa.splits = t->wide_splits;
            aa.groups = t->wide_groups;
            aa.w1_parts = t->wide_w1_parts;
            aa.colsums = t->wide_colsums;
            aa.small_grad = chunks > 1 ? p.grad : p.grad_partials;
            aa.grad = t->wide_grad;
            cuda_check(launch_wide_assemble(aa, sms, s), "wide gradient");
            const size_t total = size_t(sim->actor_params) + kCriticParams;
            if (multi) cuda_check(comm_allreduce_float(dev, t->wide_grad, total, s, err), err.c_str());
            WideAdamArgs ad{};
            ad.grad = t->wide_grad;
            ad.params = static_cast<float*>(sim->buf[MDN_BUF_ACTOR]);
            ad.m = p.actor_m;
            ad.v = p.actor_v;
            ad.count = sim->actor_params;
            ad.bias_corr = p.bias_corr + 2 * u;
            ad.learning_rate = p.learning_rate;
            ad.max_norm = p.max_norm;
            ad.norm_out = p.grad_norms + 2 * u;
            cuda_check(launch_wide_clip_adam(ad, t->wide_norm_parts, sms, s), "wide clip+adam");
            cuda_check(launch_clip_adam_critic(p, u, t->wide_grad + sim->actor_params, s), "critic clip+adam");
            continue;
        }
        if (t->tensor_cores) {
            // one gradient partial per CTA, summed in CTA order into p.grad
            PpoArgs pt = p;
            pt.fwd_grid = multi ? std::max<uint32_t>(t->tc_grid, 2) : t->tc_grid;
            cuda_check(launch_minibatch_tc(pt, t->tc_maps, u, pt.fwd_grid, s), "tensor-core minibatch");
            if (multi) cuda_check(comm_allreduce_float(dev, pt.grad, kPpoParams, s, err), err.c_str());
            cuda_check(launch_clip_adam(pt, u, pt.fwd_grid, s), "clip+adam");
            continue;
        }
        cuda_check(launch_minibatch(p, u, chunks, s), "minibatch");
        if (multi) cuda_check(comm_allreduce_float(dev, p.grad, kPpoParams, s, err), err.c_str());
        cuda_check(launch_clip_adam(p, u, chunks, s), "clip+adam");
    }
    cuda_check(launch_metrics_mean(p, t->updates, s), "metrics");
}
}  // namespace

extern "C" int mdn_ppo_create(mdn_sim* sim, uint32_t epochs, uint32_t minibatch_rows, mdn_ppo** out) {
    return guarded([&] {
        require(sim && out, MDN_ERR_INVALID, "mdn_ppo_create: null argument");
        cuda_check(cudaSetDevice(sim->dev->gpu), "cudaSetDevice");
        require(epochs >= 1 && epochs <= 4, MDN_ERR_INVALID, "PPO epochs must be 1..4");  // main.mm:1160
        auto t = std::make_unique<mdn_ppo>();
        t->sim = sim;
        t->epochs = epochs;
        t->minibatch = minibatch_rows ? minibatch_rows : 256u;
        t->rows = sim->n * sim->horizon;
        require(t->rows > 0, MDN_ERR_INVALID, "PPO requires at least one rollout row");
        t->minibatch = std::min(t->minibatch, t->rows);
        t->minibatches = (t->rows + t->minibatch - 1) / t->minibatch;
        t->updates = t->epochs * t->minibatches;
        t->starts.resize(t->minibatches);
        const uint32_t sms = uint32_t(sim->dev->sm_count);
        t->fwd_grid = std::max<uint32_t>(1, std::min<uint32_t>((t->minibatch + 63) / 64, 2 * sms));
        const uint32_t per = (t->minibatch + 2 * sms - 1) / (2 * sms);
        t->grad_chunk = std::max<uint32_t>(64, (per + 31) / 32 * 32);
        t->grad_chunks = (t->minibatch + t->grad_chunk - 1) / t->grad_chunk;
        const uint32_t chunk_bufs = std::max<uint32_t>(t->grad_chunks, 2);
        // The 64-unit actor's fused minibatch kernel (ppo.cu k_mb_fused) runs one
        // CTA per gradient chunk and writes one loss partial per CTA.
        if (!sim->wide) t->fwd_grid = sim->dev->world > 1 ? chunk_bufs : t->grad_chunks;
        const size_t mb = t->minibatch, U = t->updates, P = kPpoParams;
        // One allocation for all trainer-owned device memory.
        PpoArgs& a = t->args;
        size_t off = 0;
        auto carve = [&](size_t bytes) { const size_t o = off; off += align256(bytes); return o; };
        const size_t AP = sim->actor_params;
        const size_t CP = sim->critic_params;
        const size_t o_am = carve(AP * 4), o_av = carve(AP * 4), o_cm = carve(CP * 4),
                     o_cv = carve(CP * 4), o_sp = carve(gae_blocks(sim->n) * 8), o_st = carve(2 * 8),
                     o_sv = carve(2 * 4), o_idx = carve(U * 3 * 4), o_bias = carve(U * 2 * 4), o_ah = carve(mb * 64 * 4),
                     o_ch = carve(mb * 64 * 4), o_ad = carve(mb * 64 * 4), o_cd = carve(mb * 64 * 4),
                     o_dm = carve(mb * 4 * 4), o_dls = carve(mb * 4 * 4), o_dv = carve(mb * 4),
                     o_gp = carve(size_t(chunk_bufs) * P * 4), o_g = carve(P * 4), o_lp = carve(U * t->fwd_grid * 4 * 4),
                     o_mr = carve(U * 4 * 4), o_mm = carve(4 * 4), o_gn = carve(U * 2 * 4), o_err = carve(4);
        const cudaError_t e = cudaMalloc(&t->mem, off);
        require(e == cudaSuccess, MDN_ERR_NOMEM, std::string("cudaMalloc trainer: ") + cudaGetErrorString(e));
        char* base = static_cast<char*>(t->mem);
        cuda_check(cudaMemsetAsync(base, 0, off, sim->stream), "clear trainer memory");
        a.n = sim->n;
        a.horizon = sim->horizon;
        a.global_rows = uint64_t(t->rows) * uint64_t(sim->dev->world);
        a.gamma = .99f;        // main.mm:1193
        a.lambda = .95f;
        a.clip = .2f;
        a.value_coef = .5f;
        a.entropy_coef = sim->cfg.entropy_coef;
        a.learning_rate = sim->cfg.learning_rate;
        a.max_norm = .5f;      // main.mm:1202
        a.rewards = static_cast<float*>(sim->buf[MDN_BUF_REWARDS]);
        a.values = static_cast<float*>(sim->buf[MDN_BUF_VALUES]);
        a.next_values = static_cast<float*>(sim->buf[MDN_BUF_NEXT_VALUES]);
        a.terminated = static_cast<uint8_t*>(sim->buf[MDN_BUF_TERMINATED]);
        a.truncated = static_cast<uint8_t*>(sim->buf[MDN_BUF_TRUNCATED]);
        a.advantages = static_cast<float*>(sim->buf[MDN_BUF_ADVANTAGES]);
        a.returns = static_cast<float*>(sim->buf[MDN_BUF_RETURNS]);
        a.raw_advantages = raw_advantages_of(sim);
        a.obs = static_cast<float*>(sim->buf[MDN_BUF_OBS]);
        a.co = static_cast<float*>(sim->buf[MDN_BUF_CO]);
        a.actions = static_cast<float*>(sim->buf[MDN_BUF_ACTIONS]);
        a.logp = static_cast<float*>(sim->buf[MDN_BUF_LOGP]);
        a.actor = static_cast<float*>(sim->buf[MDN_BUF_ACTOR]);
        a.critic = static_cast<float*>(sim->buf[MDN_BUF_CRITIC]);
        a.actor_m = reinterpret_cast<float*>(base + o_am);
        a.actor_v = reinterpret_cast<float*>(base + o_av);
        a.critic_m = reinterpret_cast<float*>(base + o_cm);
        a.critic_v = reinterpret_cast<float*>(base + o_cv);
        a.stat_partials = reinterpret_cast<double*>(base + o_sp);
        a.stats = reinterpret_cast<double*>(base + o_st);
        a.stat_values = reinterpret_cast<float*>(base + o_sv);
        t->d_starts = reinterpret_cast<uint32_t*>(base + o_idx);
        t->d_bias = reinterpret_cast<float*>(base + o_bias);
        a.starts = t->d_starts;
        a.batch = t->d_starts + U;
        a.global_batch = t->d_starts + 2 * U;
        a.bias_corr = t->d_bias;
        a.mb_ah = reinterpret_cast<float*>(base + o_ah);
        a.mb_ch = reinterpret_cast<float*>(base + o_ch);
        a.mb_adelta = reinterpret_cast<float*>(base + o_ad);
        a.mb_cdelta = reinterpret_cast<float*>(base + o_cd);
        a.mb_dm = reinterpret_cast<float*>(base + o_dm);
        a.mb_dls = reinterpret_cast<float*>(base + o_dls);
        a.mb_dv = reinterpret_cast<float*>(base + o_dv);
        a.grad_partials = reinterpret_cast<float*>(base + o_gp);
        a.grad = reinterpret_cast<float*>(base + o_g);
        a.loss_partials = reinterpret_cast<float*>(base + o_lp);
        a.metric_rows = reinterpret_cast<float*>(base + o_mr);
        a.metric_mean = reinterpret_cast<float*>(base + o_mm);
        a.grad_norms = reinterpret_cast<float*>(base + o_gn);
        t->tc_error = reinterpret_cast<uint32_t*>(base + o_err);
        a.tc_error = t->tc_error;
        a.fwd_grid = t->fwd_grid;
        a.grad_chunk = t->grad_chunk;
        a.actor_b2 = sim->actor_hidden * (kActorObs + 1 + kActions);
        a.actor_log_std = a.actor_b2 + kActions;
        if (sim->wide) {
            t->wide = true;
            const uint32_t H = sim->actor_hidden, sms = uint32_t(sim->dev->sm_count);
            const size_t cap256 = (size_t(t->minibatch) + 255) / 256 * 256;
            const uint32_t m_tiles = H / 128;
            t->wide_splits = std::max<uint32_t>(1, std::min<uint32_t>((3 * sms + m_tiles - 1) / m_tiles,
                                                                      (t->minibatch + 31) / 32));
            t->wide_groups = wide_backward_groups(H, int(sms));
            size_t woff = 0;
            auto wcarve = [&](size_t bytes) { const size_t o = woff; woff += align256(bytes); return o; };
            const size_t w_part = wcarve(size_t(H / 128) * t->minibatch * 16), w_delta = wcarve(cap256 * H * 4),
                         w_w1 = wcarve(size_t(t->wide_splits) * H * kActorObs * 4),
                         w_cs = wcarve(size_t(t->wide_groups) * 5 * H * 4),
                         w_g = wcarve((size_t(sim->actor_params) + kCriticParams) * 4), w_np = wcarve(size_t(sms) * 2 * 4);
            const cudaError_t we = cudaMalloc(&t->wide_mem, woff);
            if (we != cudaSuccess) {
                cudaFree(t->mem);
                throw Error(MDN_ERR_NOMEM, std::string("cudaMalloc wide trainer: ") + cudaGetErrorString(we));
            }
            char* wb = static_cast<char*>(t->wide_mem);
            cuda_check(cudaMemsetAsync(wb, 0, woff, sim->stream), "clear wide trainer memory");
            t->wide_partials = reinterpret_cast<float*>(wb + w_part);
            t->wide_delta = reinterpret_cast<float*>(wb + w_delta);
            t->wide_w1_parts = reinterpret_cast<float*>(wb + w_w1);
            t->wide_colsums = reinterpret_cast<float*>(wb + w_cs);
            t->wide_grad = reinterpret_cast<float*>(wb + w_g);
            t->wide_norm_parts = reinterpret_cast<float*>(wb + w_np);
            a.wide_partials = t->wide_partials;
            a.wide_slices = H / 128;
            a.wide_rows_cap = t->minibatch;
            cuda_check(wide_make_map(&t->obs32_map, static_cast<const float*>(sim->buf[MDN_BUF_OBS]), kActorObs,
                                     size_t(sim->n) * sim->horizon, kActorObs * 4, 32, true),
                       "observation tensor map (32-row boxes)");
            cuda_check(wide_make_map(&t->delta_map, t->wide_delta, H, cap256, size_t(H) * 4, 32, true), "delta tensor map");
            cuda_check(wide_make_map(&t->obs256_map, static_cast<const float*>(sim->buf[MDN_BUF_OBS]), kActorObs,
                                     size_t(sim->n) * sim->horizon, kActorObs * 4, 256),
                       "observation tensor map (256-row boxes)");
            cuda_check(wide_make_map(&t->w1_128_map, static_cast<const float*>(sim->buf[MDN_BUF_ACTOR]), kActorObs, H,
                                     kActorObs * 4, 128),
                       "actor W1 tensor map (128-row boxes)");
        }
        if (sim->layered) {
            t->layered = true;
            const MlpShape& A = sim->lay->actor;
            const MlpShape& C = sim->lay->critic;
            a.actor_b2 = A.bias_offset(A.layers);
            a.actor_log_std = A.param_count() - kActions;
            t->lay_loss_ctas = layered_loss_ctas(t->minibatch);
            size_t largest = 0;  // weight-gradient partials of the largest layer launch
            for (const MlpShape* net : {&A, &C})
                for (uint32_t l = 0; l <= net->layers; l++) {
                    uint32_t chunks = 1, chunk_rows = 64;
                    layer_chunks(net->in_dim(l), net->out_dim(l), t->minibatch, sms, chunks, chunk_rows);
                    largest = std::max(largest, size_t(chunks) * (size_t(net->out_dim(l)) * net->in_dim(l) +
                                                                   net->out_dim(l)));
                }
            const size_t widest = std::max(A.hidden, C.hidden);
            size_t loff = 0;
            auto lcarve = [&](size_t bytes) { const size_t o = loff; loff += align256(bytes); return o; };
            std::vector<size_t> o_ya, o_za, o_yc, o_zc;
            for (uint32_t l = 0; l < A.layers; l++) {
                o_ya.push_back(lcarve(mb * A.hidden * 4));
                o_za.push_back(lcarve(mb * A.hidden * 4));
            }
            for (uint32_t l = 0; l < C.layers; l++) {
                o_yc.push_back(lcarve(mb * C.hidden * 4));
                o_zc.push_back(lcarve(mb * C.hidden * 4));
            }
            const size_t l_oa = lcarve(mb * 16), l_oc = lcarve(mb * 4), l_da = lcarve(mb * 16), l_dc = lcarve(mb * 4),
                         l_d0 = lcarve(mb * widest * 4), l_d1 = lcarve(mb * widest * 4),
                         l_part = lcarve(largest * 4),
                         l_cta = lcarve(size_t(t->lay_loss_ctas) * 8 * 4), l_g = lcarve((AP + CP) * 4),
                         l_n = lcarve(size_t(sms) * 2 * 4);
            const cudaError_t le = cudaMalloc(&t->lay_mem, loff);
            if (le != cudaSuccess) {
                cudaFree(t->mem);
                throw Error(MDN_ERR_NOMEM, std::string("cudaMalloc layered trainer: ") + cudaGetErrorString(le));
            }
            char* lb = static_cast<char*>(t->lay_mem);
            cuda_check(cudaMemsetAsync(lb, 0, loff, sim->stream), "clear layered trainer memory");
            auto at = [&](size_t o) { return reinterpret_cast<float*>(lb + o); };
            for (size_t o : o_ya) t->lay_ya.push_back(at(o));
            for (size_t o : o_za) t->lay_za.push_back(at(o));
            for (size_t o : o_yc) t->lay_yc.push_back(at(o));
            for (size_t o : o_zc) t->lay_zc.push_back(at(o));
            t->lay_out_a = at(l_oa);
            t->lay_out_c = at(l_oc);
            t->lay_dout_a = at(l_da);
            t->lay_dout_c = at(l_dc);
            t->lay_d[0] = at(l_d0);
            t->lay_d[1] = at(l_d1);
            t->lay_part = at(l_part);
            t->lay_cta = at(l_cta);
            t->lay_grad = at(l_g);
            t->lay_norm = at(l_n);
        }
        cuda_check(cudaMallocHost(&t->h_idx, U * 3 * 4), "pinned staging");
        cuda_check(cudaMallocHost(&t->h_bias, U * 2 * 4), "pinned staging");
        cuda_check(cudaEventCreateWithFlags(&t->staged, cudaEventDisableTiming), "event");
        cuda_check(cudaEventCreate(&t->ev_start), "event");
        cuda_check(cudaEventCreate(&t->ev_stop), "event");
        cuda_check(cudaEventRecord(t->staged, sim->stream), "event");
        cuda_check(configure_ppo_kernels(), "ppo kernel attributes");
        cuda_check(cudaStreamSynchronize(sim->stream), "mdn_ppo_create");
        sim->dev->trainers.push_back(t.get());
        *out = t.release();
    });
}

extern "C" int mdn_ppo_destroy(mdn_ppo* t) {
    return guarded([&] {
        if (!t) return;
        cuda_check(cudaSetDevice(t->sim->dev->gpu), "cudaSetDevice");
        cudaStreamSynchronize(t->sim->stream);
        if (t->graph) cudaGraphExecDestroy(t->graph);
        cudaFree(t->mem);
        cudaFree(t->wide_mem);
        cudaFree(t->lay_mem);
        cudaFreeHost(t->h_idx);
        cudaFreeHost(t->h_bias);
        cudaEventDestroy(t->staged);
        cudaEventDestroy(t->ev_start);
        cudaEventDestroy(t->ev_stop);
        auto& v = t->sim->dev->trainers;
        v.erase(std::remove(v.begin(), v.end(), t), v.end());
        delete t;
    });
}

namespace {
// main.mm:1331-1337: canonical chunk starts, shuffled by the rollout-seeded
// mt19937, reshuffled once at epoch 1 (later epochs reuse that order).
void chunk_order(uint32_t rows, uint32_t minibatch, uint32_t epochs, uint32_t rollout_index,
                 std::vector<uint32_t>& starts, std::vector<uint32_t>& out) {
    starts.clear();
    for (uint32_t s0 = 0; s0 < rows; s0 += minibatch) starts.push_back(s0);
    std::mt19937 rng(0x9e3779b9u + rollout_index * 0x85ebca6bu);
    std::shuffle(starts.begin(), starts.end(), rng);
    out.clear();
    for (uint32_t epoch = 0; epoch < epochs; epoch++) {
        if (epoch == 1) std::shuffle(starts.begin(), starts.end(), rng);
        out.insert(out.end(), starts.begin(), starts.end());
    }
}
void chunk_order(mdn_ppo* t, uint32_t rollout_index, std::vector<uint32_t>& out) {
    chunk_order(t->rows, t->minibatch, t->epochs, rollout_index, t->starts, out);
}
}  // namespace

extern "C" int mdn_minibatch_order(uint32_t rows, uint32_t minibatch, uint32_t epochs, uint32_t rollout_index,
                                   uint32_t* out, size_t count) {
    return guarded([&] {
        require(rows > 0 && minibatch > 0 && epochs > 0 && out, MDN_ERR_INVALID, "minibatch order: bad argument");
        const size_t chunks = (size_t(rows) + minibatch - 1) / minibatch;
        require(count == chunks * epochs, MDN_ERR_INVALID, "minibatch order: count must be epochs*chunks");
        std::vector<uint32_t> starts, order;
        chunk_order(rows, minibatch, epochs, rollout_index, starts, order);
        std::copy(order.begin(), order.end(), out);
    });
}

extern "C" int mdn_ppo_minibatch_order(mdn_ppo* t, uint32_t rollout_index, uint32_t* out, size_t count) {
    return guarded([&] {
        checked(t);
        require(out && count == size_t(t->updates), MDN_ERR_INVALID, "minibatch order: count must be epochs*chunks");
        std::vector<uint32_t> order;
        chunk_order(t, rollout_index, order);
        std::copy(order.begin(), order.end(), out);
    });
}

extern "C" int mdn_ppo_rollout_update(mdn_ppo* t, uint32_t rollout_index) {
    return guarded([&] {
        checked(t);
        mdn_sim* sim = t->sim;
        // PPOTrainer reads the learning rate and entropy coefficient from the
        // simulator config (main.mm:1193,1368); they are graph arguments here.
        if (sim->cfg.learning_rate != t->args.learning_rate || sim->cfg.entropy_coef != t->args.entropy_coef ||
            raw_advantages_of(sim) != t->args.raw_advantages) {
            t->args.learning_rate = sim->cfg.learning_rate;
            t->args.entropy_coef = sim->cfg.entropy_coef;
            t->args.raw_advantages = raw_advantages_of(sim);
            if (t->graph) {
                cudaGraphExecDestroy(t->graph);
                t->graph = nullptr;
            }
        }
        std::vector<uint32_t> order;
        chunk_order(t, rollout_index, order);
        require(!sim->dev->comm_failed, MDN_ERR_NCCL,
                "rollout update: the NCCL communicator was aborted after a failure; re-create it (mdn_comm_init)");
        sync_event(sim->dev, t->staged, "staging reuse");
        const uint32_t U = t->updates;
        for (uint32_t u = 0; u < U; u++) {
            const uint32_t begin = order[u];
            const uint32_t b = std::min(t->minibatch, t->rows - begin);
            require(t->optimizer_step < uint64_t(UINT32_MAX), MDN_ERR_STATE, "PPO Adam step overflow");
            const uint32_t step = uint32_t(++t->optimizer_step);
            t->h_idx[u] = begin;
            t->h_idx[U + u] = b;
            t->h_idx[2 * U + u] = b * uint32_t(sim->dev->world);
            // cpu_reference.hpp:558-559
            t->h_bias[2 * u] = 1.0f - std::pow(0.9f, float(step));
            t->h_bias[2 * u + 1] = 1.0f - std::pow(0.999f, float(step));
        }
        cuda_check(cudaMemcpyAsync(t->d_starts, t->h_idx, U * 3 * 4, cudaMemcpyHostToDevice, sim->stream), "stage");
        cuda_check(cudaMemcpyAsync(t->d_bias, t->h_bias, U * 2 * 4, cudaMemcpyHostToDevice, sim->stream), "stage");
        cuda_check(cudaEventRecord(t->staged, sim->stream), "event");
        if (!t->graph) {
            cudaGraph_t g;
            cuda_check(cudaStreamBeginCapture(sim->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
            try {
                enqueue_update(t);
            } catch (...) {
                cudaStreamEndCapture(sim->stream, &g);
                throw;
            }
            cuda_check(cudaStreamEndCapture(sim->stream, &g), "end capture");
            size_t nodes = 0;
            cudaGraphGetNodes(g, nullptr, &nodes);
            std::vector<cudaGraphNode_t> list(nodes);
            if (nodes) cudaGraphGetNodes(g, list.data(), &nodes);
            t->launches = 0;
            for (auto node : list) {
                cudaGraphNodeType type;
                if (cudaGraphNodeGetType(node, &type) == cudaSuccess && type == cudaGraphNodeTypeKernel) t->launches++;
            }
            const cudaError_t inst = cudaGraphInstantiate(&t->graph, g, 0);
            cudaGraphDestroy(g);
            cuda_check(inst, "graph instantiate");
        }
        cuda_check(cudaEventRecord(t->ev_start, sim->stream), "event");
        cuda_check(cudaGraphLaunch(t->graph, sim->stream), "update graph");
        cuda_check(cudaEventRecord(t->ev_stop, sim->stream), "event");
        t->completed_rollouts = rollout_index + 1;
    });
}

extern "C" int mdn_ppo_set_tensor_cores(mdn_ppo* t, int enabled) {
    return guarded([&] {
        checked(t);
        mdn_sim* sim = t->sim;
        require(!(enabled && sim->layered), MDN_ERR_INVALID,
                "tensor-core minibatch path: the 64-unit actor and critic only (not layered networks)");
        require(!(enabled && sim->wide), MDN_ERR_INVALID,
                "tensor-core minibatch path: the wide actor already runs on the tensor cores");
        cuda_check(cudaStreamSynchronize(sim->stream), "set tensor cores");
        if (enabled && !t->tc_maps_ready) {
            cuda_check(tc_make_maps(&t->tc_maps, static_cast<const float*>(sim->buf[MDN_BUF_OBS]),
                                    static_cast<const float*>(sim->buf[MDN_BUF_CO]), uint64_t(sim->n) * sim->horizon,
                                    static_cast<const float*>(sim->buf[MDN_BUF_ACTOR]),
                                    static_cast<const float*>(sim->buf[MDN_BUF_CRITIC])),
                       "tensor-core minibatch tensor maps");
            cuda_check(configure_tc_kernels(), "tensor-core minibatch kernel attributes");
            t->tc_grid = tc_grid(t->minibatch, sim->dev->sm_count);
            t->tc_maps_ready = true;
        }
        if (t->tensor_cores != (enabled != 0) && t->graph) {
            cudaGraphExecDestroy(t->graph);  // the update graph is captured per path
            t->graph = nullptr;
        }
        t->tensor_cores = enabled != 0;
    });
}

namespace mdn {
// A barrier wait of the tensor-core minibatch kernel that gave up (called by
// mdn_sync once the streams are idle).
void check_trainer_errors(mdn_device* dev) {
    for (mdn_ppo* t : dev->trainers) {
        if (!t->tensor_cores) continue;
        uint32_t flag = 0;
        cuda_check(cudaMemcpy(&flag, t->tc_error, sizeof(flag), cudaMemcpyDeviceToHost), "tensor-core error flag");
        require(flag == 0, MDN_ERR_TIMEOUT,
                "tensor-core minibatch kernel: a barrier wait gave up (flag " + std::to_string(flag) + ")");
    }
}
}  // namespace mdn

extern "C" int mdn_ppo_last_update_ms(mdn_ppo* t, float* ms) {
    return guarded([&] {
        checked(t);
        sync_event(t->sim->dev, t->ev_stop, "event sync");
        cuda_check(cudaEventElapsedTime(&t->last_update_ms, t->ev_start, t->ev_stop), "elapsed");
        if (ms) *ms = t->last_update_ms;
    });
}

extern "C" int mdn_ppo_metrics(mdn_ppo* t, float out[4]) {
    return guarded([&] {
        checked(t);
        require(out != nullptr, MDN_ERR_INVALID, "null out");
        cuda_check(cudaMemcpyAsync(out, t->args.metric_mean, 16, cudaMemcpyDeviceToHost, t->sim->stream), "metrics");
        sync_stream(t->sim->dev, t->sim->stream, "metrics");
    });
}

extern "C" int mdn_ppo_state(mdn_ppo* t, uint64_t* optimizer_step, uint32_t* completed_rollouts) {
    return guarded([&] {
        checked(t);
        if (optimizer_step) *optimizer_step = t->optimizer_step;
        if (completed_rollouts) *completed_rollouts = t->completed_rollouts;
    });
}

extern "C" int mdn_ppo_set_state(mdn_ppo* t, uint64_t optimizer_step, uint32_t completed_rollouts) {
    return guarded([&] {
        checked(t);
        t->optimizer_step = optimizer_step;
        t->completed_rollouts = completed_rollouts;
    });
}

extern "C" int mdn_ppo_moments(mdn_ppo* t, int which, float* host, size_t count, int upload) {
    return guarded([&] {
        checked(t);
        require(which >= 0 && which < 4 && host, MDN_ERR_INVALID, "moments: bad argument");
        float* d = which == 0 ? t->args.actor_m : which == 1 ? t->args.actor_v : which == 2 ? t->args.critic_m : t->args.critic_v;
        const size_t n = which < 2 ? size_t(t->sim->actor_params) : size_t(t->sim->critic_params);
        require(count == n, MDN_ERR_INVALID, "moments: count mismatch");
        cuda_check(upload ? cudaMemcpyAsync(d, host, n * 4, cudaMemcpyHostToDevice, t->sim->stream)
                          : cudaMemcpyAsync(host, d, n * 4, cudaMemcpyDeviceToHost, t->sim->stream),
                   "moments");
        sync_stream(t->sim->dev, t->sim->stream, "moments");
    });
}

extern "C" int mdn_ppo_grad_norms(mdn_ppo* t, float* host_rows, size_t count) {
    return guarded([&] {
        checked(t);
        require(host_rows && count == size_t(t->updates) * 2, MDN_ERR_INVALID, "grad norms: count must be 2*updates");
        cuda_check(cudaMemcpyAsync(host_rows, t->args.grad_norms, count * 4, cudaMemcpyDeviceToHost, t->sim->stream),
                   "grad norms");
        sync_stream(t->sim->dev, t->sim->stream, "grad norms");
    });
}

// ------------------------------------------------------------ checkpoints
namespace {
template <class T>
void download(void* dst, const T* src, size_t bytes, cudaStream_t s) {
    cuda_check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s), "checkpoint download");
}
}  // namespace

// read_checkpoint_header (main.mm:993-1000): the 136-byte header of any
// version 3..10, with the fields older versions lack filled as the reference
// fills them.
void mdn::read_checkpoint_header(std::ifstream& f, mdn_checkpoint_header& h) {
    std::memset(&h, 0, sizeof(h));
    f.read(reinterpret_cast<char*>(&h), 48);
    require(bool(f) && std::memcmp(h.magic, "PPOFIX1", 7) == 0 && h.version >= 3 && h.version <= 10, MDN_ERR_IO,
            "checkpoint prefix/version");
    f.read(reinterpret_cast<char*>(&h.config), 64);
    if (h.version >= 4) {
        f.read(reinterpret_cast<char*>(&h) + 112, 16);
        if (h.version >= 6) f.read(reinterpret_cast<char*>(&h) + 128, 8);
        else h.config.geometry_memory = 0;
        if (h.version == 4) h.config.velocity_contract = 0;
    } else {
        h.config.risk_coef = 0;
        h.config.entropy_coef = h.family == 7 ? .002f : .005f;
        h.config.learning_rate = .0003f;
        h.config.velocity_contract = 0;
        h.config.geometry_memory = 0;
    }
    require(bool(f), MDN_ERR_IO, "checkpoint header truncated");
}

// PPOTrainer::save_checkpoint (main.mm:1287-1320): header, actor, critic, Adam
// moments, the simulator state, and from version 8 (runtime config or tasks
// on) the runtime and task configuration, each env's episode plant and task
// state, the nominal plant and the RAPTOR controller.
extern "C" int mdn_ppo_checkpoint_save(mdn_ppo* t, const char* path, uint32_t family, uint32_t seed,
                                       uint32_t completed_rollouts) {
    return guarded([&] {
        checked(t);
        require(path != nullptr, MDN_ERR_INVALID, "null path");
        require(t->sim->dev->world == 1, MDN_ERR_INVALID, "checkpoint save: gather sharded state with world == 1");
        require(!t->sim->layered, MDN_ERR_INVALID,
                "checkpoint save: PPOFIX1 holds the one-hidden-layer tanh networks, not layered ones");
        mdn_sim* sim = t->sim;
        const std::filesystem::path p(path);
        if (p.has_parent_path()) std::filesystem::create_directories(p.parent_path());
        mdn_checkpoint_header h;
        std::memset(&h, 0, sizeof(h));
        std::memcpy(h.magic, "PPOFIX1", 7);
        const bool extended = sim->runtime.enabled || sim->task_ctl.enabled;
        h.version = extended ? 8 : 6;
        h.actor_count = sim->actor_params;
        h.critic_count = kCriticParams;
        h.horizon = sim->horizon;
        h.n = sim->n;
        h.family = family;
        h.base_seed = seed;
        h.completed_rollouts = completed_rollouts;
        h.optimizer_step = t->optimizer_step;
        h.config = sim->cfg;
        h.config.tick = 0;
        std::vector<char> blob;
        auto append_device = [&](const void* dptr, size_t bytes) {
            const size_t o = blob.size();
            blob.resize(o + bytes);
            download(blob.data() + o, dptr, bytes, sim->stream);
        };
        blob.resize(sizeof(h));
        std::memcpy(blob.data(), &h, sizeof(h));
        append_device(sim->buf[MDN_BUF_ACTOR], size_t(sim->actor_params) * 4);
        append_device(sim->buf[MDN_BUF_CRITIC], kCriticParams * 4);
        append_device(t->args.actor_m, size_t(sim->actor_params) * 4);
        append_device(t->args.actor_v, size_t(sim->actor_params) * 4);
        append_device(t->args.critic_m, kCriticParams * 4);
        append_device(t->args.critic_v, kCriticParams * 4);
        for (int id : {MDN_BUF_STATES, MDN_BUF_RUNS, MDN_BUF_WORLDS, MDN_BUF_SENSORS, MDN_BUF_POSES, MDN_BUF_COMMANDS})
            append_device(sim->buf[id], sim->bytes[id]);
        if (extended) {
            auto append_host = [&](const void* p, size_t bytes) {
                const size_t o = blob.size();
                blob.resize(o + bytes);
                std::memcpy(blob.data() + o, p, bytes);
            };
            append_host(&sim->runtime, sizeof(sim->runtime));
            append_host(&sim->task_ctl, sizeof(sim->task_ctl));
            if (sim->bytes[MDN_BUF_ENV_PHYSICS]) {
                append_device(sim->buf[MDN_BUF_ENV_PHYSICS], sim->bytes[MDN_BUF_ENV_PHYSICS]);
            } else {  // runtime config never on: every env flies the nominal plant (sim.metal:62,69)
                cuda_check(cudaStreamSynchronize(sim->stream), "checkpoint download");
                mdn_physics_params nominal;
                download(&nominal, sim->buf[MDN_BUF_PHYSICS], sizeof(nominal), sim->stream);
                cuda_check(cudaStreamSynchronize(sim->stream), "checkpoint download");
                for (uint32_t e = 0; e < sim->n; e++) append_host(&nominal, sizeof(nominal));
            }
            append_device(sim->buf[MDN_BUF_TASK_STATES], sim->bytes[MDN_BUF_TASK_STATES]);
            append_device(sim->buf[MDN_BUF_PHYSICS], sizeof(mdn_physics_params));
            append_device(sim->buf[MDN_BUF_RAPTOR], sizeof(mdn_raptor_weights));
        }
        cuda_check(cudaStreamSynchronize(sim->stream), "checkpoint download");
        const std::string tmp = std::string(path) + ".tmp";
        {
            std::ofstream f(tmp, std::ios::binary | std::ios::trunc);
            require(bool(f), MDN_ERR_IO, "cannot write PPO checkpoint: " + tmp);
            f.write(blob.data(), std::streamsize(blob.size()));
            f.flush();
            require(bool(f), MDN_ERR_IO, "PPO checkpoint write failed: " + tmp);
        }
        require(std::rename(tmp.c_str(), path) == 0, MDN_ERR_IO, std::string("cannot replace PPO checkpoint: ") + path);
    });
}

// PPOTrainer::load_checkpoint (main.mm:1209-1286) for versions 3..8. Versions
// 7-8 carry the runtime and task configuration, which must equal the
// simulator's byte for byte (configure it first; mdn_checkpoint_inspect reads
// them). Versions 9-10 (geodesic reward shaping, calibrated camera) are
// rejected: this build implements neither.
extern "C" int mdn_ppo_checkpoint_load(mdn_ppo* t, const char* path, uint32_t family, uint32_t horizon, uint32_t n,
                                       uint32_t seed) {
    return guarded([&] {
        checked(t);
        require(path != nullptr, MDN_ERR_INVALID, "null path");
        mdn_sim* sim = t->sim;
        require(!sim->layered, MDN_ERR_INVALID,
                "checkpoint load: PPOFIX1 holds the one-hidden-layer tanh networks, not layered ones");
        std::ifstream f(path, std::ios::binary);
        require(bool(f), MDN_ERR_IO, std::string("cannot open checkpoint ") + path);
        mdn_checkpoint_header h;
        read_checkpoint_header(f, h);
        require(h.version <= 8, MDN_ERR_MISMATCH,
                "checkpoint version 9+ carries reward-shaping or calibrated-camera state this build does not implement");
        require(h.actor_count == sim->actor_params && h.critic_count == kCriticParams, MDN_ERR_MISMATCH,
                "PPO checkpoint dimensions mismatch");
        require(h.family == family && h.horizon == horizon && h.n == n && h.base_seed == seed, MDN_ERR_MISMATCH,
                "PPO checkpoint config mismatch");
        require(horizon == sim->horizon && n == sim->n, MDN_ERR_MISMATCH, "PPO checkpoint does not fit this simulator");
        const mdn_sim_config& c = sim->cfg;
        require(h.config.family == c.family && h.config.n == c.n && h.config.substeps == c.substeps &&
                    h.config.sensor_period == c.sensor_period && h.config.sensor_delay == c.sensor_delay &&
                    h.config.command_delay == c.command_delay && h.config.max_steps == c.max_steps &&
                    h.config.mode == c.mode && h.config.speed == c.speed && h.config.distance == c.distance &&
                    h.config.wind == c.wind && h.config.depth_noise == c.depth_noise && h.config.dropout == c.dropout &&
                    h.config.risk_coef == c.risk_coef && h.config.entropy_coef == c.entropy_coef &&
                    h.config.learning_rate == c.learning_rate && h.config.velocity_contract == c.velocity_contract &&
                    h.config.geometry_memory == c.geometry_memory,
                MDN_ERR_MISMATCH, "PPO checkpoint simulator settings mismatch");
        std::vector<char> tmp;
        auto read_to_device = [&](void* dptr, size_t bytes) {
            tmp.resize(bytes);
            f.read(tmp.data(), std::streamsize(bytes));
            require(bool(f), MDN_ERR_IO, "truncated PPO checkpoint");
            cuda_check(cudaMemcpyAsync(dptr, tmp.data(), bytes, cudaMemcpyHostToDevice, sim->stream), "checkpoint upload");
            cuda_check(cudaStreamSynchronize(sim->stream), "checkpoint upload");
        };
        read_to_device(sim->buf[MDN_BUF_ACTOR], size_t(sim->actor_params) * 4);
        read_to_device(sim->buf[MDN_BUF_CRITIC], kCriticParams * 4);
        read_to_device(t->args.actor_m, size_t(sim->actor_params) * 4);
        read_to_device(t->args.actor_v, size_t(sim->actor_params) * 4);
        read_to_device(t->args.critic_m, kCriticParams * 4);
        read_to_device(t->args.critic_v, kCriticParams * 4);
        for (int id : {MDN_BUF_STATES, MDN_BUF_RUNS, MDN_BUF_WORLDS, MDN_BUF_SENSORS}) read_to_device(sim->buf[id], sim->bytes[id]);
        if (h.version >= 6) read_to_device(sim->buf[MDN_BUF_POSES], sim->bytes[MDN_BUF_POSES]);
        else cuda_check(cudaMemsetAsync(sim->buf[MDN_BUF_POSES], 0, sim->bytes[MDN_BUF_POSES], sim->stream), "poses");
        read_to_device(sim->buf[MDN_BUF_COMMANDS], sim->bytes[MDN_BUF_COMMANDS]);
        if (h.version >= 7) {
            mdn_runtime_config saved_runtime{};
            mdn_task_control saved_tasks{};
            f.read(reinterpret_cast<char*>(&saved_runtime), sizeof(saved_runtime));
            f.read(reinterpret_cast<char*>(&saved_tasks), h.version >= 8 ? sizeof(saved_tasks) : 144);
            require(h.version >= 8 || saved_tasks.enabled == 0, MDN_ERR_MISMATCH,
                    "task-generator semantics changed; use an explicit parameter warmstart from version7");
            require(bool(f), MDN_ERR_IO, "truncated navigation runtime configuration");
            require(std::memcmp(&saved_runtime, &sim->runtime, sizeof(saved_runtime)) == 0 &&
                        std::memcmp(&saved_tasks, &sim->task_ctl, sizeof(saved_tasks)) == 0,
                    MDN_ERR_MISMATCH, "checkpoint dynamics/task configuration mismatch");
            const size_t plants = size_t(sim->n) * sizeof(mdn_physics_params);
            if (sim->bytes[MDN_BUF_ENV_PHYSICS]) {
                read_to_device(sim->buf[MDN_BUF_ENV_PHYSICS], plants);
            } else {  // runtime config off: the stored plants are the nominal one, unused
                tmp.resize(plants);
                f.read(tmp.data(), std::streamsize(plants));
                require(bool(f), MDN_ERR_IO, "truncated PPO simulator checkpoint");
            }
            read_to_device(sim->buf[MDN_BUF_TASK_STATES], sim->bytes[MDN_BUF_TASK_STATES]);
            mdn_physics_params saved_nominal{}, nominal{};
            mdn_raptor_weights saved_raptor{};
            f.read(reinterpret_cast<char*>(&saved_nominal), sizeof(saved_nominal));
            f.read(reinterpret_cast<char*>(&saved_raptor), sizeof(saved_raptor));
            require(bool(f), MDN_ERR_IO, "truncated checkpoint nominal plant/controller");
            std::vector<mdn_raptor_weights> raptor(1);
            download(&nominal, sim->buf[MDN_BUF_PHYSICS], sizeof(nominal), sim->stream);
            download(raptor.data(), sim->buf[MDN_BUF_RAPTOR], sizeof(mdn_raptor_weights), sim->stream);
            cuda_check(cudaStreamSynchronize(sim->stream), "checkpoint compare");
            require(std::memcmp(&saved_nominal, &nominal, sizeof(nominal)) == 0 &&
                        std::memcmp(&saved_raptor, raptor.data(), sizeof(saved_raptor)) == 0,
                    MDN_ERR_MISMATCH, "checkpoint nominal plant/controller mismatch");
        } else {
            require(sim->runtime.enabled == 0 && sim->task_ctl.enabled == 0, MDN_ERR_MISMATCH,
                    "legacy resume cannot infer new dynamics/task state; use explicit parameter warmstart");
        }
        refresh_world_mirror(sim);
        char extra;
        require(!f.read(&extra, 1), MDN_ERR_IO, "PPO checkpoint has trailing data");
        require(h.optimizer_step <= uint64_t(UINT32_MAX), MDN_ERR_MISMATCH, "PPO checkpoint Adam step is too large");
        mdn_sim_config next = h.config;
        next.tick = 0;
        sim->cfg = next;
        sim->release_graphs();
        t->args.entropy_coef = next.entropy_coef;
        t->args.learning_rate = next.learning_rate;
        if (t->graph) {
            cudaGraphExecDestroy(t->graph);
            t->graph = nullptr;
        }
        t->optimizer_step = h.optimizer_step;
        t->completed_rollouts = h.completed_rollouts;
        cuda_check(cudaStreamSynchronize(sim->stream), "checkpoint load");
    });
}

// The header and the version 7-8 runtime/task blocks of a checkpoint, read
// on the host (main.mm:993-1000, 1238-1240).
extern "C" int mdn_checkpoint_inspect(const char* path, mdn_checkpoint_header* header, mdn_runtime_config* runtime,
                                      mdn_task_control* tasks) {
    return guarded([&] {
        require(path != nullptr, MDN_ERR_INVALID, "null path");
        std::ifstream f(path, std::ios::binary);
        require(bool(f), MDN_ERR_IO, std::string("cannot open checkpoint ") + path);
        mdn_checkpoint_header h;
        read_checkpoint_header(f, h);
        if (header) *header = h;
        mdn_runtime_config rt{};
        mdn_task_control tc{};
        if (h.version >= 7) {
            const uint64_t n = h.n;
            const uint64_t skip = (uint64_t(h.actor_count) * 3 + uint64_t(h.critic_count) * 3) * 4 +
                                  n * (sizeof(mdn_physics_state) + sizeof(mdn_sim_run) + sizeof(mdn_world) +
                                       uint64_t(kFrames) * kPixels * 4 + uint64_t(kFrames) * 12 * 4 +
                                       uint64_t(kFrames) * kActions * 4);
            f.seekg(std::streamoff(skip), std::ios::cur);
            f.read(reinterpret_cast<char*>(&rt), sizeof(rt));
            f.read(reinterpret_cast<char*>(&tc), h.version >= 8 ? sizeof(tc) : 144);
            require(bool(f), MDN_ERR_IO, "truncated navigation runtime configuration");
        }
        if (runtime) *runtime = rt;
        if (tasks) *tasks = tc;
    });
}

extern "C" int mdn_ppo_profile_minibatch(mdn_ppo* t, uint32_t update, float* ms) {
    return guarded([&] {
        checked(t);
        require(ms != nullptr && update < t->updates, MDN_ERR_INVALID, "profile minibatch: bad argument");
        require(t->graph != nullptr, MDN_ERR_STATE, "profile minibatch: run one rollout update first");
        require(!t->wide && !t->layered, MDN_ERR_INVALID,
                "profile minibatch: the 64-unit actor's minibatch kernels only");
        mdn_sim* sim = t->sim;
        cudaStream_t s = sim->stream;
        const bool multi = sim->dev->world > 1;
        cudaEvent_t e0, e1;
        cuda_check(cudaEventCreate(&e0), "event");
        cuda_check(cudaEventCreate(&e1), "event");
        cuda_check(cudaEventRecord(e0, s), "event");
        if (t->tensor_cores) {
            PpoArgs pt = t->args;
            pt.fwd_grid = multi ? std::max<uint32_t>(t->tc_grid, 2) : t->tc_grid;
            cuda_check(launch_minibatch_tc(pt, t->tc_maps, update, pt.fwd_grid, s), "tensor-core minibatch");
        } else {
            const uint32_t chunks = multi ? std::max<uint32_t>(t->grad_chunks, 2) : t->grad_chunks;
            cuda_check(launch_minibatch(t->args, update, chunks, s), "minibatch");
        }
        cuda_check(cudaEventRecord(e1, s), "event");
        cuda_check(cudaEventSynchronize(e1), "event");
        cuda_check(cudaEventElapsedTime(ms, e0, e1), "event");
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    });
}

extern "C" int mdn_launch_counts(mdn_sim* sim, mdn_ppo* t, uint32_t* per_policy_step, uint32_t* per_update) {
    return guarded([&] {
        if (per_policy_step) {
            require(sim != nullptr, MDN_ERR_INVALID, "launch counts: null simulator");
            *per_policy_step = uint32_t(kernels_per_step(sim->cfg, sim->wide != nullptr));
        }
        if (per_update) {
            require(t != nullptr, MDN_ERR_INVALID, "launch counts: null trainer");
            require(t->graph != nullptr, MDN_ERR_STATE, "launch counts: run one rollout update first");
            *per_update = t->launches;
        }
        (void)sim;
    });
}
