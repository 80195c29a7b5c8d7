"""Wide actor (184 -> 5120 tanh -> 4, 967,688 parameters) on the B200, through the C-ABI.

The actor forward runs as tcgen05 TF32 matrix products with fp32 accumulation.
Tolerance (stated for the tensor-core path): |mean_gpu - mean_ref| <=
TF32_ABS + TF32_REL * |mean_ref| against a float64 evaluation of ppo.hpp:65-80
on the same observations and parameters (the oracle's fp32 forward agrees with
float64 to ~1e-6 here, far inside the bound).
"""
import numpy as np
import pytest

from conftest import load_oracle_module, load_package

HIDDEN = 5120
OBS = 184
TF32_ABS = 1e-3
TF32_REL = 2e-3

pytestmark = pytest.mark.gpu


def reference_mean(obs, actor, hidden=HIDDEN):
    w1 = actor[: hidden * OBS].reshape(hidden, OBS).astype(np.float64)
    b1 = actor[hidden * OBS: hidden * OBS + hidden].astype(np.float64)
    w2 = actor[hidden * OBS + hidden: hidden * OBS + 5 * hidden].reshape(4, hidden).astype(np.float64)
    b2 = actor[hidden * OBS + 5 * hidden: hidden * OBS + 5 * hidden + 4].astype(np.float64)
    mean = np.tanh(obs.astype(np.float64) @ w1.T + b1) @ w2.T + b2
    mean[:, :3] += obs[:, OBS - 3:]
    return mean


def make_sim(layouts, n, horizon, seed=5):
    pkg = load_package()
    dev = pkg.Device(0)
    cfg = layouts.default_config(n=n, family=17, seed=seed)
    sim = pkg.Sim(dev, cfg, horizon, actor_hidden=HIDDEN)
    return pkg, dev, sim


def quiet_actor(sim, rng):
    """Non-zero b1/b2 (to exercise the biases) and log_std = -30, so the sampled
    action equals the mean to ~1e-13."""
    actor = sim.download("actor")
    actor[HIDDEN * OBS: HIDDEN * OBS + HIDDEN] = rng.normal(0, 0.1, HIDDEN).astype(np.float32)
    actor[HIDDEN * OBS + 5 * HIDDEN: HIDDEN * OBS + 5 * HIDDEN + 4] = rng.normal(0, 0.1, 4).astype(np.float32)
    actor[-4:] = -30.0
    sim.upload("actor", actor)
    return actor


def test_wide_init_matches_oracle(layouts, olib):
    _, dev, sim = make_sim(layouts, 256, 2)
    try:
        om = load_oracle_module()
        actor = np.zeros(olib.o_wide_param_count(HIDDEN), np.float32)
        critic = np.zeros(olib.o_critic_param_count(), np.float32)
        olib.o_wide_init(HIDDEN, om.ptr(actor), om.ptr(critic))
        got = sim.download("actor")
        assert got.size == 967688
        assert np.array_equal(got, actor)
        assert np.array_equal(sim.download("critic"), critic)
    finally:
        sim.close()
        dev.close()


@pytest.mark.parametrize("n,tick", [(1024, 0), (1000, 1)])
def test_wide_actor_step_matches_reference(layouts, n, tick):
    """One policy step; n = 1000 at the last tick makes the final 128-row tile
    run past the observation tensor (zero-filled by the TMA unit)."""
    _, dev, sim = make_sim(layouts, n, 2)
    try:
        actor = quiet_actor(sim, np.random.default_rng(3))
        for t in range(tick + 1):
            sim.step(t)
        dev.finish()
        obs = sim.download("obs").reshape(2, n, OBS)[tick]
        act = sim.download("actions").reshape(2, n, 4)[tick]
        mean = reference_mean(obs, actor)
        err = np.abs(act - mean)
        assert np.all(np.isfinite(act))
        assert np.all(err <= TF32_ABS + TF32_REL * np.abs(mean)), float(err.max())
        # the small-actor fields are untouched by the wide path
        assert np.all(np.isfinite(sim.download("values").reshape(2, n)[tick]))
    finally:
        sim.close()
        dev.close()


def test_wide_actor_matches_oracle_fp32_rows(layouts, olib):
    """A few rows against the oracle's fp32 restatement (bit-pinned to ppo.hpp)."""
    om = load_oracle_module()
    n = 512
    _, dev, sim = make_sim(layouts, n, 1, seed=9)
    try:
        actor = quiet_actor(sim, np.random.default_rng(11))
        sim.step(0)
        dev.finish()
        obs = sim.download("obs").reshape(n, OBS)
        act = sim.download("actions").reshape(n, 4)
        for r in (0, 1, 127, 128, 511):
            h = np.zeros(HIDDEN, np.float32)
            m = np.zeros(4, np.float32)
            olib.o_wide_actor_forward(HIDDEN, om.ptr(np.ascontiguousarray(obs[r])), om.ptr(actor), om.ptr(h),
                                      om.ptr(m))
            assert np.all(np.abs(act[r] - m) <= TF32_ABS + TF32_REL * np.abs(m)), (r, act[r], m)
    finally:
        sim.close()
        dev.close()


def test_wide_rollout_graph(layouts):
    """collect() captures the wide forward into the rollout graph; the last
    tick's actions match the reference forward and the barrier flag stays clear."""
    n, horizon = 2048, 4
    _, dev, sim = make_sim(layouts, n, horizon, seed=21)
    try:
        actor = quiet_actor(sim, np.random.default_rng(5))
        sim.collect()
        sim.collect()
        dev.finish()  # raises on a wide-kernel barrier timeout
        obs = sim.download("obs").reshape(horizon, n, OBS)[horizon - 1]
        act = sim.download("actions").reshape(horizon, n, 4)[horizon - 1]
        mean = reference_mean(obs, actor)
        assert np.all(np.abs(act - mean) <= TF32_ABS + TF32_REL * np.abs(mean))
    finally:
        sim.close()
        dev.close()


# ---------------------------------------------------------------- PPO update
# One full-batch update (epochs = 1, minibatch = all rows): after Adam's first
# step the actor's first moment is 0.1 x the clipped gradient, which is
# compared with a float64 evaluation of the same gradient (loss derivatives
# from the oracle's sample_loss_and_grad, ppo.hpp:144-181; per-sample
# gradients summed as actor_backward_sample, ppo.hpp:269-287, sums them).
# Tolerance for the tensor-core parts (dW1, db1, dW2: TF32 products, fp32
# accumulation): relative L2 error <= GRAD_REL_L2 and per-element
# |m - m_ref| <= GRAD_ABS * max|m_ref|. b2 and log_std are fp32 sums of loss
# derivatives that depend on the TF32 means, scaled by the actor's global-norm
# clip (whose norm carries the TF32 error too): relative 5e-3 plus 1e-3 of the
# block's largest entry (log-std sums cancel). The critic is independent of the
# actor's precision: relative 1e-3.
GRAD_REL_L2 = 1e-2
GRAD_ABS = 1e-2


def expected_moments(olib, om, rollout, actor, critic, adv, ret, entropy_coef, hidden=HIDDEN):
    obs, co, act, logp, values = rollout
    rows = obs.shape[0]
    H = hidden
    w1 = actor[: H * OBS].reshape(H, OBS).astype(np.float64)
    b1 = actor[H * OBS: H * OBS + H].astype(np.float64)
    w2 = actor[H * OBS + H: H * OBS + 5 * H].reshape(4, H).astype(np.float64)
    b2 = actor[H * OBS + 5 * H: H * OBS + 5 * H + 4].astype(np.float64)
    log_std = actor[-4:].copy()
    hid = np.tanh(obs.astype(np.float64) @ w1.T + b1)
    mean = hid @ w2.T + b2
    mean[:, :3] += obs[:, OBS - 3:]
    mean32 = mean.astype(np.float32)
    cw1 = critic[: 64 * 32].reshape(64, 32).astype(np.float64)
    cb1 = critic[64 * 32: 64 * 33].astype(np.float64)
    cw2 = critic[64 * 33: 64 * 34].astype(np.float64)
    cb2 = float(critic[64 * 34])
    chid = np.tanh(co.astype(np.float64) @ cw1.T + cb1)
    value = (chid @ cw2 + cb2).astype(np.float32)
    dm = np.zeros((rows, 4), np.float32)
    dls = np.zeros((rows, 4), np.float32)
    dv = np.zeros(rows, np.float32)
    loss = np.zeros(4, np.float32)
    for r in range(rows):
        d_m = np.zeros(4, np.float32)
        d_l = np.zeros(4, np.float32)
        d_v = np.zeros(1, np.float32)
        olib.o_sample_loss_and_grad(om.ptr(np.ascontiguousarray(act[r])), om.ptr(np.ascontiguousarray(mean32[r])),
                                    om.ptr(log_std), float(logp[r]), float(value[r]), float(adv[r]),
                                    float(ret[r]), float(rows), 0.2, 0.5, float(entropy_coef), om.ptr(d_m),
                                    om.ptr(d_l), om.ptr(d_v), om.ptr(loss))
        dm[r], dls[r], dv[r] = d_m, d_l, d_v[0]
    dm64 = dm.astype(np.float64)
    delta = (dm64 @ w2) * (1.0 - hid * hid)
    g_w1 = delta.T @ obs.astype(np.float64)
    g_b1 = delta.sum(0)
    g_w2 = dm64.T @ hid
    g_actor = np.concatenate([g_w1.ravel(), g_b1, g_w2.ravel(), dm64.sum(0), dls.astype(np.float64).sum(0)])
    cdelta = np.outer(dv.astype(np.float64), cw2) * (1.0 - chid * chid)
    g_critic = np.concatenate([(cdelta.T @ co.astype(np.float64)).ravel(), cdelta.sum(0),
                               (dv.astype(np.float64)[:, None] * chid).sum(0), [dv.astype(np.float64).sum()]])
    out = []
    for g in (g_actor, g_critic):
        norm = np.sqrt(np.sum(g * g))
        scale = min(1.0, 0.5 / norm)
        out.append((0.1 * scale * g, norm))
    return out


def test_wide_ppo_update_gradient(layouts, olib):
    pkg = load_package()
    om = load_oracle_module()
    n, horizon = 256, 4
    dev = pkg.Device(0)
    cfg = layouts.default_config(n=n, family=17, seed=13)
    sim = pkg.Sim(dev, cfg, horizon, actor_hidden=HIDDEN)
    tr = pkg.PPOTrainer(sim, epochs=1, minibatch=n * horizon)
    try:
        actor = sim.download("actor")
        actor[HIDDEN * OBS: HIDDEN * OBS + HIDDEN] = np.random.default_rng(2).normal(0, 0.1, HIDDEN).astype(np.float32)
        sim.upload("actor", actor)
        critic = sim.download("critic")
        sim.collect()
        dev.finish()
        rows = n * horizon
        rollout = (sim.download("obs").reshape(rows, OBS), sim.download("co").reshape(rows, 32),
                   sim.download("actions").reshape(rows, 4), sim.download("logp"), sim.download("values"))
        tr.rollout_update(0)
        dev.finish()
        adv, ret = sim.download("advantages"), sim.download("returns")
        (m_actor_ref, norm_a), (m_critic_ref, norm_c) = expected_moments(
            olib, om, rollout, actor, critic, adv, ret, float(cfg["entropy_coef"]))
        m_actor = tr.moments(0).astype(np.float64)
        m_critic = tr.moments(2).astype(np.float64)
        norms = tr.grad_norms(1)[0]
        assert m_actor.size == 967688
        H = HIDDEN
        tc = slice(0, H * OBS + 5 * H)          # dW1, db1, dW2: tensor-core sums
        small = slice(H * OBS + 5 * H, None)    # b2, log_std
        rel = np.linalg.norm(m_actor[tc] - m_actor_ref[tc]) / np.linalg.norm(m_actor_ref[tc])
        assert rel <= GRAD_REL_L2, rel
        assert np.max(np.abs(m_actor[tc] - m_actor_ref[tc])) <= GRAD_ABS * np.max(np.abs(m_actor_ref[tc]))
        assert np.allclose(m_actor[small], m_actor_ref[small], rtol=5e-3, atol=1e-3 * np.max(np.abs(m_actor_ref[small])))
        assert np.allclose(m_critic, m_critic_ref, rtol=1e-3, atol=1e-4 * np.max(np.abs(m_critic_ref)))
        assert abs(norms[0] - norm_a) <= 1e-2 * norm_a
        assert abs(norms[1] - norm_c) <= 1e-4 * norm_c
        # Adam's first step moves every parameter by at most lr (plus rounding)
        after = sim.download("actor")
        lr = float(cfg["learning_rate"])
        assert np.all(np.isfinite(after))
        assert np.max(np.abs(after[:-4] - actor[:-4])) <= lr * 1.001
    finally:
        tr.close()
        sim.close()
        dev.close()


def test_wide_ppo_update_minibatches(layouts):
    """Several minibatches and epochs through the captured update graph: the
    update completes, parameters stay finite, the barrier flag stays clear, and
    a second rollout + update runs on the updated weights."""
    pkg = load_package()
    n, horizon = 1024, 8
    dev = pkg.Device(0)
    cfg = layouts.default_config(n=n, family=17, seed=17)
    sim = pkg.Sim(dev, cfg, horizon, actor_hidden=HIDDEN)
    tr = pkg.PPOTrainer(sim, epochs=2, minibatch=n * horizon // 4)
    try:
        before = sim.download("actor")
        for k in range(2):
            sim.collect()
            tr.rollout_update(k)
        dev.finish()
        after = sim.download("actor")
        assert np.all(np.isfinite(after)) and not np.array_equal(before, after)
        assert np.all(np.isfinite(tr.metric_mean))
        assert np.all(np.isfinite(tr.grad_norms(8)))
    finally:
        tr.close()
        sim.close()
        dev.close()
