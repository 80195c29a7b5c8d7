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
