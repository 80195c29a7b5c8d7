"""Wide actor (967,688 parameters: 184 -> 5120 tanh -> 4), CPU only.

Pins the oracle's width-generic restatement (o_wide_*) against the reference's
ppo.hpp operators compiled at FIXED_PPO_HIDDEN_DIM=5120 (oracle/_ref/libref_wide.so),
bit for bit, and checks the initialisation stream of main.mm:548-555 against
the 64-unit build at the shared prefix.
"""
import numpy as np
import pytest

from conftest import load_oracle_module

HIDDEN = 5120
OBS = 184


@pytest.fixture(scope="module")
def wlib():
    lib = load_oracle_module().load_ref_wide()
    if lib is None:
        pytest.skip("oracle/_ref/libref_wide.so not built: the reference sources are not on this machine")
    return lib


def wide_params(olib, hidden=HIDDEN):
    ptr = load_oracle_module().ptr
    actor = np.zeros(olib.o_wide_param_count(hidden), np.float32)
    critic = np.zeros(olib.o_critic_param_count(), np.float32)
    olib.o_wide_init(hidden, ptr(actor), ptr(critic))
    return actor, critic


def test_wide_param_count(olib, wlib):
    assert olib.o_wide_param_count(HIDDEN) == 967688 == wlib.refw_actor_param_count()
    assert wlib.refw_hidden() == HIDDEN
    assert olib.o_wide_param_count(64) == olib.o_actor_param_count()


def test_wide_init_matches_64_unit_stream(olib, oracle_mod, layouts, raptor):
    # With hidden = 64 the width-generic init must equal the simulator's own
    # (cpu_reference.hpp:89-103 == main.mm:548-555).
    a64, c64 = wide_params(olib, 64)
    cfg = layouts.default_config(n=4, family=1, seed=3)
    sim = oracle_mod.OracleSim(layouts, cfg, 2, raptor)
    assert np.array_equal(a64, sim.buf("actor"))
    assert np.array_equal(c64, sim.buf("critic"))
    # Wide: W1 draws are the first 5120*184 normals of the same stream, x 0.04.
    aw, _ = wide_params(olib, HIDDEN)
    assert np.array_equal(aw[: 64 * OBS], a64[: 64 * OBS])
    assert np.all(aw[HIDDEN * OBS: HIDDEN * OBS + HIDDEN] == 0.0)          # b1
    assert np.all(aw[-4:] == -1.0)                                          # log_std
    assert abs(float(np.std(aw[: HIDDEN * OBS])) - 0.04) < 1e-3


def test_wide_actor_forward_bitwise(olib, wlib):
    ptr = load_oracle_module().ptr
    actor, _ = wide_params(olib)
    rng = np.random.default_rng(7)
    actor[HIDDEN * OBS: HIDDEN * OBS + HIDDEN] = rng.normal(0, 0.1, HIDDEN).astype(np.float32)  # nonzero b1
    rows = 6
    obs = rng.uniform(-1, 1, (rows, OBS)).astype(np.float32)
    ref_h = np.zeros((rows, HIDDEN), np.float32)
    ref_m = np.zeros((rows, 4), np.float32)
    wlib.refw_actor_forward(ptr(obs), ptr(actor), rows, ptr(ref_h), ptr(ref_m))
    for r in range(rows):
        h = np.zeros(HIDDEN, np.float32)
        m = np.zeros(4, np.float32)
        olib.o_wide_actor_forward(HIDDEN, ptr(obs[r]), ptr(actor), ptr(h), ptr(m))
        assert np.array_equal(h, ref_h[r]) and np.array_equal(m, ref_m[r])
    # and against float64 arithmetic
    w1 = actor[: HIDDEN * OBS].reshape(HIDDEN, OBS).astype(np.float64)
    b1 = actor[HIDDEN * OBS: HIDDEN * OBS + HIDDEN].astype(np.float64)
    w2 = actor[HIDDEN * OBS + HIDDEN: HIDDEN * OBS + 5 * HIDDEN].reshape(4, HIDDEN).astype(np.float64)
    hid = np.tanh(obs.astype(np.float64) @ w1.T + b1)
    mean = hid @ w2.T
    mean[:, :3] += obs[:, OBS - 3:]
    assert np.max(np.abs(mean - ref_m)) < 1e-5
