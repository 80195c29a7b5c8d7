"""Deployment export (NAVPOL1 / NAVWID4) against the reference's own readers and
writer (deployment.hpp, navigation_wide_deployment.hpp compiled unmodified into
oracle/_ref/libref_deploy.so).

CPU: libmdn's host writer (mdn_policy_write) produces the byte-identical NAVPOL1
file that NavigationPolicy::write_file writes for the same weights; the wide
NAVWID4 file loads in WideNavigationPolicy and evaluates to the oracle's forward.
GPU: a simulator's actor exported after a PPO update loads back exactly.
"""
import ctypes

import numpy as np
import pytest

from conftest import load_oracle_module, load_package


@pytest.fixture(scope="module")
def dlib():
    lib = load_oracle_module().load_ref_deploy()
    if lib is None:
        pytest.skip("oracle/_ref/libref_deploy.so not built: the reference sources are not on this machine")
    return lib


@pytest.fixture
def source(tmp_path):
    p = tmp_path / "checkpoint.bin"
    p.write_bytes(bytes(range(256)) * 37 + b"PPOFIX1")
    return p


def fnv1a64(data):
    h = 14695981039346656037
    for b in data:
        h ^= b
        h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def test_navpol1_byte_identical(dlib, olib, tmp_path, source):
    om = load_oracle_module()
    pkg = load_package()
    actor = np.zeros(olib.o_wide_param_count(64), np.float32)
    critic = np.zeros(olib.o_critic_param_count(), np.float32)
    olib.o_wide_init(64, om.ptr(actor), om.ptr(critic))
    actor += np.random.default_rng(1).normal(0, 0.01, actor.size).astype(np.float32)
    ours, theirs = tmp_path / "ours.navpol", tmp_path / "ref.navpol"
    pkg.write_policy(ours, actor, 64, source, 1.75)
    assert dlib.refd_write_navpol(str(theirs).encode(), om.ptr(actor), 1.75, str(source).encode()) == 1
    assert ours.read_bytes() == theirs.read_bytes()
    w = np.zeros(12104, np.float32)
    h = ctypes.c_uint64()
    ms = ctypes.c_float()
    assert dlib.refd_load_navpol(str(ours).encode(), om.ptr(w), ctypes.byref(h), ctypes.byref(ms)) == 1
    assert np.array_equal(w, actor) and ms.value == np.float32(1.75)
    assert h.value == fnv1a64(source.read_bytes())


def test_navwid4_loads_and_evaluates(dlib, olib, tmp_path, source):
    om = load_oracle_module()
    pkg = load_package()
    hidden = 5120
    actor = np.zeros(olib.o_wide_param_count(hidden), np.float32)
    critic = np.zeros(olib.o_critic_param_count(), np.float32)
    olib.o_wide_init(hidden, om.ptr(actor), om.ptr(critic))
    actor[hidden * 184: hidden * 185] = np.random.default_rng(2).normal(0, 0.1, hidden).astype(np.float32)
    path = tmp_path / "wide.navwid"
    pkg.write_policy(path, actor, hidden, source, 1.5)
    rows = 3
    obs = np.random.default_rng(3).uniform(0, 1, (rows, 184)).astype(np.float32)
    mean = np.zeros((rows, 4), np.float32)
    vel = np.zeros((rows, 4), np.float32)
    h = ctypes.c_uint64()
    got = dlib.refd_wide_eval(str(path).encode(), om.ptr(obs), rows, om.ptr(mean), om.ptr(vel), ctypes.byref(h))
    assert got == hidden
    assert h.value == fnv1a64(source.read_bytes())
    for r in range(rows):
        hid = np.zeros(hidden, np.float32)
        m = np.zeros(4, np.float32)
        olib.o_wide_actor_forward(hidden, om.ptr(np.ascontiguousarray(obs[r])), om.ptr(actor), om.ptr(hid), om.ptr(m))
        assert np.array_equal(m, mean[r])  # same fp32 operation order as ppo.hpp:65-80


def test_export_rejects_bad_input(tmp_path, source):
    pkg = load_package()
    actor = np.full(12104, np.nan, np.float32)
    with pytest.raises(pkg.MdnError):
        pkg.write_policy(tmp_path / "x", actor, 64, source, 1.5)
    with pytest.raises(pkg.MdnError):
        pkg.write_policy(tmp_path / "y", np.zeros(12104, np.float32), 64, tmp_path / "missing", 1.5)
    assert not (tmp_path / "x").exists() and not (tmp_path / "y").exists()


@pytest.mark.gpu
@pytest.mark.parametrize("hidden", [64, 5120])
def test_export_after_update(dlib, tmp_path, source, hidden):
    om = load_oracle_module()
    pkg = load_package()
    dev = pkg.Device(0)
    cfg = pkg.layouts.default_config(n=256, family=17, seed=4)
    sim = pkg.Sim(dev, cfg, 4, actor_hidden=None if hidden == 64 else hidden)
    tr = pkg.PPOTrainer(sim, epochs=1, minibatch=512)
    try:
        sim.collect()
        tr.rollout_update(0)
        dev.finish()
        path = tmp_path / "policy.bin"
        sim.export_policy(path, source, 1.5)
        actor = sim.download("actor")
        if hidden == 64:
            w = np.zeros(12104, np.float32)
            h = ctypes.c_uint64()
            ms = ctypes.c_float()
            assert dlib.refd_load_navpol(str(path).encode(), om.ptr(w), ctypes.byref(h), ctypes.byref(ms)) == 1
            assert np.array_equal(w, actor)
        else:
            obs = sim.download("obs").reshape(-1, 184)[:2].copy()
            mean = np.zeros((2, 4), np.float32)
            vel = np.zeros((2, 4), np.float32)
            h = ctypes.c_uint64()
            assert dlib.refd_wide_eval(str(path).encode(), om.ptr(obs), 2, om.ptr(mean), om.ptr(vel),
                                       ctypes.byref(h)) == hidden
            assert np.all(np.isfinite(mean))
    finally:
        tr.close()
        sim.close()
        dev.close()


# ----------------------------------------------------- deployment probe
# The reference checks a deployed policy on eight probe observations
# (main.mm:1001-1042): NavigationPolicy::raw_mean of the exported file must
# equal the fixed PPO actor within 2e-5. Replayed here on the reference's own
# exported policy (tests/golden/ref_navpol_rooms.bin, trained weights).
PROBE_GATE = 2e-5


def probe_observation(sample):
    """deployment_probe_observation (main.mm:1001-1015)."""
    obs = np.zeros(184, np.float32)
    for i in range(160):
        obs[i] = np.float32(0.20) + np.float32(0.01) * np.float32((i * 13 + sample * 7) % 70)
    c = 160
    angle = np.float32(-0.7) + np.float32(0.2) * np.float32(sample)
    obs[c + 0] = np.cos(angle)
    obs[c + 1] = np.sin(angle)
    obs[c + 2] = 0.1
    obs[c + 3] = np.float32(0.3) + np.float32(0.04) * np.float32(sample)
    obs[c + 4:c + 21] = (0.1, -0.05, 0.02, 0.01, -0.02, 0.03, 0.0, 0.0, 1.0, 0.05, -0.03, 0.0, 0.02, 0.01, 0.02,
                         -0.01, 0.0)
    obs[181:184] = (0.08, -0.04, 0.02)
    return obs


def golden_policy():
    from conftest import GOLDEN
    path = GOLDEN / "ref_navpol_rooms.bin"
    raw = path.read_bytes()
    assert raw[:8] == b"NAVPOL1\x00"
    header = np.frombuffer(raw, "<u4", 6, 8)
    assert tuple(header) == (1, 184, 64, 4, 17, 12104)
    return path, np.frombuffer(raw, np.float32, 12104, 64).copy()


def f64_means(actor, obs):
    w1 = actor[:64 * 184].reshape(64, 184).astype(np.float64)
    b1 = actor[64 * 184:64 * 185].astype(np.float64)
    w2 = actor[64 * 185:64 * 189].reshape(4, 64).astype(np.float64)
    b2 = actor[64 * 189:64 * 189 + 4].astype(np.float64)
    m = np.tanh(obs.astype(np.float64) @ w1.T + b1) @ w2.T + b2
    m[:, :3] += obs[:, 181:184]
    return m


def test_reference_policy_probe_cpu(dlib):
    """The reference's reader on its own exported policy against a float64
    forward of the same weights (the probe's own gate)."""
    path, actor = golden_policy()
    obs = np.stack([probe_observation(s) for s in range(8)])
    got = np.zeros((8, 4), np.float32)
    assert dlib.refd_navpol_eval(str(path).encode(), obs.ctypes.data_as(ctypes.c_void_p), 8,
                                 got.ctypes.data_as(ctypes.c_void_p)) == 1
    assert np.max(np.abs(got - f64_means(actor, obs))) < PROBE_GATE


@pytest.mark.gpu
def test_reference_policy_probe_gpu():
    """The reference's trained policy uploaded into a simulator, evaluated on
    the GPU (mdn_sim_actor_means) on the probe observations: within the
    probe's 2e-5 of the float64 forward and of the reference's own reader."""
    pkg = load_package()
    path, actor = golden_policy()
    obs = np.stack([probe_observation(s) for s in range(8)])
    dev = pkg.Device(0)
    sim = pkg.Sim(dev, pkg.layouts.default_config(n=16, family=1), 2)
    try:
        sim.upload("actor", actor)
        got = sim.actor_means(obs)
        assert np.max(np.abs(got - f64_means(actor, obs))) < PROBE_GATE
        lib = load_oracle_module().load_ref_deploy()
        if lib is not None:
            ref = np.zeros((8, 4), np.float32)
            assert lib.refd_navpol_eval(str(path).encode(), obs.ctypes.data_as(ctypes.c_void_p), 8,
                                        ref.ctypes.data_as(ctypes.c_void_p)) == 1
            assert np.max(np.abs(got - ref)) < PROBE_GATE
        # a trained actor also drives a rollout without non-finite values
        sim.collect()
        assert np.isfinite(sim.download("actions")).all()
    finally:
        sim.close()
        dev.close()
