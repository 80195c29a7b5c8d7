"""Per-episode plant variation on the GPU (NavigationRuntimeConfig,
sim_reset_one sim.metal:62-82, sim_advance :287) against the CPU oracle.

Every episode reset draws the env's plant from its own seed; the drawn plants
(MDN_BUF_ENV_PHYSICS) and the per-rotor hover RPMs are compared bit for bit,
at reset and after the resets inside a teacher-forced rollout; the integrated
state within RTOL/ATOL = 1e-5 per step, flags and counters bitwise. Then the
navigation_training::configure / validate_rollout contract.
"""
import numpy as np
import pytest

from conftest import load_oracle_module, load_package

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-5
STATE_KEYS = ("states", "runs", "worlds", "sensors", "poses", "commands", "task_states", "env_physics")


def close(a, b, what):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    bad = ~(np.abs(a - b) <= ATOL + RTOL * np.abs(b))
    bad &= ~(np.isnan(a) & np.isnan(b))
    assert not bad.any(), f"{what}: {bad.sum()} differ; worst {np.nanmax(np.abs(a - b)):.3e}"


def floats(structured):
    return np.frombuffer(np.ascontiguousarray(structured).tobytes(), np.float32)


CASES = [
    dict(amplitude=1.0, cfg=dict(family=1, max_steps=5, wind=0.4), strict=False),
    dict(amplitude=0.4, cfg=dict(family=17, max_steps=4, sensor_delay=1, command_delay=1), strict=False),
    dict(amplitude=1.0, cfg=dict(family=3, max_steps=6), strict=True),  # some draws rejected: NaN-mass plants
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_domain_steps_match_oracle(case):
    pkg, om = load_package(), load_oracle_module()
    L = pkg.layouts
    raptor = pkg.default_raptor()
    dev = pkg.Device(0)
    c = CASES[case]
    n, T = 256, 10
    cfg = L.default_config(**{**dict(n=n, speed=1.0, distance=3.0, seed=17 + case), **c["cfg"]})
    rt = pkg.runtime_config(c["amplitude"])
    if c["strict"]:
        rt["domain_range"]["minimum_thrust_to_weight"] = 1.46  # near the median draw at amplitude 1
    gpu = pkg.Sim(dev, cfg, T, raptor=raptor)
    ora = om.OracleSim(L, cfg, T, raptor)
    try:
        gpu.set_runtime(rt)
        gpu.reset()
        ora.set_runtime(rt)
        ora.reset()
        plants = gpu.download("env_physics")
        assert plants.tobytes() == ora.buf("env_physics").tobytes(), "reset plants"
        assert gpu.download("states").tobytes() == ora.buf("states").tobytes(), "reset states (hover rpm)"
        masses = plants["mass"]
        if c["strict"]:
            assert np.isnan(masses).any() and np.isfinite(masses).any()
        else:
            assert np.isfinite(masses).all() and np.unique(masses).size > n // 2
        for t in range(T):
            for name in STATE_KEYS:
                gpu.upload(name, ora.buf(name))
            gpu.step(t)
            ora.step(t)
            rows = slice(t * n, (t + 1) * n)
            for name in ("terminated", "truncated", "contact_id"):
                assert np.array_equal(gpu.download(name)[rows], ora.buf(name)[rows]), f"t={t} {name}"
            close(gpu.download("rewards")[rows], ora.buf("rewards")[rows], f"t={t} rewards")
            rs_g, rs_o = gpu.download("runs"), ora.buf("runs")
            for f in ("steps", "episodes", "collisions", "rng"):
                assert np.array_equal(rs_g[f], rs_o[f]), f"t={t} runs.{f}"
            assert gpu.download("env_physics").tobytes() == ora.buf("env_physics").tobytes(), f"t={t} plants"
            close(floats(gpu.download("states")), floats(ora.buf("states")), f"t={t} states")
        assert ora.buf("runs")["episodes"].sum() > n // 4  # resets drew fresh plants
    finally:
        gpu.close()
        dev.close()


def test_zero_amplitude_runtime_is_nominal():
    """runtime.enabled with amplitude 0 integrates exactly the nominal plant."""
    pkg = load_package()
    L = pkg.layouts
    dev = pkg.Device(0)
    cfg = L.default_config(n=512, family=2, seed=8, speed=1.0, max_steps=7, wind=0.3)
    a, b = pkg.Sim(dev, cfg, 8), pkg.Sim(dev, cfg, 8)
    try:
        b.set_runtime(pkg.runtime_config(0.0))
        b.reset()
        a.collect()
        b.collect()
        for name in ("states", "runs", "worlds", "obs", "rewards", "terminated", "truncated"):
            assert a.download(name).tobytes() == b.download(name).tobytes(), name
        nominal = a.download("physics")
        assert b.download("env_physics").tobytes() == nominal.tobytes() * 512
    finally:
        a.close()
        b.close()
        dev.close()


def test_configure_and_validate():
    """navigation_training::configure / validate_rollout (navigation_training.hpp:16-35)."""
    pkg = load_package()
    L = pkg.layouts
    dev = pkg.Device(0)
    cfg = L.default_config(n=128, family=1, mode=22, speed=1.5, distance=8.0, seed=3, max_steps=400)
    sim = pkg.Sim(dev, cfg, 4)
    try:
        control = pkg.task_control(2, 1)
        sim.configure_tasks(control, domain_amplitude=0.7)
        plants = sim.download("env_physics")
        assert np.isfinite(plants["mass"]).all() and np.unique(plants["mass"]).size > 64
        if (sim.download("task_states")["generation_status"] == 4).all():
            sim.validate_tasks()
        rt = pkg.runtime_config(1.0)
        rt["domain_range"]["minimum_thrust_to_weight"] = 50.0  # every draw rejected
        sim.set_runtime(rt)
        sim.reset()
        assert np.isnan(sim.download("env_physics")["mass"]).all()
        with pytest.raises(pkg.MdnError, match="task generation rejected|episode dynamics sample rejected"):
            sim.validate_tasks()
        sim.collect()  # NaN plants integrate to invalid states and end their episodes as collisions
        assert sim.download("terminated").any()
        # A frozen bank and the task generator cannot both own the world.
        bank_path = pkg.PACKAGE_DIR.parent / "tests" / "golden" / "challenge_bank_small.jsonl"
        import json
        h = json.loads(bank_path.read_text().splitlines()[0])["world_source_sha256"]
        sim.set_challenge_bank(pkg.ChallengeBank(bank_path, "train", h).worlds())
        with pytest.raises(pkg.MdnError, match="frozen bank"):
            sim.configure_tasks(control)
    finally:
        sim.close()
        dev.close()


def test_checkpoint_v8_roundtrip(tmp_path):
    """PPOFIX1 version 8 (main.mm:1287-1320): runtime + task blocks, per-env
    plants and task states; resume continues bit-identically."""
    pkg = load_package()
    L = pkg.layouts
    dev = pkg.Device(0)
    cfg = L.default_config(n=128, family=1, mode=22, speed=1.5, distance=8.0, seed=3, max_steps=400)
    T = 8
    control = pkg.task_control(2, 1)
    control["config"]["max_nav_steps"] = 5  # resets (fresh plants) inside every rollout
    sim, sim2 = pkg.Sim(dev, cfg, T), pkg.Sim(dev, cfg, T)
    tr, tr2 = pkg.PPOTrainer(sim, epochs=1), pkg.PPOTrainer(sim2, epochs=1)
    path = tmp_path / "v8.bin"
    try:
        sim.configure_tasks(control, 0.6)
        sim.collect()
        tr.rollout_update(0)
        tr.save_checkpoint(path, 1, 3, 1)
        h, rt, tc = pkg.checkpoint_inspect(path)
        assert int(h["version"]) == 8
        assert rt.tobytes() == pkg.runtime_config(0.6).tobytes()
        assert tc.tobytes() == np.array(control, L.TASK_CONTROL).tobytes()
        with pytest.raises(pkg.MdnError, match="dynamics/task configuration mismatch|legacy resume"):
            tr2.load_checkpoint(path, 1, T, 128, 3)
        sim2.configure_tasks(control, 0.6)
        tr2.load_checkpoint(path, 1, T, 128, 3)
        for k in ("actor", "critic", "states", "runs", "worlds", "sensors", "commands", "task_states", "env_physics"):
            assert sim2.download(k).tobytes() == sim.download(k).tobytes(), k
        sim.collect()
        tr.rollout_update(1)
        sim2.collect()
        tr2.rollout_update(1)
        for k in ("actor", "env_physics", "task_states", "states"):
            assert sim2.download(k).tobytes() == sim.download(k).tobytes(), k
        # a version 8 file does not resume into a legacy (runtime/tasks off) simulator
        sim3 = pkg.Sim(dev, cfg, T)
        tr3 = pkg.PPOTrainer(sim3, epochs=1)
        with pytest.raises(pkg.MdnError):
            tr3.load_checkpoint(path, 1, T, 128, 3)
        tr3.close()
        sim3.close()
    finally:
        tr.close()
        tr2.close()
        sim.close()
        sim2.close()
        dev.close()
