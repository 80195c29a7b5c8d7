"""The reference's own PPOFIX1 checkpoints load and resume on the GPU.

Two checkpoints written by the reference's Metal trainer (copied from its
assets/checkpoints by tests/golden/make_fixtures.py) are loaded through
mdn_ppo_checkpoint_load (PPOTrainer::load_checkpoint, main.mm:1209-1320):

* version 6, guided-stress: 128 environments of family 7 with 2/1-tick delays,
  wind, depth noise, dropout and geometry memory, 30 rollouts / 960 Adam steps
  into training. Every loaded buffer equals the file bytes; then one resumed
  rollout (teacher-forced step by step against the CPU oracle) and the resumed
  PPO update (2 epochs x 256-row chunks, Adam steps 961-992 from the stored
  moments) match the oracle at the tolerances of tests/test_gpu_ppo.py.
* version 8, local-waypoint-fast: mode 22 with goal-arrival tasks and the
  runtime block. The simulator is configured from the file's own runtime and
  task blocks (as navigation_training::configure does before a resume), every
  loaded block equals the file bytes, and resumed steps match the oracle
  teacher-forced.
"""
import numpy as np
import pytest

from conftest import GOLDEN, load_oracle_module, load_package

pytestmark = pytest.mark.gpu

V6 = GOLDEN / "ref_ckpt_v6_guided_stress.bin"
V8 = GOLDEN / "ref_ckpt_v8_local_waypoint.bin"
STATE_KEYS = ("states", "runs", "worlds", "sensors", "poses", "commands")
ROLL = ("obs", "co", "actions", "logp", "values", "rewards", "next_values", "terminated", "truncated")


@pytest.fixture(scope="module")
def pkg():
    return load_package()


@pytest.fixture(scope="module")
def om():
    return load_oracle_module()


@pytest.fixture(scope="module")
def device(pkg):
    return pkg.Device(0)


def close(a, b, what, rtol=1e-5, atol=1e-5):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    bad = ~(np.abs(a - b) <= atol + rtol * np.abs(b))
    bad &= ~(np.isnan(a) & np.isnan(b))
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} differ; worst |d|={np.nanmax(np.abs(a - b)):.3e}"


def floats(structured):
    return np.frombuffer(np.ascontiguousarray(structured).tobytes(), np.float32)


def file_blocks(L, path):
    """Slices of a PPOFIX1 file in its layout (main.mm:978-1000,1209-1320)."""
    raw = path.read_bytes()
    h, _, _ = load_package().checkpoint_inspect(path)
    n = int(h["n"])
    A, C = int(h["actor_count"]), int(h["critic_count"])
    sizes = [("actor", A * 4), ("critic", C * 4), ("actor_m", A * 4), ("actor_v", A * 4), ("critic_m", C * 4),
             ("critic_v", C * 4), ("states", n * L.STATE.itemsize), ("runs", n * L.RUN.itemsize),
             ("worlds", n * L.WORLD.itemsize), ("sensors", n * 8 * 320 * 4), ("poses", n * 8 * 12 * 4),
             ("commands", n * 8 * 4 * 4)]
    if int(h["version"]) >= 7:
        sizes += [("runtime", L.RUNTIME_CONFIG.itemsize), ("task_control", L.TASK_CONTROL.itemsize),
                  ("env_physics", n * L.PARAMS.itemsize), ("task_states", n * L.TASK_STATE.itemsize),
                  ("nominal", L.PARAMS.itemsize), ("raptor", L.RAPTOR.itemsize)]
    out, off = {}, 136
    for name, size in sizes:
        out[name] = raw[off:off + size]
        off += size
    assert off == len(raw), "layout does not cover the file"
    return h, out


def sim_from_checkpoint(pkg, device, path, epochs=2):
    h, rt, tc = pkg.checkpoint_inspect(path)
    cfg = np.array(h["config"], pkg.layouts.CONFIG)
    sim = pkg.Sim(device, cfg, int(h["horizon"]), raptor=pkg.default_raptor())
    if int(h["version"]) >= 7 and int(tc["enabled"]):
        # navigation_training::configure, then the file's own runtime block (the
        # reference runner that wrote it kept per-episode plants off)
        sim.configure_tasks(tc, float(rt["domain_amplitude"]))
        sim.set_runtime(rt)
    tr = pkg.PPOTrainer(sim, epochs=epochs)
    tr.load_checkpoint(path, int(h["family"]), int(h["horizon"]), int(h["n"]), int(h["base_seed"]))
    return h, rt, tc, cfg, sim, tr


def check_loaded(pkg, sim, tr, blocks):
    for name in ("actor", "critic") + STATE_KEYS:
        assert sim.download(name).tobytes() == blocks[name], f"loaded {name}"
    for which, name in enumerate(("actor_m", "actor_v", "critic_m", "critic_v")):
        assert tr.moments(which).tobytes() == blocks[name], f"loaded {name}"
    if "task_states" in blocks:
        for name in ("task_states", "env_physics"):
            assert sim.download(name).tobytes() == blocks[name], f"loaded {name}"


def teacher_forced(gpu, ora, T, n, keys, hint_tol=1e-5, tasks=False):
    for t in range(T):
        for name in keys:
            gpu.upload(name, ora.buf(name))
        gpu.step(t)
        ora.step(t)
        rows = slice(t * n, (t + 1) * n)
        close(gpu.download("obs").reshape(T * n, 184)[rows], ora.buf("obs").reshape(T * n, 184)[rows],
              f"t={t} obs", atol=hint_tol)
        close(gpu.download("co").reshape(T * n, 32)[rows], ora.buf("co").reshape(T * n, 32)[rows], f"t={t} co")
        for name in ("actions", "logp", "values", "rewards", "next_values"):
            close(gpu.download(name).reshape(T * n, -1)[rows], ora.buf(name).reshape(T * n, -1)[rows],
                  f"t={t} {name}", atol=1e-4 if name == "logp" else 1e-5)
        for name in ("terminated", "truncated", "contact_id"):
            assert np.array_equal(gpu.download(name)[rows], ora.buf(name)[rows]), f"t={t} {name}"
        rs_g, rs_o = gpu.download("runs"), ora.buf("runs")
        for f in ("steps", "episodes", "successes", "collisions", "timeouts", "rng"):
            assert np.array_equal(rs_g[f], rs_o[f]), f"t={t} runs.{f}"
        close(floats(gpu.download("states")), floats(ora.buf("states")), f"t={t} states")
        wg, wo = gpu.download("worlds"), ora.buf("worlds")
        if tasks:
            # task resets draw goal directions with cosf/sinf (navigation_tasks.hpp:400-482):
            # last-ulp goal differences, as in tests/test_gpu_tasks.py
            assert np.array_equal(wg["count"], wo["count"]), f"t={t} world counts"
            close(floats(wg), floats(wo), f"t={t} worlds")
        else:
            assert wg.tobytes() == wo.tobytes(), f"t={t} worlds"


def bias(olib, steps):
    return (np.array([olib.o_pow_correction(0.9, int(s)) for s in steps], np.float32),
            np.array([olib.o_pow_correction(0.999, int(s)) for s in steps], np.float32))


def test_reference_v6_checkpoint_loads_and_resumes(pkg, om, device):
    L = pkg.layouts
    _, blocks = file_blocks(L, V6)
    h, rt, tc, cfg, sim, tr = sim_from_checkpoint(pkg, device, V6)
    try:
        assert int(h["version"]) == 6 and int(cfg["geometry_memory"]) == 1
        check_loaded(pkg, sim, tr, blocks)
        step0, done = int(h["optimizer_step"]), int(h["completed_rollouts"])
        assert tr.state() == (step0, done)
        n, T = int(h["n"]), int(h["horizon"])
        ora = om.OracleSim(L, cfg, T, sim.raptor)
        for name in ("actor", "critic") + STATE_KEYS:
            ora.buf(name)[:] = sim.download(name)
        teacher_forced(sim, ora, T, n, STATE_KEYS)
        # the resumed update, from the GPU's rollout and the stored Adam state
        for name in ROLL:
            ora.buf(name)[:] = sim.download(name)
        for bid, name in zip((100, 101, 102, 103), ("actor_m", "actor_v", "critic_m", "critic_v")):
            ora.buf(bid)[:] = np.frombuffer(blocks[name], np.float32)
        U = 2 * (n * T // 256)
        order = tr.minibatch_order(done, U)
        tr.rollout_update(done)
        assert tr.state() == (step0 + U, done + 1)
        ora.gae(True)
        assert np.array_equal(sim.download("advantages"), ora.buf("advantages"))
        b1, b2 = bias(ora.lib, range(step0 + 1, step0 + U + 1))
        out_o, norms_o = ora.train_rollout(256, 2, order, b1, b2)
        norms_g = tr.grad_norms(U).ravel()
        print(f"grad norms: worst relative difference {np.max(np.abs(norms_g - norms_o) / norms_o):.3e}")
        np.testing.assert_allclose(norms_g, norms_o, rtol=1e-4)
        lr = float(cfg["learning_rate"])
        for which, bid, pname in ((0, 100, "actor"), (2, 102, "critic")):
            p_g, p_o, m_o = sim.download(pname), ora.buf(pname), ora.buf(bid)
            diff = np.abs(p_g.astype(np.float64) - p_o)
            bad = diff > np.maximum(1e-7 + 1e-5 * np.abs(p_o), 1e-3 * lr * U)
            tiny = np.abs(m_o) <= 1e-4 * np.abs(m_o).max()
            print(f"{pname}: {int(bad.sum())} beyond tolerance, worst |d| = {diff.max():.3e}")
            assert not (bad & ~tiny).any(), f"{pname}: {int((bad & ~tiny).sum())} parameters differ"
            assert (diff <= 2.0001 * lr * U).all()
        np.testing.assert_allclose(tr.metric_mean, out_o, rtol=1e-3, atol=1e-6)
    finally:
        tr.close()
        sim.close()


def test_reference_v8_checkpoint_loads_and_resumes(pkg, om, device):
    L = pkg.layouts
    _, blocks = file_blocks(L, V8)
    h, rt, tc, cfg, sim, tr = sim_from_checkpoint(pkg, device, V8)
    try:
        assert int(h["version"]) == 8 and int(cfg["mode"]) == 22 and int(tc["enabled"]) == 1
        assert rt.tobytes() == blocks["runtime"] and tc.tobytes() == blocks["task_control"]
        check_loaded(pkg, sim, tr, blocks)
        assert tr.state() == (int(h["optimizer_step"]), int(h["completed_rollouts"]))
        n, T = int(h["n"]), int(h["horizon"])
        ora = om.OracleSim(L, cfg, T, sim.raptor)
        ora.set_task_control(tc)
        ora.set_runtime(rt)
        ora.reset()
        keys = STATE_KEYS + ("task_states", "env_physics")
        for name in ("actor", "critic") + keys:
            ora.buf(name)[:] = sim.download(name)
        teacher_forced(sim, ora, T, n, keys, tasks=True)
        for f in ("step_count", "terminal", "stable_ticks", "generation_status", "valid"):
            assert np.array_equal(sim.download("task_states")[f], ora.buf("task_states")[f]), f
        tr.rollout_update(int(h["completed_rollouts"]))
        device.finish()
        assert np.isfinite(sim.download("actor")).all() and np.isfinite(tr.metric_mean).all()
    finally:
        tr.close()
        sim.close()
