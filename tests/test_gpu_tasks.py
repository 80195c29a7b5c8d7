"""Goal-arrival tasks and the sim_act mode table on the GPU against the oracle.

The task contract (sim_reset_navigation_task, sim.metal:125-141; the
navigation_task_step override of sim_advance, sim.metal:307-317) and the
evaluation/training modes of sim_act (sim.metal:229-270) run through the C-ABI
and are compared step by step, teacher-forced, with the CPU oracle, whose
task operators are pinned bit for bit to navigation_tasks.hpp.

Tolerances, stated: integers (status, counters, flags, termination) bit-exact;
fp32 within RTOL = 1e-5 relative + ATOL = 1e-5 absolute. Task generation draws
directions with cosf/sinf and the start quaternion with cosf/sinf of the half
yaw, so generated starts and goals match to the last ulp (RTOL), not bitwise.
"""
import numpy as np
import pytest

from conftest import load_oracle_module, load_package

pytestmark = pytest.mark.gpu

RTOL = 1e-5
ATOL = 1e-5
STATE_KEYS = ("states", "runs", "worlds", "sensors", "poses", "commands", "task_states")
TASK_INTS = ("generation_status", "valid", "generation_attempts", "family", "stage", "objective", "max_nav_steps",
             "step_count", "stable_ticks", "was_inside_goal", "waypoint_event_latched", "terminal",
             "witness_point_count")
TASK_FLOATS = ("start_position", "start_yaw_rad", "start_velocity_world", "goal_position", "initial_distance_m",
               "previous_distance_m", "difficulty", "start_clearance_m", "goal_clearance_m",
               "direct_segment_clearance_m", "witness_min_clearance_m", "witness_length_m", "stable_time_s",
               "last_executed_world_command", "witness_points")


@pytest.fixture(scope="module")
def pkg():
    return load_package()


@pytest.fixture(scope="module")
def om():
    return load_oracle_module()


@pytest.fixture(scope="module")
def device(pkg):
    return pkg.Device(0)


@pytest.fixture(scope="module")
def raptor(pkg):
    return pkg.default_raptor()


def close(a, b, what, rtol=RTOL, atol=ATOL):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    bad = ~(np.abs(a - b) <= atol + rtol * np.abs(b))
    bad &= ~(np.isnan(a) & np.isnan(b))
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} differ; worst |d|={np.nanmax(np.abs(a - b)):.3e}"


def floats(structured):
    return np.frombuffer(np.ascontiguousarray(structured).tobytes(), np.float32)


def compare_tasks(g, o, what):
    for f in TASK_INTS:
        assert np.array_equal(g[f], o[f]), f"{what} task.{f}"
    for f in TASK_FLOATS:
        close(g[f], o[f], f"{what} task.{f}")


def pair(pkg, om, device, raptor, cfg, T, control, domain_amplitude=0.0):
    gpu = pkg.Sim(device, cfg, T, raptor=raptor)
    gpu.configure_tasks(control, domain_amplitude)
    ora = om.OracleSim(pkg.layouts, cfg, T, raptor)
    ora.set_task_control(control)
    ora.set_runtime(pkg.runtime_config(domain_amplitude))  # navigation_training.hpp:20-22
    ora.reset()
    return gpu, ora


TASK_CASES = [
    dict(stage=0, family=0, mode=22),
    dict(stage=1, family=0, mode=22),
    dict(stage=2, family=1, mode=22),
    dict(stage=2, family=2, mode=0),
    dict(stage=2, family=4, mode=17, eval=1),
    dict(stage=2, family=5, mode=22, wind=0.3, sensor_delay=1, command_delay=1),
    dict(stage=2, family=12, mode=22),
    # navigation_training::train / evaluate: mode 22 / 17 with geometry memory
    dict(stage=2, family=12, mode=22, geometry_memory=1),
    dict(stage=1, family=0, mode=17, geometry_memory=1, eval=1),
]


@pytest.mark.parametrize("case", TASK_CASES, ids=[str(c) for c in TASK_CASES])
def test_task_reset_matches_oracle(pkg, om, device, raptor, case):
    case = dict(case)
    stage = case.pop("stage")
    cfg = pkg.layouts.default_config(**{**dict(n=200, speed=1.5, distance=8.0, seed=31, max_steps=400), **case})
    gpu, ora = pair(pkg, om, device, raptor, cfg, 4, pkg.task_control(stage, int(cfg["family"])))
    try:
        compare_tasks(gpu.download("task_states"), ora.buf("task_states"), "reset")
        assert (ora.buf("task_states")["generation_status"] == 4).mean() > 0.9
        close(floats(gpu.download("states")), floats(ora.buf("states")), "reset states")
        rg, ro = gpu.download("runs"), ora.buf("runs")
        for f in ("yaw", "initial_distance", "reference_position", "desired_velocity"):
            close(rg[f], ro[f], f"reset runs.{f}")
        wg, wo = gpu.download("worlds"), ora.buf("worlds")
        assert np.array_equal(wg["count"], wo["count"])
        close(floats(wg), floats(wo), "reset worlds")
    finally:
        gpu.close()


@pytest.mark.parametrize("family", [1, 2, 12])
def test_task_detour_witnesses_match_oracle(pkg, om, device, raptor, family):
    """Forced detours (require_detour) on long goals: every task's witness is a
    dogleg, so the warp-split segment scan and its early stop on failing
    doglegs are exercised; witness choice and clearances match the oracle."""
    cfg = pkg.layouts.default_config(n=256, family=family, mode=22, speed=1.5, distance=8.0, seed=5, max_steps=400)
    control = pkg.task_control(2, family)
    control["config"]["require_detour"] = 1
    control["config"]["goal_distance_max_m"] = 20.0
    gpu, ora = pair(pkg, om, device, raptor, cfg, 4, control)
    try:
        to = ora.buf("task_states")
        compare_tasks(gpu.download("task_states"), to, "detour reset")
        ready = to["generation_status"] == 4
        assert ready.mean() > 0.5
        assert (to["witness_point_count"][ready] >= 3).all()
        close(floats(gpu.download("worlds")), floats(ora.buf("worlds")), "detour worlds")
    finally:
        gpu.close()


@pytest.mark.parametrize("case", TASK_CASES, ids=[str(c) for c in TASK_CASES])
def test_task_teacher_forced_steps(pkg, om, device, raptor, case):
    case = dict(case)
    stage = case.pop("stage")
    n, T = 160, 10
    cfg = pkg.layouts.default_config(**{**dict(n=n, speed=1.5, distance=8.0, seed=13, max_steps=400), **case})
    control = pkg.task_control(stage, int(cfg["family"]))
    control["config"]["max_nav_steps"] = 6  # task timeouts and resets inside the window
    gpu, ora = pair(pkg, om, device, raptor, cfg, T, control)
    try:
        for t in range(T):
            for name in STATE_KEYS:
                gpu.upload(name, ora.buf(name))
            gpu.step(t)
            ora.step(t)
            rows = slice(t * n, (t + 1) * n)
            for name in ("actions", "logp", "values", "rewards", "next_values"):
                g = gpu.download(name).reshape(T * n, -1)[rows]
                o = ora.buf(name).reshape(T * n, -1)[rows]
                close(g, o, f"t={t} {name}", atol=1e-4 if name == "logp" else ATOL)
            for name in ("terminated", "truncated", "contact_id"):
                assert np.array_equal(gpu.download(name)[rows], ora.buf(name)[rows]), f"t={t} {name}"
            rs_g, rs_o = gpu.download("runs"), ora.buf("runs")
            for f in ("steps", "successes", "collisions", "timeouts", "episodes", "rng"):
                assert np.array_equal(rs_g[f], rs_o[f]), f"t={t} runs.{f}"
            compare_tasks(gpu.download("task_states"), ora.buf("task_states"), f"t={t}")
            close(floats(gpu.download("states")), floats(ora.buf("states")), f"t={t} states")
            close(gpu.download("commands"), ora.buf("commands"), f"t={t} commands")
        assert ora.buf("runs")["episodes"].sum() > 0  # resets with new tasks were exercised
    finally:
        gpu.close()


MODE_CASES = [2, 3, 9, 12, 16, 17, 18, 19, 20, 21, 22, 5]


@pytest.mark.parametrize("mode", MODE_CASES)
def test_mode_table_teacher_forced(pkg, om, device, raptor, mode):
    n, T = 128, 6
    cfg = pkg.layouts.default_config(n=n, family=12, mode=mode, speed=1.0, distance=3.0, seed=21, sensor_delay=1,
                                     command_delay=1)
    gpu = pkg.Sim(device, cfg, T, raptor=raptor)
    ora = om.OracleSim(pkg.layouts, cfg, T, raptor)
    try:
        for t in range(T):
            for name in STATE_KEYS[:-1]:
                gpu.upload(name, ora.buf(name))
            gpu.step(t)
            ora.step(t)
            rows = slice(t * n, (t + 1) * n)
            for name in ("actions", "logp", "values", "rewards"):
                g = gpu.download(name).reshape(T * n, -1)[rows]
                o = ora.buf(name).reshape(T * n, -1)[rows]
                close(g, o, f"mode {mode} t={t} {name}", atol=1e-4 if name == "logp" else ATOL)
            close(gpu.download("commands"), ora.buf("commands"), f"mode {mode} t={t} commands")
            rs_g, rs_o = gpu.download("runs"), ora.buf("runs")
            for f in ("previous_nav", "desired_velocity", "yaw"):
                close(rs_g[f], rs_o[f], f"mode {mode} t={t} runs.{f}")
            for name in ("terminated", "truncated"):
                assert np.array_equal(gpu.download(name)[rows], ora.buf(name)[rows]), f"mode {mode} t={t} {name}"
    finally:
        gpu.close()


def test_validate_tasks_and_config_checks(pkg, device, raptor):
    cfg = pkg.layouts.default_config(n=64, family=1, mode=22, speed=1.5, distance=8.0, seed=3, max_steps=400)
    sim = pkg.Sim(device, cfg, 4, raptor=raptor)
    try:
        with pytest.raises(pkg.MdnError):
            sim.validate_tasks()  # legacy episodes carry no tasks
        control = pkg.task_control(2, 1)
        sim.configure_tasks(control)
        statuses = sim.download("task_states")["generation_status"]
        if (statuses == 4).all():
            sim.validate_tasks()
        bad = control.copy()
        bad["config"]["nav_period_s"] = np.float32(0.04)
        with pytest.raises(pkg.MdnError):
            sim.configure_tasks(bad)  # task/simulator clock mismatch
        for amplitude in (1.5, -0.1, float("nan")):
            with pytest.raises(pkg.MdnError):
                sim.configure_tasks(control, domain_amplitude=amplitude)  # domain amplitude must be 0..1
        invalid = control.copy()
        invalid["config"]["goal_radius_m"] = np.float32(0.0)
        sim.configure_tasks(invalid)  # accepted like the reference; every env reports status 1
        assert (sim.download("task_states")["generation_status"] == 1).all()
        with pytest.raises(pkg.MdnError):
            sim.validate_tasks()
        sim.collect()
    finally:
        sim.close()
