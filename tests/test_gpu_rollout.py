"""Rollout kernels on the GPU against the CPU oracle (through the C-ABI).

Parity bar (north_star): integer outputs bit-exact (termination, truncation,
contact id, counters); fp32 state, depth and observations within 1e-5 relative
per step. Geometry, the range ring, poses and the depth/context part of the
observation are compared bitwise (same IEEE operations). Per-step comparison is
teacher-forced: after every step the oracle's full simulator state is uploaded
into the GPU simulator, so each step starts from identical inputs.

Tolerances, stated: RTOL = 1e-5 relative, ATOL = 1e-5 absolute (|x| <= 1e-5 +
1e-5*|ref|) for everything that passes through a learned network or a
transcendental function (CUDA and libm differ in the last ulp).
"""
import numpy as np
import pytest

from conftest import GOLDEN, load_oracle_module, load_package

pytestmark = pytest.mark.gpu

RTOL = 1e-5
ATOL = 1e-5
STATE_KEYS = ("states", "runs", "worlds", "sensors", "poses", "commands")
RUN_FLOATS = ("hidden", "motors", "previous_nav", "desired_velocity", "yaw", "path", "elapsed", "peak_speed",
              "min_clearance", "initial_distance", "success_time", "total_path", "total_elapsed", "final_progress",
              "reference_position")


@pytest.fixture(scope="module")
def pkg():
    return load_package()


@pytest.fixture(scope="module")
def device(pkg):
    d = pkg.Device(0)
    yield d


@pytest.fixture(scope="module")
def om():
    return load_oracle_module()


def close(a, b, what, rtol=RTOL, atol=ATOL, grazing=0.0):
    """Elementwise |a - b| <= atol + rtol |b|. `grazing` > 0 lets that fraction
    of the elements (at least one) exceed it: depth rays that graze a moving
    sphere turn a last-ulp difference of its sinf-placed centre into a larger
    range difference (the intersection distance scales it by 1/sqrt(disc))."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    bad = ~(np.abs(a - b) <= atol + rtol * np.abs(b))
    bad &= ~(np.isnan(a) & np.isnan(b))
    allowed = max(1, int(grazing * bad.size)) if grazing > 0 else 0
    assert bad.sum() <= allowed, f"{what}: {bad.sum()} of {bad.size} differ; worst |d|={np.nanmax(np.abs(a - b)):.3e}"


def floats(structured):
    return np.frombuffer(np.ascontiguousarray(structured).tobytes(), np.float32)


def make_pair(pkg, om, raptor, cfg, horizon):
    L = pkg.layouts
    gpu = pkg.Sim(pkg_device(), cfg, horizon, raptor=raptor)
    ora = om.OracleSim(L, cfg, horizon, raptor)
    return gpu, ora


_DEV = {}


def pkg_device():
    return _DEV["dev"]


@pytest.fixture(scope="module", autouse=True)
def _register(device):
    _DEV["dev"] = device


@pytest.fixture(scope="module")
def raptor(pkg):
    return pkg.default_raptor()


CONFIGS = [
    dict(family=1),
    dict(family=2),
    dict(family=3),
    dict(family=0),
    dict(family=1, sensor_delay=2, command_delay=2, wind=0.3),
    dict(family=12, sensor_delay=1, command_delay=1, wind=0.5, depth_noise=0.05, dropout=0.1),
    dict(family=13),
    dict(family=7, risk_coef=0.5, max_steps=7),
    dict(family=1, sensor_period=2, velocity_contract=0, distance=5.0),
    dict(family=1, mode=1),
    dict(family=4, eval=1, max_steps=9),
    dict(family=17),
    dict(family=18, sensor_delay=2, command_delay=2),
    dict(family=19),
    dict(family=20, max_steps=40),
    dict(family=13, geometry_memory=1, sensor_delay=2),
    dict(family=1, geometry_memory=1, mode=22, command_delay=1, sensor_period=2),
]


@pytest.mark.parametrize("extra", CONFIGS, ids=[str(c) for c in CONFIGS])
def test_reset_bitwise(pkg, om, raptor, extra):
    cfg = pkg.layouts.default_config(**{**dict(n=300, speed=1.0, distance=3.0, seed=5), **extra})
    gpu, ora = make_pair(pkg, om, raptor, cfg, 4)
    try:
        for name in STATE_KEYS + ("actor", "critic"):
            assert gpu.download(name).tobytes() == ora.buf(name).tobytes(), name
    finally:
        gpu.close()


@pytest.mark.parametrize("extra", CONFIGS, ids=[str(c) for c in CONFIGS])
def test_teacher_forced_steps(pkg, om, raptor, extra):
    n, T = 256, 12
    cfg = pkg.layouts.default_config(**{**dict(n=n, speed=1.0, distance=3.0, seed=9), **extra})
    gpu, ora = make_pair(pkg, om, raptor, cfg, T)
    # Depth noise draws Box-Muller normals (logf/cosf, sim.metal:154-156), and
    # the bounded moving spheres of the mixed-capability courses (families 18,
    # 20) place their centres with sinf (world.hpp:32-41): ranges of rays that
    # meet them match to the last ulp only, so compare those with RTOL.
    movers = 1e-4 if int(cfg["family"]) in (18, 20) else 0.0
    exact_depth = float(cfg["depth_noise"]) == 0.0 and movers == 0.0
    try:
        for t in range(T):
            # identical inputs: the oracle's state becomes the GPU's state
            for name in STATE_KEYS:
                gpu.upload(name, ora.buf(name))
            gpu.step(t)
            ora.step(t)
            rows = slice(t * n, (t + 1) * n)
            obs_g = gpu.download("obs").reshape(T * n, 184)[rows]
            obs_o = ora.buf("obs").reshape(T * n, 184)[rows]
            # depth pool + 21 context features: same IEEE operations -> bitwise
            if exact_depth:
                assert np.array_equal(obs_g[:, :181], obs_o[:, :181]), f"t={t} obs[:181]"
            else:
                close(obs_g[:, :181], obs_o[:, :181], f"t={t} obs[:181]", grazing=movers)
            close(obs_g[:, 181:], obs_o[:, 181:], f"t={t} guidance hint")
            co_g = gpu.download("co").reshape(T * n, 32)[rows]
            co_o = ora.buf("co").reshape(T * n, 32)[rows]
            if exact_depth:
                assert np.array_equal(co_g, co_o), f"t={t} critic obs"
            else:  # clearance and obstacle offsets include the sinf-placed movers
                close(co_g, co_o, f"t={t} critic obs")
            for name in ("actions", "logp", "values", "rewards", "next_values"):
                g = gpu.download(name).reshape(T * n, -1)[rows]
                o = ora.buf(name).reshape(T * n, -1)[rows]
                close(g, o, f"t={t} {name}", atol=1e-4 if name == "logp" else ATOL)
            for name in ("terminated", "truncated", "contact_id"):
                g = gpu.download(name)[rows]
                o = ora.buf(name)[rows]
                assert np.array_equal(g, o), f"t={t} {name}"
            # post-step simulator state
            rs_g, rs_o = gpu.download("runs"), ora.buf("runs")
            for f in ("steps", "successes", "collisions", "timeouts", "episodes"):
                assert np.array_equal(rs_g[f], rs_o[f]), f"t={t} runs.{f}"
            assert np.array_equal(rs_g["rng"], rs_o["rng"]), f"t={t} runs.rng"
            close(floats(gpu.download("states")), floats(ora.buf("states")), f"t={t} states")
            for f in RUN_FLOATS:
                close(rs_g[f], rs_o[f], f"t={t} runs.{f}")
            assert gpu.download("worlds").tobytes() == ora.buf("worlds").tobytes(), f"t={t} worlds"
            if exact_depth:
                assert np.array_equal(gpu.download("sensors"), ora.buf("sensors")), f"t={t} sensors"
            else:
                close(gpu.download("sensors"), ora.buf("sensors"), f"t={t} sensors", grazing=movers)
            assert np.array_equal(gpu.download("poses"), ora.buf("poses")), f"t={t} poses"
            close(gpu.download("commands"), ora.buf("commands"), f"t={t} commands")
    finally:
        gpu.close()


GRAPH_CASES = [(dict(n=1000, family=1, speed=1.0, distance=4.0, seed=3), 16),
               # short episodes: resets inside the rollout, run by the next step's k_sense
               # (odd horizon: the reset-list phase restarts with each collect)
               (dict(n=777, family=18, speed=1.0, distance=3.0, seed=5, sensor_delay=2, command_delay=2,
                     max_steps=5), 7),
               (dict(n=300, family=13, speed=1.0, distance=3.0, seed=7, max_steps=4, risk_coef=0.5,
                     depth_noise=0.05, wind=0.3), 8),
               (dict(n=333, family=18, speed=1.0, distance=3.0, seed=9, eval=1, max_steps=3), 6),
               # more listed resets per step than the sensing kernel has reset-worker warps
               (dict(n=20000, family=18, speed=1.0, distance=3.0, seed=11, sensor_delay=2, command_delay=2,
                     max_steps=3), 6)]


@pytest.mark.parametrize("case", range(len(GRAPH_CASES)))
def test_collect_graph_equals_steps(pkg, raptor, case):
    """collect() replays a captured CUDA graph in which each step's ended
    episodes are reset by the next step's sensing kernel (the last step
    flushes them); it must equal step-by-step launches, over two replays."""
    fields, T = GRAPH_CASES[case]
    cfg = pkg.layouts.default_config(**fields)
    a = pkg.Sim(pkg_device(), cfg, T, raptor=raptor)
    b = pkg.Sim(pkg_device(), cfg, T, raptor=raptor)
    try:
        for rep in range(2):  # the second replay continues the episodes
            a.collect()
            for t in range(T):
                b.step(t)
            for name in STATE_KEYS + ("obs", "co", "actions", "logp", "values", "rewards", "next_values",
                                      "terminated", "truncated", "contact_id"):
                assert a.download(name).tobytes() == b.download(name).tobytes(), f"replay {rep}: {name}"
        runs = a.download("runs")
        assert runs["steps"].max() > T or runs["episodes"].sum() > 0
        if fields.get("max_steps", 1000) < T and not fields.get("eval"):
            assert runs["episodes"].sum() >= fields["n"], "episodes ended inside the rollout"
    finally:
        a.close()
        b.close()


def test_free_run_vs_reference_trace(pkg, raptor):
    """The reference's own CPU path (compiled unmodified, recorded in
    tests/golden/ref_trace.npz) free-running from reset: the first observation
    row is bit-exact; later steps stay within a loose drift bound."""
    ref = np.load(GOLDEN / "ref_trace.npz")
    for family in (1, 3):
        cfg = pkg.layouts.default_config(n=24, family=family, speed=1.0, distance=3.0, seed=42)
        sim = pkg.Sim(pkg_device(), cfg, 6, raptor=raptor)
        try:
            assert sim.download("worlds").tobytes() == ref[f"f{family}_worlds0"].tobytes()
            assert sim.download("states").tobytes() == ref[f"f{family}_states0"].tobytes()
            sim.collect()
            obs = sim.download("obs").reshape(6, 24, 184)
            robs = ref[f"f{family}_obs"].reshape(6, 24, 184)
            assert np.array_equal(obs[0, :, :181], robs[0, :, :181])
            close(obs, robs, f"family {family} obs over 6 steps", rtol=1e-3, atol=1e-3)
            assert np.array_equal(sim.download("terminated"), ref[f"f{family}_terminated"])
            close(floats(sim.download("states")), floats(ref[f"f{family}_states6"]), "final states", rtol=1e-3,
                  atol=1e-3)
        finally:
            sim.close()


def test_custom_room_matches_oracle(pkg, om, raptor):
    """BASELINE room x[-2,8] y[-5,5] z[0,4] as a parameter (world.hpp:73-74,85 generalised)."""
    room = np.array([-2, -5, 0, 8, 5, 4], np.float32)
    cfg = pkg.layouts.default_config(n=128, family=1, speed=1.0, distance=3.0, seed=2)
    gpu = pkg.Sim(pkg_device(), cfg, 4, raptor=raptor, room=room)
    ora = om.OracleSim(pkg.layouts, cfg, 4, raptor, room=room)
    try:
        for t in range(4):
            for name in STATE_KEYS:
                gpu.upload(name, ora.buf(name))
            gpu.step(t)
            ora.step(t)
        assert np.array_equal(gpu.download("sensors"), ora.buf("sensors"))
        assert np.array_equal(gpu.download("co"), ora.buf("co"))
        assert np.array_equal(gpu.download("terminated"), ora.buf("terminated"))
    finally:
        gpu.close()


def test_rejects_unsupported_config(pkg, raptor):
    with pytest.raises(pkg.MdnError):
        pkg.Sim(pkg_device(), pkg.layouts.default_config(n=8, sensor_delay=7), 4, raptor=raptor)
    with pytest.raises(pkg.MdnError):
        pkg.Sim(pkg_device(), pkg.layouts.default_config(n=0), 4, raptor=raptor)


ACTOR_CASES = [(1, 320, {}), (4, 320, {}),
               # a partial last 64-environment pass of the quad actor's staged rows
               (4, 333, {}),
               # more than 2 x SMs x 64 environments: quad blocks loop over several passes
               (4, 19000, {}),
               # evaluation mode skips environments whose episode has finished
               (4, 333, dict(eval=1, max_steps=3)), (1, 333, dict(eval=1, max_steps=3))]


@pytest.mark.parametrize("threads,n,extra", ACTOR_CASES, ids=[f"t{t}-n{n}-{e}" for t, n, e in ACTOR_CASES])
def test_actor_kernels_match_oracle(pkg, om, raptor, threads, n, extra, monkeypatch):
    """Both 64-unit actor kernels (one thread per environment, and four threads
    per environment for small shards; MDN_ACT_THREADS picks one at simulator
    creation) against the oracle, teacher-forced."""
    monkeypatch.setenv("MDN_ACT_THREADS", str(threads))
    T = 6
    cfg = pkg.layouts.default_config(**{**dict(n=n, family=18, speed=1.0, distance=3.0, seed=13, sensor_delay=2,
                                               command_delay=2, mode=17), **extra})
    gpu, ora = make_pair(pkg, om, raptor, cfg, T)
    try:
        for t in range(T):
            for name in STATE_KEYS:
                gpu.upload(name, ora.buf(name))
            gpu.step(t)
            ora.step(t)
            rows = slice(t * n, (t + 1) * n)
            for name in ("actions", "logp", "values"):
                g = gpu.download(name).reshape(T * n, -1)[rows]
                o = ora.buf(name).reshape(T * n, -1)[rows]
                close(g, o, f"t={t} {name}", atol=1e-4 if name == "logp" else ATOL)
            close(gpu.download("commands"), ora.buf("commands"), f"t={t} commands")
            rs_g, rs_o = gpu.download("runs"), ora.buf("runs")
            assert np.array_equal(rs_g["rng"], rs_o["rng"]), f"t={t} rng"
            close(rs_g["desired_velocity"], rs_o["desired_velocity"], f"t={t} desired velocity")
    finally:
        gpu.close()


GROUP_CASES = [dict(family=18, sensor_delay=2, command_delay=2), dict(family=12, depth_noise=0.05, wind=0.3),
               dict(family=13, max_steps=5, risk_coef=0.5)]


@pytest.mark.parametrize("group", [1, 2, 4, 8])
@pytest.mark.parametrize("case", range(len(GROUP_CASES)))
def test_advance_lane_groups_match_oracle(pkg, om, raptor, group, case, monkeypatch):
    """k_advance with 1, 2, 4 and 8 lanes per environment (plan_step picks by shard
    size; MDN_ADVANCE_GROUP forces one) against the oracle, teacher-forced, with
    episode ends and resets inside the window."""
    monkeypatch.setenv("MDN_ADVANCE_GROUP", str(group))
    n, T = 256, 8
    cfg = pkg.layouts.default_config(**{**dict(n=n, speed=1.0, distance=3.0, seed=31 + case, max_steps=6),
                                        **GROUP_CASES[case]})
    gpu, ora = make_pair(pkg, om, raptor, cfg, T)
    movers = 1e-4 if int(cfg["family"]) in (18, 20) else 0.0
    try:
        for t in range(T):
            for name in STATE_KEYS:
                gpu.upload(name, ora.buf(name))
            gpu.step(t)
            ora.step(t)
            rows = slice(t * n, (t + 1) * n)
            for name in ("terminated", "truncated", "contact_id"):
                assert np.array_equal(gpu.download(name)[rows], ora.buf(name)[rows]), f"t={t} {name}"
            for name in ("rewards", "next_values"):
                close(gpu.download(name)[rows], ora.buf(name)[rows], f"t={t} {name}")
            rs_g, rs_o = gpu.download("runs"), ora.buf("runs")
            for f in ("steps", "episodes", "rng"):
                assert np.array_equal(rs_g[f], rs_o[f]), f"t={t} runs.{f}"
            close(floats(gpu.download("states")), floats(ora.buf("states")), f"t={t} states")
            assert gpu.download("worlds").tobytes() == ora.buf("worlds").tobytes(), f"t={t} worlds"
            if movers:
                close(gpu.download("sensors"), ora.buf("sensors"), f"t={t} sensors", grazing=movers)
        assert ora.buf("runs")["episodes"].sum() > 0
    finally:
        gpu.close()


def test_delay_rehearsal_teacher_forced(pkg, om, raptor):
    """Delay rehearsal (NAV_DELAY_REHEARSAL, sim.metal:14-24) switched on at
    run time under mode 22: every other group of four environments trains
    without delays, wind, depth noise or dropout. Reset and teacher-forced
    steps against the oracle with the same switch; the clean groups are
    checked directly too (zero wind)."""
    n, T = 256, 8
    cfg = pkg.layouts.default_config(n=n, family=1, mode=22, speed=1.0, distance=3.0, seed=17, sensor_delay=2,
                                     command_delay=2, wind=0.4, depth_noise=0.05, dropout=0.1, max_steps=6)
    gpu, ora = make_pair(pkg, om, raptor, cfg, T)
    try:
        gpu.set_delay_rehearsal(True)
        gpu.reset()
        ora.set_delay_rehearsal(True)
        ora.reset()
        for name in STATE_KEYS:
            assert gpu.download(name).tobytes() == ora.buf(name).tobytes(), f"reset {name}"
        clean = (np.arange(n) // 4) % 2 == 0
        wind = gpu.download("worlds")["wind"][:, 0]
        assert (wind[clean] == 0).all() and (wind[~clean] != 0).all()
        for t in range(T):
            for name in STATE_KEYS:
                gpu.upload(name, ora.buf(name))
            gpu.step(t)
            ora.step(t)
            rows = slice(t * n, (t + 1) * n)
            # depth noise goes through logf/cosf: ranges and features at 1e-5
            close(gpu.download("obs").reshape(T * n, 184)[rows], ora.buf("obs").reshape(T * n, 184)[rows],
                  f"t={t} obs")
            close(gpu.download("co").reshape(T * n, 32)[rows], ora.buf("co").reshape(T * n, 32)[rows], f"t={t} co")
            for name in ("actions", "values", "rewards", "next_values"):
                close(gpu.download(name).reshape(T * n, -1)[rows], ora.buf(name).reshape(T * n, -1)[rows],
                      f"t={t} {name}")
            for name in ("terminated", "truncated", "contact_id"):
                assert np.array_equal(gpu.download(name)[rows], ora.buf(name)[rows]), f"t={t} {name}"
            rs_g, rs_o = gpu.download("runs"), ora.buf("runs")
            for f in ("steps", "episodes", "rng"):
                assert np.array_equal(rs_g[f], rs_o[f]), f"t={t} runs.{f}"
            for f in ("previous_nav", "desired_velocity"):
                close(rs_g[f], rs_o[f], f"t={t} runs.{f}")
            close(floats(gpu.download("states")), floats(ora.buf("states")), f"t={t} states")
            assert gpu.download("worlds").tobytes() == ora.buf("worlds").tobytes(), f"t={t} worlds"
        assert ora.buf("runs")["episodes"].sum() > 0
    finally:
        gpu.close()


def test_bounded_mover_samples_gpu(pkg, om, raptor):
    """The reference's bounded-motion check (navigation_motion_check.mm:19-32)
    on the GPU: 1,001 environments, each with the one moving sphere at time
    i * 0.02 s and the vehicle 1 m from its surface. The sensing kernel's
    critic observation gives the clearance (feature 19, x5) and the sphere's
    offset (features 21-23, x10): the clearance is 1 (gate 1e-5) and both
    match the oracle's wclearance / wc within 1e-5."""
    olib = om.load_oracle()
    L = pkg.layouts
    n = 1001
    cfg = L.default_config(n=n, family=1, seed=2, max_steps=50)
    sim = pkg.Sim(pkg_device(), cfg, 2, raptor=raptor)
    try:
        worlds = sim.download("worlds")
        states = sim.download("states")
        runs = sim.download("runs")
        worlds[:] = np.zeros((), L.WORLD)
        want_cl, want_c, points = [], [], []
        for i in range(n):
            w = worlds[i:i + 1]
            w["count"] = 1
            o = w["obstacles"][0, 0]
            o["kind"] = 3
            o["center"] = (6, 0, 1.5)
            o["size"] = (0.28, 2.7, -1.57079632679)
            o["velocity"] = (0, 0.8, 0)
            w["goal"] = (8, 0, 1.5)
            t = np.float32(i) * np.float32(0.02)
            c = np.zeros(3, np.float32)
            olib.o_wc(om.ptr(worlds[i]["obstacles"]), t, om.ptr(c))
            p = np.array([c[0] + np.float32(0.28) + np.float32(0.18) + np.float32(1), c[1], c[2]], np.float32)
            want_cl.append(olib.o_wclearance(om.ptr(worlds[i:i + 1]), None, om.ptr(p), t, None))
            want_c.append(c)
            points.append(p)
            runs[i]["elapsed"] = t
        points = np.array(points)
        states["position"] = points
        sim.upload("worlds", worlds)
        sim.upload("states", states)
        sim.upload("runs", runs)
        sim.step(0)
        co = sim.download("co").reshape(2, n, 32)[0].astype(np.float64)
        cl = co[:, 19] * 5.0
        assert np.all(np.abs(cl - 1.0) < 1e-5), np.max(np.abs(cl - 1.0))
        close(cl, np.array(want_cl), "clearance vs oracle")
        close(co[:, 21:24] * 10.0 + points, np.array(want_c), "sphere centre vs oracle")
    finally:
        sim.close()


def test_report_matches_run_records(pkg, raptor):
    """Sim::report (main.mm:599-602) reduced on the GPU equals the same
    aggregates of the downloaded run records: counters exactly, float totals
    (summed in double) within 1e-12 relative, minimum clearance and peak speed
    exactly."""
    cfg = pkg.layouts.default_config(n=5000, family=18, speed=1.0, distance=3.0, seed=21, max_steps=6)
    sim = pkg.Sim(pkg_device(), cfg, 8, raptor=raptor)
    try:
        sim.collect()
        sim.collect()
        rep = sim.report()
        runs = sim.download("runs")
        assert runs["episodes"].sum() > 0
        for key in ("episodes", "successes", "collisions", "timeouts"):
            assert rep[key] == float(runs[key].astype(np.float64).sum()), key
        for key in ("success_time", "total_path", "total_elapsed", "final_progress"):
            want = float(runs[key].astype(np.float64).sum())
            assert abs(rep[key] - want) <= 1e-12 * max(abs(want), 1.0), key
        assert rep["min_clearance"] == float(min(12.0, runs["min_clearance"].min()))
        assert rep["peak_speed"] == float(max(0.0, runs["peak_speed"].max()))
    finally:
        sim.close()
