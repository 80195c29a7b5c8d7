"""Pin the C restatement (oracle/liboracle.so) to the reference.

Against the reference's golden fixtures (RAPTOR official sequence, rl-tools L2F
fixtures, the analytic ray / GAE / normalisation / Adam cases of main.mm and
ppo.hpp) and, bit for bit, against the reference's own CPU path compiled
unmodified (oracle/_ref). CPU only.
"""
import numpy as np
import pytest

from conftest import physics_fixture, raptor_fixture_sequence

P = None


@pytest.fixture(scope="module", autouse=True)
def _ptr(oracle_mod, olib):
    global P
    P = oracle_mod.ptr
    # oracle/_ref is a g++ build: g++ evaluates the three draws inside
    # wgenerate_mixed's wadd_table argument list (world.hpp:180) right to left,
    # the reference platforms left to right. Compare like with like here; the
    # product follows the reference platforms (tests/test_gpu_*.py).
    olib.o_set_argument_order(1)
    yield
    olib.o_set_argument_order(0)


def f3(*v):
    return np.array(v, np.float32)


def test_raptor_official_sequence(olib, raptor):
    # main.mm:127-137: 16-step official RAPTOR sequence, gate 2e-5.
    obs, exp = raptor_fixture_sequence()
    h = raptor["initial_hidden_state"].copy()
    a = np.zeros(4, np.float32)
    err = 0.0
    for t in range(16):
        o = obs[t].copy()
        olib.o_raptor_forward(P(raptor), P(o), P(h), P(a))
        err = max(err, float(np.abs(a - exp[t]).max()))
    assert err < 2e-5, err


def test_raptor_bitwise_vs_reference(olib, rlib, raptor):
    rng = np.random.default_rng(0)
    for _ in range(200):
        o = rng.uniform(-1.5, 1.5, 22).astype(np.float32)
        h0 = rng.uniform(-1, 1, 16).astype(np.float32)
        h1, h2 = h0.copy(), h0.copy()
        a1, a2 = np.zeros(4, np.float32), np.zeros(4, np.float32)
        olib.o_raptor_forward(P(raptor), P(o), P(h1), P(a1))
        rlib.ref_raptor_forward(P(raptor), P(o), P(h2), P(a2))
        assert np.array_equal(h1, h2) and np.array_equal(a1, a2)


def test_physics_fixtures(olib, rlib, layouts):
    # main.mm:138-176: 64 cases x 8 steps from rl-tools, gate 2e-5.
    params, recs = physics_fixture(layouts)
    default = np.zeros((), layouts.PARAMS)
    olib.o_physics_default(P(default))
    assert default.tobytes() == params.tobytes()  # rl_physics_crazyflie_default == fixture params
    out = np.zeros((), layouts.STATE)
    out2 = np.zeros((), layouts.STATE)
    err = 0.0
    for r in recs:
        s = np.array(r["state"], layouts.STATE)
        act = np.array(r["action"], np.float32)
        wind = np.array(r["wind"], np.float32)
        olib.o_physics_step(P(s), P(act), P(wind), P(params), P(out))
        rlib.ref_physics_step(P(s), P(act), P(wind), P(params), P(out2))
        assert out.tobytes() == out2.tobytes()
        e = np.frombuffer(out.tobytes(), np.float32) - np.frombuffer(np.array(r["expected"]).tobytes(), np.float32)
        err = max(err, float(np.abs(e).max()))
    assert err < 2e-5, err


def test_analytic_rays(olib):
    # main.mm:108-115 known answers.
    assert abs(olib.o_wray_sphere(P(f3(0, 0, 0)), P(f3(1, 0, 0)), P(f3(3, 0, 0)), 1) - 2) < 1e-6
    assert abs(olib.o_wray_sphere(P(f3(3, 0, 0)), P(f3(1, 0, 0)), P(f3(3, 0, 0)), 1) - 1) < 1e-6
    assert olib.o_wray_sphere(P(f3(0, 2, 0)), P(f3(1, 0, 0)), P(f3(3, 0, 0)), 1) == 1000
    assert abs(olib.o_wray_sphere(P(f3(0, 1, 0)), P(f3(1, 0, 0)), P(f3(3, 0, 0)), 1) - 3) < 1e-6
    assert abs(olib.o_wray_box(P(f3(0, 0, 0)), P(f3(1, 0, 0)), P(f3(3, 0, 0)), P(f3(1, 1, 1))) - 2) < 1e-6
    assert olib.o_wray_box(P(f3(0, 2, 0)), P(f3(1, 0, 0)), P(f3(3, 0, 0)), P(f3(1, 1, 1))) == 1000
    assert abs(olib.o_wray_cylinder(P(f3(0, 0, 0)), P(f3(1, 0, 0)), P(f3(3, 0, 0)), 1, 1) - 2) < 1e-6
    assert abs(olib.o_wray_cylinder(P(f3(3, 0, 3)), P(f3(0, 0, -1)), P(f3(3, 0, 0)), 1, 1) - 2) < 1e-6


def test_moving_sphere_and_range_clamp(olib, layouts):
    # main.mm:122-123: moving sphere, independent collision, max range clamp.
    w = np.zeros((), layouts.WORLD)
    w["count"] = 1
    o = w["obstacles"][0]
    o["kind"] = 1
    o["center"] = (3, 0, 1.5)
    o["size"] = (0.5, 0, 0)
    o["velocity"] = (-1, 0, 0)
    assert abs(olib.o_wray(P(w), None, P(f3(0, 0, 1.5)), P(f3(1, 0, 0)), 1) - 1.5) < 1e-6
    assert olib.o_wclearance(P(w), None, P(f3(2, 0, 1.5)), 1, None) < 0
    w["count"] = 0
    assert olib.o_wray(P(w), None, P(f3(0, 0, 2.5)), P(f3(1, 0, 0)), 0) == 12


@pytest.mark.parametrize("family", list(range(17)))
def test_wgenerate_bitwise(olib, rlib, layouts, family):
    # Family 6 draws three values inside one call's argument list; g++ (which
    # built oracle/_ref) evaluates them right to left, the reference platforms
    # left to right. Pin against the g++ build with the g++ order.
    for seed in range(1, 60):
        a = np.zeros((), layouts.WORLD)
        b = np.zeros((), layouts.WORLD)
        olib.o_wgenerate(P(a), seed * 2654435761 % 2**32, family, 3.0 + (seed % 7))
        rlib.ref_wgenerate(P(b), seed * 2654435761 % 2**32, family, 3.0 + (seed % 7))
        assert a.tobytes() == b.tobytes(), (family, seed)


def test_family6_reference_platform_order(olib, layouts):
    """Left-to-right (reference platform) order differs from the g++ order only
    in the three table dimensions of family 6; every other field matches."""
    for seed in range(1, 40):
        olib.o_set_argument_order(0)
        a = np.zeros((), layouts.WORLD)
        olib.o_wgenerate(P(a), seed * 2654435761 % 2**32, 6, 5.0)
        olib.o_set_argument_order(1)
        b = np.zeros((), layouts.WORLD)
        olib.o_wgenerate(P(b), seed * 2654435761 % 2**32, 6, 5.0)
        assert a["count"] == b["count"] == 10
        # obstacles 5.. (counter, sphere, poles, low box) use later draws: identical
        assert a["obstacles"][5:].tobytes() == b["obstacles"][5:].tobytes()


def test_training_family_mixture(olib, rlib):
    for family in (0, 1, 7, 9, 12, 13):
        for seed in range(1, 200):
            r1 = np.array([seed * 747796405 % 2**32 or 1], np.uint32)
            r2 = r1.copy()
            assert olib.o_wtraining_family(family, P(r1)) == rlib.ref_wtraining_family(family, P(r2))
            assert r1[0] == r2[0]


def random_worlds(olib, layouts, count, seed):
    rng = np.random.default_rng(seed)
    worlds = np.zeros(count, layouts.WORLD)
    for i in range(count):
        olib.o_wgenerate(P(worlds[i:i + 1]), int(rng.integers(1, 2**32 - 1)), int(i % 4), float(rng.uniform(3, 8)))
        if i % 5 == 4:  # bounded moving spheres (kind 3) as in the combined courses
            for j in range(4):
                o = worlds[i]["obstacles"][8 + j] if worlds[i]["count"] >= 8 + j else None
            k = min(int(worlds[i]["count"]), 12)
            for j in range(4):
                o = worlds[i]["obstacles"][k + j]
                o["kind"] = 3
                o["center"] = rng.uniform((0, -4, 0.5), (10, 4, 4)).astype(np.float32)
                o["size"] = (rng.uniform(0.2, 0.5), rng.uniform(0.5, 2.0), rng.uniform(0, 6.28))
                v = rng.normal(size=3)
                o["velocity"] = (v / np.linalg.norm(v) * rng.uniform(0.5, 2.0)).astype(np.float32)
            worlds[i]["count"] = k + 4
    return worlds


def motion_check_world(layouts):
    """navigation_motion_check.mm:20-24: one bounded moving sphere (kind 3),
    centre (6, 0, 1.5), radius 0.28, amplitude 2.7, phase -pi/2, speed 0.8
    along y."""
    w = np.zeros((), layouts.WORLD)
    w["count"] = 1
    o = w["obstacles"][0]
    o["kind"] = 3
    o["center"] = (6, 0, 1.5)
    o["size"] = (0.28, 2.7, -1.57079632679)
    o["velocity"] = (0, 0.8, 0)
    return w


def test_bounded_mover_samples(olib, rlib, layouts):
    """The reference's bounded-motion check (navigation_motion_check.mm:19-32):
    1,001 times over 20 s; 1 m from the sphere's surface the clearance is 1
    and the depth along -x is 1.18 (gate 1e-5); restatement == reference."""
    w = motion_check_world(layouts)
    for i in range(1001):
        t = np.float32(i) * np.float32(0.02)
        c = np.zeros(3, np.float32)
        olib.o_wc(P(w["obstacles"]), t, P(c))
        point = np.array([c[0] + np.float32(0.28) + np.float32(0.18) + np.float32(1), c[1], c[2]], np.float32)
        cl = olib.o_wclearance(P(w), None, P(point), t, None)
        ray = olib.o_wray(P(w), None, P(point), P(f3(-1, 0, 0)), t)
        assert abs(cl - 1) < 1e-5 and abs(ray - 1.18) < 1e-5, (i, cl, ray)
        assert cl == rlib.ref_wclearance(P(w), P(point), t)
        assert ray == rlib.ref_wray(P(w), P(point), P(f3(-1, 0, 0)), t)


def test_world_rays_bitwise(olib, rlib, layouts):
    # main.mm:116-121 style: many worlds x 320 camera rays, CPU restatement vs reference.
    worlds = random_worlds(olib, layouts, 64, 1)
    rng = np.random.default_rng(2)
    for i in range(64):
        p = rng.uniform((-1, -3, 0.3), (9, 3, 4)).astype(np.float32)
        t = np.float32(rng.uniform(0, 5))
        q = rng.normal(size=4)
        q /= np.linalg.norm(q)
        for k in range(0, 320, 7):
            d = np.zeros(3, np.float32)
            olib.o_pixel_ray(1.0, 0.75, k, P(d))
            d2 = np.zeros(3, np.float32)
            rlib.ref_pixel_ray(1.0, 0.75, k, P(d2))
            assert np.array_equal(d, d2)
            dd = rng.normal(size=3).astype(np.float32)
            for ray in (d, dd / np.float32(np.linalg.norm(dd))):
                ray = ray.astype(np.float32)
                a = olib.o_wray(P(worlds[i:i + 1]), None, P(p), P(ray), t)
                b = rlib.ref_wray(P(worlds[i:i + 1]), P(p), P(ray), t)
                assert a == b or (np.isnan(a) and np.isnan(b))
        a = olib.o_wclearance(P(worlds[i:i + 1]), None, P(p), t, None)
        b = rlib.ref_wclearance(P(worlds[i:i + 1]), P(p), t)
        assert a == b


def test_guidance_bitwise(olib, rlib):
    rng = np.random.default_rng(3)
    for i in range(300):
        cur = rng.uniform(0.2, 12, 80).astype(np.float32)
        cur[rng.random(80) < 0.3] = 12.0
        prev = np.clip(cur + rng.normal(0, 0.3, 80), 0, 12).astype(np.float32)
        goal = rng.normal(size=3).astype(np.float32)
        vel = rng.normal(0, 1, 3).astype(np.float32)
        dist = np.float32(rng.uniform(0, 10))
        h1, h2 = np.zeros(3, np.float32), np.zeros(3, np.float32)
        olib.o_nav_guidance(P(cur), P(prev), P(goal), dist, P(vel), 0.05, 0.75, P(h1))
        rlib.ref_nav_guidance(P(cur), P(prev), P(goal), dist, P(vel), 0.05, 0.75, P(h2))
        assert np.array_equal(h1, h2), i


def test_guidance_memory_bitwise(olib, rlib):
    rng = np.random.default_rng(4)
    for i in range(40):
        cur = rng.uniform(0.2, 12, 80).astype(np.float32)
        prev = np.clip(cur + rng.normal(0, 0.3, 80), 0, 12).astype(np.float32)
        ring = rng.uniform(0.05, 12.5, 8 * 320).astype(np.float32)
        poses = np.zeros((8, 12), np.float32)
        for f in range(8):
            q = rng.normal(size=4)
            q /= np.linalg.norm(q)
            w, x, y, z = q
            poses[f, :3] = rng.uniform(-1, 1, 3)
            poses[f, 3:] = [1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
                            2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
                            2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)]
        cp = poses[int(rng.integers(0, 8))].copy()
        goal = rng.normal(size=3).astype(np.float32)
        vel = rng.normal(0, 1, 3).astype(np.float32)
        h1, h2 = np.zeros(3, np.float32), np.zeros(3, np.float32)
        args = (np.float32(rng.uniform(0.5, 9)), P(vel), 0.05, 0.75, P(ring), P(poses.ravel()), P(cp),
                int(rng.integers(0, 8)), int(rng.integers(0, 9)))
        olib.o_nav_guidance_memory(P(cur), P(prev), P(goal), *args, P(h1), 0.0)
        rlib.ref_nav_guidance_memory(P(cur), P(prev), P(goal), *args, P(h2), 0.0)
        assert np.array_equal(h1, h2), i


def test_gae_known_case(olib):
    # main.mm:286-297: T=3, N=2 with one termination and one truncation.
    r = np.array([1, 2, 3, 4, 5, 6], np.float32)
    v = np.array([.1, .2, .3, .4, .5, .6], np.float32)
    nv = np.array([.2, .3, .4, .5, .6, .7], np.float32)
    term = np.array([0, 0, 1, 0, 0, 0], np.uint8)
    trunc = np.array([0, 0, 0, 1, 0, 0], np.uint8)
    adv, ret = np.zeros(6, np.float32), np.zeros(6, np.float32)
    olib.o_compute_gae(3, 2, P(r), P(v), P(nv), P(term), P(trunc), 0.99, 0.95, P(adv), P(ret))
    # direct float64 evaluation of the same recursion
    exp_adv = np.zeros(6)
    for env in range(2):
        carry = 0.0
        for t in (2, 1, 0):
            k = t * 2 + env
            boot = 0.0 if term[k] else nv[k]
            delta = r[k] + 0.99 * boot - v[k]
            carry = delta + (0.0 if (term[k] or trunc[k]) else 0.99 * 0.95 * carry)
            exp_adv[k] = carry
    assert np.allclose(adv, exp_adv, atol=2e-5)
    assert np.allclose(ret, exp_adv + v, atol=2e-5)


def test_normalization_known_case(olib):
    # main.mm:301-314 (no-op clip radius): standardised advantages.
    x = np.array([-40, -2, -1, 0, 1, 2, 10, 40], np.float32)
    y = x.copy()
    olib.o_normalize_advantages(P(y), 8)
    m = x.mean()
    assert np.allclose(y, (x - m) / np.sqrt(((x - m) ** 2).mean() + 1e-8), atol=2e-6)


def test_ppo_operators_bitwise(olib, rlib):
    rng = np.random.default_rng(5)
    T, N = 7, 33
    r = rng.normal(size=T * N).astype(np.float32)
    v = rng.normal(size=T * N).astype(np.float32)
    nv = rng.normal(size=T * N).astype(np.float32)
    term = (rng.random(T * N) < 0.1).astype(np.uint8)
    trunc = ((rng.random(T * N) < 0.05) & (term == 0)).astype(np.uint8)
    a1, r1, a2, r2 = (np.zeros(T * N, np.float32) for _ in range(4))
    olib.o_compute_gae(T, N, P(r), P(v), P(nv), P(term), P(trunc), 0.99, 0.95, P(a1), P(r1))
    rlib.ref_compute_gae(T, N, P(r), P(v), P(nv), P(term), P(trunc), 0.99, 0.95, P(a2), P(r2))
    assert np.array_equal(a1, a2) and np.array_equal(r1, r2)
    olib.o_normalize_advantages(P(a1), a1.size)
    rlib.ref_normalize_advantages(P(a2), a2.size)
    assert np.array_equal(a1, a2)
    for i in range(200):
        act = rng.normal(size=4).astype(np.float32)
        mean = rng.normal(size=4).astype(np.float32)
        ls = rng.uniform(-2, 0.5, 4).astype(np.float32)
        old = np.float32(rng.normal(-3, 2))
        outs = [[np.zeros(4, np.float32), np.zeros(4, np.float32), np.zeros(1, np.float32), np.zeros(4, np.float32)]
                for _ in range(2)]
        args = (old, np.float32(rng.normal()), np.float32(rng.normal()), np.float32(rng.normal()), 256.0, 0.2, 0.5, 0.005)
        olib.o_sample_loss_and_grad(P(act), P(mean), P(ls), *args, *[P(x) for x in outs[0]])
        rlib.ref_sample_loss_and_grad(P(act), P(mean), P(ls), *args, *[P(x) for x in outs[1]])
        for x, y in zip(*outs):
            assert np.array_equal(x, y), i


def test_adam_known_case(olib):
    # ppo.hpp:254-266: one Adam step from zero moments.
    p = np.array([1.0], np.float32)
    g = np.array([0.25], np.float32)
    m = np.zeros(1, np.float32)
    v = np.zeros(1, np.float32)
    olib.o_adam_update(P(p), P(g), P(m), P(v), 1, olib.o_pow_correction(0.9, 1), olib.o_pow_correction(0.999, 1), 0.01)
    assert abs(m[0] - 0.1 * 0.25) < 2e-3 and abs(v[0] - 0.001 * 0.0625) < 2e-3
    assert abs(p[0] - (1 - 0.01 * (0.025 / 0.1) / (np.sqrt(0.0000625 / 0.001) + 1e-8))) < 2e-3


def test_reference_self_tests(rlib):
    assert rlib.ref_run_cpu_self_tests() == 1  # ppo.hpp:204-267 finite differences + Adam


def _compare(a, b, what):
    assert a.tobytes() == b.tobytes(), what


@pytest.mark.parametrize("family,extra", [
    (1, {}), (2, {}), (3, {}),
    (1, dict(sensor_delay=2, command_delay=2, wind=0.3)),
    (12, dict(sensor_delay=1, command_delay=1, wind=0.5, depth_noise=0.05, dropout=0.1)),
    (13, dict(geometry_memory=1, sensor_delay=2)),
    (1, dict(risk_coef=0.5, max_steps=6)),
])
def test_rollout_trace_bitwise(oracle_mod, layouts, raptor, olib, rlib, family, extra):
    """Whole policy steps of the restatement against cpu_reference::Trainer, bit for bit."""
    cfg = layouts.default_config(n=48, family=family, speed=1.0, distance=3.0, seed=7, **extra)
    T = 10
    osim = oracle_mod.OracleSim(layouts, cfg, T, raptor, lib=olib)
    ref = oracle_mod.RefTrainer(layouts, cfg, T, raptor, lib=rlib)
    for name in ("states", "runs", "worlds", "actor", "critic", "sensors", "commands"):
        _compare(osim.buf(name), ref.buf(name), ("init", name))
    for t in range(T):
        osim.step(t)
        ref.step(t)
        for name in ("states", "runs", "worlds", "sensors", "poses", "commands"):
            _compare(osim.buf(name), ref.buf(name), (t, name))
    for name in ("obs", "co", "actions", "logp", "values", "rewards", "next_values", "terminated", "truncated"):
        _compare(osim.buf(name), ref.buf(name), name)
    osim.gae(True)
    ref.lib.ref_gae_normalize(ref.h)
    _compare(osim.buf("advantages"), ref.buf("advantages"), "advantages")
    _compare(osim.buf("returns"), ref.buf("returns"), "returns")


def test_minibatch_update_bitwise(oracle_mod, layouts, raptor, olib, rlib):
    """One rollout update (2 epochs of shuffled 256-row chunks, clip + Adam) bit for bit."""
    cfg = layouts.default_config(n=40, family=1, speed=1.0, distance=3.0, seed=11)
    T = 16
    osim = oracle_mod.OracleSim(layouts, cfg, T, raptor, lib=olib)
    ref = oracle_mod.RefTrainer(layouts, cfg, T, raptor, lib=rlib)
    for t in range(T):
        osim.step(t)
        ref.step(t)
    osim.gae(True)
    ref.lib.ref_gae_normalize(ref.h)
    rows = 40 * T
    chunks = (rows + 255) // 256
    order = np.zeros(2 * chunks, np.uint32)
    rlib.ref_minibatch_order(rows, 256, 0, 2, P(order))
    steps = np.arange(1, 2 * chunks + 1)
    b1 = np.array([olib.o_pow_correction(0.9, int(s)) for s in steps], np.float32)
    b2 = np.array([olib.o_pow_correction(0.999, int(s)) for s in steps], np.float32)
    out_o, _ = osim.train_rollout(256, 2, order, b1, b2)
    out_r = np.zeros(4, np.float32)
    rlib.ref_train_rollout(ref.h, 0, P(out_r))
    _compare(osim.buf("actor"), ref.buf("actor"), "actor")
    _compare(osim.buf("critic"), ref.buf("critic"), "critic")
    for i in range(100, 104):
        _compare(osim.buf(i), ref.buf(i), ("moment", i))
    assert np.array_equal(out_o, out_r)


def test_delay_rehearsal_matches_reference_build(oracle_mod, layouts, raptor, olib):
    """NAV_DELAY_REHEARSAL (sim.metal:14-24, cpu_reference.hpp:219-223): the
    restatement's switch against cpu_reference compiled with
    -DNAV_DELAY_REHEARSAL=1 (oracle/_ref/libref_rehearsal.so), under mode 22.
    The reference's CPU sampling loop has no mode-22 action map, so the pin is
    taken where the switch acts before the action: the reset's wind, and the
    observation's sensor delay, depth noise and dropout, teacher-forced step by
    step. The command delay reads the same predicate."""
    rl = oracle_mod.load_ref(rehearsal=True)
    if rl is None:
        pytest.skip("oracle/_ref not built: the reference sources are not on this machine")
    n, T = 48, 6
    cfg = layouts.default_config(n=n, family=1, mode=22, speed=1.0, distance=3.0, seed=5, sensor_delay=2,
                                 command_delay=2, wind=0.4, depth_noise=0.05, dropout=0.1)
    osim = oracle_mod.OracleSim(layouts, cfg, T, raptor, lib=olib)
    osim.set_delay_rehearsal(True)
    osim.reset()
    ref = oracle_mod.RefTrainer(layouts, cfg, T, raptor, lib=rl)
    for name in ("states", "runs", "worlds", "sensors", "commands"):
        _compare(osim.buf(name), ref.buf(name), ("reset", name))
    clean = (np.arange(n) // 4) % 2 == 0
    wind = osim.buf("worlds")["wind"][:, 0]
    assert (wind[clean] == 0).all() and (wind[~clean] != 0).all()
    for t in range(T):
        for name in ("states", "runs", "worlds", "sensors", "poses", "commands"):
            ref.buf(name)[:] = osim.buf(name)
        osim.observe(t)
        rl.ref_step_observe(ref.h, t)
        for name in ("obs", "co"):
            width = 184 if name == "obs" else 32
            _compare(osim.buf(name).reshape(T, n, width)[t], ref.buf(name).reshape(T, n, width)[t], (t, name))
        _compare(osim.buf("sensors"), ref.buf("sensors"), (t, "sensors"))
        osim.act(t)
        osim.advance(t)
