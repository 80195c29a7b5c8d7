"""Mixed-capability distribution (family 18 = BASELINE configs 2 and 4), CPU only.

The reference has no generator for these lanes; the oracle's restatement is
checked against the stated distribution here and the CUDA generator against the
oracle bit for bit (tests/test_gpu_rollout.py, families 18-20).
"""
import numpy as np
import pytest

from conftest import load_oracle_module

ROOM_LO = np.array([-2.0, -5.0, 0.0], np.float32)
ROOM_HI = np.array([14.0, 5.0, 5.0], np.float32)


def gen(olib, layouts, family, seed):
    om = load_oracle_module()
    w = np.zeros(1, layouts.WORLD)
    olib.o_wgenerate(om.ptr(w), seed, family, 4.0)
    return w[0]


def box_sdf(p, c, e):
    k = np.abs(p - c) - e
    return np.linalg.norm(np.maximum(k, 0.0)) + min(max(k.max(), -np.inf), 0.0)


def test_lane_split(olib):
    lanes = [olib.o_mixed_lane_family(g) for g in range(16)]
    assert lanes == [17, 17, 19, 20] * 4
    counts = {f: lanes.count(f) for f in (17, 19, 20)}
    assert counts == {17: 8, 19: 4, 20: 4}  # 50 / 25 / 25 %


@pytest.mark.parametrize("seed", range(1, 40))
def test_long_goal_family(olib, layouts, seed):
    w = gen(olib, layouts, 19, seed * 7919)
    g = np.array(w["goal"])
    start = np.array([0.0, 0.0, 1.5], np.float32)
    assert w["family"] == 19 and 1 <= w["count"] <= 16
    assert -1.5 <= g[0] <= 13.5 and -4.5 <= g[1] <= 4.5 and 1.0 <= g[2] <= 2.0
    for o in w["obstacles"][: w["count"]]:
        assert o["kind"] == 0
        c, e = np.array(o["center"]), np.array(o["size"])
        assert np.all(c >= ROOM_LO) and c[0] <= 14.0 and np.all((e >= 0.2) & (e <= 1.0))
        assert box_sdf(start, c, e) > 0.5 and box_sdf(g, c, e) > 0.5


@pytest.mark.parametrize("seed", range(1, 40))
def test_combined_course_family(olib, layouts, seed):
    w = gen(olib, layouts, 20, seed * 104729)
    g = np.array(w["goal"], np.float64)
    start = np.array([0.0, 0.0, 1.5])
    obs = w["obstacles"][: w["count"]]
    statics = [o for o in obs if o["kind"] == 0]
    movers = [o for o in obs if o["kind"] == 3]
    assert len(statics) <= 12 and len(movers) <= 4 and len(statics) + len(movers) == w["count"]
    assert all(o["kind"] in (0, 3) for o in obs)
    # statics first, then movers (the generator appends movers after the boxes)
    assert [o["kind"] for o in obs] == sorted(o["kind"] for o in obs)
    for m in movers:
        radius, amplitude, phase = (float(x) for x in m["size"])
        v = np.array(m["velocity"], np.float64)
        speed = np.linalg.norm(v)
        assert 0.2 <= radius <= 0.5 and 0.5 <= amplitude <= 2.0 and 0.0 <= phase <= 6.2832
        assert 0.5 - 1e-5 <= speed <= 2.0 + 1e-5
        d = v / speed
        c = np.array(m["center"], np.float64)
        # the whole swept segment (world.hpp:32-41 keeps the sphere within
        # centre +- amplitude * direction) stays clear of the boxes
        for f in np.linspace(-amplitude, amplitude, 41):
            p = c + d * f
            for b in statics:
                assert box_sdf(p, np.array(b["center"]), np.array(b["size"])) > radius + 0.04
            assert np.linalg.norm(p - start) > radius + 0.49
            assert np.linalg.norm(p - g) > radius + 0.29


def test_movers_present_on_average(olib, layouts):
    movers = [sum(o["kind"] == 3 for o in gen(olib, layouts, 20, s)["obstacles"][: gen(olib, layouts, 20, s)["count"]])
              for s in range(1, 200)]
    assert np.mean(movers) > 2.0


def test_mixed_reset_assigns_lanes(oracle_mod, layouts, raptor):
    cfg = layouts.default_config(n=64, family=18, seed=3, sensor_delay=2, command_delay=2)
    sim = oracle_mod.OracleSim(layouts, cfg, 2, raptor)
    fam = sim.buf("worlds")["family"]
    assert list(fam[:8]) == [17, 17, 19, 20, 17, 17, 19, 20]
