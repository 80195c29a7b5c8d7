"""Pin the goal-arrival task contract of the C restatement to the reference.

navigation_tasks.hpp is compiled unmodified into oracle/_ref; its generator
(:343-482), physical start (:486-495), step reward/termination (:499-548) and
segment clearance (:240-252) are compared with the restatement bit for bit,
and libmdn's mdn_task_settings with navigation_task_default_config plus the
overrides of navigation_training::task_settings (navigation_training.hpp:7-14).
CPU only.
"""
import numpy as np
import pytest

from conftest import load_package

P = None

# (stage, family): open and hold use family 0, clutter its five static families.
CASES = [(0, 0), (1, 0), (2, 1), (2, 2), (2, 4), (2, 5), (2, 12)]


@pytest.fixture(scope="module", autouse=True)
def _ptr(oracle_mod, olib):
    global P
    P = oracle_mod.ptr
    # oracle/_ref is a g++ build: g++ evaluates the draws inside the wv(...)
    # argument lists of the generators right to left; compare like with like.
    olib.o_set_argument_order(1)
    yield
    olib.o_set_argument_order(0)


def _ref_config(rlib, layouts, stage, family, difficulty):
    c = np.zeros((), layouts.TASK_CONFIG)
    assert rlib.ref_task_default_config(stage, family, difficulty, P(c)) == 1
    return c


@pytest.mark.parametrize("stage,family", CASES)
def test_task_settings_match_reference(rlib, layouts, stage, family):
    capi_mod = load_package().capi
    for difficulty in (0.0, 0.35, 1.0):
        ref = _ref_config(rlib, layouts, stage, family, difficulty)
        # navigation_training::task_settings overrides
        ref["time_cost_per_s"] = np.float32(0.2)
        ref["command_smoothness_weight"] = np.float32(0.05)
        ref["initial_speed_max_mps"] = np.float32(0.5 if stage == 1 else 1.0)
        mine = capi_mod.task_settings(stage, family, difficulty)
        assert mine.tobytes() == ref.tobytes(), (stage, family, difficulty)


@pytest.mark.parametrize("stage,family", CASES)
def test_generate_task_bitwise(olib, rlib, layouts, stage, family):
    for difficulty in (0.0, 0.5, 1.0):
        cfg = _ref_config(rlib, layouts, stage, family, difficulty)
        cfg["initial_speed_max_mps"] = np.float32(1.0)
        for seed in range(24):
            rng0 = np.uint32(seed * 2654435761 % 2**32 ^ 0x9e3779b9)
            wo, wr = np.zeros((), layouts.WORLD), np.zeros((), layouts.WORLD)
            to, tr = np.zeros((), layouts.TASK_STATE), np.zeros((), layouts.TASK_STATE)
            ro, rr = np.array([rng0], np.uint32), np.array([rng0], np.uint32)
            so = olib.o_generate_task(P(wo), P(to), P(ro), P(cfg), None)
            sr = rlib.ref_generate_task(P(wr), P(tr), P(rr), P(cfg))
            assert so == sr, (stage, family, seed)
            assert to.tobytes() == tr.tobytes(), (stage, family, seed, to, tr)
            assert wo.tobytes() == wr.tobytes(), (stage, family, seed)
            assert ro[0] == rr[0]
            if so == 4:
                so_, sr_ = np.zeros((), layouts.STATE), np.zeros((), layouts.STATE)
                olib.o_task_apply_start(P(to), P(so_))
                rlib.ref_task_apply_start(P(tr), P(sr_))
                assert so_.tobytes() == sr_.tobytes()


def test_generation_mostly_ready(olib, rlib, layouts):
    """The default recipes almost always produce a task within the attempt bound."""
    for stage, family in CASES:
        cfg = _ref_config(rlib, layouts, stage, family, 0.5)
        ready = 0
        for seed in range(32):
            w, t = np.zeros((), layouts.WORLD), np.zeros((), layouts.TASK_STATE)
            rng = np.array([seed * 747796405 % 2**32], np.uint32)
            ready += olib.o_generate_task(P(w), P(t), P(rng), P(cfg), None) == 4
        assert ready >= 30, (stage, family, ready)


def test_invalid_configs_rejected_like_reference(olib, rlib, layouts):
    base = _ref_config(rlib, layouts, 2, 1, 0.5)
    mutations = [
        ("generation_version", 2), ("family", 3), ("goal_radius_m", 0.0), ("scene_distance_m", 11.0),
        ("max_nav_steps", 0), ("minimum_endpoint_clearance_m", 0.1), ("difficulty", 1.5),
    ]
    for field, value in mutations:
        cfg = base.copy()
        cfg[field] = value
        wo, wr = np.zeros((), layouts.WORLD), np.zeros((), layouts.WORLD)
        to, tr = np.zeros((), layouts.TASK_STATE), np.zeros((), layouts.TASK_STATE)
        ro, rr = np.array([5], np.uint32), np.array([5], np.uint32)
        so = olib.o_generate_task(P(wo), P(to), P(ro), P(cfg), None)
        sr = rlib.ref_generate_task(P(wr), P(tr), P(rr), P(cfg))
        assert so == sr and so in (1, 5), (field, so, sr)
        assert to.tobytes() == tr.tobytes(), field
    cfg = base.copy()
    cfg["goal_max_xyz"][0] = 14.0  # goal box leaves the room by less than the endpoint clearance
    t = np.zeros((), layouts.TASK_STATE)
    assert olib.o_generate_task(P(np.zeros((), layouts.WORLD)), P(t), P(np.array([1], np.uint32)), P(cfg), None) == 1


def test_task_step_bitwise(olib, rlib, layouts):
    rng = np.random.default_rng(3)
    for stage, family in CASES:
        cfg = _ref_config(rlib, layouts, stage, family, 0.5)
        cfg["max_nav_steps"] = 40
        w = np.zeros((), layouts.WORLD)
        task = np.zeros((), layouts.TASK_STATE)
        r = np.array([17], np.uint32)
        assert olib.o_generate_task(P(w), P(task), P(r), P(cfg), None) == 4
        to, tr = task.copy(), task.copy()
        goal = task["goal_position"].astype(np.float32)
        for k in range(60):
            # approach the goal, then hover inside it slowly (stable hold), with contacts late
            frac = np.float32(min(1.0, k / 20.0))
            pos = (task["start_position"] * (1 - frac) + goal * frac + rng.normal(0, 0.02, 3)).astype(np.float32)
            vel = rng.normal(0, 0.2 if k > 20 else 1.0, 3).astype(np.float32)
            cmd = rng.normal(0, 0.5, 4).astype(np.float32)
            contact = int(k == 55)
            timeout = int(k == 58)
            oo, orr = np.zeros(8, np.uint32), np.zeros(8, np.uint32)
            olib.o_task_step(P(to), P(cfg), P(pos), P(vel), P(cmd), contact, timeout, P(oo))
            rlib.ref_task_step(P(tr), P(cfg), P(pos), P(vel), P(cmd), contact, timeout, P(orr))
            assert oo.tobytes() == orr.tobytes(), (stage, family, k)
            assert to.tobytes() == tr.tobytes(), (stage, family, k)
        assert tr["terminal"] == 1


def test_segment_clearance_bitwise(olib, rlib, layouts):
    rng = np.random.default_rng(5)
    for family in (1, 2, 4, 5):
        w = np.zeros((), layouts.WORLD)
        olib.o_wgenerate(P(w), 1234 + family, family, np.float32(8.0))
        for _ in range(20):
            a = rng.uniform([-1, -4, 0.5], [13, 4, 4.5]).astype(np.float32)
            b = rng.uniform([-1, -4, 0.5], [13, 4, 4.5]).astype(np.float32)
            co = olib.o_task_segment_clearance(P(w), None, P(a), P(b))
            cr = rlib.ref_task_segment_clearance(P(w), P(a), P(b))
            assert np.float32(co).tobytes() == np.float32(cr).tobytes()
