"""Frozen challenge banks on the host: libmdn's JSONL loader, SHA-256 and
level sampler (csrc/bank.cpp) against the checkers.

  - the loader against oracle/bank.py (parse_level / load_split restated,
    challenge_evaluation.hpp:163-313) on the fixtures made by the reference's
    own generator (tests/golden/make_challenge_bank.py) and, when the reference
    checkout is present, on its bank files; every record check is exercised
    with a mutated record;
  - SHA-256 against hashlib;
  - the sampler against the reference's challenge_training.hpp compiled
    unmodified (oracle/_ref/libref_bank.so) and oracle/bank.py: schedules,
    failure scores and the CHTRN1 sidecar bytes over several rollouts.
"""
import copy
import ctypes
import hashlib
import json
import pathlib

import numpy as np
import pytest

from conftest import GOLDEN, REFERENCE, ROOT, _load_module, load_oracle_module, load_package

SMALL = GOLDEN / "challenge_bank_small.jsonl"
MIRRORED = GOLDEN / "challenge_bank_mirrored_small.jsonl"
REFERENCE_BANKS = REFERENCE / "evidence" / "inputs"
INVALID = 0xFFFFFFFF


def obank():
    return _load_module("mdn_oracle_bank", ROOT / "oracle" / "bank.py")


def world_hash(path):
    return json.loads(path.read_text().splitlines()[0])["world_source_sha256"]


def compare_split(path, split):
    pkg, ob = load_package(), obank()
    h = world_hash(path)
    ours = pkg.ChallengeBank(path, split, h)
    theirs, bank_hash = ob.load_split(str(path), split, h, pkg.layouts.WORLD)
    assert len(ours) == len(theirs) and ours.bank_sha256 == bank_hash
    worlds = ours.worlds()
    for i, lv in enumerate(theirs):
        assert worlds[i].tobytes() == np.array(lv["world"], pkg.layouts.WORLD).tobytes(), (path.name, split, i)
        rec = ours.level(i)
        for key in ("family", "seed", "base_seed", "environment_index", "witness_sample_count", "witness_point_count",
                    "mirrored", "line_number", "failure_id", "split", "family_name", "geometry_contract",
                    "difficulty_band", "scene_sha256", "world_source_sha256"):
            assert rec[key] == lv[key], (key, i)
        for key in ("distance", "difficulty", "direct_route_clearance_m", "witness_min_clearance_m"):
            assert np.float32(rec[key]) == np.float32(lv[key]), (key, i)
        assert np.array_equal(rec["witness_route"], lv["witness_route"])
    ours.close()
    return len(theirs)


@pytest.mark.parametrize("path", [SMALL, MIRRORED], ids=["identity", "mirrored"])
@pytest.mark.parametrize("split", ["train", "dev", "final"])
def test_loader_matches_restatement(path, split):
    assert compare_split(path, split) == 12


@pytest.mark.skipif(not REFERENCE_BANKS.exists(), reason="reference bank files not on this machine")
@pytest.mark.parametrize("name", ["challenge-bank-v1", "challenge-bank-mirrored-v1", "course-bank-v1"])
def test_reference_bank_files(name):
    total = sum(compare_split(REFERENCE_BANKS / f"{name}.jsonl", s) for s in ("train", "dev", "final"))
    assert total == len((REFERENCE_BANKS / f"{name}.jsonl").read_text().splitlines())


@pytest.mark.skipif(not (REFERENCE / "challenge_bank.py").exists(),
                    reason="reference generator not on this machine")
def test_fixtures_come_from_the_reference_generator(tmp_path):
    import importlib.util
    spec = importlib.util.spec_from_file_location("rcb", str(REFERENCE / "challenge_bank.py"))
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    h = hashlib.sha256((REFERENCE / "world.hpp").read_bytes()).hexdigest()
    records = gen.build_records(20261001, 4, 8.0, [14, 15, 16], h, False)
    text = "".join(json.dumps(r, sort_keys=True, separators=(",", ":")) + "\n" for r in records)
    assert text == SMALL.read_text()


def test_sha256_matches_hashlib(tmp_path):
    pkg = load_package()
    rng = np.random.default_rng(0)
    for size in (0, 3, 55, 56, 63, 64, 65, 119, 200_003):
        p = tmp_path / f"f{size}"
        data = rng.integers(0, 256, size, dtype=np.uint8).tobytes()
        p.write_bytes(data)
        assert pkg.sha256_file(p) == hashlib.sha256(data).hexdigest()
    with pytest.raises(pkg.MdnError):
        pkg.sha256_file(tmp_path / "missing")


# --------------------------------------------------------------- rejections
def first_record(split="train", family=14):
    for line in SMALL.read_text().splitlines():
        r = json.loads(line)
        if r["split"] == split and r["family"] == family:
            return r
    raise AssertionError




def set_obstacles(r, n):
    r["obstacles"] = [copy.deepcopy(r["obstacles"][0]) for _ in range(n)]


RECORD_CASES = [
    ("record_type", lambda r: r.update(record_type="course"), "unsupported record_type"),
    ("schema", lambda r: r.update(schema_version=2), "unsupported schema_version"),
    ("schema_float", lambda r: r.update(schema_version=1.5), "unsigned 32-bit integer"),
    ("split", lambda r: r.update(split="test"), "has invalid split"),
    ("family", lambda r: r.update(family=13), "family must be 14, 15, or 16"),
    ("family_bool", lambda r: r.update(family=True), "family must be 14, 15, or 16"),
    ("family_name", lambda r: r.update(family_name="x"), "family label/geometry contract"),
    ("transform", lambda r: r.update(coordinate_transform="rotate"), "unsupported coordinate transform"),
    ("mirror_contract", lambda r: r.update(coordinate_transform="mirror_y"), "family label/geometry contract"),
    ("seed", lambda r: r.update(seed=(r["seed"] + 1) & 0xFFFFFFFF), "seed does not match"),
    ("difficulty", lambda r: r.update(difficulty=1.0), "difficulty must be in [0,1)"),
    ("difficulty_range", lambda r: r.update(difficulty=1e39), "outside float32 range"),
    ("band", lambda r: r.update(difficulty_band="easy" if r["difficulty_band"] != "easy" else "hard"),
     "difficulty band does not match"),
    ("band_name", lambda r: r.update(difficulty_band="tough"), "invalid difficulty_band"),
    ("scene_hash", lambda r: r.update(scene_sha256="ABC"), "malformed source hashes"),
    ("config_index", lambda r: r["sim_config"].update(environment_index=r["environment_index"] + 1),
     "sim_config does not match"),
    ("distance", lambda r: r["sim_config"].update(distance=11.0), "distance must be in [3,10]"),
    ("room", lambda r: r["room_bounds"].update(x=[-3.0, 14.0]), "room bounds incompatible"),
    ("room_pair", lambda r: r["room_bounds"].update(z=[0.0]), "axis must have two values"),
    ("goal_len", lambda r: r.update(goal=r["goal"][:2]), "must contain exactly 3 values"),
    ("goal_type", lambda r: r.update(goal="north"), "must be an array"),
    ("goal_missing", lambda r: r.pop("goal"), "missing field goal"),
    ("body", lambda r: r.update(body_radius_m=0.2), "body radius differs"),
    ("too_many", lambda r: set_obstacles(r, 17), "more than 16 obstacles"),
    ("kind", lambda r: r["obstacles"][0].update(kind=3), "obstacle kind must be"),
    ("negative", lambda r: r["obstacles"][0].update(half_extent=[-0.1, 1.0, 1.0]), "size cannot be negative"),
    ("zero", lambda r: r["obstacles"][0].update(half_extent=[0.0, 1.0, 1.0]), "non-positive collision dimension"),
    ("outside", lambda r: r["obstacles"][0].update(center=[13.9, 0.0, 2.5]), "outside the fixed room bounds"),
    ("unsafe", lambda r: r["obstacles"].append(
        {"kind": 1, "center": [0.0, 0.0, 1.5], "half_extent": [0.3, 0.0, 0.0], "velocity": [0.0, 0.0, 0.0]}),
     "unsafe start or goal"),
    ("direct", lambda r: r.update(direct_route_clearance_m=0.0), "obstructed-route/witness-clearance contract"),
    ("samples", lambda r: r.update(witness_sample_count=0), "obstructed-route/witness-clearance contract"),
    ("route_short", lambda r: r.update(witness_route=r["witness_route"][:1]), "needs at least two points"),
    ("route_end", lambda r: r["witness_route"][-1].__setitem__(0, r["witness_route"][-1][0] + 0.01),
     "endpoints do not match"),
]


def write_bank(path, lines):
    path.write_text("".join(line + "\n" for line in lines))
    return path


def expect_both(path, split, h, needle):
    pkg, ob = load_package(), obank()
    with pytest.raises(pkg.MdnError) as ours:
        pkg.ChallengeBank(path, split, h)
    assert needle in str(ours.value), str(ours.value)
    with pytest.raises((ob.BankError, OSError)) as theirs:
        ob.load_split(str(path), split, h, pkg.layouts.WORLD)
    assert needle in str(theirs.value) or isinstance(theirs.value, OSError), str(theirs.value)


@pytest.mark.parametrize("name,mutate,needle", RECORD_CASES, ids=[c[0] for c in RECORD_CASES])
def test_record_checks(tmp_path, name, mutate, needle):
    r = first_record()
    mutate(r)
    path = write_bank(tmp_path / "bank.jsonl", [json.dumps(r)])
    expect_both(path, "train", world_hash(SMALL), needle)


def test_file_checks(tmp_path):
    h = world_hash(SMALL)
    lines = SMALL.read_text().splitlines()
    expect_both(write_bank(tmp_path / "a", lines[:2]), "train", "0" * 64, "hash does not match")
    expect_both(write_bank(tmp_path / "b", [lines[0], "", lines[1]]), "train", h, "blank JSONL row at line 2")
    expect_both(write_bank(tmp_path / "c", [lines[0], "{"]), "train", h, "invalid JSON object at line 2")
    expect_both(write_bank(tmp_path / "d", [lines[0], "[1, 2]"]), "train", h, "invalid JSON object at line 2")
    expect_both(write_bank(tmp_path / "e", [lines[0], lines[0]]), "train", h, "duplicate failure_id")
    expect_both(write_bank(tmp_path / "f", lines[:2]), "test", h, "split must be train, dev, or final")
    train_only = [x for x in lines if json.loads(x)["split"] == "train"]
    expect_both(write_bank(tmp_path / "g", train_only), "dev", h, "no records for requested split dev")
    pkg = load_package()
    with pytest.raises(pkg.MdnError):
        pkg.ChallengeBank(tmp_path / "missing.jsonl", "train", h)
    # Whitespace and key order inside a row do not matter; CRLF line ends are whitespace.
    r = json.loads(lines[0])
    crlf = tmp_path / "h"
    crlf.write_bytes((json.dumps(r, indent=1).replace("\n", " ") + "\r\n").encode())
    assert len(pkg.ChallengeBank(crlf, "train", h)) == 1


# --------------------------------------------------------------- sampler
SETTINGS = [
    dict(selection=0, rehearsal_environments=0, focus_family=0),
    dict(selection=1, rehearsal_environments=2, focus_family=0),
    dict(selection=1, rehearsal_environments=0, focus_family=15, uniform_floor=0.75, score_staleness_mix=0.25),
    dict(selection=0, rehearsal_environments=3, focus_family=16, sampler_seed=0),
    dict(selection=1, rehearsal_environments=1, focus_family=0, uniform_floor=0.5, score_staleness_mix=1.0,
         sampler_seed=987654321),
]


def evidence(schedule, active, H, rng):
    """Rollout evidence consistent with a schedule: an env that ends its
    episode at tick t plays schedule slot t + 1 from the next tick."""
    E = schedule.shape[0]
    ids = np.zeros((H, E), np.uint32)
    term = np.zeros((H, E), np.uint8)
    trunc = np.zeros((H, E), np.uint8)
    active = active.copy()
    for t in range(H):
        for e in range(E):
            ids[t, e] = active[e]
            if rng.random() < 0.3:
                (term if rng.random() < 0.7 else trunc)[t, e] = 1
                active[e] = schedule[e, t + 1]
    gae = rng.normal(0.0, 1.5, (H, E)).astype(np.float32)
    return gae, term, trunc, ids, active


class RefSampler:
    """The reference's ChallengeTraining through oracle/_ref/libref_bank.so."""

    def __init__(self, lib, level_file, world_hash, E, H, s):
        self.lib, self.E, self.H = lib, E, H
        u = np.array([E, H, s.get("sampler_seed", 1), s.get("rehearsal_environments", 0), s.get("selection", 0),
                      s.get("focus_family", 0)], np.uint32)
        h = ctypes.c_void_p()
        self.ok(lib.refb_create(str(level_file).encode(), world_hash.encode(), u.ctypes.data,
                                s.get("uniform_floor", 0.5), s.get("score_staleness_mix", 0.5), ctypes.byref(h)))
        self.h = h

    def ok(self, rc):
        if rc != 0:
            raise RuntimeError(self.lib.refb_error().decode())

    def initial(self):
        out = np.zeros((self.E, self.H + 1), np.uint32)
        self.ok(self.lib.refb_initial_schedule(self.h, out.ctypes.data))
        return out

    def next(self, active, rollout):
        out = np.zeros((self.E, self.H + 1), np.uint32)
        a = np.ascontiguousarray(active, np.uint32)
        self.ok(self.lib.refb_next_schedule(self.h, a.ctypes.data, self.E, rollout, out.ctypes.data))
        return out

    def observe(self, gae, term, trunc, ids, rollout):
        self.ok(self.lib.refb_observe(self.h, gae.ctypes.data, term.ctypes.data, trunc.ctypes.data, ids.ctypes.data,
                                      rollout))

    def level(self, i):
        score, done = np.zeros(1, np.float32), np.zeros(1, np.uint64)
        self.ok(self.lib.refb_level(self.h, i, score.ctypes.data, done.ctypes.data))
        return score[0], int(done[0])

    def save(self, path, ckpt, completed, active):
        a = np.ascontiguousarray(active, np.uint32)
        self.ok(self.lib.refb_save(self.h, str(path).encode(), ckpt.encode(), completed, a.ctypes.data, self.E))

    def close(self):
        self.lib.refb_destroy(self.h)


def all_levels(path, h):
    pkg, ob = load_package(), obank()
    levels = []
    for split in ("train", "dev", "final"):
        levels += ob.load_split(str(path), split, h, pkg.layouts.WORLD)[0]
    return sorted(levels, key=lambda lv: lv["line_number"])


@pytest.mark.parametrize("case", range(len(SETTINGS)))
def test_sampler_matches_reference(tmp_path, case):
    pkg, ob = load_package(), obank()
    s = SETTINGS[case]
    E, H = 11, 6
    h = world_hash(SMALL)
    levels, bank_hash = ob.load_split(str(SMALL), "train", h, pkg.layouts.WORLD)
    ours = pkg.ChallengeSampler(SMALL, h, environment_count=E, horizon=H, **s)
    port = ob.ChallengeTraining(levels, bank_hash, h, environment_count=E, horizon=H, **s)
    rlib = load_oracle_module().load_ref_bank()
    ref = None
    if rlib is not None:
        level_file = tmp_path / "levels.bin"
        ob.write_level_file(level_file, all_levels(SMALL, h), bank_hash, pkg.layouts.WORLD)
        ref = RefSampler(rlib, level_file, h, E, H, s)
    try:
        assert tuple(ours.control().tolist()) == port.control() == (1, 12, H + 1, H)
        rng = np.random.default_rng(case)
        sched = ours.initial_schedule()
        assert np.array_equal(sched, port.initial_schedule())
        if ref:
            assert np.array_equal(sched, ref.initial())
        R = s.get("rehearsal_environments", 0)
        assert np.all(sched[:R] == INVALID) and np.all(sched[R:] < 12)
        active = sched[:, 0].copy()
        assert np.array_equal(ours.active_ids(), active)
        for rollout in range(5):
            if rollout:
                sched = ours.next_schedule(active, rollout)
                assert np.array_equal(sched, port.next_schedule(active, rollout)), rollout
                if ref:
                    assert np.array_equal(sched, ref.next(active, rollout)), rollout
                assert np.array_equal(sched[:, 0], active)
            gae, term, trunc, ids, active = evidence(sched, active, H, rng)
            ours.observe_raw_gae(gae, term, trunc, ids, rollout)
            port.observe_raw_gae(gae, term, trunc, ids, rollout)
            if ref:
                ref.observe(gae, term, trunc, ids, rollout)
            for lvl in range(12):
                score, done, visit = ours.level_stats(lvl)
                assert np.float32(score) == port.scores[lvl] and done == port.completed[lvl], (rollout, lvl)
                assert visit == port.last_visit[lvl]
                if ref:
                    assert (np.float32(score), done) == ref.level(lvl), (rollout, lvl)
        if s.get("selection") == 1:
            assert port.completed.sum() > 0
        ckpt = hashlib.sha256(b"checkpoint").hexdigest()
        ours.save_state(tmp_path / "ours" / "replay.state", ckpt, 5, active)
        data = (tmp_path / "ours" / "replay.state").read_bytes()
        assert len(data) == 256 + 12 * (4 + 8 * 3) + E * (8 + 4 * 3)
        assert data == port.state_bytes(ckpt, 5, active)
        if ref:
            ref.save(tmp_path / "ref.state", ckpt, 5, active)
            assert data == (tmp_path / "ref.state").read_bytes()
        # Resume: a fresh sampler restores the ids and continues identically.
        again = pkg.ChallengeSampler(SMALL, h, environment_count=E, horizon=H, **s)
        assert np.array_equal(again.load_state(tmp_path / "ours" / "replay.state", ckpt, 5), active)
        assert np.array_equal(again.next_schedule(active, 5), ours.next_schedule(active, 5))
        with pytest.raises(pkg.MdnError):
            again.load_state(tmp_path / "ours" / "replay.state", hashlib.sha256(b"other").hexdigest(), 5)
        with pytest.raises(pkg.MdnError):
            again.load_state(tmp_path / "ours" / "replay.state", ckpt, 4)
        (tmp_path / "short.state").write_bytes(data[:-1])
        with pytest.raises(pkg.MdnError):
            again.load_state(tmp_path / "short.state", ckpt, 5)
        (tmp_path / "long.state").write_bytes(data + b"\0")
        with pytest.raises(pkg.MdnError):
            again.load_state(tmp_path / "long.state", ckpt, 5)
        again.close()
    finally:
        ours.close()
        if ref:
            ref.close()


def test_sampler_rejections(tmp_path):
    pkg = load_package()
    h = world_hash(SMALL)
    for bad in (dict(environment_count=0), dict(horizon=0), dict(environment_count=2),
                dict(environment_count=5, rehearsal_environments=3), dict(focus_family=13), dict(selection=2),
                dict(uniform_floor=0.4), dict(score_staleness_mix=1.5)):
        with pytest.raises(pkg.MdnError):
            pkg.ChallengeSampler(SMALL, h, **bad)
    s = pkg.ChallengeSampler(SMALL, h, environment_count=6, horizon=4, rehearsal_environments=1)
    sched = s.initial_schedule()
    active = sched[:, 0].copy()
    wrong = active.copy()
    wrong[1] = wrong[2]  # env 1 plays family 14, env 2 family 15
    with pytest.raises(pkg.MdnError, match="family quota"):
        s.next_schedule(wrong, 1)
    rehearsal = active.copy()
    rehearsal[0] = active[1]
    with pytest.raises(pkg.MdnError, match="rehearsal environment"):
        s.next_schedule(rehearsal, 1)
    ids = np.tile(active, (4, 1))
    ids[2, 3] = active[3] + 3 if active[3] + 3 < 12 else active[3] - 3
    z = np.zeros((4, 6), np.uint8)
    with pytest.raises(pkg.MdnError, match="changed before episode completion"):
        s.observe_raw_gae(np.ones((4, 6), np.float32), z, z, ids, 0)
    bad_gae = np.ones((4, 6), np.float32)
    bad_gae[0, 4] = np.nan
    s2 = pkg.ChallengeSampler(SMALL, h, environment_count=6, horizon=4, rehearsal_environments=1)
    s2.initial_schedule()
    with pytest.raises(pkg.MdnError, match="non-finite"):
        s2.observe_raw_gae(bad_gae, z, z, np.tile(active, (4, 1)), 0)
    with pytest.raises(pkg.MdnError, match="SHA-256"):
        s.save_state(tmp_path / "x", "short", 1, active)
    missing = tmp_path / "bank_without_16.jsonl"
    write_bank(missing, [x for x in SMALL.read_text().splitlines() if json.loads(x)["family"] != 16])
    with pytest.raises(pkg.MdnError, match="must contain each family 14, 15, and 16"):
        pkg.ChallengeSampler(missing, h)
    s.close()
    s2.close()
