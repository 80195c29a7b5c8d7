"""TEST INFRASTRUCTURE ONLY: a Python restatement of the reference's frozen
challenge-bank host code, the checker for libmdn's C++ version (csrc/bank.cpp).

  load_split        challenge_evaluation::load_split / parse_level
                    (challenge_evaluation.hpp:163-313), JSON read with the
                    standard json module, numbers rounded to float32 as the
                    reference's required_float does (:135-139).
  ChallengeTraining challenge_training::ChallengeTraining
                    (challenge_training.hpp:53-427): schedules, failure scores,
                    the CHTRN1 sidecar.

Pinned: the sampler against the reference's own challenge_training.hpp
compiled unmodified (oracle/_ref/libref_bank.so); the loader against the
reference's bank files and generator (challenge_bank.py) through the fixtures
in tests/golden. The reference's own JSONL reader needs Foundation and is not
built here. Only tests/ may import this module.
"""
import hashlib
import json
import math
import os
import struct

import numpy as np

F32_MAX = float(np.finfo(np.float32).max)
ENV_STRIDE, ENV_OFFSET = 747796405, 2891336453
INVALID = 0xFFFFFFFF
MASK = 0xFFFFFFFF


class BankError(ValueError):
    pass


def fail(message):
    raise BankError("challenge bank: " + message)


def f32(x):
    return float(np.float32(x))


def _field(obj, name, where):
    if name not in obj:
        fail(f"{where} missing field {name}")
    return obj[name]


def _obj(v, where):
    if not isinstance(v, dict):
        fail(f"{where} must be an object")
    return v


def _arr(v, where):
    if not isinstance(v, list):
        fail(f"{where} must be an array")
    return v


def _str(v, where):
    if not isinstance(v, str):
        fail(f"{where} must be a string")
    return v


def _num(v, where):
    # NSJSONSerialization yields NSNumber for booleans too.
    if isinstance(v, bool):
        v = 1.0 if v else 0.0
    if not isinstance(v, (int, float)):
        fail(f"{where} must be a number")
    v = float(v)
    if not math.isfinite(v):
        fail(f"{where} must be finite")
    return v


def _uint(v, where):
    n = _num(v, where)
    if n < 0 or n > 4294967295.0 or math.floor(n) != n:
        fail(f"{where} must be an unsigned 32-bit integer")
    return int(n)


def _float(v, where):
    n = _num(v, where)
    if abs(n) > F32_MAX:
        fail(f"{where} is outside float32 range")
    return f32(n)


def _vec3(v, where):
    a = _arr(v, where)
    if len(a) != 3:
        fail(f"{where} must contain exactly 3 values")
    return [_float(a[k], f"{where}[{k}]") for k in range(3)]


def _clearance(world, p):
    """wclearance at t = 0 for kinds 0-2 (world.hpp:84-99), float32 steps."""
    F = np.float32
    p = [F(x) for x in p]
    best = min(min(p[0] + F(2), F(14) - p[0]), min(min(p[1] + F(5), F(5) - p[1]), min(p[2], F(5) - p[2]))) - F(0.18)
    for o in world["obstacles"][: int(world["count"])]:
        q = [p[k] - (F(o["center"][k]) + F(0) * F(o["velocity"][k])) for k in range(3)]
        s = [F(x) for x in o["size"]]
        if o["kind"] == 1:
            d = F(np.sqrt(q[0] * q[0] + q[1] * q[1] + q[2] * q[2])) - s[0]
        elif o["kind"] == 2:
            a = F(np.sqrt(q[0] * q[0] + q[1] * q[1])) - s[0]
            b = F(abs(q[2])) - s[2]
            d = F(np.sqrt(max(a, F(0)) * max(a, F(0)) + max(b, F(0)) * max(b, F(0)))) + min(max(a, b), F(0))
        else:
            k = [F(abs(q[j])) - s[j] for j in range(3)]
            m = [max(x, F(0)) for x in k]
            d = F(np.sqrt(m[0] * m[0] + m[1] * m[1] + m[2] * m[2])) + min(max(k[0], max(k[1], k[2])), F(0))
        best = min(best, F(d - F(0.18)))
    return best


FAMILY_NAMES = {14: "bent_hallway_corner", 15: "connected_rooms_offset_doors_furniture",
                16: "vertical_over_under_choice"}


def parse_level(record, line_number, world_dtype):
    """One JSONL record -> dict with the level's fields and its WWorld."""
    where = f"JSONL line {line_number}"
    if _str(_field(record, "record_type", where), where + ".record_type") != "challenge":
        fail(where + " has an unsupported record_type")
    if _uint(_field(record, "schema_version", where), where + ".schema_version") != 1:
        fail(where + " has an unsupported schema_version")
    lv = {"line_number": line_number}
    lv["failure_id"] = _str(_field(record, "failure_id", where), where + ".failure_id")
    lv["split"] = _str(_field(record, "split", where), where + ".split")
    if lv["split"] not in ("train", "dev", "final"):
        fail(where + " has invalid split")
    fam = lv["family"] = _uint(_field(record, "family", where), where + ".family")
    if fam < 14 or fam > 16:
        fail(where + " family must be 14, 15, or 16")
    lv["family_name"] = _str(_field(record, "family_name", where), where + ".family_name")
    lv["geometry_contract"] = _str(_field(record, "geometry_contract", where), where + ".geometry_contract")
    transform = _str(record["coordinate_transform"], where + ".coordinate_transform") \
        if "coordinate_transform" in record else "identity"
    mirrored = transform == "mirror_y"
    if transform != "identity" and not mirrored:
        fail(where + " unsupported coordinate transform")
    lv["mirrored"] = int(mirrored)
    corner = ("connected partitions force south turn, east hall, then north turn" if mirrored
              else "connected partitions force north turn, east hall, then south turn")
    contract = {14: corner, 15: "offset doors with intermediate table detour",
                16: "cross low barrier above, overhang below, then choose over or under slab"}[fam]
    if lv["family_name"] != FAMILY_NAMES[fam] or lv["geometry_contract"] != contract:
        fail(where + " family label/geometry contract does not match its family id")
    lv["seed"] = _uint(_field(record, "seed", where), where + ".seed")
    lv["environment_index"] = _uint(_field(record, "environment_index", where), where + ".environment_index")
    lv["difficulty"] = _float(_field(record, "difficulty", where), where + ".difficulty")
    if lv["difficulty"] < 0 or lv["difficulty"] >= 1:
        fail(where + " difficulty must be in [0,1)")
    lv["difficulty_band"] = _str(_field(record, "difficulty_band", where), where + ".difficulty_band")
    if lv["difficulty_band"] not in ("easy", "medium", "hard"):
        fail(where + " has invalid difficulty_band")
    d = np.float32(lv["difficulty"])
    band = "easy" if d < np.float32(1.0) / np.float32(3.0) else "medium" if d < np.float32(2.0) / np.float32(3.0) \
        else "hard"
    if lv["difficulty_band"] != band:
        fail(where + " difficulty band does not match its difficulty value")
    lv["scene_sha256"] = _str(_field(record, "scene_sha256", where), where + ".scene_sha256")
    lv["world_source_sha256"] = _str(_field(record, "world_source_sha256", where), where + ".world_source_sha256")
    hexd = set("0123456789abcdef")
    if not all(len(h) == 64 and set(h) <= hexd for h in (lv["scene_sha256"], lv["world_source_sha256"])):
        fail(where + " has malformed source hashes")
    cfg = _obj(_field(record, "sim_config", where), where + ".sim_config")
    if _uint(_field(cfg, "family", where), where + ".sim_config.family") != fam or \
            _uint(_field(cfg, "environment_index", where), where + ".sim_config.environment_index") != \
            lv["environment_index"]:
        fail(where + " sim_config does not match record family/index")
    lv["base_seed"] = _uint(_field(cfg, "seed", where), where + ".sim_config.seed")
    lv["distance"] = _float(_field(cfg, "distance", where), where + ".sim_config.distance")
    if lv["distance"] < 3.0 or lv["distance"] > 10.0:
        fail(where + " distance must be in [3,10]")
    st = (lv["base_seed"] + lv["environment_index"] * ENV_STRIDE + ENV_OFFSET) & MASK
    st ^= (st << 13) & MASK
    st ^= st >> 17
    st ^= (st << 5) & MASK
    if st != lv["seed"]:
        fail(where + " seed does not match simulator environment seed derivation")
    bounds = _obj(_field(record, "room_bounds", where), where + ".room_bounds")
    for axis, (lo_e, hi_e) in zip("xyz", ((-2, 14), (-5, 5), (0, 5))):
        pair = _arr(_field(bounds, axis, where + ".room_bounds"), where + ".room_bounds")
        if len(pair) != 2:
            fail(where + ".room_bounds axis must have two values")
        lo = np.float32(_float(pair[0], where + ".room_bounds lower"))
        hi = np.float32(_float(pair[1], where + ".room_bounds upper"))
        if abs(lo - np.float32(lo_e)) > np.float32(1e-5) or abs(hi - np.float32(hi_e)) > np.float32(1e-5):
            fail(where + " uses room bounds incompatible with world.hpp")
    goal = _vec3(_field(record, "goal", where), where + ".goal")
    wind = _vec3(_field(record, "wind", where), where + ".wind")
    if abs(_num(_field(record, "body_radius_m", where), where + ".body_radius_m") - 0.18) > 1e-5:
        fail(where + " body radius differs from simulator collision model")
    w = np.zeros((), world_dtype)
    w["family"], w["seed"], w["goal"], w["wind"] = fam, lv["seed"], goal, wind
    obstacles = _arr(_field(record, "obstacles", where), where + ".obstacles")
    if len(obstacles) > 16:
        fail(where + " contains more than 16 obstacles")
    w["count"] = len(obstacles)
    for i, ob in enumerate(obstacles):
        ob = _obj(ob, where + ".obstacles[]")
        kind = _uint(_field(ob, "kind", where), where + ".obstacle.kind")
        if kind > 2:
            fail(where + " obstacle kind must be AABB(0), sphere(1), or cylinder(2)")
        c = _vec3(_field(ob, "center", where), where + ".obstacle.center")
        s = _vec3(_field(ob, "half_extent", where), where + ".obstacle.half_extent")
        v = _vec3(_field(ob, "velocity", where), where + ".obstacle.velocity")
        if any(x < 0 for x in s):
            fail(where + " obstacle size cannot be negative")
        o = w["obstacles"][i]
        o["kind"], o["center"], o["size"], o["velocity"] = kind, c, s, v
        if (kind == 0 and min(s) <= 0) or (kind == 1 and s[0] <= 0) or (kind == 2 and (s[0] <= 0 or s[2] <= 0)):
            fail(where + " obstacle has a non-positive collision dimension")
        F = np.float32
        for axis, (lo, hi) in enumerate(((-2.0, 14.0), (-5.0, 5.0), (0.0, 5.0))):
            ext = s[axis] if kind == 0 else s[0] if kind == 1 else (s[2] if axis == 2 else s[0])
            if F(c[axis]) - F(ext) < F(lo) - F(1e-4) or F(c[axis]) + F(ext) > F(hi) + F(1e-4):
                fail(where + " obstacle extends outside the fixed room bounds")
    start = [0.0, 0.0, 1.5]
    if _clearance(w, start) <= np.float32(0.04) or _clearance(w, goal) <= np.float32(0.04):
        fail(where + " has an unsafe start or goal for the 0.18 m vehicle")
    lv["direct_route_clearance_m"] = _float(_field(record, "direct_route_clearance_m", where),
                                            where + ".direct_route_clearance_m")
    lv["witness_min_clearance_m"] = _float(_field(record, "witness_min_clearance_m", where),
                                           where + ".witness_min_clearance_m")
    lv["witness_sample_count"] = _uint(_field(record, "witness_sample_count", where), where + ".witness_sample_count")
    if lv["direct_route_clearance_m"] >= np.float32(-0.02) or lv["witness_min_clearance_m"] <= np.float32(0.04) or \
            lv["witness_sample_count"] == 0:
        fail(where + " does not satisfy the stored obstructed-route/witness-clearance contract")
    route = _arr(_field(record, "witness_route", where), where + ".witness_route")
    if len(route) < 2:
        fail(where + " witness_route needs at least two points")
    pts = np.array([_vec3(p, where + ".witness_route[]") for p in route], np.float32)
    F = np.float32
    if any(abs(pts[0, a] - F(start[a])) > F(1e-5) or abs(pts[-1, a] - F(goal[a])) > F(1e-5) for a in range(3)):
        fail(where + " witness route endpoints do not match the simulator start and stored goal")
    lv["witness_route"] = pts
    lv["witness_point_count"] = len(route)
    lv["world"] = w
    return lv


def load_split(path, split, expected_world_hash, world_dtype):
    """Levels of one split and the file's SHA-256 (load_split, :282-313)."""
    if split not in ("train", "dev", "final"):
        fail("split must be train, dev, or final")
    with open(path, "rb") as f:
        raw = f.read()
    bank_hash = hashlib.sha256(raw).hexdigest()
    selected, ids = [], set()
    lines = raw.split(b"\n")
    if lines and lines[-1] == b"":
        lines.pop()
    for number, line in enumerate(lines, 1):
        if not line:
            fail(f"blank JSONL row at line {number}")
        try:
            record = json.loads(line.decode("utf-8"))
        except (ValueError, UnicodeDecodeError):
            record = None
        if not isinstance(record, dict):
            fail(f"invalid JSON object at line {number}")
        lv = parse_level(record, number, world_dtype)
        if lv["world_source_sha256"] != expected_world_hash:
            fail("bank world.hpp hash does not match the running binary source")
        if lv["failure_id"] in ids:
            fail("duplicate failure_id: " + lv["failure_id"])
        ids.add(lv["failure_id"])
        if lv["split"] == split:
            selected.append(lv)
    if not selected:
        fail("bank contains no records for requested split " + split)
    return selected, bank_hash


def write_level_file(path, levels, bank_hash, world_dtype):
    """The flat level file that oracle/ref/bank_shim's load_split reads."""
    code = {"train": 0, "dev": 1, "final": 2}
    with open(path, "wb") as f:
        f.write(b"MDNLVL1\x00" + struct.pack("<I", len(levels)) + bank_hash.encode())
        for lv in levels:
            f.write(struct.pack("<II", code[lv["split"]], lv["family"]))
            f.write(np.array(lv["world"], world_dtype).tobytes())


class ChallengeTraining:
    """challenge_training::ChallengeTraining restated (challenge_training.hpp:53-427)."""

    HEADER = struct.Struct("<8s8I2Q2f64s64s64s")

    def __init__(self, levels, bank_hash, world_hash, environment_count=128, horizon=32, sampler_seed=1,
                 rehearsal_environments=0, selection=0, uniform_floor=0.5, score_staleness_mix=0.5, focus_family=0):
        self.E, self.H = environment_count, horizon
        if self.E == 0 or self.H == 0:
            raise ValueError("challenge training needs nonzero environments and horizon")
        if self.E < 3 or rehearsal_environments > self.E - 3:
            raise ValueError("rehearsal must leave at least three bank environments")
        if focus_family not in (0, 14, 15, 16):
            raise ValueError("focused challenge family must be14,15,16 or0 for balanced")
        if selection not in (0, 1):
            raise ValueError("unsupported challenge level selection mode")
        self.uniform_floor = np.float32(uniform_floor)
        self.mix = np.float32(score_staleness_mix)
        if not (0.5 <= self.uniform_floor <= 1.0):
            raise ValueError("failure-weighted replay uniform floor must be in [0.5,1]")
        if not (0.0 <= self.mix <= 1.0):
            raise ValueError("score/staleness mix must be in [0,1]")
        self.R, self.selection, self.focus = rehearsal_environments, selection, focus_family
        self.levels = [lv for lv in levels if lv["split"] == "train"]
        self.bank_hash, self.world_hash = bank_hash, world_hash
        self.family_levels = {}
        for i, lv in enumerate(self.levels):
            self.family_levels.setdefault(lv["family"], []).append(i)
        for fam in (14, 15, 16):
            if not self.family_levels.get(fam):
                raise ValueError(f"train bank is missing family {fam}")
        self.families = [14, 15, 16]
        L = len(self.levels)
        self.scores = np.zeros(L, np.float32)
        self.last_visit = np.zeros(L, np.uint64)
        self.last_score = np.zeros(L, np.uint64)
        self.completed = np.zeros(L, np.uint64)
        self.abs_gae = np.zeros(self.E, np.float64)
        self.count = np.zeros(self.E, np.uint32)
        self.episode_level = np.full(self.E, INVALID, np.uint32)
        self.active = np.zeros(0, np.uint32)
        self.rng = sampler_seed or 1
        self.last_rollout = 0
        self.weights = {}

    def control(self):
        return (1, len(self.levels), self.H + 1, self.H)

    def _u32(self):
        x = self.rng or 1
        x ^= (x << 13) & MASK
        x ^= x >> 17
        x ^= (x << 5) & MASK
        self.rng = x or 1
        return self.rng

    def _uniform(self):
        return self._u32() / 4294967296.0

    def _uniform_index(self, cand):
        return cand[(self._u32() * len(cand)) >> 32]

    def _family(self, env):
        return self.focus if self.focus else self.families[(env - self.R) % len(self.families)]

    def _validate(self, env, level):
        if env < self.R:
            if level != INVALID:
                raise ValueError("rehearsal environment contains a bank level")
            return
        if level >= len(self.levels):
            raise ValueError("active challenge id is outside the train bank")
        if self.levels[level]["family"] != self._family(env):
            raise ValueError("active challenge id violates its fixed per-environment family quota")

    def _refresh(self):
        self.weights = {}
        if self.selection != 1:
            return
        mix = float(self.mix)
        for fam in self.families:
            cand = self.family_levels[fam]
            by_score = sorted(cand, key=lambda a: (-float(self.scores[a]), a))
            by_age = sorted(cand, key=lambda a: (int(self.last_visit[a]), a))
            spos = {lvl: r for r, lvl in enumerate(by_score)}
            apos = {lvl: r for r, lvl in enumerate(by_age)}
            self.weights[fam] = [mix / float(spos[lvl] + 1) + (1.0 - mix) / float(apos[lvl] + 1) for lvl in cand]

    def _sample(self, fam):
        cand = self.family_levels[fam]
        if self.selection == 0 or self._uniform() < float(self.uniform_floor):
            return self._uniform_index(cand)
        w = self.weights[fam]
        total = 0.0
        for x in w:
            total += x
        target = self._uniform() * total
        for i, x in enumerate(w):
            target -= x
            if target <= 0:
                return cand[i]
        return cand[-1]

    def initial_schedule(self):
        out = np.zeros((self.E, self.H + 1), np.uint32)
        self._refresh()
        for env in range(self.E):
            if env < self.R:
                out[env] = INVALID
                continue
            fam = self._family(env)
            for t in range(self.H + 1):
                out[env, t] = self._sample(fam)
        self.active = out[:, 0].copy()
        return out

    def next_schedule(self, active, rollout_index):
        active = np.asarray(active, np.uint32)
        self.last_rollout = rollout_index
        self._refresh()
        out = np.zeros((self.E, self.H + 1), np.uint32)
        for env in range(self.E):
            self._validate(env, int(active[env]))
            out[env, 0] = active[env]
        self.active = active.copy()
        for env in range(self.E):
            if env < self.R:
                out[env, 1:] = INVALID
                continue
            fam = self._family(env)
            for t in range(1, self.H + 1):
                out[env, t] = self._sample(fam)
        return out

    def observe_raw_gae(self, gae, term, trunc, ids, rollout_index):
        gae, ids = np.asarray(gae, np.float32).ravel(), np.asarray(ids, np.uint32).ravel()
        term, trunc = np.asarray(term).ravel(), np.asarray(trunc).ravel()
        for t in range(self.H):
            for env in range(self.E):
                row = t * self.E + env
                level = int(ids[row])
                if env < self.R:
                    if level != INVALID:
                        raise ValueError("rehearsal transition contains a bank level")
                    continue
                if level >= len(self.levels):
                    raise ValueError("transition level id is outside the frozen train bank")
                if self.episode_level[env] == INVALID:
                    self.episode_level[env] = level
                if self.episode_level[env] != level:
                    raise ValueError("active challenge level changed before episode completion")
                v = float(gae[row])
                if not math.isfinite(v):
                    raise ValueError("raw GAE is non-finite")
                self.abs_gae[env] += abs(v)
                self.count[env] += 1
                self.last_visit[level] = rollout_index
                if term[row] or trunc[row]:
                    self.scores[level] = np.float32(self.abs_gae[env] / float(self.count[env]))
                    self.last_score[level] = rollout_index
                    self.completed[level] += 1
                    self.abs_gae[env] = 0.0
                    self.count[env] = 0
                    self.episode_level[env] = INVALID
        self.last_rollout = rollout_index

    def state_bytes(self, checkpoint_hash, completed_rollouts, active):
        """The CHTRN1 v3 sidecar's bytes (save_state, :204-232)."""
        active = np.asarray(active, np.uint32)
        for env in range(self.E):
            self._validate(env, int(active[env]))
        self.active = active.copy()
        head = self.HEADER.pack(b"CHTRN1\x00\x00", 3, self.selection, self.E, self.H, len(self.levels), self.rng,
                                self.focus, self.R, self.last_rollout, completed_rollouts, float(self.uniform_floor),
                                float(self.mix), self.bank_hash.encode(), self.world_hash.encode(),
                                checkpoint_hash.encode())
        return head + b"".join(a.tobytes() for a in (
            self.scores, self.last_visit, self.last_score, self.completed, self.abs_gae, self.count,
            self.episode_level, self.active))


def sha256_of(path):
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def fixtures_dir():
    return os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "tests", "golden")
