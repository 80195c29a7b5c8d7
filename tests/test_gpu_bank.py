"""Frozen challenge banks on the GPU (sim_apply_challenge_world, sim.metal:95-122,
143, 326, 330) against the CPU oracle, through the C-ABI.

Bank levels replace the procedural world at reset (schedule slot 0) and at
every in-step episode reset (slot tick + 1); level id 0xffffffff plays a
rehearsal world; a level id past the bank or a slot past the schedule keeps
the procedural world. Worlds, level ids and integer outputs are compared
bitwise; fp32 state within RTOL/ATOL = 1e-5 (as the rollout parity tests).
Then a whole bank-training loop: sampler schedules -> GPU rollouts -> PPO
update -> raw GAE and transition ids back into the sampler.
"""
import json

import numpy as np
import pytest

from conftest import GOLDEN, load_oracle_module, load_package

pytestmark = pytest.mark.gpu

SMALL = GOLDEN / "challenge_bank_small.jsonl"
INVALID = 0xFFFFFFFF
RTOL = ATOL = 1e-5
STATE_KEYS = ("states", "runs", "worlds", "sensors", "poses", "commands", "bank_active_ids")


def world_hash():
    return json.loads(SMALL.read_text().splitlines()[0])["world_source_sha256"]


def close(a, b, what):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    bad = ~(np.abs(a - b) <= ATOL + RTOL * np.abs(b))
    assert not bad.any(), f"{what}: {bad.sum()} differ; worst {np.nanmax(np.abs(a - b)):.3e}"


def floats(structured):
    return np.frombuffer(np.ascontiguousarray(structured).tobytes(), np.float32)


def schedule_for(n, stride, seed):
    rng = np.random.default_rng(seed)
    s = rng.integers(0, 12, (n, stride)).astype(np.uint32)
    s[::7] = INVALID       # rehearsal rows (even and odd envs: families 12 and 13)
    s[5] = 99              # unknown level: the procedural world stays
    s[11, 1::2] = INVALID  # rehearsal resets between bank levels
    return s


CASES = [
    dict(cfg=dict(family=12, wind=0.3, max_steps=5), stride=None),
    dict(cfg=dict(family=1, sensor_delay=1, command_delay=1, max_steps=4), stride=3),
    dict(cfg=dict(family=17, max_steps=6, risk_coef=0.5), stride=None),
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_bank_steps_match_oracle(case):
    pkg, om = load_package(), load_oracle_module()
    L = pkg.layouts
    raptor = pkg.default_raptor()
    dev = pkg.Device(0)
    n, T = 200, 12
    c = CASES[case]
    stride = c["stride"] or T + 1
    cfg = L.default_config(**{**dict(n=n, speed=1.0, distance=4.0, seed=21 + case), **c["cfg"]})
    bank = pkg.ChallengeBank(SMALL, "train", world_hash())
    worlds = bank.worlds()
    control = (1, len(worlds), stride, T)
    sched = schedule_for(n, stride, case)
    gpu = pkg.Sim(dev, cfg, T, raptor=raptor)
    ora = om.OracleSim(L, cfg, T, raptor)
    try:
        # before any bank: every env's active id is "none"
        assert np.all(gpu.download("bank_active_ids") == INVALID)
        gpu.set_challenge_bank(worlds, control)
        gpu.set_bank_schedule(sched)
        gpu.reset()
        ora.set_challenge_bank(worlds, control)
        ora.buf("bank_schedule")[:] = sched.ravel()
        ora.reset()
        for name in STATE_KEYS:
            assert gpu.download(name).tobytes() == ora.buf(name).tobytes(), f"reset {name}"
        active = gpu.download("bank_active_ids")
        assert np.array_equal(active[::7], np.full(len(active[::7]), INVALID, np.uint32))
        assert active[5] == INVALID  # 99 is not a level: nothing was applied
        plays = active[(active != INVALID)]
        assert plays.size > 0 and np.all(plays < 12)
        w = gpu.download("worlds")
        for i in np.flatnonzero(active != INVALID)[:20]:
            ref = worlds[active[i]].copy()
            ref["wind"] = (0.0 if (cfg["family"] in (12, 13) and i % 2 == 0) else cfg["wind"], 0.0, 0.0)
            assert w[i].tobytes() == ref.tobytes(), i
        resets = 0
        for t in range(T):
            for name in STATE_KEYS:
                gpu.upload(name, ora.buf(name))
            gpu.step(t)
            ora.step(t)
            rows = slice(t * n, (t + 1) * n)
            for name in ("terminated", "truncated", "contact_id", "bank_transition_ids"):
                assert np.array_equal(gpu.download(name)[rows], ora.buf(name)[rows]), f"t={t} {name}"
            for name in ("rewards", "next_values"):
                close(gpu.download(name)[rows], ora.buf(name)[rows], f"t={t} {name}")
            assert gpu.download("worlds").tobytes() == ora.buf("worlds").tobytes(), f"t={t} worlds"
            assert np.array_equal(gpu.download("bank_active_ids"), ora.buf("bank_active_ids")), f"t={t} active"
            rs_g, rs_o = gpu.download("runs"), ora.buf("runs")
            for f in ("steps", "episodes", "rng"):
                assert np.array_equal(rs_g[f], rs_o[f]), f"t={t} runs.{f}"
            close(rs_g["initial_distance"], rs_o["initial_distance"], f"t={t} initial distance")
            close(floats(gpu.download("states")), floats(ora.buf("states")), f"t={t} states")
            done = (gpu.download("terminated")[rows] | gpu.download("truncated")[rows]) != 0
            resets += int(done.sum())
        assert resets > n // 2  # slots past 0 were exercised
        trans = gpu.download("bank_transition_ids").reshape(T, n)
        assert np.all(trans[:, ::7] == INVALID)
    finally:
        gpu.close()
        bank.close()
        dev.close()


def test_bank_off_is_legacy_and_ids_invalid():
    pkg = load_package()
    L = pkg.layouts
    dev = pkg.Device(0)
    cfg = L.default_config(n=256, family=3, seed=4, max_steps=5)
    a, b = pkg.Sim(dev, cfg, 6), pkg.Sim(dev, cfg, 6)
    bank = pkg.ChallengeBank(SMALL, "train", world_hash())
    try:
        b.set_challenge_bank(bank.worlds())
        b.set_challenge_bank(None)  # switched off again before any reset
        b.reset()
        a.collect()
        b.collect()
        for name in ("states", "worlds", "rewards", "terminated"):
            assert a.download(name).tobytes() == b.download(name).tobytes(), name
        assert np.all(b.download("bank_active_ids") == INVALID)
        assert np.all(b.download("bank_transition_ids") == INVALID)
    finally:
        bank.close()
        a.close()
        b.close()
        dev.close()


def test_bank_training_loop():
    """main.mm:2400-2492 in miniature: initial schedule + reset, then per
    rollout next_schedule from the device's active ids, collect, PPO update,
    and the raw GAE / terminal flags / transition ids into the sampler."""
    pkg, om = load_package(), load_oracle_module()
    L = pkg.layouts
    dev = pkg.Device(0)
    n, T = 384, 16
    cfg = L.default_config(n=n, family=12, seed=3, speed=1.0, max_steps=8)
    sim = pkg.Sim(dev, cfg, T)
    sampler = pkg.ChallengeSampler(SMALL, world_hash(), environment_count=n, horizon=T, rehearsal_environments=8,
                                   selection=1)
    trainer = pkg.PPOTrainer(sim, epochs=1, minibatch=1536)
    try:
        c = sampler.control()
        sim.set_challenge_bank(sampler.bank.worlds(), c)
        sim.set_bank_schedule(sampler.initial_schedule())
        sim.reset()
        assert np.array_equal(sim.download("bank_active_ids"), sampler.active_ids())
        for rollout in range(3):
            if rollout:
                sim.set_bank_schedule(sampler.next_schedule(sim.download("bank_active_ids"), rollout))
            sim.collect()
            trainer.rollout_update(rollout)
            dev.finish()
            raw = sim.download("raw_advantages")
            # the raw copy is the GAE before normalisation (ppo.hpp:108-126)
            adv = np.zeros(n * T, np.float32)
            ret = np.zeros(n * T, np.float32)
            olib = om.load_oracle()
            args = [sim.download(k) for k in ("rewards", "values", "next_values", "terminated", "truncated")]
            olib.o_compute_gae(T, n, *[om.ptr(np.ascontiguousarray(a)) for a in args], 0.99, 0.95, om.ptr(adv),
                               om.ptr(ret))
            close(raw, adv, f"rollout {rollout} raw GAE")
            assert not np.allclose(raw, sim.download("advantages"))  # the normalised copy differs
            sampler.observe_raw_gae(raw, sim.download("terminated"), sim.download("truncated"),
                                    sim.download("bank_transition_ids"), rollout)
        stats = [sampler.level_stats(i) for i in range(len(sampler.bank))]
        assert sum(s[1] for s in stats) > 0 and all(np.isfinite(s[0]) for s in stats)
    finally:
        trainer.close()
        sampler.close()
        sim.close()
        dev.close()


def test_bank_evaluate_matches_oracle(tmp_path):
    """challenge_evaluation::run (challenge_evaluation.hpp:352-497) through
    mdn_bank_evaluate: the 38-column CSV and the BankScore of a checkpoint on the
    train split equal an oracle replay of the same batch (worlds, per-level policy
    seeds, evaluation mode); outcomes bitwise, episode metrics within 1e-3."""
    import csv
    pkg, om = load_package(), load_oracle_module()
    L = pkg.layouts
    dev = pkg.Device(0)
    cfg = L.default_config(n=64, family=1, speed=1.0, distance=3.0, seed=8)
    sim = pkg.Sim(dev, cfg, 8)
    tr = pkg.PPOTrainer(sim)
    try:
        sim.collect()
        tr.rollout_update(0)
        ck = tmp_path / "ck.bin"
        tr.save_checkpoint(ck, 1, 8, 1)
        actor, critic = sim.download("actor"), sim.download("critic")
        steps = 30
        out = tmp_path / "eval" / "train.csv"
        score = pkg.evaluate_bank(dev, ck, SMALL, "train", world_hash(), out, mode=17, speed=1.5, max_steps=steps)
        rows = list(csv.reader(out.open()))
        header, rows = rows[0], rows[1:]
        assert len(header) == 38 and header[0] == "failure_id" and header[-1] == "world_source_sha256"
        assert len(rows) == 12 and not (tmp_path / "eval" / "train.csv.tmp").exists()
        bank = pkg.ChallengeBank(SMALL, "train", world_hash())
        levels = [bank.level(i) for i in range(12)]
        worlds = bank.worlds()
        col = {name: k for k, name in enumerate(header)}
        for r, lv in zip(rows, levels):
            assert r[col["failure_id"]] == lv["failure_id"] and r[col["split"]] == "train"
            assert r[col["checkpoint_sha256"]] == pkg.sha256_file(ck) and r[col["bank_sha256"]] == bank.bank_sha256
            assert r[col["physics_invalid"]] == "not_instrumented" and int(r[col["max_steps"]]) == steps
            route = np.array(json.loads(r[col["witness_route_json"]]), np.float32)
            assert np.array_equal(route, lv["witness_route"])  # 9 significant digits round-trip float32
        ocfg = L.default_config(n=12, family=0, mode=17, seed=levels[0]["seed"], eval=1, speed=1.5,
                                distance=levels[0]["distance"], max_steps=steps, wind=0.0,
                                velocity_contract=int(cfg["velocity_contract"]), geometry_memory=0)
        ora = om.OracleSim(L, ocfg, 32, pkg.default_raptor())
        ora.buf("actor")[:] = actor
        ora.buf("critic")[:] = critic
        ora.buf("worlds")[:] = worlds
        runs = ora.buf("runs")
        for i, lv in enumerate(levels):
            runs["rng"][i] = (lv["base_seed"] + lv["environment_index"] * 747796405 + 2891336453) & 0xFFFFFFFF
            runs["steps"][i] = 0
            g = worlds["goal"][i].astype(np.float32)
            runs["initial_distance"][i] = np.sqrt(g[0] * g[0] + g[1] * g[1] + (g[2] - np.float32(1.5)) ** 2)
            runs["reference_position"][i] = (0.0, 0.0, 1.5)
        for t in range(steps):
            ora.step(t % 32)
        runs = ora.buf("runs")
        for i, r in enumerate(rows):
            for name, field in (("episodes", "episodes"), ("success", "successes"), ("collision", "collisions"),
                                ("timeout", "timeouts")):
                assert int(r[col[name]]) == int(runs[field][i]), (i, name)
            for name, value in (("progress", runs["final_progress"][i]), ("path_m", runs["path"][i]),
                                ("elapsed_s", runs["elapsed"][i]), ("peak_speed_mps", runs["peak_speed"][i]),
                                ("min_clearance_m", runs["min_clearance"][i])):
                assert float(r[col[name]]) == pytest.approx(float(value), rel=1e-3, abs=1e-3), (i, name)
        assert score["episodes"] == 12 and score["successes"] == int(runs["successes"].sum())
        assert score["family_episodes"] == [4, 4, 4]
        with pytest.raises(pkg.MdnError):
            pkg.evaluate_bank(dev, ck, SMALL, "train", world_hash(), out, mode=5)
        with pytest.raises(pkg.MdnError):
            pkg.evaluate_bank(dev, ck, SMALL, "train", world_hash(), out, max_steps=401)
    finally:
        tr.close()
        sim.close()
        dev.close()
