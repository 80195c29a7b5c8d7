"""The C++ host veneer (include/mdn.hpp): Device / Sim / PPOTrainer and the
navigation_training helpers (navigation_training.hpp:7-170) over the C-ABI.

CPU: a C++ program that uses every part of the veneer compiles and links
against libmdn.so. GPU: the program evaluates a fresh actor twice (identical
scores, a 128-row CSV with the reference's columns), trains two task rollouts
from a warm-start checkpoint, resumes for a third, and leaves the checkpoint,
best checkpoint and history the reference's train() leaves.
"""
import os
import pathlib
import subprocess

import numpy as np
import pytest

from conftest import ROOT, load_oracle_module, load_package

PROGRAM = ROOT / "tests" / "cpp" / "veneer_check.cpp"
CSV_HEADER = ("seed,env,stage,family,mode,domain_amplitude,start_x,start_y,start_z,start_yaw,initial_vx,initial_vy,"
              "initial_vz,goal_x,goal_y,goal_z,initial_distance_m,direct_clearance_m,witness_length_m,mass_kg,success,"
              "collision,timeout,time_s,path_m,goal_error_m,final_speed_mps,hold_s,peak_speed_mps,"
              "min_sphere_clearance_m,success_rule")


def build(out):
    lib_dir = ROOT / "metal-drone-nav_b200"
    cmd = ["g++", "-std=c++17", "-O1", f"-I{ROOT / 'include'}", str(PROGRAM), f"-L{lib_dir}", "-lmdn",
           f"-Wl,-rpath,{lib_dir}", "-o", str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    return out


def test_veneer_compiles_and_links(tmp_path):
    assert (ROOT / "metal-drone-nav_b200" / "libmdn.so").exists()
    build(tmp_path / "veneer_check")


@pytest.mark.gpu
def test_veneer_evaluate_and_train(tmp_path):
    exe = build(tmp_path / "veneer_check")
    env = dict(os.environ, MDN_RAPTOR=str(ROOT / "metal-drone-nav_b200" / "assets" / "raptor.bin"))
    r = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    lines = {ln.split()[0]: ln.split()[1:] for ln in r.stdout.splitlines() if ln.split()}
    assert lines["eval"] == lines["eval_again"], "evaluation is not deterministic"
    success, collision, timeout, _ = (float(x) for x in lines["eval"])
    # the fresh actor's means for an all-0.5 observation: the float64 forward
    # of the reference's initial parameters (main.mm:548-555) within 1e-5
    om = load_oracle_module()
    olib = om.load_oracle()
    actor = np.zeros(olib.o_wide_param_count(64), np.float32)
    critic = np.zeros(olib.o_critic_param_count(), np.float32)
    olib.o_wide_init(64, om.ptr(actor), om.ptr(critic))
    x = np.full(184, 0.5)
    w1, b1 = actor[:64 * 184].reshape(64, 184).astype(np.float64), actor[64 * 184:64 * 185].astype(np.float64)
    w2, b2 = actor[64 * 185:64 * 189].reshape(4, 64).astype(np.float64), actor[64 * 189:64 * 189 + 4].astype(np.float64)
    want = np.tanh(w1 @ x + b1) @ w2.T + b2
    want[:3] += 0.5
    assert np.allclose([float(v) for v in lines["means"]], want, rtol=1e-5, atol=1e-6)
    assert abs(success + collision + timeout - 1.0) < 1e-6
    rows = (tmp_path / "eval.csv").read_text().splitlines()
    assert rows[0] == CSV_HEADER and len(rows) == 129
    pkg = load_package()
    h, _, _ = pkg.checkpoint_inspect(tmp_path / "task.bin")
    assert int(h["completed_rollouts"]) == 3 and int(h["n"]) == 128 and int(h["family"]) == 1
    assert (tmp_path / "task.bin.best").exists()
    history = (tmp_path / "task.bin.history.csv").read_text().splitlines()
    assert history[0].startswith("rollout,total_transitions") and len(history) == 1 + 1 + 3
