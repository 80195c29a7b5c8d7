"""Regenerate the golden fixtures in this folder from the reference checkout.

Run where the reference sources are present ($MDN_REFERENCE, else a folder
named `reference` beside this repository):
    python tests/golden/make_fixtures.py [reference_root]

Copies, byte for byte, the reference's golden data files that the tests
replay, and the frozen RAPTOR controller the product ships as runtime data:
  raptor.bin   RAPTOR1 weights + RPFIX1 16-step official sequence
               (assets/raptor.bin; format raptor.hpp:25-40, main.mm:127-137)
  physics.bin  RLPHYS1 L2F fixtures, 64 cases x 8 steps generated from rl-tools
               (assets/physics.bin; format main.mm:138-176, reference.cpp:83-156)
  ../../metal-drone-nav_b200/assets/raptor.bin  the same RAPTOR1 file
  ref_ckpt_v6_guided_stress.bin   PPOFIX1 v6 checkpoint of the reference's own
               training (assets/checkpoints/guided-stress.bin.best; layout
               main.mm:978-1000,1209-1320): 128 envs, family 7, geometry memory
  ref_ckpt_v8_local_waypoint.bin  PPOFIX1 v8 checkpoint with the runtime and
               task blocks (assets/checkpoints/local-waypoint-fast-experimental
               .bin.best): 128 envs, mode 22, goal-arrival tasks
  ref_navpol_rooms.bin  a NAVPOL1 deployment file the reference exported from
               its own training (assets/navigation-rooms-experimental.bin;
               format deployment.hpp:41-88): trained actor weights for the
               deployment probe (main.mm:1001-1042)
Then writes ref_trace.npz: a short teacher-forced trace of the reference's own
CPU path (oracle/_ref, compiled unmodified), used by GPU tests on machines
without the reference sources.
"""
import pathlib
import shutil
import sys
import importlib.util

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parents[1]


def _load(name, path, pkg_dir=None):
    spec = importlib.util.spec_from_file_location(
        name, path, submodule_search_locations=[str(pkg_dir)] if pkg_dir else None)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


CHECKPOINTS = {"ref_ckpt_v6_guided_stress.bin": "guided-stress.bin.best",
               "ref_ckpt_v8_local_waypoint.bin": "local-waypoint-fast-experimental.bin.best"}


def copy_checkpoints(ref):
    """The reference's own training checkpoints the resume tests load."""
    for mine, theirs in CHECKPOINTS.items():
        shutil.copyfile(ref / "assets" / "checkpoints" / theirs, HERE / mine)


def reference_root(ref_root=None):
    import os
    return pathlib.Path(ref_root or os.environ.get("MDN_REFERENCE") or ROOT.parent / "reference")


def main(ref_root=None):
    ref = reference_root(ref_root)
    copy_checkpoints(ref)
    shutil.copyfile(ref / "assets" / "navigation-rooms-experimental.bin", HERE / "ref_navpol_rooms.bin")
    shutil.copyfile(ref / "assets" / "raptor.bin", HERE / "raptor.bin")
    shutil.copyfile(ref / "assets" / "physics.bin", HERE / "physics.bin")
    (ROOT / "metal-drone-nav_b200" / "assets").mkdir(parents=True, exist_ok=True)
    shutil.copyfile(ref / "assets" / "raptor.bin", ROOT / "metal-drone-nav_b200" / "assets" / "raptor.bin")

    layouts = _load("mdn_layouts", ROOT / "metal-drone-nav_b200" / "layouts.py")
    oracle = _load("mdn_oracle_py", ROOT / "oracle" / "oracle.py")
    oracle.build(ref)
    raptor = layouts.load_raptor_file(HERE / "raptor.bin")
    out = {}
    # Teacher-forced trace: 24 envs of family 1 (8 boxes) and a short horizon;
    # state after every step of the reference's own CPU path.
    for family in (1, 3):
        cfg = layouts.default_config(n=24, family=family, speed=1.0, distance=3.0, seed=42)
        tr = oracle.RefTrainer(layouts, cfg, 6, raptor)
        out[f"f{family}_worlds0"] = tr.buf("worlds").copy()
        out[f"f{family}_states0"] = tr.buf("states").copy()
        out[f"f{family}_runs0"] = tr.buf("runs").copy()
        for t in range(6):
            tr.step(t)
            out[f"f{family}_states{t+1}"] = tr.buf("states").copy()
            out[f"f{family}_runs{t+1}"] = tr.buf("runs").copy()
        for name in ("obs", "co", "actions", "logp", "values", "rewards", "next_values", "terminated", "truncated"):
            out[f"f{family}_{name}"] = tr.buf(name).copy()
        tr.lib.ref_gae_normalize(tr.h)
        out[f"f{family}_advantages"] = tr.buf("advantages").copy()
        out[f"f{family}_returns"] = tr.buf("returns").copy()
        loss = np.zeros(4, np.float32)
        tr.lib.ref_train_rollout(tr.h, 0, oracle.ptr(loss))
        out[f"f{family}_actor_after"] = tr.buf("actor").copy()
        out[f"f{family}_critic_after"] = tr.buf("critic").copy()
        out[f"f{family}_loss"] = loss
    np.savez_compressed(HERE / "ref_trace.npz", **out)
    print("wrote", sorted(p.name for p in HERE.iterdir()))


if __name__ == "__main__":
    main(*sys.argv[1:])
