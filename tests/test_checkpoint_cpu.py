"""PPOFIX1 checkpoint layout on the host (main.mm:984-1000, 1209-1320).

mdn_checkpoint_inspect reads the reference's own checkpoints (assets/
checkpoints, versions 6-9) when the reference checkout is present: header
fields, the version 7/8 runtime and task blocks, and file sizes that match the
layout libmdn writes (version 8 = version 6 + runtime + task control + per-env
plants + task states + nominal plant + RAPTOR weights).
"""
import pathlib

import numpy as np
import pytest

from conftest import REFERENCE, load_package

CKPTS = REFERENCE / "assets" / "checkpoints"


def v6_bytes(h):
    n = int(h["n"])
    return (136 + (int(h["actor_count"]) * 3 + int(h["critic_count"]) * 3) * 4 +
            n * (68 + 184 + 676 + 8 * 320 * 4 + 8 * 12 * 4 + 8 * 4 * 4))


@pytest.mark.skipif(not CKPTS.exists(), reason="reference checkpoints not on this machine")
def test_inspect_reference_checkpoints():
    pkg = load_package()
    L = pkg.layouts
    stress = pkg.runtime_config(0.0)["domain_range"]
    seen = set()
    for path in sorted(CKPTS.iterdir()):
        h, rt, tc = pkg.checkpoint_inspect(path)
        v = int(h["version"])
        seen.add(v)
        size = path.stat().st_size
        n = int(h["n"])
        extra = 56 + (148 if v >= 8 else 144) + n * (L.PARAMS.itemsize + L.TASK_STATE.itemsize) + \
            L.PARAMS.itemsize + L.RAPTOR.itemsize
        if v == 6:
            assert size == v6_bytes(h), path.name
            assert rt.tobytes() == bytes(56) and tc["enabled"] == 0
        elif v in (7, 8):
            assert size == v6_bytes(h) + extra, path.name
            assert rt["domain_range"].tobytes() == stress.tobytes()
            assert tc["enabled"] == 1 and tc["config"]["nav_period_s"] == np.float32(0.05)
            if rt["enabled"]:
                assert rt.tobytes() == pkg.runtime_config(float(rt["domain_amplitude"])).tobytes()
        elif v == 9:  # + TrainingPotentialControl, TrainingPotentialGridSpec, field hash
            assert size == v6_bytes(h) + extra + 16 + 44 + 64, path.name
    assert {6, 7, 8}.issubset(seen)


def test_inspect_rejects_bad_files(tmp_path):
    pkg = load_package()
    bad = tmp_path / "x.bin"
    bad.write_bytes(b"PPOFIX2\0" + bytes(200))
    with pytest.raises(pkg.MdnError):
        pkg.checkpoint_inspect(bad)
    with pytest.raises(pkg.MdnError):
        pkg.checkpoint_inspect(tmp_path / "missing.bin")
