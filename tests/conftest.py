"""Shared fixtures. `gpu` marks tests that need a CUDA device (run on a B200)."""
import importlib.util
import os
import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
# The reference checkout (read only by CPU pin tests that skip without it):
# $MDN_REFERENCE, else a folder named `reference` beside this repository.
REFERENCE = pathlib.Path(os.environ.get("MDN_REFERENCE") or ROOT.parent / "reference")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def _load_module(name, path, package_dir=None):
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(
        name, path, submodule_search_locations=[str(package_dir)] if package_dir else None)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_package():
    """The product package (its folder name is not a Python identifier)."""
    pkg = ROOT / "metal-drone-nav_b200"
    return _load_module("mdn_b200", pkg / "__init__.py", pkg)


def load_oracle_module():
    return _load_module("mdn_oracle_py", ROOT / "oracle" / "oracle.py")


@pytest.fixture(scope="session")
def layouts():
    return load_package().layouts


@pytest.fixture(scope="session")
def oracle_mod():
    return load_oracle_module()


@pytest.fixture(scope="session")
def olib(oracle_mod):
    return oracle_mod.load_oracle()


@pytest.fixture(scope="session")
def rlib(oracle_mod):
    lib = oracle_mod.load_ref()
    if lib is None:
        pytest.skip("oracle/_ref not built: the reference sources are not on this machine")
    return lib


@pytest.fixture(scope="session")
def raptor(layouts):
    return layouts.load_raptor_file(GOLDEN / "raptor.bin")


def raptor_fixture_sequence():
    """RPFIX1 block after the weights: 16x22 observations, 16x4 expected actions."""
    raw = (GOLDEN / "raptor.bin").read_bytes()
    off = 16 + 8336
    assert raw[off:off + 8] == b"RPFIX1\x00\x00"
    obs = np.frombuffer(raw, np.float32, 16 * 22, off + 20).reshape(16, 22)
    exp = np.frombuffer(raw, np.float32, 64, off + 20 + 16 * 22 * 4).reshape(16, 4)
    return obs, exp


def physics_fixture(layouts):
    """RLPHYS1 (main.mm:138-176): header, params, then (state, action, wind, expected) records."""
    raw = (GOLDEN / "physics.bin").read_bytes()
    assert raw[:8] == b"RLPHYS1\x00"
    version, cases, horizon = np.frombuffer(raw, "<u4", 3, 8)
    assert version == 1
    params = np.frombuffer(raw, layouts.PARAMS, 1, 20).copy().reshape(())
    rec = np.dtype([("state", layouts.STATE), ("action", "<f4", 4), ("wind", "<f4", 3), ("expected", layouts.STATE)])
    recs = np.frombuffer(raw, rec, int(cases * horizon), 20 + 352).copy()
    return params, recs
