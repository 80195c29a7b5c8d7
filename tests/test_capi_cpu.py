"""CPU-side checks of the C-ABI library: it loads, exports every entry point
include/mdn.h declares, host-only logic matches the reference, and calls fail
with a status (not a crash) when there is no GPU. No kernel runs here."""
import ctypes
import re

import numpy as np
import pytest

from conftest import GOLDEN, ROOT, load_package, physics_fixture


@pytest.fixture(scope="module")
def pkg():
    return load_package()


def declared_symbols():
    text = (ROOT / "include" / "mdn.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+char\s*\*|int|void|uint32_t)\s+(mdn_\w+)\s*\(", text, re.M)))


def test_header_symbols_exported(pkg):
    lib = pkg.lib()
    names = declared_symbols()
    assert len(names) >= 35
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # every declared entry point has a typed binding in the Python veneer
    assert set(names) <= set(pkg.capi.SIGNATURES), set(names) - set(pkg.capi.SIGNATURES)


def test_layout_sizes(pkg):
    L = pkg.layouts
    assert (L.STATE.itemsize, L.PARAMS.itemsize, L.WORLD.itemsize, L.RUN.itemsize, L.CONFIG.itemsize,
            L.RAPTOR.itemsize, L.CHECKPOINT_HEADER.itemsize) == (68, 352, 676, 184, 84, 8336, 136)


def test_rollout_shape_layout(pkg):
    """mdn_rollout_shape_default writes exactly the 60-byte struct the Python
    layout describes (guard bytes after it stay untouched); the layered fields
    default to one tanh hidden layer."""
    L = pkg.layouts
    raw = np.full(L.SHAPE.itemsize + 16, 0xA5, np.uint8)
    pkg.lib().mdn_rollout_shape_default(raw.ctypes.data_as(ctypes.c_void_p))
    assert np.all(raw[L.SHAPE.itemsize:] == 0xA5)
    shape = raw[:L.SHAPE.itemsize].view(L.SHAPE)[0]
    assert (shape["actor_obs_dim"], shape["critic_obs_dim"], shape["actor_hidden"], shape["critic_hidden"]) == \
        (184, 32, 64, 64)
    assert (shape["actor_layers"], shape["critic_layers"], shape["actor_activation"], shape["critic_activation"]) == \
        (0, 0, 0, 0)
    assert list(shape["room_min"]) == [-2.0, -5.0, 0.0] and list(shape["room_max"]) == [14.0, 5.0, 5.0]


def test_defaults_match_reference(pkg, olib, oracle_mod):
    L = pkg.layouts
    lib = pkg.lib()
    c = np.zeros((), L.CONFIG)
    lib.mdn_sim_config_default(c.ctypes.data)
    assert c.tobytes() == L.default_config().tobytes()  # SimConfig{} (main.mm:462-463)
    p = np.zeros((), L.PARAMS)
    lib.mdn_physics_crazyflie_default(p.ctypes.data)
    q = np.zeros((), L.PARAMS)
    olib.o_physics_default(oracle_mod.ptr(q))
    params, _ = physics_fixture(L)
    assert p.tobytes() == q.tobytes() == params.tobytes()


def test_raptor_loader(pkg):
    w = pkg.default_raptor()
    assert w.tobytes() == pkg.layouts.load_raptor_file(GOLDEN / "raptor.bin").tobytes()
    bad = np.zeros((), pkg.layouts.RAPTOR)
    assert pkg.lib().mdn_raptor_load(str(GOLDEN / "physics.bin").encode(), bad.ctypes.data) == 5  # MDN_ERR_IO


@pytest.mark.parametrize("rows,mb,epochs", [(512 * 64, 256, 2), (40 * 16, 256, 2), (8192 * 128, 131072, 4),
                                            (1000, 256, 3), (256, 256, 1)])
def test_minibatch_order_bitwise(pkg, rlib, oracle_mod, rows, mb, epochs):
    """Chunk permutations are integer work: bit-exact with the reference's
    std::mt19937 + std::shuffle (main.mm:1331-1337)."""
    for rollout in (0, 1, 7, 123):
        mine = pkg.capi.minibatch_order(rows, mb, epochs, rollout)
        ref = np.zeros_like(mine)
        rlib.ref_minibatch_order(rows, mb, rollout, epochs, oracle_mod.ptr(ref))
        assert np.array_equal(mine, ref)


def test_no_gpu_is_a_status_not_a_crash(pkg):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    status = pkg.lib().mdn_device_open(0, ctypes.byref(h))
    assert status in (1, 2)
    assert pkg.lib().mdn_last_error()
    with pytest.raises(pkg.MdnError):
        pkg.Device(0)
