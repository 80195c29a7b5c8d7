"""PPO update kernels on the GPU against the CPU oracle (through the C-ABI).

GAE + advantage normalisation: bit-exact (same float recursion; fp64 sums).
One Adam step (one minibatch chunk, one epoch): actor/critic parameters,
Adam moments and gradient norms within RTOL 1e-5 / ATOL 1e-7 of the oracle
fed the same rollout. A parameter may differ by up to 2*lr only where its
gradient is at float-rounding level (Adam's first step is sign(g)*lr, so a
rounding-size gradient can flip sign); the test bounds those by the oracle's
first moment.
"""
import numpy as np
import pytest

from conftest import load_oracle_module, load_package

pytestmark = pytest.mark.gpu

ROLL = ("obs", "co", "actions", "logp", "values", "rewards", "next_values", "terminated", "truncated")


@pytest.fixture(scope="module")
def pkg():
    return load_package()


@pytest.fixture(scope="module")
def device(pkg):
    return pkg.Device(0)


@pytest.fixture(scope="module")
def om():
    return load_oracle_module()


def rollout_pair(pkg, om, device, n, T, minibatch, epochs, family=1, seed=4):
    cfg = pkg.layouts.default_config(n=n, family=family, speed=1.0, distance=3.0, seed=seed)
    raptor = pkg.default_raptor()
    sim = pkg.Sim(device, cfg, T, raptor=raptor)
    tr = pkg.PPOTrainer(sim, epochs=epochs, minibatch=minibatch)
    sim.collect()
    ora = om.OracleSim(pkg.layouts, cfg, T, raptor)
    for name in ROLL + ("actor", "critic"):
        ora.buf(name)[:] = sim.download(name)
    return sim, tr, ora


def bias(olib_, steps):
    return (np.array([olib_.o_pow_correction(0.9, int(s)) for s in steps], np.float32),
            np.array([olib_.o_pow_correction(0.999, int(s)) for s in steps], np.float32))


def test_gae_normalisation_bitwise(pkg, om, device):
    sim, tr, ora = rollout_pair(pkg, om, device, n=512, T=64, minibatch=256, epochs=1)
    try:
        tr.rollout_update(0)
        ora.gae(True)
        assert np.array_equal(sim.download("returns"), ora.buf("returns"))
        assert np.array_equal(sim.download("advantages"), ora.buf("advantages"))
    finally:
        tr.close()
        sim.close()


@pytest.mark.parametrize("n,T,mb", [(32, 8, 256), (512, 32, 16384)])
def test_single_adam_step(pkg, om, device, n, T, mb):
    sim, tr, ora = rollout_pair(pkg, om, device, n=n, T=T, minibatch=mb, epochs=1)
    try:
        order = tr.minibatch_order(0, 1)
        tr.rollout_update(0)
        ora.gae(True)
        b1, b2 = bias(ora.lib, [1])
        out_o, norms_o = ora.train_rollout(mb, 1, order, b1, b2)
        norms_g = tr.grad_norms(1)
        np.testing.assert_allclose(norms_g.ravel(), norms_o[:2], rtol=1e-5)
        for which, name, pname in ((0, 100, "actor"), (2, 102, "critic")):
            m_g, m_o = tr.moments(which), ora.buf(name)
            np.testing.assert_allclose(m_g, m_o, rtol=1e-4, atol=1e-6 * np.abs(m_o).max())
            p_g, p_o = sim.download(pname), ora.buf(pname)
            lr = float(sim.cfg["learning_rate"])
            diff = np.abs(p_g - p_o)
            bad = diff > 1e-7 + 1e-5 * np.abs(p_o)
            # only rounding-level gradients may flip Adam's first step
            tiny = np.abs(m_o) <= 1e-4 * np.abs(m_o).max()
            assert not (bad & ~tiny).any(), f"{pname}: {int((bad & ~tiny).sum())} params differ"
            assert (diff <= 2.0001 * lr).all()
        np.testing.assert_allclose(tr.metric_mean, out_o, rtol=1e-4, atol=1e-6)
    finally:
        tr.close()
        sim.close()


def test_two_epochs_of_chunks(pkg, om, device):
    """Reference schedule: 2 epochs x shuffled 256-row chunks (main.mm:1331-1378)."""
    n, T = 64, 16
    sim, tr, ora = rollout_pair(pkg, om, device, n=n, T=T, minibatch=256, epochs=2)
    try:
        U = 2 * (n * T // 256)
        order = tr.minibatch_order(0, U)
        assert np.array_equal(order, pkg.capi.minibatch_order(n * T, 256, 2, 0))
        tr.rollout_update(0)
        ora.gae(True)
        b1, b2 = bias(ora.lib, range(1, U + 1))
        out_o, norms_o = ora.train_rollout(256, 2, order, b1, b2)
        np.testing.assert_allclose(tr.grad_norms(U).ravel(), norms_o, rtol=1e-3)
        lr = float(sim.cfg["learning_rate"])
        for pname in ("actor", "critic"):
            p_g, p_o = sim.download(pname), ora.buf(pname)
            diff = np.abs(p_g - p_o)
            assert np.quantile(diff, 0.999) <= 1e-5, pname
            assert diff.max() <= 2 * U * lr, pname
        assert tr.optimizer_step == U
    finally:
        tr.close()
        sim.close()


def test_checkpoint_roundtrip(pkg, device, tmp_path):
    """PPOFIX1 v6 save/load (main.mm:1209-1320) restores params, moments and state."""
    cfg = pkg.layouts.default_config(n=64, family=1, speed=1.0, distance=3.0, seed=8)
    sim = pkg.Sim(device, cfg, 8)
    tr = pkg.PPOTrainer(sim)
    sim.collect()
    tr.rollout_update(0)
    path = tmp_path / "ck.bin"
    tr.save_checkpoint(path, 1, 8, 1)
    snap = {k: sim.download(k) for k in ("actor", "critic", "states", "runs", "worlds", "sensors", "poses", "commands")}
    moments = [tr.moments(i) for i in range(4)]
    sim2 = pkg.Sim(device, cfg, 8)
    tr2 = pkg.PPOTrainer(sim2)
    try:
        tr2.load_checkpoint(path, 1, 8, 64, 8)
        for k, v in snap.items():
            assert sim2.download(k).tobytes() == v.tobytes(), k
        for i in range(4):
            assert np.array_equal(tr2.moments(i), moments[i])
        assert tr2.state() == (tr.optimizer_step, 1)
        with pytest.raises(pkg.MdnError):
            tr2.load_checkpoint(path, 1, 8, 64, 9)  # base seed mismatch
        # resumed training is bit-identical to uninterrupted training
        sim.collect()
        tr.rollout_update(1)
        sim2.collect()
        tr2.rollout_update(1)
        assert sim.download("actor").tobytes() == sim2.download("actor").tobytes()
    finally:
        tr2.close()
        sim2.close()
        tr.close()
        sim.close()
