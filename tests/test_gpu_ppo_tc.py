"""The tensor-core PPO minibatch kernel (ppo_tc.cu, mdn_ppo_set_tensor_cores)
against the fp32 CPU oracle.

TF32 tolerance, stated: the products read their fp32 operands with a 10-bit
mantissa (relative rounding up to 2^-10), so the forward pre-activations, the
losses and every gradient sum differ from fp32 at the 1e-3 level. The bar is
a relative L2 difference of at most 1e-2 per parameter block of the first
update's gradient (read back as Adam's first moment, 0.1 x the clipped
gradient), gradient norms within 1e-2 relative, loss metrics within 1e-2
relative (+1e-5 absolute), and the result independent of scheduling (two runs
equal bit for bit). Cases: many tiles per CTA (both epilogue groups, the
shared-memory ring wrapping), a ragged last tile, a minibatch shorter than the
grid (CTAs without rows write zero partials), and two epochs.
"""
import numpy as np
import pytest

from conftest import load_oracle_module, load_package

pytestmark = pytest.mark.gpu

ROLL = ("obs", "co", "actions", "logp", "values", "rewards", "next_values", "terminated", "truncated")
A_BLOCKS = {"W1": (0, 64 * 184), "b1": (64 * 184, 64 * 185), "W2": (64 * 185, 64 * 189), "b2": (64 * 189, 64 * 189 + 4),
            "log_std": (64 * 189 + 4, 64 * 189 + 8)}
C_BLOCKS = {"cW1": (0, 64 * 32), "cb1": (64 * 32, 64 * 33), "cw2": (64 * 33, 64 * 34), "cb2": (64 * 34, 64 * 34 + 1)}


@pytest.fixture(scope="module")
def pkg():
    return load_package()


@pytest.fixture(scope="module")
def om():
    return load_oracle_module()


@pytest.fixture(scope="module")
def device(pkg):
    return pkg.Device(0)


def bias(olib, steps):
    return (np.array([olib.o_pow_correction(0.9, int(s)) for s in steps], np.float32),
            np.array([olib.o_pow_correction(0.999, int(s)) for s in steps], np.float32))


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def run_tc(pkg, device, cfg, T, mb, epochs):
    sim = pkg.Sim(device, cfg, T, raptor=pkg.default_raptor())
    tr = pkg.PPOTrainer(sim, epochs=epochs, minibatch=mb)
    tr.set_tensor_cores(True)
    sim.collect()
    return sim, tr


@pytest.mark.parametrize("n,T,mb,epochs", [(2048, 32, 65536, 1), (300, 16, 1000, 1), (1024, 16, 8192, 2)],
                         ids=["mb65536_multi_tile", "ragged_and_empty_ctas", "two_epochs"])
def test_tensor_core_update_matches_oracle(pkg, om, device, n, T, mb, epochs):
    cfg = pkg.layouts.default_config(n=n, family=18, speed=1.0, distance=3.0, seed=23, sensor_delay=2,
                                     command_delay=2)
    sim, tr = run_tc(pkg, device, cfg, T, mb, epochs)
    try:
        ora = om.OracleSim(pkg.layouts, cfg, T, sim.raptor)
        for name in ROLL + ("actor", "critic"):
            ora.buf(name)[:] = sim.download(name)
        rows = n * T
        U = epochs * (-(-rows // mb))
        order = tr.minibatch_order(0, U)
        tr.rollout_update(0)
        device.finish()
        ora.gae(True)
        assert np.array_equal(sim.download("advantages"), ora.buf("advantages"))
        b1, b2 = bias(ora.lib, range(1, U + 1))
        # first update alone in the oracle: its gradient is Adam's first moment / 0.1
        if U == 1:
            out_o, norms_o = ora.train_rollout(mb, epochs, order, b1, b2)
            for which, bid, blocks in ((0, 100, A_BLOCKS), (2, 102, C_BLOCKS)):
                m_g, m_o = tr.moments(which), ora.buf(bid)
                for name, (lo, hi) in blocks.items():
                    err = rel_l2(m_g[lo:hi], m_o[lo:hi])
                    print(f"{name}: relative L2 {err:.2e}")
                    assert err <= 1e-2, name
            np.testing.assert_allclose(tr.grad_norms(U).ravel(), norms_o, rtol=1e-2)
            np.testing.assert_allclose(tr.metric_mean, out_o, rtol=1e-2, atol=1e-5)
        else:
            out_o, norms_o = ora.train_rollout(mb, epochs, order, b1, b2)
            g = tr.grad_norms(U).ravel()
            print(f"grad norms over {U} updates: worst relative {np.max(np.abs(g - norms_o) / norms_o):.2e}")
            np.testing.assert_allclose(g, norms_o, rtol=2e-2)
            lr = float(sim.cfg["learning_rate"])
            for pname in ("actor", "critic"):
                d = np.abs(sim.download(pname).astype(np.float64) - ora.buf(pname))
                assert (d <= 2.0001 * lr * U).all(), pname
                assert np.mean(d > 0.5 * lr) < 0.02, pname  # Adam steps agree in sign almost everywhere
            np.testing.assert_allclose(tr.metric_mean, out_o, rtol=2e-2, atol=1e-5)
        assert np.isfinite(sim.download("actor")).all()
    finally:
        tr.close()
        sim.close()


def test_tensor_core_update_is_deterministic(pkg, device):
    cfg = pkg.layouts.default_config(n=1024, family=17, seed=5)
    results = []
    for _ in range(2):
        sim, tr = run_tc(pkg, device, cfg, 32, 16384, 1)
        try:
            tr.rollout_update(0)
            device.finish()
            results.append((sim.download("actor").tobytes(), sim.download("critic").tobytes(),
                            tr.moments(0).tobytes(), tr.grad_norms(2).tobytes()))
        finally:
            tr.close()
            sim.close()
    assert results[0] == results[1]


def test_tensor_core_switch_matches_fp32_path(pkg, device):
    """The same rollout updated once by each path: the two gradients agree
    within the TF32 bar, and switching back restores the fp32 kernel."""
    cfg = pkg.layouts.default_config(n=512, family=1, seed=9)
    sim = pkg.Sim(device, cfg, 32)
    try:
        sim.collect()
        saved = {k: sim.download(k) for k in ("actor", "critic")}
        grads = []
        for enabled in (False, True, False):
            for k, v in saved.items():
                sim.upload(k, v)
            tr = pkg.PPOTrainer(sim, epochs=1, minibatch=16384)
            tr.set_tensor_cores(enabled)
            tr.rollout_update(0)
            device.finish()
            grads.append(np.concatenate([tr.moments(0), tr.moments(2)]))
            tr.close()
        assert rel_l2(grads[1], grads[0]) <= 1e-2
        assert grads[2].tobytes() == grads[0].tobytes()
    finally:
        sim.close()
