"""CPU checks of the float64 restatement of the layered networks (oracle/mlp.py).

The reference has no layered networks, so their parity is unpinned by it; the
restatement is checked here on its own terms: at one tanh hidden layer of 64
units its initial parameters equal the reference path's (the C oracle's
o_wide_init, pinned to main.mm:548-555), and its gradients equal finite
differences of its own loss.
"""
import numpy as np
import pytest

from conftest import ROOT, _load_module


@pytest.fixture(scope="module")
def mlp():
    return _load_module("mdn_oracle_mlp", ROOT / "oracle" / "mlp.py")


def test_one_layer_init_equals_reference(mlp, olib, oracle_mod):
    a_net = mlp.Net(184, 64, 1, 4, "tanh", log_std=True)
    c_net = mlp.Net(32, 64, 1, 1)
    actor, critic = mlp.init(a_net, c_net)
    ref_a = np.zeros(olib.o_wide_param_count(64), np.float32)
    ref_c = np.zeros(olib.o_critic_param_count(), np.float32)
    olib.o_wide_init(64, oracle_mod.ptr(ref_a), oracle_mod.ptr(ref_c))
    assert actor.size == ref_a.size == 12104 and critic.size == ref_c.size
    # numpy's float32 log/cos may differ from libm's in the last place
    assert np.allclose(actor, ref_a, rtol=2e-6, atol=1e-9)
    assert np.allclose(critic, ref_c, rtol=2e-6, atol=1e-9)


def test_layouts_and_counts(mlp):
    a = mlp.Net(184, 480, 4, 4, "gelu", log_std=True)
    c = mlp.Net(32, 512, 2, 1)
    assert a.param_count() == 184 * 480 + 480 + 3 * (480 * 480 + 480) + 4 * 480 + 4 + 4
    assert c.param_count() == 32 * 512 + 512 + 512 * 512 + 512 + 512 + 1
    w_off, b_off = a.offsets()[4]
    assert b_off == w_off + 4 * 480 and b_off + 4 + 4 == a.param_count()


@pytest.mark.parametrize("kind,critic_in", [("tanh", 32), ("gelu", 32), ("tanh", 64)])
def test_gradient_matches_finite_differences(mlp, kind, critic_in):
    """critic_in 64: the control-state critic's input width."""
    rng = np.random.default_rng(3)
    a_net = mlp.Net(184, 7, 3, 4, kind, log_std=True)
    c_net = mlp.Net(critic_in, 5, 2, 1, kind)
    actor = rng.normal(0, 0.3, a_net.param_count())
    actor[-4:] = rng.uniform(-1.5, -0.5, 4)
    critic = rng.normal(0, 0.3, c_net.param_count())
    rows = 9
    obs = rng.normal(0, 1, (rows, 184))
    co = rng.normal(0, 1, (rows, critic_in))
    actions = rng.normal(0, 1, (rows, 4))
    adv = rng.normal(0, 1, rows)
    ret = rng.normal(0, 1, rows)
    # logp_old so that every ratio sits well inside the clip range (no kinks)
    mean = mlp.actor_means(a_net, actor, obs)
    d = (actions - mean) * np.exp(-actor[-4:])
    logp = np.sum(-0.5 * (d * d + 2.0 * actor[-4:] + mlp.LOG_2PI), axis=1)
    logp_old = logp + rng.uniform(-0.05, 0.05, rows)
    ec = 0.005

    def loss(a, c):
        m = mlp.actor_means(a_net, a, obs)
        v = mlp.critic_values(c_net, c, co)
        dd = (actions - m) * np.exp(-a[-4:])
        lp = np.sum(-0.5 * (dd * dd + 2.0 * a[-4:] + mlp.LOG_2PI), axis=1)
        ratio = np.exp(lp - logp_old)
        policy = -np.minimum(ratio * adv, np.clip(ratio, 0.8, 1.2) * adv)
        value = 0.5 * 0.5 * (v - ret) ** 2
        entropy = -ec * np.sum(a[-4:] + 0.5 * (1.0 + mlp.LOG_2PI))
        return np.sum(policy + value) / rows + entropy

    g_a, g_c, _ = mlp.gradient(a_net, c_net, actor, critic, obs, co, actions, logp_old, adv, ret, ec, rows)
    eps = 1e-6
    for params, grad, which in ((actor, g_a, 0), (critic, g_c, 1)):
        for i in rng.choice(params.size, 40, replace=False):
            plus, minus = params.copy(), params.copy()
            plus[i] += eps
            minus[i] -= eps
            if which == 0:
                fd = (loss(plus, critic) - loss(minus, critic)) / (2 * eps)
            else:
                fd = (loss(actor, plus) - loss(actor, minus)) / (2 * eps)
            assert abs(fd - grad[i]) <= 1e-6 + 1e-5 * abs(fd), (which, i, fd, grad[i])
