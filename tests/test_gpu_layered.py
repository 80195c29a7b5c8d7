"""Layered actor/critic networks on the B200, through the C-ABI.

The reference's networks have one hidden layer of tanh units; the layered
shapes (BASELINE configs 0/1/3: a 2 x 64 actor, 2 x 128 and 2 x 512 critics,
a 4 x 480 GELU actor) are this build's own, so their parity is unpinned by the
reference and checked against the float64 restatement in oracle/mlp.py.
The GPU computes in fp32 (dense kernels, fmaf dot products in input order);
tolerances, stated per check:
  - rollout means and values: |gpu - f64| <= 2e-5 + 1e-4 |f64|;
  - first-update gradient (read back as Adam's first moment, 0.1 x the
    clipped gradient): relative L2 error <= 1e-4 per network, per element
    <= 1e-3 of the network's largest entry; gradient norms within 1e-4.
"""
import numpy as np
import pytest

from conftest import ROOT, _load_module, load_package

pytestmark = pytest.mark.gpu

SHAPES = {
    # BASELINE config 0's 2 x 64 tanh actor with config 1's 2 x 128 critic
    "2x64-tanh/2x128": dict(actor_hidden=64, actor_layers=2, critic_hidden=128, critic_layers=2),
    # BASELINE config 3's 4 x 480 GELU actor with its 2 x 512 critic
    "4x480-gelu/2x512": dict(actor_hidden=480, actor_layers=4, actor_activation="gelu", critic_hidden=512,
                             critic_layers=2),
    # the delay-training build's control-state critic: 64 inputs, 1 x 64 tanh
    # (FIXED_PPO_CRITIC_OBS_DIM=64 with NAV_CRITIC_CONTROL_STATE, sim.metal:166-180)
    "control-state-critic": dict(critic_obs_dim=64),
}


@pytest.fixture(scope="module")
def mlp():
    return _load_module("mdn_oracle_mlp", ROOT / "oracle" / "mlp.py")


def nets(mlp, shape):
    a = mlp.Net(184, shape.get("actor_hidden", 64), shape.get("actor_layers", 1), 4, shape.get("actor_activation", "tanh"),
                log_std=True)
    c = mlp.Net(shape.get("critic_obs_dim", 32), shape.get("critic_hidden", 64), shape.get("critic_layers", 1), 1,
                shape.get("critic_activation", "tanh"))
    return a, c


def make(layouts, shape, n, horizon, seed=5, **cfg):
    pkg = load_package()
    dev = pkg.Device(0)
    c = layouts.default_config(**{**dict(n=n, family=17, seed=seed), **cfg})
    sim = pkg.Sim(dev, c, horizon, **shape)
    return pkg, dev, sim


@pytest.mark.parametrize("name", list(SHAPES))
def test_layered_init(layouts, mlp, name):
    a_net, c_net = nets(mlp, SHAPES[name])
    _, dev, sim = make(layouts, SHAPES[name], 64, 2)
    try:
        actor, critic = sim.download("actor"), sim.download("critic")
        assert actor.size == a_net.param_count() and critic.size == c_net.param_count()
        ra, rc = mlp.init(a_net, c_net)
        assert np.allclose(actor, ra, rtol=2e-6, atol=1e-9) and np.allclose(critic, rc, rtol=2e-6, atol=1e-9)
    finally:
        sim.close()
        dev.close()


def test_one_layer_actor_keeps_reference_init(layouts):
    """A layered simulator whose actor is the reference's 1 x 64 tanh draws it
    first from the same stream: bit-identical to the default simulator's."""
    pkg = load_package()
    dev = pkg.Device(0)
    cfg = layouts.default_config(n=64, family=17, seed=1)
    a = pkg.Sim(dev, cfg, 2)
    b = pkg.Sim(dev, cfg, 2, critic_hidden=128)
    try:
        assert np.array_equal(a.download("actor"), b.download("actor"))
        assert b.critic_params == 32 * 128 + 128 + 128 + 1
    finally:
        a.close()
        b.close()
        dev.close()


def quiet(sim, a_net, rng):
    """Non-zero biases everywhere and log_std = -30, so the sampled action
    equals the mean to ~1e-13."""
    actor = sim.download("actor")
    for l in range(a_net.layers + 1):
        _, b_off = a_net.offsets()[l]
        o = a_net.dims()[l][1]
        actor[b_off: b_off + o] = rng.normal(0, 0.1, o).astype(np.float32)
    actor[-4:] = -30.0
    sim.upload("actor", actor)
    return actor


def close(got, ref, what):
    got = np.asarray(got, np.float64)
    bad = np.abs(got - ref) > 2e-5 + 1e-4 * np.abs(ref)
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size}, worst {np.max(np.abs(got - ref))}"


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("collect", [False, True])
def test_layered_rollout_matches_f64(layouts, mlp, name, collect):
    """Actions (= means), values and bootstrap values of a rollout with episode
    ends inside it, single steps or the captured graph."""
    shape = SHAPES[name]
    a_net, c_net = nets(mlp, shape)
    n, T = 777, 5
    _, dev, sim = make(layouts, shape, n, T, seed=11, family=18, speed=1.0, distance=3.0, max_steps=3)
    try:
        rng = np.random.default_rng(7)
        actor = quiet(sim, a_net, rng)
        critic = sim.download("critic")
        critic[-1] = 0.3
        sim.upload("critic", critic)
        if collect:
            sim.collect()
        else:
            for t in range(T):
                sim.step(t)
        dev.finish()
        obs = sim.download("obs").reshape(T, n, 184)
        co = sim.download("co").reshape(T, n, c_net.inp)
        acts = sim.download("actions").reshape(T, n, 4)
        values = sim.download("values").reshape(T, n)
        nxt = sim.download("next_values").reshape(T, n)
        done = (sim.download("terminated") | sim.download("truncated")).reshape(T, n).astype(bool)
        assert done.any()
        for t in range(T):
            close(acts[t], mlp.actor_means(a_net, actor, obs[t]), f"t={t} means")
            close(values[t], mlp.critic_values(c_net, critic, co[t]), f"t={t} values")
        compared = 0
        for t in range(T - 1):
            # the bootstrap value of a continuing environment is the value of
            # its next critic observation (the same state)
            keep = ~done[t]
            compared += int(keep.sum())
            close(nxt[t][keep], mlp.critic_values(c_net, critic, co[t + 1][keep]), f"t={t} next values")
        assert compared >= 2 * n
    finally:
        sim.close()
        dev.close()


@pytest.mark.parametrize("name", list(SHAPES))
def test_layered_update_gradient(layouts, mlp, name):
    """One full-batch update: Adam's first moments against the float64 gradient."""
    shape = SHAPES[name]
    a_net, c_net = nets(mlp, shape)
    pkg = load_package()
    n, T = 256, 4
    _, dev, sim = make(layouts, shape, n, T, seed=13)
    tr = pkg.PPOTrainer(sim, epochs=1, minibatch=n * T)
    try:
        rng = np.random.default_rng(2)
        actor = sim.download("actor")
        actor[:-4] += rng.normal(0, 0.02, actor.size - 4).astype(np.float32)
        sim.upload("actor", actor)
        critic = sim.download("critic")
        sim.collect()
        dev.finish()
        rows = n * T
        obs = sim.download("obs").reshape(rows, 184)
        co = sim.download("co").reshape(rows, c_net.inp)
        acts = sim.download("actions").reshape(rows, 4)
        logp = sim.download("logp")
        tr.rollout_update(0)
        dev.finish()
        adv, ret = sim.download("advantages"), sim.download("returns")
        g_a, g_c, sums = mlp.gradient(a_net, c_net, actor, critic, obs, co, acts, logp, adv, ret,
                                      float(sim.cfg["entropy_coef"]), rows)
        norms = tr.grad_norms(1)[0]
        for which, g, norm in ((0, g_a, norms[0]), (2, g_c, norms[1])):
            ref, ref_norm = mlp.first_moments(g)
            got = tr.moments(which).astype(np.float64)
            assert got.size == ref.size
            rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
            assert rel <= 1e-4, (which, rel)
            assert np.max(np.abs(got - ref)) <= 1e-3 * np.max(np.abs(ref)), which
            assert abs(norm - ref_norm) <= 1e-4 * ref_norm, (which, norm, ref_norm)
        metrics = tr.metric_mean
        assert abs(metrics[3] - sums[3] / rows) <= 1e-5  # mean ratio
        assert abs(metrics[1] - sums[1]) <= 1e-4 * abs(sums[1]) + 1e-7
    finally:
        tr.close()
        sim.close()
        dev.close()


def test_control_state_observation_matches_oracle(layouts):
    """The 64-input critic observation of every step, single steps through
    episode ends, against the oracle's restatement of sim_critic_obs
    (sim.metal:159-180) on the state the step started from. Inputs 0..31 and
    the control-state inputs are bit-exact except 52/53 (sine and cosine of
    the yaw error: CUDA's atan2f/sinf/cosf against the C library's, within
    2e-6). Also: the 32-input simulator's rows are unchanged by the wider
    layout (same seed, same first step)."""
    pkg = load_package()
    om = _load_module("mdn_oracle_py", ROOT / "oracle" / "oracle.py")
    n, T = 700, 6
    # family 17 (static clutter rooms): no sinf-placed movers, so the clearance
    # and obstacle-offset inputs are bit-exact too
    _, dev, sim = make(layouts, dict(critic_obs_dim=64), n, T, seed=21, family=17, speed=1.0, distance=3.0,
                       max_steps=4, sensor_delay=2, command_delay=2)
    ora = om.OracleSim(layouts, sim.cfg, T, sim.raptor)
    try:
        assert sim.critic_params == 64 * 64 + 64 + 64 + 1
        ended, live = 0, 0.0
        for t in range(T):
            pre = {k: sim.download(k) for k in ("states", "worlds", "runs")}
            sim.step(t)
            dev.finish()
            co = sim.download("co").reshape(T, n, 64)[t]
            ref = ora.critic_obs_rows(pre["states"], pre["worlds"], pre["runs"], 64)
            exact = np.r_[0:52, 54:64]
            assert np.array_equal(co[:, exact], ref[:, exact]), f"t={t}: {np.argwhere(co[:, exact] != ref[:, exact])[:4]}"
            assert np.max(np.abs(co[:, 52:54] - ref[:, 52:54])) <= 2e-6, t
            live = max(live, float(np.abs(co[:, 32:48]).max()) * float(np.abs(co[:, 48:52]).max()))
            ended += int((sim.download("terminated") | sim.download("truncated")).reshape(T, n)[t].sum())
        assert ended > 0 and live > 0  # episode ends; a non-zero RAPTOR hidden state and rotor speeds
    finally:
        sim.close()
        dev.close()
    # the same first step of the 32-input simulator writes the same first 32 inputs
    dev = pkg.Device(0)
    cfg = layouts.default_config(n=n, family=18, seed=21, speed=1.0, distance=3.0, max_steps=4, sensor_delay=2,
                                 command_delay=2)
    narrow = pkg.Sim(dev, cfg, T)
    wide = pkg.Sim(dev, cfg, T, critic_obs_dim=64)
    try:
        narrow.step(0)
        wide.step(0)
        dev.finish()
        assert np.array_equal(narrow.download("co").reshape(T, n, 32)[0],
                              wide.download("co").reshape(T, n, 64)[0, :, :32])
    finally:
        narrow.close()
        wide.close()
        dev.close()


def test_control_state_rejects_other_widths(layouts):
    pkg = load_package()
    dev = pkg.Device(0)
    try:
        for dim in (16, 48, 128):
            with pytest.raises(pkg.MdnError):
                pkg.Sim(dev, layouts.default_config(n=64, family=17, seed=1), 2, critic_obs_dim=dim)
    finally:
        dev.close()


def test_layered_minibatches_deterministic(layouts):
    """Several minibatches and epochs: finite, and two identical trainers end
    with bit-identical parameters (fixed-order gradient sums)."""
    pkg = load_package()
    shape = SHAPES["4x480-gelu/2x512"]
    out = []
    for _ in range(2):
        _, dev, sim = make(layouts, shape, 512, 8, seed=3)
        tr = pkg.PPOTrainer(sim, epochs=2, minibatch=1000)
        try:
            for k in range(2):
                sim.collect()
                tr.rollout_update(k)
            dev.finish()
            a, c = sim.download("actor"), sim.download("critic")
            assert np.isfinite(a).all() and np.isfinite(c).all()
            out.append((a, c))
        finally:
            tr.close()
            sim.close()
            dev.close()
    assert np.array_equal(out[0][0], out[1][0]) and np.array_equal(out[0][1], out[1][1])


def test_layered_rejects_reference_formats(layouts, tmp_path):
    pkg = load_package()
    _, dev, sim = make(layouts, SHAPES["2x64-tanh/2x128"], 64, 2)
    tr = pkg.PPOTrainer(sim, epochs=1, minibatch=128)
    try:
        with pytest.raises(pkg.MdnError):
            tr.save_checkpoint(str(tmp_path / "x.bin"), 17, 5, 0)
        with pytest.raises(pkg.MdnError):
            sim.export_policy(str(tmp_path / "p.bin"), "x")
        with pytest.raises(pkg.MdnError):
            tr.set_tensor_cores(True)
    finally:
        tr.close()
        sim.close()
        dev.close()
