"""CPU checks of the oracle's control-state critic observation (sim.metal:166-180).

The reference computes the 64-input critic observation of its delay-training
build (FIXED_PPO_CRITIC_OBS_DIM=64, NAV_CRITIC_CONTROL_STATE=1) only in its
Metal kernel, so no reference CPU result pins it. The oracle's restatement
(o_critic_obs_rows) is checked here on its own terms: its first 32 inputs are
the oracle's own sim_critic_obs rows of the same state, bit for bit, and its
32 control-state inputs equal an independent numpy float32 restatement of
sim.metal:166-180 (bit for bit, the yaw error's sine and cosine within 1e-6:
numpy's float32 arctan2/sin/cos against the C library's).
"""
import numpy as np


def test_control_state_rows(layouts, oracle_mod, raptor):
    n, T = 48, 5
    cfg = layouts.default_config(n=n, family=18, seed=9, speed=1.0, distance=3.0, max_steps=3)
    ora = oracle_mod.OracleSim(layouts, cfg, T, raptor)
    seen_hidden = seen_rpm = False
    for t in range(T):
        pre = {k: ora.buf(k).copy() for k in ("states", "worlds", "runs")}
        ora.step(t)
        co32 = ora.critic_obs_rows(pre["states"], pre["worlds"], pre["runs"], 32)
        co64 = ora.critic_obs_rows(pre["states"], pre["worlds"], pre["runs"], 64)
        assert np.array_equal(co32, ora.buf("co").reshape(T, n, 32)[t]), t
        assert np.array_equal(co64[:, :32], co32), t

        st, run, w = pre["states"], pre["runs"], pre["worlds"]
        f = np.float32
        ctl = co64[:, 32:]
        assert np.array_equal(ctl[:, 0:16], run["hidden"])
        assert np.array_equal(ctl[:, 16:20], st["rpm"])
        assert np.array_equal(ctl[:, 22:26], run["previous_nav"])
        assert np.array_equal(ctl[:, 26:29], run["desired_velocity"] / f(2))
        q = st["orientation_wxyz"]
        yaw = np.arctan2(f(2) * (q[:, 0] * q[:, 3] + q[:, 1] * q[:, 2]),
                         f(1) - f(2) * (q[:, 2] * q[:, 2] + q[:, 3] * q[:, 3]))
        err = run["yaw"] - yaw
        assert np.max(np.abs(ctl[:, 20] - np.sin(err))) <= 1e-6
        assert np.max(np.abs(ctl[:, 21] - np.cos(err))) <= 1e-6
        g = w["goal"] - st["position"]
        v = st["linear_velocity"]
        dist = np.sqrt(g[:, 0] * g[:, 0] + g[:, 1] * g[:, 1] + g[:, 2] * g[:, 2])
        closing = (g[:, 0] * v[:, 0] + g[:, 1] * v[:, 1] + g[:, 2] * v[:, 2]) / np.maximum(dist, f(1e-6)) / f(4)
        assert np.array_equal(ctl[:, 29], closing)
        assert np.array_equal(ctl[:, 30], dist / f(10))
        assert np.array_equal(ctl[:, 31], np.sqrt(v[:, 0] * v[:, 0] + v[:, 1] * v[:, 1] + v[:, 2] * v[:, 2]) / f(4))
        seen_hidden = seen_hidden or np.abs(ctl[:, 0:16]).max() > 0
        seen_rpm = seen_rpm or np.abs(ctl[:, 16:20]).max() > 0
    assert seen_hidden and seen_rpm


def test_control_state_at_the_goal(layouts, oracle_mod, raptor):
    """Goal at the drone's position: the goal-closing speed divides by the
    1e-6 floor of the distance (sim.metal:178), so it stays finite (zero), and
    the distance input is zero. Identity attitude with run yaw 0.3: yaw error
    0.3 (sine/cosine of it)."""
    cfg = layouts.default_config(n=2, family=17, seed=3)
    ora = oracle_mod.OracleSim(layouts, cfg, 1, raptor)
    st, w, run = ora.buf("states").copy(), ora.buf("worlds").copy(), ora.buf("runs").copy()
    st["orientation_wxyz"] = [1.0, 0.0, 0.0, 0.0]
    st["linear_velocity"] = [[0.5, -1.0, 2.0], [0.0, 0.0, 0.0]]
    w["goal"] = st["position"]
    run["yaw"] = 0.3
    ctl = ora.critic_obs_rows(st, w, run, 64)[:, 32:]
    assert np.all(np.isfinite(ctl))
    assert np.all(ctl[:, 29] == 0.0) and np.all(ctl[:, 30] == 0.0)
    assert np.allclose(ctl[:, 20], np.sin(np.float32(0.3)), atol=1e-7)
    assert np.allclose(ctl[:, 21], np.cos(np.float32(0.3)), atol=1e-7)
    assert ctl[0, 31] == np.float32(np.sqrt(np.float32(0.25 + 1.0 + 4.0))) / np.float32(4)
    assert ctl[1, 31] == 0.0
