"""TEST INFRASTRUCTURE ONLY: float64 restatement of the layered actor and critic.

The reference's networks have one hidden layer of tanh units (ppo.hpp:35-45);
deeper or GELU networks exist only in this build (mdn_rollout_shape's
actor_layers / critic_layers / *_activation). Parity for them is unpinned by
the reference: this restatement of the same formulas in float64 is the check.
It follows the reference where the reference has a counterpart:
  - parameters flat per layer, W [out][in] row-major then b [out], the actor's
    log_std[4] last (ppo.hpp:35-45 at one layer);
  - initialisation from the seed-1789 xorshift/Box-Muller stream of
    main.mm:548-555 (first layer 0.04 / 0.15, output layer 0.01 / 0.1, as the
    reference; hidden-to-hidden layers 1/sqrt(fan_in)), actor before critic;
  - the geometry prior obs[181..183] added to means 0..2 (ppo.hpp:77);
  - the clipped-PPO loss and its derivatives (ppo.hpp:144-181), the loss scale
    1/B, and per-network global-norm clipping to 0.5 (main.mm:1202).

Only tests/ import this module. The product never does.
"""
import numpy as np
from scipy.special import erf

LOG_2PI = 1.8378770664093453
OBS, CO, ACTIONS = 184, 32, 4


class Net:
    def __init__(self, inp, hidden, layers, out, activation="tanh", log_std=False):
        self.inp, self.hidden, self.layers, self.out = int(inp), int(hidden), int(layers), int(out)
        self.activation = activation
        self.log_std = log_std

    def dims(self):
        """(in, out) of each layer, the output layer last."""
        d = [(self.inp if l == 0 else self.hidden, self.hidden) for l in range(self.layers)]
        return d + [(self.hidden, self.out)]

    def offsets(self):
        """(weight offset, bias offset) of each layer."""
        out, off = [], 0
        for i, o in self.dims():
            out.append((off, off + i * o))
            off += i * o + o
        return out

    def param_count(self):
        i, o = self.dims()[-1]
        return self.offsets()[-1][1] + o + (ACTIONS if self.log_std else 0)

    def layer(self, params, l):
        i, o = self.dims()[l]
        w_off, b_off = self.offsets()[l]
        w = params[w_off: w_off + i * o].reshape(o, i).astype(np.float64)
        b = params[b_off: b_off + o].astype(np.float64)
        return w, b


def act(z, kind):
    if kind == "tanh":
        return np.tanh(z)
    return 0.5 * z * (1.0 + erf(z / np.sqrt(2.0)))


def act_grad(z, kind):
    if kind == "tanh":
        t = np.tanh(z)
        return 1.0 - t * t
    return 0.5 * (1.0 + erf(z / np.sqrt(2.0))) + z * np.exp(-0.5 * z * z) / np.sqrt(2.0 * np.pi)


def init(actor_net, critic_net):
    """Initial float32 parameters, the stream order of main.mm:548-555."""
    state = [1789]

    def unit():
        s = state[0]
        s ^= (s << 13) & 0xFFFFFFFF
        s ^= s >> 17
        s ^= (s << 5) & 0xFFFFFFFF
        state[0] = s
        return np.float32(s >> 8) * np.float32(1.0 / 16777216.0)

    def normal():
        u = max(unit(), np.float32(1e-7))
        r = np.sqrt(np.float32(-2.0) * np.log(np.float32(u)))
        return np.float32(r * np.cos(np.float32(6.2831853) * unit()))

    def fill(net, first, last):
        p = np.zeros(net.param_count(), np.float32)
        for l, ((i, o), (w_off, _)) in enumerate(zip(net.dims(), net.offsets())):
            scale = first if l == 0 else (last if l == net.layers else np.float32(1.0) / np.sqrt(np.float32(i)))
            for k in range(i * o):
                p[w_off + k] = normal() * np.float32(scale)
        if net.log_std:
            p[-ACTIONS:] = -1.0
        return p

    actor = fill(actor_net, np.float32(0.04), np.float32(0.01))
    critic = fill(critic_net, np.float32(0.15), np.float32(0.1))
    return actor, critic


def forward(net, params, x, out_bias=True):
    """Float64 forward over rows x: (inputs of each layer, pre-activations of
    each hidden layer, output layer without / with its bias)."""
    xs, zs = [np.asarray(x, np.float64)], []
    h = xs[0]
    for l in range(net.layers):
        w, b = net.layer(params, l)
        z = h @ w.T + b
        zs.append(z)
        h = act(z, net.activation)
        xs.append(h)
    w, b = net.layer(params, net.layers)
    out = h @ w.T + (b if out_bias else 0.0)
    return xs, zs, out


def actor_means(net, params, obs):
    """Means of the actor: output layer + b2 + the geometry prior (ppo.hpp:65-80)."""
    _, _, out = forward(net, params, obs)
    out[:, :3] += np.asarray(obs, np.float64)[:, OBS - 3:]
    return out


def critic_values(net, params, co):
    return forward(net, params, co)[2][:, 0]


def loss_derivatives(mean, value, log_std, actions, logp_old, adv, ret, scale, entropy_coef, clip=0.2,
                     value_coef=0.5):
    """ppo.hpp:144-181 per row in float64: d mean, d log_std, d value and the
    four loss sums (policy, value, entropy, ratio)."""
    log_std = np.asarray(log_std, np.float64)
    a = np.asarray(actions, np.float64)
    inv_var = np.exp(-2.0 * log_std)
    d = (a - mean) * np.exp(-log_std)
    logp = np.sum(-0.5 * (d * d + 2.0 * log_std + LOG_2PI), axis=1)
    raw = logp - np.asarray(logp_old, np.float64)
    ratio = np.exp(np.clip(raw, -20.0, 20.0))
    adv = np.asarray(adv, np.float64)
    ret = np.asarray(ret, np.float64)
    clipped = np.clip(ratio, 1.0 - clip, 1.0 + clip)
    chosen = np.minimum(ratio * adv, clipped * adv)
    in_range = (raw >= -20.0) & (raw <= 20.0)
    active = in_range & np.where(adv >= 0.0, ratio <= 1.0 + clip, ratio >= 1.0 - clip)
    dlogp = np.where(active, -ratio * adv * scale, 0.0)[:, None]
    diff = a - mean
    dm = dlogp * diff * inv_var
    dls = dlogp * (diff * diff * inv_var - 1.0) - entropy_coef * scale
    dv = value_coef * (value - ret) * scale
    entropy = -entropy_coef * np.sum(log_std + 0.5 * (1.0 + LOG_2PI)) * scale
    sums = np.array([np.sum(-chosen * scale), np.sum(0.5 * value_coef * (value - ret) ** 2 * scale),
                     entropy * len(ratio), np.sum(ratio)])
    return dm, dls, dv, sums


def backward(net, params, xs, zs, dout, grad):
    """Per-layer gradients of the summed output deltas, written into grad."""
    dy = np.asarray(dout, np.float64)
    for l in range(net.layers, -1, -1):
        w, _ = net.layer(params, l)
        w_off, b_off = net.offsets()[l]
        grad[w_off: w_off + w.size] = (dy.T @ xs[l]).ravel()
        grad[b_off: b_off + w.shape[0]] = dy.sum(0)
        if l:
            dy = (dy @ w) * act_grad(zs[l - 1], net.activation)


def gradient(actor_net, critic_net, actor, critic, obs, co, actions, logp_old, adv, ret, entropy_coef, batch):
    """Float64 gradients of one minibatch (rows given), the loss scale 1/batch.
    Returns (actor gradient, critic gradient, loss sums)."""
    xa, za, out_a = forward(actor_net, actor, obs, out_bias=True)
    mean = out_a.copy()
    mean[:, :3] += np.asarray(obs, np.float64)[:, OBS - 3:]
    xc, zc, out_c = forward(critic_net, critic, co)
    value = out_c[:, 0]
    dm, dls, dv, sums = loss_derivatives(mean, value, actor[-ACTIONS:], actions, logp_old, adv, ret,
                                         1.0 / max(float(batch), 1.0), entropy_coef)
    g_actor = np.zeros(actor_net.param_count())
    g_critic = np.zeros(critic_net.param_count())
    backward(actor_net, actor, xa, za, dm, g_actor)
    g_actor[-ACTIONS:] = dls.sum(0)
    backward(critic_net, critic, xc, zc, dv[:, None], g_critic)
    return g_actor, g_critic, sums


def first_moments(g, max_norm=0.5):
    """Adam's first moment after one step from zero: 0.1 x the clipped gradient."""
    norm = float(np.sqrt(np.sum(g * g)))
    return 0.1 * min(1.0, max_norm / norm) * g, norm
