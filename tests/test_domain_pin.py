"""Per-episode plant variation (physics_domain.hpp) on the CPU.

The oracle's rl_physics_sample_domain restatement (mdn_oracle.c
o_physics_sample_domain) equals the reference's own physics_domain.hpp,
compiled unmodified into oracle/_ref/libref_oracle.so, bit for bit: accept /
reject flag, the varied plant, the 17 sample floats and the RNG state after
the draws, over seeds, amplitudes (0 to 1 and out of range) and ranges
(the stress range, rejecting thrust-to-weight floors, malformed ranges).
libmdn's stress range equals rl_physics_domain_stress_range.
"""
import numpy as np
import pytest

from conftest import load_oracle_module, load_package


def params(olib, layouts):
    p = np.zeros((), layouts.PARAMS)
    olib.o_physics_default(load_oracle_module().ptr(p))
    return p


def stress(layouts):
    r = np.zeros((), layouts.DOMAIN_RANGE)
    load_package().lib().mdn_domain_stress_range(r.ctypes.data)
    return r


def test_stress_range_matches_reference(rlib, layouts):
    ours = stress(layouts)
    ref = np.zeros((), layouts.DOMAIN_RANGE)
    rlib.ref_domain_stress_range(ref.ctypes.data)
    assert ours.tobytes() == ref.tobytes()


def ranges(layouts):
    base = stress(layouts)
    out = [("stress", base)]
    strict = base.copy()
    strict["minimum_thrust_to_weight"] = 1.46  # draws span about 1.26-1.70 at amplitude 1: some fail
    out.append(("strict", strict))
    wide = base.copy()
    wide["mass_scale_min"], wide["mass_scale_max"] = 0.5, 1.6
    wide["thrust_gain_min"], wide["thrust_gain_max"] = 0.6, 1.3
    out.append(("wide", wide))
    for field, value in (("mass_scale_min", 0.0), ("thrust_gain_max", 0.5), ("minimum_thrust_to_weight", 0.9),
                         ("rising_lag_scale_max", float("nan"))):
        bad = base.copy()
        bad[field] = value
        out.append((f"bad_{field}", bad))
    return out


@pytest.mark.parametrize("amplitude", [0.0, 0.25, 0.8, 1.0, 1.5, -0.1, float("nan")])
def test_sample_domain_matches_reference(olib, rlib, layouts, amplitude):
    om = load_oracle_module()
    nominal = params(olib, layouts)
    accepted = rejected = 0
    for name, rng_range in ranges(layouts):
        for seed in (1, 7, 0x3F84D5B5, 0xFFFFFFFF, 0, 123456789, 0x9E3779B9, 42):
            a_rng = np.array([seed], np.uint32)
            b_rng = a_rng.copy()
            va, vb = np.zeros((), layouts.PARAMS), np.zeros((), layouts.PARAMS)
            sa, sb = np.zeros(17, np.float32), np.zeros(17, np.float32)
            ok_a = olib.o_physics_sample_domain(om.ptr(nominal), om.ptr(a_rng), amplitude, om.ptr(rng_range),
                                                om.ptr(va), om.ptr(sa))
            ok_b = rlib.ref_physics_sample_domain(om.ptr(nominal), om.ptr(b_rng), amplitude, om.ptr(rng_range),
                                                  om.ptr(vb), om.ptr(sb))
            assert ok_a == ok_b, (name, seed)
            assert a_rng[0] == b_rng[0], (name, seed)
            if ok_a:
                accepted += 1
                assert va.tobytes() == vb.tobytes(), (name, seed)
                assert sa.tobytes() == sb.tobytes(), (name, seed)
            else:
                rejected += 1
    if amplitude == 0.25 or amplitude == 0.8:
        assert accepted and rejected


def test_zero_amplitude_is_nominal(olib, layouts):
    om = load_oracle_module()
    nominal = params(olib, layouts)
    rng = np.array([99], np.uint32)
    varied = np.zeros((), layouts.PARAMS)
    assert olib.o_physics_sample_domain(om.ptr(nominal), om.ptr(rng), 0.0, om.ptr(stress(layouts)), om.ptr(varied),
                                        None) == 1
    assert varied.tobytes() == nominal.tobytes() and rng[0] == 99  # no draws


def test_episode_seed(olib, layouts):
    """sim_domain_episode_seed (sim.metal:50-54) against a direct restatement."""
    om = load_oracle_module()
    rt = load_package().runtime_config(0.5)
    for cfg_seed, env, episode in ((42, 0, 0), (1, 17, 3), (0xFFFFFFFF, 65535, 1000), (5, 2, 0xFFFFFFFF)):
        M = 0xFFFFFFFF
        s = (int(rt["domain_seed"]) ^ cfg_seed ^ (((env + 1) * 0x9E3779B9) & M) ^ (((episode + 1) * 0x85EBCA6B) & M))
        s ^= s >> 16
        s = (s * 0x7FEB352D) & M
        s ^= s >> 15
        s = (s * 0x846CA68B) & M
        s ^= s >> 16
        assert olib.o_domain_episode_seed(om.ptr(rt), cfg_seed, env, episode) == (s or 1)
