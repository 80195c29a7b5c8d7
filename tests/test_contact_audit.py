"""Mechanical contact audit (vehicle_geometry.hpp GJK, navigation_contact.metal).

CPU: the reference's own vg_world_contact (compiled unmodified into
oracle/_ref/libref_oracle.so) on known poses, as the checker's sanity.
GPU: with the audit enabled, each policy step's audit record of every
environment that did not reset in that step equals the reference's
vg_world_contact of the downloaded post-step pose, byte for byte.
"""
import numpy as np
import pytest

from conftest import load_oracle_module, load_package

AUDIT = np.dtype([("physical_clearance_m", "<f4"), ("safety_clearance_m", "<f4"), ("contact", "<u4"),
                  ("ambiguous", "<u4")])


def ref_audit(rlib, pos, quat, world, t, margin=0.04):
    om = load_oracle_module()
    out = np.zeros(1, AUDIT)
    p = np.ascontiguousarray(pos, np.float32)
    q = np.ascontiguousarray(quat, np.float32)
    w = np.ascontiguousarray(world)
    rlib.ref_vg_world_contact(om.ptr(p), om.ptr(q), om.ptr(w), float(t), float(margin), om.ptr(out))
    return out[0]


def one_box_world(layouts, center, half):
    w = np.zeros(1, layouts.WORLD)
    w["count"] = 1
    w["obstacles"][0, 0]["kind"] = 0
    w["obstacles"][0, 0]["center"] = center
    w["obstacles"][0, 0]["size"] = half
    return w


def test_reference_audit_sanity(rlib, layouts):
    ident = [1.0, 0.0, 0.0, 0.0]
    w = one_box_world(layouts, [3.0, 0.0, 1.5], [0.5, 0.5, 0.5])
    free = ref_audit(rlib, [1.0, 0.0, 1.5], ident, w, 0.0)
    assert free["contact"] == 0 and free["ambiguous"] == 0
    # the rotor discs reach furthest ahead: 28 mm centre + 22.5 mm radius
    assert abs(float(free["physical_clearance_m"]) - (3.0 - 0.5 - 1.0 - 0.0505)) < 1e-4
    assert abs(float(free["safety_clearance_m"]) - (float(free["physical_clearance_m"]) - 0.04)) < 1e-6
    inside = ref_audit(rlib, [2.6, 0.0, 1.5], ident, w, 0.0)
    assert inside["contact"] == 1 and inside["physical_clearance_m"] == 0.0
    floor = ref_audit(rlib, [1.0, 0.0, 0.002], ident, w, 0.0)
    assert floor["contact"] == 1
    mover = np.zeros(1, layouts.WORLD)
    mover["count"] = 1
    mover["obstacles"][0, 0]["kind"] = 3
    mover["obstacles"][0, 0]["size"] = [0.3, 1.0, 0.0]
    assert ref_audit(rlib, [1.0, 0.0, 1.5], ident, mover, 0.0)["ambiguous"] == 1


@pytest.mark.gpu
@pytest.mark.parametrize("family", [1, 2, 3, 17, 18])
def test_gpu_audit_matches_reference(rlib, layouts, family):
    pkg = load_package()
    dev = pkg.Device(0)
    n, T = 512, 8
    cfg = layouts.default_config(n=n, family=family, seed=11, speed=1.0, distance=3.0)
    sim = pkg.Sim(dev, cfg, T)
    try:
        sim.set_contact_audit(True, 0.04)
        checked = 0
        for t in range(T):
            sim.step(t)
            dev.finish()
            audit = sim.download("contact_audit").reshape(T, n)[t]
            states = sim.download("states")
            runs = sim.download("runs")
            worlds = sim.download("worlds")
            reset = (sim.download("terminated").reshape(T, n)[t] | sim.download("truncated").reshape(T, n)[t]) != 0
            for i in range(n):
                if reset[i]:
                    continue  # the audited pose was replaced by the new episode's start
                ref = ref_audit(rlib, states[i]["position"], states[i]["orientation_wxyz"], worlds[i:i + 1],
                                runs[i]["elapsed"])
                assert audit[i].tobytes() == ref.tobytes(), (t, i, audit[i], ref)
                checked += 1
        assert checked > n * T // 2
        if family == 18:  # moving spheres are outside the reference audit's shapes: ambiguous
            assert audit["ambiguous"][3::4].mean() > 0.5
    finally:
        sim.close()
        dev.close()


@pytest.mark.gpu
def test_audit_off_changes_nothing(layouts):
    pkg = load_package()
    dev = pkg.Device(0)
    cfg = layouts.default_config(n=256, family=17, seed=5)
    a, b = pkg.Sim(dev, cfg, 4), pkg.Sim(dev, cfg, 4)
    try:
        b.set_contact_audit(True)
        a.collect()
        b.collect()
        dev.finish()
        for name in ("states", "obs", "actions", "rewards", "terminated"):
            assert a.download(name).tobytes() == b.download(name).tobytes(), name
    finally:
        a.close()
        b.close()
        dev.close()
