"""The depth kernel's divide-free quotient (csrc/mdn_device.cuh div_by_rcp:
a * RN(1/d) with two fused residual corrections, Markstein's method) returns
the IEEE-rounded quotient bit for bit on the ray tests' operand ranges. The
ranges themselves are compared bitwise against the oracle by the rollout
parity tests; this checks the arithmetic on 2^31 random operand pairs."""
import pytest

from conftest import load_package

pytestmark = pytest.mark.gpu


def test_division_matches_ieee():
    pkg = load_package()
    dev = pkg.Device(0)
    try:
        for seed in (1, 0x5EED):
            assert dev.selftest_division(1 << 30, seed) == 0
    finally:
        dev.close()
