"""B200-native metal-drone-nav rollout/PPO hot path (host side).

The compute path is libmdn.so: CUDA kernels for sm_100a behind the C-ABI in
include/mdn.h (built from csrc/ by build()). This package is a thin Python
veneer over that C-ABI with the reference's host API names (Sim, PPOTrainer;
main.mm:516-603,1110-1476). There is no CPU fallback: without libmdn.so the
constructors raise.
"""
import pathlib
import subprocess

from . import layouts  # noqa: F401
from .capi import (ChallengeBank, ChallengeSampler, Device, MdnError, PPOTrainer, Sim, challenge_settings,  # noqa: F401
                   checkpoint_inspect, default_raptor, evaluate_bank, gather_rollout_evidence, lib, runtime_config,
                   sha256_file, task_control, task_settings, write_policy)

PACKAGE_DIR = pathlib.Path(__file__).resolve().parent


def build(jobs=8):
    """Compile libmdn.so for sm_100a in-tree (nvcc cross-compiles without a GPU)."""
    subprocess.run(["make", "-s", "-j", str(jobs), "-C", str(PACKAGE_DIR / "csrc")], check=True)
    return PACKAGE_DIR / "libmdn.so"
