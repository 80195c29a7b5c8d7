"""B200-native metal-drone-nav rollout/PPO hot path (host side).

The compute path is libmdn.so (CUDA kernels for sm_100a behind the C-ABI in
include/mdn.h). This package is a thin Python veneer over that C-ABI with the
reference's host API names (Sim, PPOTrainer; main.mm:516-603,1110-1476).
"""
from . import layouts  # noqa: F401
