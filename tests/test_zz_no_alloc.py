"""mdn_gae_normalize_static: the allocation-free GAE + advantage normalisation.

Some callers cannot call cudaMalloc on their hot path: a framework whose caching
allocator owns all device memory, or a loop that runs under a fixed latency
budget. For them libmdn offers this one entry point, whose
scratch is a fixed array compiled into the library. This test calls it through
the C-ABI on a real rollout, twice in a row (the shared scratch keeps the first
call's contents), and checks each result against the existing entry point,
mdn_ppo_rollout_update, whose first phase computes the same advantages and
returns from the same buffers. Tolerance: bit-exact, as the GPU GAE tests use.
It also checks the size limit is refused with an error, not a fault, and the
case the header advertises for graph users: after one warm-up call, the call
captured into a CUDA graph on a non-default stream and replayed on new
rollouts.
"""
import ctypes

import numpy as np
import pytest

from conftest import load_package

pytestmark = pytest.mark.gpu


def test_static_gae_matches_trainer():
    import torch

    pkg = load_package()
    lib = pkg.lib()
    dev = pkg.Device(0)
    n, T = 512, 32
    cfg = pkg.layouts.default_config(n=n, family=17, seed=3)
    sim = pkg.Sim(dev, cfg, T)
    tr = pkg.PPOTrainer(sim, epochs=1, minibatch=n * T)
    try:
        inputs = [sim.buffer(name)[0] for name in ("rewards", "values", "next_values", "terminated", "truncated")]
        for call in range(2):
            sim.collect()
            dev.finish()
            adv = torch.empty(n * T, dtype=torch.float32, device="cuda")
            ret = torch.empty(n * T, dtype=torch.float32, device="cuda")
            status = lib.mdn_gae_normalize_static(*[ctypes.c_void_p(p) for p in inputs], ctypes.c_void_p(adv.data_ptr()),
                                                  ctypes.c_void_p(ret.data_ptr()), T, n, 0.99, 0.95, None)
            assert status == 0, lib.mdn_last_error()
            torch.cuda.synchronize()
            tr.rollout_update(call)
            dev.finish()
            assert np.array_equal(adv.cpu().numpy(), sim.download("advantages")), f"call {call}: advantages"
            assert np.array_equal(ret.cpu().numpy(), sim.download("returns")), f"call {call}: returns"
        too_many = 4096 * 256 + 1
        status = lib.mdn_gae_normalize_static(*[ctypes.c_void_p(p) for p in inputs], ctypes.c_void_p(adv.data_ptr()),
                                              ctypes.c_void_p(ret.data_ptr()), 1, too_many, 0.99, 0.95, None)
        assert status == 1 and b"scratch limit" in lib.mdn_last_error()
    finally:
        tr.close()
        sim.close()


def test_static_gae_captured_in_graph():
    import torch

    pkg = load_package()
    lib = pkg.lib()
    dev = pkg.Device(0)
    n, T = 384, 16
    cfg = pkg.layouts.default_config(n=n, family=17, seed=11)
    sim = pkg.Sim(dev, cfg, T)
    tr = pkg.PPOTrainer(sim, epochs=1, minibatch=n * T)
    graph = None
    try:
        inputs = [sim.buffer(name)[0] for name in ("rewards", "values", "next_values", "terminated", "truncated")]
        adv = torch.empty(n * T, dtype=torch.float32, device="cuda")
        ret = torch.empty(n * T, dtype=torch.float32, device="cuda")
        args = [ctypes.c_void_p(p) for p in inputs] + [ctypes.c_void_p(adv.data_ptr()), ctypes.c_void_p(ret.data_ptr()),
                                                       T, n, 0.99, 0.95]
        sim.collect()
        dev.finish()
        assert lib.mdn_gae_normalize_static(*args, None) == 0, lib.mdn_last_error()  # warm-up: scratch address
        torch.cuda.synchronize()
        stream = torch.cuda.Stream()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            status = lib.mdn_gae_normalize_static(*args, ctypes.c_void_p(stream.cuda_stream))
        assert status == 0, lib.mdn_last_error()
        for call in range(2):
            sim.collect()
            dev.finish()
            adv.fill_(float("nan"))
            ret.fill_(float("nan"))
            graph.replay()
            torch.cuda.synchronize()
            tr.rollout_update(call)
            dev.finish()
            assert np.array_equal(adv.cpu().numpy(), sim.download("advantages")), f"replay {call}: advantages"
            assert np.array_equal(ret.cpu().numpy(), sim.download("returns")), f"replay {call}: returns"
    finally:
        graph = None
        torch.cuda.synchronize()
        tr.close()
        sim.close()
