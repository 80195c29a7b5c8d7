"""Multi-GPU trainer parity: two ranks over NCCL equal one GPU.

Two processes (tests/multirank_gpu_worker.py under torch.distributed.run)
each simulate 256 of 512 global environments and run one rollout and one PPO
update, with libmdn allreducing the advantage statistics (fp64) and every
minibatch gradient over NCCL. This process then runs the same 512 environments
on one GPU. With a minibatch of whole time steps, global minibatch k is the
union of the ranks' chunk k (T-major rows), so the two updates see the same
rows and the same 1/B loss scale:

* every rank's rollout slice equals the one-GPU rollout bit for bit (global
  environment ids, the same per-environment kernels);
* normalised advantages and returns are bit-identical (one fp64 partial per
  rank, summed exactly);
* both ranks hold bit-identical parameters (replicated Adam);
* gradient norms of every update within 1e-5 relative and Adam-updated
  parameters within 1e-5 relative + 1e-7 absolute of the one-GPU update (the
  gradient sums add the same rows in another order), except parameters whose
  accumulated gradient is at rounding level, bounded by 2*lr per update.

Three update paths run: the fp32 kernel, the tensor-core kernel (whose
TMA loads read only this GPU's own memory) and the layered networks (a 2 x 64
actor and a 2 x 128 critic, whose flat gradient is allreduced the same way).
Needs two GPUs; NVLS is off (NCCL_NVLS_ENABLE=0).
"""
import os
import pathlib
import socket
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT, load_package

pytestmark = pytest.mark.gpu

N_RANK, HORIZON, EPOCHS, MB_STEPS, WORLD = 256, 16, 2, 2, 2


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.skipif(gpu_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mode", [0, 1, 2], ids=["fp32_update", "tensor_core_update", "layered_update"])
def test_two_ranks_equal_one_gpu(tmp_path, mode):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MASTER_ADDR="127.0.0.1")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={WORLD}", "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           str(ROOT / "tests" / "multirank_gpu_worker.py"), str(tmp_path), str(N_RANK), str(HORIZON), str(EPOCHS),
           str(MB_STEPS), str(mode)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    ranks = [np.load(tmp_path / f"rank{k}.npz") for k in range(WORLD)]

    sys.path.insert(0, str(ROOT / "tests"))
    import multirank_gpu_worker as worker
    pkg = load_package()
    dev = pkg.Device(0)
    n = N_RANK * WORLD
    sim = pkg.Sim(dev, worker.config(pkg, n), HORIZON, **worker.shape(mode))
    tr = pkg.PPOTrainer(sim, epochs=EPOCHS, minibatch=MB_STEPS * n)
    if mode == 1:
        tr.set_tensor_cores(True)
    try:
        sim.collect()
        U = EPOCHS * (HORIZON // MB_STEPS)
        order = tr.minibatch_order(0, U)
        tr.rollout_update(0)
        dev.finish()
        one = {k: sim.download(k) for k in worker.SAVE}
        assert int(one["terminated"].sum() + one["truncated"].sum()) > 0, "no episode ended in the rollout"
        for k, rk in enumerate(ranks):
            sl = slice(k * N_RANK, (k + 1) * N_RANK)
            for name in ("obs", "co", "actions", "logp", "values", "rewards", "next_values", "terminated",
                         "truncated", "advantages", "returns"):
                g = one[name].reshape(HORIZON, n, -1)[:, sl]
                assert np.array_equal(rk[name].reshape(HORIZON, N_RANK, -1), g), f"rank {k} {name}"
            for name in ("states", "sensors"):
                per = one[name].reshape(n, -1)[sl]
                assert rk[name].reshape(N_RANK, -1).tobytes() == per.tobytes(), f"rank {k} {name}"
            assert np.array_equal(rk["order"].astype(np.int64) * WORLD, order), "chunk order (row starts)"
        for name in ("actor", "critic", "grad_norms"):
            assert ranks[0][name].tobytes() == ranks[1][name].tobytes(), f"replicas differ: {name}"
        rel = np.abs(ranks[0]["grad_norms"] - tr.grad_norms(U)) / tr.grad_norms(U)
        print(f"grad norms: worst relative difference {rel.max():.3e}")
        np.testing.assert_allclose(ranks[0]["grad_norms"], tr.grad_norms(U), rtol=1e-5)
        lr = float(sim.cfg["learning_rate"])
        for pname, which in (("actor", 0), ("critic", 2)):
            p_g, p_o = ranks[0][pname], one[pname]
            m_o = tr.moments(which)
            diff = np.abs(p_g.astype(np.float64) - p_o)
            bad = diff > 1e-7 + 1e-5 * np.abs(p_o)
            tiny = np.abs(m_o) <= 1e-4 * np.abs(m_o).max()
            print(f"{pname}: {int(bad.sum())} beyond 1e-5, worst {diff.max():.3e}")
            assert not (bad & ~tiny).any(), f"{pname}: {int((bad & ~tiny).sum())} parameters differ"
            assert (diff <= 2.0001 * lr * U).all()
    finally:
        tr.close()
        sim.close()
        dev.close()
