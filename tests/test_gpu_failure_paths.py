"""Failure detection without a GPU fault.

* A bounded barrier wait that nothing completes gives up after its limit and
  surfaces as MDN_ERR_TIMEOUT on the host; the context stays usable.
* A rank that leaves between steps: the surviving rank's next collective
  cannot complete, its host wait aborts the NCCL communicator within the
  deadline (MDN_NCCL_TIMEOUT_S) and raises MDN_ERR_NCCL, and later updates are
  refused. Two GPUs, NVLS off; the leaving rank has nothing in flight.
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


def gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def test_barrier_wait_times_out():
    pkg = load_package()
    dev = pkg.Device(0)
    try:
        with pytest.raises(pkg.MdnError) as e:
            dev.selftest_barrier_timeout(2_000_000)  # ~1 ms at 2 GHz; nothing arrives
        assert e.value.code == pkg.capi.ERR["TIMEOUT"]
        dev.selftest_barrier_timeout(2_000_000, arrive=True)
        # the context is still usable afterwards
        sim = pkg.Sim(dev, pkg.layouts.default_config(n=64, family=1, seed=2), 2)
        sim.collect()
        dev.finish()
        assert np.isfinite(sim.download("states").view(np.float32)).all()
        sim.close()
    finally:
        dev.close()


@pytest.mark.skipif(gpu_count() < 2, reason="needs two GPUs")
def test_lost_rank_aborts_the_collective(tmp_path):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MDN_NCCL_TIMEOUT_S="20", MASTER_ADDR="127.0.0.1")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={port}",
           str(ROOT / "tests" / "multirank_failure_worker.py"), str(tmp_path)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    out = tmp_path / "rank0.txt"
    progress = tmp_path / "rank0.progress"
    seen = progress.read_text() if progress.exists() else "(no progress file)"
    assert out.exists(), "rank 0 phases:\n" + seen + "\n" + r.stdout[-1500:] + r.stderr[-1500:]
    first, second, waited = out.read_text().splitlines()
    nccl = pkg_err_code("NCCL")
    assert first.startswith(f"code {nccl}"), first
    assert second.startswith(f"code {nccl}"), second
    assert float(waited) < 120


def pkg_err_code(name):
    return load_package().capi.ERR[name]
