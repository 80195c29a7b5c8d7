"""One rank of the multi-GPU parity check (launched by tests/test_gpu_multirank.py
under torch.distributed.run, one process per GPU).

Each rank opens its GPU, joins libmdn's NCCL communicator (the unique id is
passed over a gloo process group), simulates its shard of the global
environments (rank r owns global env ids [r*n, (r+1)*n)), runs one rollout and
one PPO update whose gradients and advantage statistics are allreduced by
libmdn over NCCL, and saves its buffers to <outdir>/rank<r>.npz for the parent
test to compare with a one-GPU run of all environments.

  argv: outdir envs_per_rank horizon epochs minibatch_time_steps mode
  mode: 0 fp32 update, 1 tensor-core update, 2 layered networks (LAYERED)
"""
import datetime
import os
import pathlib
import sys

import numpy as np

sys.path.insert(0, str(pathlib.Path(__file__).resolve().parent))
from conftest import load_package  # noqa: E402

SAVE = ("obs", "co", "actions", "logp", "values", "rewards", "next_values", "terminated", "truncated",
        "advantages", "returns", "actor", "critic", "states", "sensors")


# BASELINE config 0's 2 x 64 actor with config 1's 2 x 128 critic
LAYERED = dict(actor_hidden=64, actor_layers=2, critic_hidden=128, critic_layers=2)


def shape(mode):
    return LAYERED if mode == 2 else {}


def config(pkg, n):
    return pkg.layouts.default_config(n=n, family=18, seed=7, sensor_delay=2, command_delay=2, max_steps=10)


def main():
    outdir = pathlib.Path(sys.argv[1])
    n, horizon, epochs, mb_steps, mode = (int(x) for x in sys.argv[2:7])
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    import torch.distributed as dist
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    pkg = load_package()
    dev = pkg.Device(local)
    obj = [pkg.Device.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    dev.comm_init(rank, world, obj[0])
    sim = pkg.Sim(dev, config(pkg, n), horizon, **shape(mode))
    tr = pkg.PPOTrainer(sim, epochs=epochs, minibatch=mb_steps * n)
    if mode == 1:
        tr.set_tensor_cores(True)
    sim.collect()
    tr.rollout_update(0)
    dev.finish()
    U = epochs * (horizon // mb_steps)
    out = {k: sim.download(k) for k in SAVE}
    out["grad_norms"] = tr.grad_norms(U)
    out["order"] = tr.minibatch_order(0, U)
    out["m_actor"] = tr.moments(0)
    out["m_critic"] = tr.moments(2)
    np.savez(outdir / f"rank{rank}.npz", **out)
    tr.close()
    sim.close()
    dev.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
