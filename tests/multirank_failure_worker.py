"""One rank of the lost-rank check (launched by tests/test_gpu_failure_paths.py
under torch.distributed.run, one process per GPU, NCCL_NVLS_ENABLE=0).

Both ranks run one rollout and one PPO update over libmdn's NCCL
communicator. Then, between steps, with none of its kernels or collectives in
flight, rank 1 leaves (exits). Rank 0 runs the next rollout and update: the
update's allreduce can never complete, so libmdn's host wait must abort the
communicator and raise MDN_ERR_NCCL within MDN_NCCL_TIMEOUT_S, and a further
update must be refused at once. Rank 0 writes what it saw to <outdir>/rank0.txt
and each phase it reaches, with its time, to <outdir>/rank0.progress.

  argv: outdir
"""
import datetime
import os
import pathlib
import sys
import time

sys.path.insert(0, str(pathlib.Path(__file__).resolve().parent))
from conftest import load_package  # noqa: E402


def main():
    outdir = pathlib.Path(sys.argv[1])
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
    sim = pkg.Sim(dev, pkg.layouts.default_config(n=128, family=1, seed=3), 8)
    tr = pkg.PPOTrainer(sim, epochs=1, minibatch=512)
    sim.collect()
    tr.rollout_update(0)
    dev.finish()
    dist.barrier()  # both ranks are between steps, nothing in flight
    if rank == 1:
        os._exit(0)  # leaves without a word, as a crashed rank would
    t0 = time.time()
    progress = open(outdir / "rank0.progress", "w", buffering=1)

    def phase(name):
        progress.write(f"{time.time() - t0:8.2f} {name}\n")

    phase("rank 1 gone")
    sim.collect()
    phase("collect enqueued")
    try:
        tr.rollout_update(1)
        phase("update enqueued")
        dev.finish()
        first = "no error"
    except pkg.MdnError as e:
        first = f"code {e.code}: {e}"
    phase(f"first update: {first}")
    waited = time.time() - t0
    try:
        tr.rollout_update(2)
        second = "no error"
    except pkg.MdnError as e:
        second = f"code {e.code}: {e}"
    phase(f"second update: {second}")
    (outdir / "rank0.txt").write_text(f"{first}\n{second}\n{waited:.1f}\n")
    os._exit(0)


if __name__ == "__main__":
    sys.exit(main())
