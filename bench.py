#!/usr/bin/env python
"""Benchmark of the B200 rollout/PPO hot path (BASELINE.json metric).

Metric: policy env-steps/s at 65,536 environments, one env-step = depth ray
casting + observation + actor + 5 RAPTOR/L2F substeps (the reference's
Sim::collect, main.mm:576-598); PPO update ms reported beside it
(PPOTrainer::rollout_update, main.mm:1321-1384).

One bench step = one rollout of `--horizon` policy steps over all
environments, then one PPO update (4 epochs x 16 minibatches by default).
`value` = env-steps of the K timed rollouts / device time of those rollouts
(CUDA events on the simulator stream, max over ranks). `e2e` = the same
metric through the public C-ABI with the policy uploaded from pinned host
memory and the episode report read back every step, host wall clock.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mdn|reference]

Under torchrun each rank drives one GPU with envs/N environments (global env
ids, identical worlds to the 1-GPU run); PPO gradients and advantage
statistics are allreduced with NCCL.
"""
import argparse
import ctypes
import importlib.util
import json
import os
import pathlib
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
METRIC = "policy env-steps/sec at 65,536 envs (physics+RAPTOR+depth+actor); PPO update ms"


def _load(name, path, package_dir=None):
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(
        name, path, submodule_search_locations=[str(package_dir)] if package_dir else None)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def package():
    d = ROOT / "metal-drone-nav_b200"
    return _load("mdn_b200", d / "__init__.py", d)


def oracle_module():
    return _load("mdn_oracle_py", ROOT / "oracle" / "oracle.py")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mdn", choices=["mdn", "reference"])
    ap.add_argument("--envs", type=int, default=65536, help="environments over all ranks")
    ap.add_argument("--horizon", type=int, default=128)
    ap.add_argument("--epochs", type=int, default=4)
    ap.add_argument("--minibatches", type=int, default=16)
    ap.add_argument("--family", type=int, default=18,
                    help="18 = mixed capability (BASELINE configs 2/4: 50%% static clutter, 25%% long-goal rooms, "
                         "25%% combined courses with movers); 17 = static clutter only")
    ap.add_argument("--delay", type=int, default=2,
                    help="sensor and command delay in policy ticks (2 = the 100 ms buffers of BASELINE config 2)")
    ap.add_argument("--actor-hidden", type=int, default=64,
                    help="64 = the reference's 12,104-parameter actor; 5120 = the 967,688-parameter wide actor "
                         "(BASELINE config 3), evaluated on the tcgen05 tensor cores")
    ap.add_argument("--ppo-fp32", action="store_true",
                    help="run the timed PPO updates on the fp32 parity path instead of the tcgen05 TF32 kernel")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the BASELINE config 0 and config 1 measurements")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-wide", action="store_true", help="skip the wide-actor (BASELINE config 3) measurement")
    return ap.parse_args()


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    FIELDS = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, bus=None):
        self.bus = bus  # PCI bus number of the benchmarked GPU (torch reports an int)
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        rows = [r for r in self.rows if len(r) >= 9]
        if self.bus is not None:
            def bus_of(field):
                try:
                    return int(field.split(":")[-2], 16)
                except (ValueError, IndexError):
                    return None
            mine = [r for r in rows if bus_of(r[1]) == int(self.bus)]
            rows = mine or rows
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({names[k] for r in rows for k in range(4) if r[5 + k].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# -------------------------------------------------------------- distributed
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self):
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, values):
        if not self.pg:
            return list(values)
        import torch
        t = torch.tensor(list(values), dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return t.tolist()

    def broadcast_bytes(self, data):
        if not self.pg:
            return data
        obj = [data]
        self.pg.broadcast_object_list(obj, src=0)
        return obj[0]

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# ------------------------------------------------------------ work counts
def sense_bytes_per_env():
    # state 68 + run 184 + world 676 + previous range frame 1280 read; range frame
    # 1280 + pose 48 + actor obs 736 + critic obs 128 written.
    return 68 + 184 + 676 + 1280 + 1280 + 48 + 736 + 128


def kernel_work(mean_obstacles):
    """Algorithmic FLOP and bytes per environment of each rollout kernel:
    depth 320 rays x (obstacles + room) x 26 FLOP per ray-primitive test plus
    30 per ray, observation and guidance 10,400; actor 2*(184*64 + 64*4) and
    critic 2*(32*64 + 64); advance 5 RAPTOR substeps of 3,904, RK4 2,200,
    clearance 1,260 and the bootstrap critic."""
    rays = 320
    depth = rays * (mean_obstacles + 1) * 26 + rays * 30
    return {
        "sense": {"flop": depth + 10400, "bytes": sense_bytes_per_env()},
        "act": {"flop": 2 * (184 * 64 + 64 * 4) + 2 * (32 * 64 + 64), "bytes": 736 + 128 + 184 + 16 + 4 + 4 + 16 + 184},
        "advance": {"flop": 19520 + 2200 + 1260 + 2 * (32 * 64 + 64), "bytes": 2 * (68 + 184) + 676 + 4 * 4 + 2 + 4},
    }


# PPO update, per row and epoch of a minibatch: HBM bytes the minibatch kernel
# must read (observation 184 floats, critic observation 32, action 4, old
# log-prob, advantage, return) and its arithmetic (forward, deltas and weight
# gradients of both networks, cpu_reference.hpp:437-551).
PPO_BYTES_PER_ROW = 184 * 4 + 32 * 4 + 4 * 4 + 4 + 4 + 4
PPO_GEMM_FLOP_PER_ROW = 2 * 2 * (184 + 32) * 64          # forward + weight-gradient products
PPO_FLOP_PER_ROW = PPO_GEMM_FLOP_PER_ROW + 2 * (64 * 4 + 64) * 2 + 6 * 64 * 2 + 2 * 64 * 4 + 200


def ppo_roofline(trainer, minibatch_rows, dist, peaks, fp32_peak):
    """Minibatch kernel of the update (one launch = one minibatch's gradient
    partials and their sum), timed with CUDA events on the simulator stream,
    against the measured HBM copy peak (its bound) and the tensor / FP32 peak."""
    ms = float(np.median([trainer.profile_minibatch(u % trainer.updates) for u in range(3)]))
    (ms,) = dist.max([ms])
    t = ms * 1e-3
    gbs = minibatch_rows * PPO_BYTES_PER_ROW / t / 1e9
    hbm = peaks.get("hbm_gbs", 6650.0)
    tensor = trainer.tensor_cores
    tflops = minibatch_rows * (PPO_GEMM_FLOP_PER_ROW if tensor else PPO_FLOP_PER_ROW) / t / 1e12
    compute_peak = peaks.get("bf16_tflops", 1590.0) / 2.0 if tensor else fp32_peak
    return {"kernel": "k_mb_tc" if tensor else "k_mb_fused", "ms_per_minibatch": ms, "minibatch_rows": minibatch_rows,
            "bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
            "bytes_per_row_epoch": PPO_BYTES_PER_ROW,
            "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
            "compute": {"achieved": tflops, "unit": "TFLOP/s", "peak": compute_peak,
                        "frac": tflops / compute_peak,
                        "flop_per_row_epoch": PPO_GEMM_FLOP_PER_ROW if tensor else PPO_FLOP_PER_ROW,
                        "peak_source": "half the measured bf16 dense rate (TF32 tensor cores)" if tensor
                        else "measured pure-FMA FP32 kernel, this run"}}


def read_profile_traffic(kernel):
    """DRAM bytes per environment measured by ncu (profiles/<kernel>_traffic.txt)."""
    f = ROOT / "profiles" / f"{kernel}_traffic.txt"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.startswith("dram_bytes_per_env:"):
            return float(line.split(":", 1)[1])
    return None


# ------------------------------------------------------------ wide actor
WIDE_HIDDEN = 5120
WIDE_ENVS = 16384


def measure_wide(pkg, dev, dist, args, peaks):
    """BASELINE config 3 on this rank's share: 16,384 environments (over all
    ranks), the 967,688-parameter actor (184 -> 5120 tanh -> 4) on tcgen05 TF32,
    T=128 rollouts, PPO 4 epochs x 16 minibatches. One warm-up rollout + update,
    then two timed ones (CUDA events on the simulator stream, max over ranks)."""
    L = pkg.layouts
    n = WIDE_ENVS // dist.world
    horizon, epochs, minibatches, steps = 128, 4, 16, 2
    cfg = L.default_config(n=n, family=17, seed=43)
    sim = pkg.Sim(dev, cfg, horizon, actor_hidden=WIDE_HIDDEN)
    tr = pkg.PPOTrainer(sim, epochs=epochs, minibatch=n * horizon // minibatches)
    try:
        sim.collect()
        tr.rollout_update(0)
        dev.finish()
        dist.barrier()
        c_ms, u_ms = 0.0, 0.0
        for k in range(steps):
            sim.collect()
            c_ms += sim.last_collect_ms()
            tr.rollout_update(1 + k)
            u_ms += tr.last_update_ms()
        dev.finish()
        c_ms, u_ms = dist.max([c_ms, u_ms])
        rows = WIDE_ENVS * horizon
        # algorithmic tensor-core work per row and epoch: forward, backward
        # recompute and dW1, each 2 x 184 x 5120 multiply-adds
        flop = 3 * 2 * 184 * WIDE_HIDDEN * rows * epochs
        upd_s = u_ms / steps * 1e-3
        # aggregate over the ranks against the ranks' combined peak
        tf32_peak = peaks.get("bf16_tflops", 1590.0) / 2.0 * dist.world
        return {"config": "BASELINE config 3: 16,384 envs, 184->5120->4 tanh actor (967,688 params) on tcgen05 TF32, "
                          "32->64->1 critic, T=128, PPO 4 epochs x 16 minibatches",
                "env_steps_per_s": rows * steps / (c_ms * 1e-3), "rollout_ms": c_ms / steps,
                "ppo_update_ms": u_ms / steps,
                "ppo_tensor_roofline": {"bound": "tensor", "achieved": flop / upd_s / 1e12, "peak": tf32_peak,
                                        "unit": "TFLOP/s", "frac": flop / upd_s / 1e12 / tf32_peak,
                                        "peak_source": "half the measured bf16 dense rate (tf32 issues at half the "
                                                       "bf16 rate on tcgen05), times the GPU count"}}
    finally:
        tr.close()
        sim.close()


# ------------------------------------------------------------ CPU baseline
def cpu_model():
    """The host CPU's model name (first /proc/cpuinfo entry)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_reference_sample(layouts, n, policy_steps, family, warmup=0, threads=None, delay=0, ppo=True,
                         own_update=False):
    """The reference's own CPU path (oracle/_ref: cpu_reference.hpp compiled
    unmodified) on a bounded sample: `n` environments of the benchmark's
    worlds, `warmup` untimed then `policy_steps` timed policy steps (each one
    ref_step over every environment, timed on its own), then the PPO cost per
    row-epoch."""
    om = oracle_module()
    ref = om.load_ref()
    kind = "reference"
    if ref is None:
        return None
    olib = om.load_oracle()
    threads = threads or os.cpu_count()
    ref.ref_set_threads(threads)
    cfg = layouts.default_config(n=n, family=1, seed=42, sensor_delay=delay, command_delay=delay)
    raptor = layouts.load_raptor_file(ROOT / "metal-drone-nav_b200" / "assets" / "raptor.bin")
    tr = om.RefTrainer(layouts, cfg, warmup + policy_steps, raptor, lib=ref)
    worlds = tr.buf("worlds")
    runs = tr.buf("runs")
    # The benchmark's worlds (families 17-20) drawn as the simulator's reset
    # draws them (seed per env, sim.metal:56-58), generated by the C
    # restatement: the reference has no generator for these families.
    rng = np.zeros(1, np.uint32)

    def world_for(i):
        fam = olib.o_mixed_lane_family(int(i)) if family == 18 else olib.o_wtraining_family(family, om.ptr(rng))
        seed = olib.o_wrng(om.ptr(rng))
        olib.o_wgenerate(om.ptr(worlds[i:i + 1]), seed, fam, 4.0)

    for i in range(n):
        rng[0] = (42 + i * 747796405 + 2891336453) & 0xFFFFFFFF
        world_for(i)
    step_s = []
    for t in range(warmup + policy_steps):
        before = runs["episodes"].copy()
        t0 = time.perf_counter()
        ref.ref_step(tr.h, t)
        if t >= warmup:
            step_s.append(time.perf_counter() - t0)
        # An episode the reference reset inside the step (cpu_reference.hpp
        # reset_env, its own family-1 generator, inside the timed step) gets a
        # world of the benchmark's families for its next steps, outside the
        # timed region.
        for i in np.nonzero(runs["episodes"] != before)[0]:
            rng[0] = runs["rng"][i]
            world_for(i)
    collect_s = float(sum(step_s))
    update_ms = None
    if own_update:
        # the reference's own update of this rollout: GAE + normalisation, then
        # 2 epochs of shuffled 256-row chunks (cpu_reference.hpp:571-608)
        loss = np.zeros(4, np.float32)
        t1 = time.perf_counter()
        ref.ref_gae_normalize(tr.h)
        ref.ref_train_rollout(tr.h, 0, om.ptr(loss))
        update_ms = (time.perf_counter() - t1) * 1e3
    out = {"env_steps_per_s": n * policy_steps / collect_s, "collect_s": collect_s, "threads": threads,
           "step_ms": collect_s / policy_steps * 1e3, "kind": kind, "cpu_model": cpu_model(), "update_ms": update_ms,
           "sample": f"{n} envs x {policy_steps} policy steps of cpu_reference::Trainer (compiled unmodified, "
                     f"OpenMP stand-ins for GCD/Accelerate) on family-{family} worlds (also after in-step resets), "
                     f"delays {delay}, {threads} threads"}
    if ppo:
        # PPO: one train_rollout over a small trainer -> seconds per row-epoch
        small = om.RefTrainer(layouts, layouts.default_config(n=1024, family=1, seed=42), 4, raptor, lib=ref)
        for t in range(4):
            ref.ref_step(small.h, t)
        ref.ref_gae_normalize(small.h)
        loss = np.zeros(4, np.float32)
        t1 = time.perf_counter()
        ref.ref_train_rollout(small.h, 0, om.ptr(loss))
        update_s = time.perf_counter() - t1
        out["per_row_epoch_s"] = update_s / (1024 * 4 * 2)
        out["sample"] += "; PPO cost from one train_rollout over 1024x4 rows (2 epochs x 256-row chunks)"
    return out


def measure_config0(pkg, dev):
    """BASELINE config 0, the reference's own CPU-runnable workload: 512
    environments of the baseline clutter scenes (family 17), T = 64, then GAE
    and the reference's update schedule (2 epochs x 256-row chunks) on the
    fp32 parity path. The reference's CPU path runs the same rollout and
    update at all host cores and at one core."""
    L = pkg.layouts
    n, T = 512, 64
    sim = pkg.Sim(dev, L.default_config(n=n, family=17, seed=0), T)
    tr = pkg.PPOTrainer(sim, epochs=2, minibatch=256)
    try:
        sim.collect()
        tr.rollout_update(0)
        dev.finish()
        c, u = [], []
        for k in range(3):
            sim.collect()
            c.append(sim.last_collect_ms())
            tr.rollout_update(k + 1)
            u.append(tr.last_update_ms())
        dev.finish()
    finally:
        tr.close()
        sim.close()
    out = {"config": "BASELINE config 0: 512 envs, family-17 scenes (16 boxes, goal 2-8 m), T=64, GAE, "
                     "PPO 2 epochs x 256-row chunks (fp32 parity path)",
           "gpu": {"env_steps_per_s": n * T / (np.mean(c) * 1e-3), "rollout_ms": float(np.mean(c)),
                   "ppo_update_ms": float(np.mean(u))}}
    for label, threads in (("cpu_all_cores", None), ("cpu_one_core", 1)):
        r = cpu_reference_sample(L, n, T, 17, threads=threads, ppo=False, own_update=True)
        if r is not None:
            out[label] = {"env_steps_per_s": r["env_steps_per_s"], "rollout_ms": r["collect_s"] * 1e3,
                          "ppo_update_ms": r["update_ms"], "cores": r["threads"], "cpu_model": r["cpu_model"],
                          "kind": r["kind"]}
    return out


def measure_config1(pkg, dev):
    """8,192 environments on the goal-arrival task path
    (navigation_tasks.hpp clutter stage, family 1 static rooms, goal band
    2-20 m), T = 128, PPO 4 epochs x 8 minibatches on the tensor-core path."""
    L = pkg.layouts
    n, T = 8192, 128
    sim = pkg.Sim(dev, L.default_config(n=n, family=1, mode=22, speed=1.5, distance=8.0, seed=7, max_steps=400), T)
    control = pkg.task_control(2, 1)
    control["config"]["goal_distance_max_m"] = 20.0
    sim.configure_tasks(control, 0.0)
    tr = pkg.PPOTrainer(sim, epochs=4, minibatch=n * T // 8)
    tr.set_tensor_cores(True)
    try:
        sim.collect()
        tr.rollout_update(0)
        dev.finish()
        c, u = [], []
        for k in range(2):
            sim.collect()
            c.append(sim.last_collect_ms())
            tr.rollout_update(k + 1)
            u.append(tr.last_update_ms())
        tr.set_tensor_cores(False)
        tr.rollout_update(3)
        dev.finish()
        fp32_ms = tr.last_update_ms()
    finally:
        tr.close()
        sim.close()
    return {"config": "BASELINE config 1: 8,192 envs, goal-arrival tasks (clutter stage, family-1 rooms, goals "
                      "2-20 m), T=128, PPO 4 epochs x 8 minibatches of 131,072 rows",
            "env_steps_per_s": n * T / (np.mean(c) * 1e-3), "rollout_ms": float(np.mean(c)),
            "ppo_update_ms": float(np.mean(u)), "ppo_update_ms_fp32_path": fp32_ms}


def layered_flop_per_row(actor, critic):
    """Forward multiply-add FLOPs of one row through both layered networks
    (the update does about three times this: forward, deltas, weight gradients)."""
    def net(inp, hidden, layers, out):
        dims = [(inp if l == 0 else hidden, hidden) for l in range(layers)] + [(hidden, out)]
        return sum(2 * i * o for i, o in dims)
    return net(184, actor[0], actor[1], 4) + net(32, critic[0], critic[1], 1)


def measure_layered(pkg, dev, label, n, T, epochs, minibatch, shape, cfg, fp32_peak, steps=2, tasks=None):
    """One BASELINE configuration with layered networks (fp32 dense kernels):
    one warm-up rollout + update, then `steps` timed ones (CUDA events)."""
    sim = pkg.Sim(dev, cfg, T, **shape)
    if tasks is not None:
        sim.configure_tasks(tasks, 0.0)
    tr = pkg.PPOTrainer(sim, epochs=epochs, minibatch=minibatch)
    try:
        sim.collect()
        tr.rollout_update(0)
        dev.finish()
        c, u = [], []
        for k in range(steps):
            sim.collect()
            c.append(sim.last_collect_ms())
            tr.rollout_update(k + 1)
            u.append(tr.last_update_ms())
        dev.finish()
    finally:
        tr.close()
        sim.close()
    a = (shape.get("actor_hidden", 64), shape.get("actor_layers", 1))
    cr = (shape.get("critic_hidden", 64), shape.get("critic_layers", 1))
    fwd = layered_flop_per_row(a, cr)
    # update work: forward + weight gradients + deltas (all but the first layer's)
    first = 2 * 184 * a[0] + 2 * 32 * cr[0]
    update_flop = (3 * fwd - first) * n * T * epochs
    upd_s = float(np.mean(u)) * 1e-3
    return {"config": label, "env_steps_per_s": n * T / (np.mean(c) * 1e-3), "rollout_ms": float(np.mean(c)),
            "ppo_update_ms": float(np.mean(u)),
            "ppo_compute_roofline": {"bound": "fp32", "achieved": update_flop / upd_s / 1e12, "peak": fp32_peak,
                                     "unit": "TFLOP/s", "frac": update_flop / upd_s / 1e12 / fp32_peak,
                                     "flop_per_row_epoch": 3 * fwd - first,
                                     "peak_source": "measured (pure-FMA kernel, this run)"}}


def measure_layered_configs(pkg, dev, fp32_peak):
    """The network shapes BASELINE configs 0, 1 and 3 name (the reference has
    only one-hidden-layer tanh networks; these run on the layered path)."""
    L = pkg.layouts
    out = {}
    out["0"] = measure_layered(
        pkg, dev, "BASELINE config 0 with its 2x64 tanh actor: 512 envs, family 17, T=64, PPO 2 epochs x 256-row "
                  "chunks", 512, 64, 2, 256, dict(actor_hidden=64, actor_layers=2),
        L.default_config(n=512, family=17, seed=0), fp32_peak, steps=3)
    control = pkg.task_control(2, 1)
    control["config"]["goal_distance_max_m"] = 20.0
    out["1"] = measure_layered(
        pkg, dev, "BASELINE config 1 with its 2x128 critic: 8,192 envs, goal-arrival tasks (goals 2-20 m), T=128, "
                  "PPO 4 epochs x 8 minibatches, fp32", 8192, 128, 4, 8192 * 128 // 8,
        dict(critic_hidden=128, critic_layers=2),
        L.default_config(n=8192, family=1, mode=22, speed=1.5, distance=8.0, seed=7, max_steps=400), fp32_peak,
        tasks=control)
    out["3"] = measure_layered(
        pkg, dev, "BASELINE config 3 with its 4x480 GELU actor and 2x512 critic: 16,384 envs, family 17, T=128, "
                  "PPO 4 epochs x 16 minibatches, fp32 CUDA cores", 16384, 128, 4, 16384 * 128 // 16,
        dict(actor_hidden=480, actor_layers=4, actor_activation="gelu", critic_hidden=512, critic_layers=2),
        L.default_config(n=16384, family=17, seed=43), fp32_peak, steps=1)
    return out


def run_reference_arm(args, dist, out_fd):
    if dist.rank != 0:
        return 0
    layouts = package().layouts
    envs = args.envs
    om = oracle_module()
    if om.load_ref() is None:
        emit({"impl": "reference", "unavailable": "oracle/_ref not built (reference sources absent)"}, out_fd)
        return 0
    # each step = one policy step over all environments, timed on its own
    s = cpu_reference_sample(layouts, envs, args.steps, args.family, warmup=args.warmup, delay=args.delay)
    value = s["env_steps_per_s"]
    rows = envs * args.horizon
    line = {
        "metric": METRIC, "value": value, "unit": "env-steps/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": s["step_ms"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "impl": "reference",
        "config": workload_config(args),
        "step": f"one policy step of all {envs:,} environments (the GPU arm's step is a {args.horizon}-step rollout "
                f"plus a PPO update)",
        "ppo_update_ms_extrapolated": s["per_row_epoch_s"] * rows * args.epochs * 1e3,
        "cpu_model": s["cpu_model"],
        "cpu_baseline": {"value": value, "unit": "env-steps/s", "cores": s["threads"], "kind": s["kind"],
                         "sample": s["sample"] + f" ({args.warmup} untimed warm-up steps)"},
        "e2e": {"value": value, "unit": "env-steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line, out_fd)
    return 0


def workload_config(args):
    actor = ("184->64->4 tanh actor" if args.actor_hidden == 64 else
             f"184->{args.actor_hidden}->4 tanh actor on tcgen05 TF32")
    scene = ("mixed capability (50% static clutter rooms of 16 boxes, 25% long-goal rooms, 25% combined courses of "
             "12 boxes + 4 bounded movers)" if args.family == 18 else f"family-{args.family} worlds")
    return {"workload": f"BASELINE config 4 on one shard set: {args.envs:,} envs, {scene}, {args.delay}-tick "
                        f"(100 ms at 2) sensor and command delays, 20x16 depth rays, {actor}, 32->64->1 critic, "
                        f"T={args.horizon} rollouts, PPO {args.epochs} epochs x {args.minibatches} minibatches",
            "envs": args.envs, "horizon": args.horizon, "family": args.family, "delay_ticks": args.delay,
            "epochs": args.epochs,
            "minibatches": args.minibatches, "actor_hidden": args.actor_hidden,
            "parallelism": f"dp{args.gpus} (envs sharded)",
            "l2": f"inputs larger than L2 (obs buffer {args.envs * args.horizon * 184 * 4 / 1e9:.2f} GB per rollout "
                  f"against a 126 MB L2)"}


# ------------------------------------------------------------------ main
def emit(line, fd):
    """Write the one JSON result line to the saved stdout."""
    os.write(fd, (json.dumps(line) + "\n").encode())


def main():
    # Libraries (NCCL's version banner, warnings) may print to fd 1; the driver
    # reads exactly one JSON line from stdout. Keep the real stdout for that line
    # and send everything else to stderr.
    out_fd = os.dup(1)
    sys.stdout.flush()
    os.dup2(2, 1)
    args = parse()
    dist = Dist()
    if args.impl == "reference":
        return run_reference_arm(args, dist, out_fd)
    dist.init()
    pkg = package()
    L = pkg.layouts
    world = dist.world
    assert args.envs % world == 0, "envs must divide evenly over ranks"
    n = args.envs // world
    dev = pkg.Device(dist.local)
    if world > 1:
        uid = dist.broadcast_bytes(pkg.Device.comm_unique_id() if dist.rank == 0 else None)
        dev.comm_init(dist.rank, world, uid)
    cfg = L.default_config(n=n, family=args.family, seed=42, sensor_delay=args.delay, command_delay=args.delay)
    sim = pkg.Sim(dev, cfg, args.horizon, actor_hidden=None if args.actor_hidden == 64 else args.actor_hidden)
    rows = n * args.horizon
    minibatch = rows // args.minibatches
    trainer = pkg.PPOTrainer(sim, epochs=args.epochs, minibatch=minibatch)
    if args.actor_hidden == 64 and not args.ppo_fp32:
        trainer.set_tensor_cores(True)  # the minibatch products on tcgen05 (TF32)

    for w in range(args.warmup):
        sim.collect()
        trainer.rollout_update(w)
    dev.finish()
    per_step, per_update = trainer.launch_counts()

    # ---- device-timed region
    import torch
    torch.cuda.set_device(dist.local)
    bus = None
    try:
        bus = torch.cuda.get_device_properties(dist.local).pci_bus_id
    except Exception:
        pass
    clocks = ClockSampler(bus)
    clocks.start()
    dist.barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    collect_ms, update_ms = [], []
    for k in range(args.steps):
        sim.collect()
        collect_ms.append(sim.last_collect_ms())
        trainer.rollout_update(args.warmup + k)
        update_ms.append(trainer.last_update_ms())
    dev.finish()
    torch.cuda.synchronize()
    dist.barrier()
    wall = time.perf_counter() - wall0
    clk = clocks.stop()
    c_ms, u_ms, wall_max = dist.max([sum(collect_ms), sum(update_ms), wall])
    env_steps = args.envs * args.horizon * args.steps
    value = env_steps / (c_ms * 1e-3)

    # ---- end to end through the C-ABI: policy from pinned host memory in,
    # episode report out, every step; host wall clock.
    actor = sim.download("actor")
    critic = sim.download("critic")
    pinned_a = torch.from_numpy(actor).pin_memory()
    pinned_c = torch.from_numpy(critic).pin_memory()
    h2d = actor.nbytes + critic.nbytes
    d2h = 10 * 8  # Sim::report's ten aggregates (reduced on the GPU)
    dist.barrier()
    torch.cuda.synchronize()
    e0 = time.perf_counter()
    for k in range(args.steps):
        sim.upload_raw("actor", pinned_a.data_ptr(), actor.nbytes)
        sim.upload_raw("critic", pinned_c.data_ptr(), critic.nbytes)
        sim.collect()
        sim.report()
    dev.finish()
    torch.cuda.synchronize()
    dist.barrier()
    (e2e_wall,) = dist.max([time.perf_counter() - e0])
    e2e_value = env_steps / e2e_wall

    peaks_file = ROOT / "MEASURED_PEAKS.json"
    peaks = json.loads(peaks_file.read_text()) if peaks_file.exists() else {}
    # ---- per-kernel roofline of one policy step (CUDA events between launches)
    prof = np.mean([sim.profile_step(t % args.horizon) for t in range(8)], axis=0)
    prof = dist.max(prof.tolist())
    names = ("sense", "act", "advance")
    dominant = int(np.argmax(prof))
    worlds = sim.download("worlds")
    mean_obstacles = float(np.mean(worlds["count"]))
    work = kernel_work(mean_obstacles)
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    hbm_src = "measured" if "hbm_gbs" in peaks else "fallback"
    fp32_peak = dev.fp32_peak_tflops()
    dom = names[dominant]
    t_s = prof[dominant] * 1e-3
    achieved_gbs = work[dom]["bytes"] * n / t_s / 1e9
    traffic = read_profile_traffic(dom)
    kernels = {}
    for i, nm in enumerate(names):
        ts = prof[i] * 1e-3
        kernels[nm] = {"ms": prof[i], "gb_s": work[nm]["bytes"] * n / ts / 1e9,
                       "tflop_s": work[nm]["flop"] * n / ts / 1e12,
                       "fp32_frac": work[nm]["flop"] * n / ts / 1e12 / fp32_peak}

    # ---- PPO update: the minibatch kernel against its roof, and the fp32
    # parity path of the same update (one more rollout update, after timing)
    ppo_roof, ppo_fp32 = None, None
    if args.actor_hidden == 64:
        ppo_roof = ppo_roofline(trainer, minibatch, dist, peaks, fp32_peak)
        if trainer.tensor_cores:
            trainer.set_tensor_cores(False)
            trainer.rollout_update(args.warmup + args.steps)
            dev.finish()
            (fp32_ms,) = dist.max([trainer.last_update_ms()])
            ppo_fp32 = {"ppo_update_ms": fp32_ms, "roofline": ppo_roofline(trainer, minibatch, dist, peaks, fp32_peak),
                        "note": "the fp32 CUDA-core kernel that keeps the reference's summation order (the parity "
                                "path), one update of the same workload after the timed region"}
            trainer.set_tensor_cores(True)

    line = {
        "metric": METRIC, "value": value, "unit": "env-steps/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": (c_ms + u_ms) / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (procedural worlds, seeded)",
        "config": workload_config(args),
        "ppo_update_ms": u_ms / args.steps,
        "ppo_path": ("tcgen05 TF32 minibatch products, fp32 accumulation, GAE / clip / Adam in fp32"
                     if trainer.tensor_cores else "fp32 CUDA cores in the reference's summation order"),
        "ppo_roofline": ppo_roof,
        "ppo_update_fp32": ppo_fp32,
        "rollout_ms": c_ms / args.steps,
        "wall_s": wall_max,
        "e2e": {"value": e2e_value, "unit": "env-steps/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "note": "policy uploaded from pinned host memory, rollout, Sim::report read back; PPO update excluded "
                        "as in the metric"},
        "gpu_launches": args.steps * (args.horizon * per_step + per_update),
        "roofline": {"bound": "hbm", "kernel": "k_" + dom, "achieved": achieved_gbs,
                     "peak": hbm_peak, "unit": "GB/s", "frac": achieved_gbs / hbm_peak,
                     "traffic": None if traffic is None else traffic * n, "peak_source": hbm_src,
                     "note": "the sensing kernel is bound by FP32 instruction issue, not HBM: its fraction of the "
                             "FP32 peak is compute_roofline; this line is its bytes against the HBM roof"},
        "compute_roofline": {"bound": "fp32", "kernel": "k_" + dom, "achieved": kernels[dom]["tflop_s"],
                             "peak": fp32_peak, "unit": "TFLOP/s", "frac": kernels[dom]["fp32_frac"],
                             "peak_source": "measured (pure-FMA kernel, this run)"},
        "kernels": kernels,
        "clocks": clk,
    }
    if not args.no_wide and args.actor_hidden == 64:
        line["wide_actor"] = measure_wide(pkg, dev, dist, args, peaks)
    if world == 1 and not args.no_secondary:
        line["baseline_configs"] = {"0": measure_config0(pkg, dev), "1": measure_config1(pkg, dev)}
        line["layered_networks"] = measure_layered_configs(pkg, dev, fp32_peak)
    if world == 1 and dist.rank == 0 and not args.no_cpu_baseline:
        s = cpu_reference_sample(L, args.envs, 2, args.family, warmup=1, delay=args.delay)
        if s is not None:
            one = cpu_reference_sample(L, 4096, 2, args.family, warmup=1, threads=1, delay=args.delay, ppo=False)
            line["cpu_baseline"] = {"value": s["env_steps_per_s"], "unit": "env-steps/s", "cores": s["threads"],
                                    "kind": s["kind"], "sample": s["sample"], "cpu_model": s["cpu_model"],
                                    "ppo_update_ms_extrapolated": s["per_row_epoch_s"] * args.envs * args.horizon
                                    * args.epochs * 1e3,
                                    "one_core": {"value": one["env_steps_per_s"], "unit": "env-steps/s", "cores": 1,
                                                 "sample": one["sample"]}}
    if dist.rank == 0:
        emit(line, out_fd)
    trainer.close()
    sim.close()
    dev.close()
    dist.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
