"""ctypes binding of libmdn.so (include/mdn.h) with the reference host API.

`Device`, `Sim` and `PPOTrainer` mirror the reference's Metal, Sim and
PPOTrainer classes (main.mm:44-72, 516-603, 1110-1476): same method names and
argument meaning, errors raised as exceptions (the reference's require()
throws std::runtime_error, main.mm:27). Buffers the reference exposes as
MTLBuffer.contents are reached with download/upload (host copies).

The CUDA library is required: constructing a Device without libmdn.so raises.
"""
import ctypes
import os
import pathlib

import numpy as np

from . import layouts

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "libmdn.so"
RAPTOR_PATH = HERE / "assets" / "raptor.bin"

_P = ctypes.c_void_p
_U = ctypes.c_uint32
_lib = None


class MdnError(RuntimeError):
    """A non-zero status from libmdn; .code is the MDN_ERR_* value."""

    def __init__(self, code, message):
        super().__init__(f"[{code}] {message}")
        self.code = code


ERR = dict(OK=0, INVALID=1, CUDA=2, NOMEM=3, TIMEOUT=4, IO=5, MISMATCH=6, NCCL=7, STATE=8)

# exported symbol -> (restype, argtypes)
SIGNATURES = {
    "mdn_last_error": (ctypes.c_char_p, []),
    "mdn_abi_version": (_U, []),
    "mdn_sim_config_default": (None, [_P]),
    "mdn_rollout_shape_default": (None, [_P]),
    "mdn_physics_crazyflie_default": (None, [_P]),
    "mdn_raptor_load": (ctypes.c_int, [ctypes.c_char_p, _P]),
    "mdn_device_open": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(_P)]),
    "mdn_device_close": (ctypes.c_int, [_P]),
    "mdn_sync": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_double)]),
    "mdn_sim_create": (ctypes.c_int, [_P, _P, _P, _U, _P, _P, ctypes.POINTER(_P)]),
    "mdn_sim_destroy": (ctypes.c_int, [_P]),
    "mdn_sim_reset": (ctypes.c_int, [_P]),
    "mdn_sim_set_config": (ctypes.c_int, [_P, _P]),
    "mdn_sim_get_config": (ctypes.c_int, [_P, _P]),
    "mdn_sim_collect": (ctypes.c_int, [_P, _U]),
    "mdn_sim_step": (ctypes.c_int, [_P, _U]),
    "mdn_sim_buffer": (ctypes.c_int, [_P, ctypes.c_int, ctypes.POINTER(_P), ctypes.POINTER(ctypes.c_size_t)]),
    "mdn_sim_download": (ctypes.c_int, [_P, ctypes.c_int, _P, ctypes.c_size_t, ctypes.c_size_t]),
    "mdn_sim_upload": (ctypes.c_int, [_P, ctypes.c_int, _P, ctypes.c_size_t, ctypes.c_size_t]),
    "mdn_sim_report": (ctypes.c_int, [_P, _P]),
    "mdn_sim_dims": (ctypes.c_int, [_P, _P, _P, _P, _P]),
    "mdn_task_settings": (ctypes.c_int, [_U, _U, ctypes.c_float, _P]),
    "mdn_sim_configure_tasks": (ctypes.c_int, [_P, _P, ctypes.c_float]),
    "mdn_sim_validate_tasks": (ctypes.c_int, [_P]),
    "mdn_sim_last_collect_ms": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_float)]),
    "mdn_sim_profile_step": (ctypes.c_int, [_P, _U, _P]),
    "mdn_sim_actor_means": (ctypes.c_int, [_P, _P, _U, _P]),
    "mdn_launch_counts": (ctypes.c_int, [_P, _P, ctypes.POINTER(_U), ctypes.POINTER(_U)]),
    "mdn_policy_write": (ctypes.c_int, [ctypes.c_char_p, _P, _U, ctypes.c_char_p, ctypes.c_float]),
    "mdn_sim_export_policy": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_float]),
    "mdn_sim_set_contact_audit": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_float]),
    "mdn_sim_set_delay_rehearsal": (ctypes.c_int, [_P, ctypes.c_int]),
    "mdn_device_fp32_peak": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_double)]),
    "mdn_selftest_barrier_timeout": (ctypes.c_int, [_P, ctypes.c_uint64, ctypes.c_int]),
    "mdn_selftest_division": (ctypes.c_int, [_P, ctypes.c_uint64, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64)]),
    "mdn_ppo_create": (ctypes.c_int, [_P, _U, _U, ctypes.POINTER(_P)]),
    "mdn_ppo_destroy": (ctypes.c_int, [_P]),
    "mdn_ppo_rollout_update": (ctypes.c_int, [_P, _U]),
    "mdn_ppo_metrics": (ctypes.c_int, [_P, _P]),
    "mdn_ppo_state": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(_U)]),
    "mdn_ppo_set_state": (ctypes.c_int, [_P, ctypes.c_uint64, _U]),
    "mdn_ppo_moments": (ctypes.c_int, [_P, ctypes.c_int, _P, ctypes.c_size_t, ctypes.c_int]),
    "mdn_ppo_grad_norms": (ctypes.c_int, [_P, _P, ctypes.c_size_t]),
    "mdn_minibatch_order": (ctypes.c_int, [_U, _U, _U, _U, _P, ctypes.c_size_t]),
    "mdn_ppo_minibatch_order": (ctypes.c_int, [_P, _U, _P, ctypes.c_size_t]),
    "mdn_ppo_last_update_ms": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_float)]),
    "mdn_ppo_set_tensor_cores": (ctypes.c_int, [_P, ctypes.c_int]),
    "mdn_ppo_profile_minibatch": (ctypes.c_int, [_P, ctypes.c_uint32, ctypes.POINTER(ctypes.c_float)]),
    "mdn_ppo_checkpoint_save": (ctypes.c_int, [_P, ctypes.c_char_p, _U, _U, _U]),
    "mdn_ppo_checkpoint_load": (ctypes.c_int, [_P, ctypes.c_char_p, _U, _U, _U, _U]),
    "mdn_gae_normalize_static": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _U, _U, ctypes.c_float,
                                                 ctypes.c_float, _P]),
    "mdn_sim_set_challenge_bank": (ctypes.c_int, [_P, _P, _P]),
    "mdn_domain_stress_range": (None, [_P]),
    "mdn_sim_set_runtime": (ctypes.c_int, [_P, _P]),
    "mdn_checkpoint_inspect": (ctypes.c_int, [ctypes.c_char_p, _P, _P, _P]),
    "mdn_bank_evaluate": (ctypes.c_int, [_P, _P, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p,
                                         ctypes.c_char_p, _U, ctypes.c_float, _U, _P]),
    "mdn_sha256_file": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p]),
    "mdn_bank_load": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(_P)]),
    "mdn_bank_free": (ctypes.c_int, [_P]),
    "mdn_bank_info": (ctypes.c_int, [_P, ctypes.POINTER(_U), ctypes.c_char_p]),
    "mdn_bank_level_get": (ctypes.c_int, [_P, _U, _P, _P]),
    "mdn_bank_worlds": (ctypes.c_int, [_P, _P, _U]),
    "mdn_bank_level_text": (ctypes.c_char_p, [_P, _U, ctypes.c_int]),
    "mdn_bank_witness_route": (ctypes.c_int, [_P, _U, _P, _U, ctypes.POINTER(_U)]),
    "mdn_challenge_settings_default": (None, [_P]),
    "mdn_challenge_create": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, _P, ctypes.POINTER(_P)]),
    "mdn_challenge_destroy": (ctypes.c_int, [_P]),
    "mdn_challenge_bank": (ctypes.c_int, [_P, ctypes.POINTER(_P)]),
    "mdn_challenge_control": (ctypes.c_int, [_P, _P]),
    "mdn_challenge_initial_schedule": (ctypes.c_int, [_P, _P]),
    "mdn_challenge_next_schedule": (ctypes.c_int, [_P, _P, ctypes.c_uint64, _P]),
    "mdn_challenge_active_ids": (ctypes.c_int, [_P, _P]),
    "mdn_challenge_observe_raw_gae": (ctypes.c_int, [_P, _P, _P, _P, _P, ctypes.c_uint64]),
    "mdn_challenge_level_stats": (ctypes.c_int, [_P, _U, ctypes.POINTER(ctypes.c_float),
                                                  ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]),
    "mdn_challenge_save_state": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_uint64, _P]),
    "mdn_challenge_load_state": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_uint64, _P]),
    "mdn_comm_unique_id": (ctypes.c_int, [_P]),
    "mdn_comm_init": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_int, _P]),
    "mdn_comm_destroy": (ctypes.c_int, [_P]),
}


def lib(path=None):
    """Load libmdn.so (in-tree). Raises when it is missing: there is no fallback."""
    global _lib
    if _lib is None:
        p = pathlib.Path(path or os.environ.get("MDN_LIB", LIB_PATH))
        if not p.exists():
            raise MdnError(ERR["INVALID"], f"libmdn.so not built at {p}; run __graft_entry__.build()")
        L = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status):
    if status != 0:
        raise MdnError(status, lib().mdn_last_error().decode())


def _ptr(a):
    return a.ctypes.data_as(_P)


def minibatch_order(rows, minibatch, epochs, rollout_index):
    """Chunk order of one rollout update, computed on the host (mdn_minibatch_order)."""
    chunks = -(-rows // minibatch)
    out = np.zeros(chunks * epochs, np.uint32)
    check(lib().mdn_minibatch_order(rows, minibatch, epochs, rollout_index, _ptr(out), out.size))
    return out


def task_settings(stage, family, difficulty=0.5):
    """navigation_training::task_settings: a ready task config (mdn_task_settings)."""
    c = np.zeros((), layouts.TASK_CONFIG)
    check(lib().mdn_task_settings(stage, family, difficulty, _ptr(c)))
    return c


def task_control(stage, family, difficulty=0.5):
    """navigation_training::task_settings as an enabled task control."""
    ctl = np.zeros((), layouts.TASK_CONTROL)
    ctl["enabled"] = 1
    ctl["config"] = task_settings(stage, family, difficulty)
    return ctl


def default_raptor():
    w = np.zeros((), layouts.RAPTOR)
    check(lib().mdn_raptor_load(str(RAPTOR_PATH).encode(), _ptr(w)))
    return w


class Device:
    """The reference's `Metal` object: one CUDA device (main.mm:44-72)."""

    def __init__(self, gpu=0):
        self.h = _P()
        check(lib().mdn_device_open(gpu, ctypes.byref(self.h)))
        self.gpu = gpu

    def finish(self):
        """Metal::finish: wait for queued work, raise device errors, return GPU seconds."""
        s = ctypes.c_double()
        check(lib().mdn_sync(self.h, ctypes.byref(s)))
        return s.value

    def fp32_peak_tflops(self):
        v = ctypes.c_double()
        check(lib().mdn_device_fp32_peak(self.h, ctypes.byref(v)))
        return v.value

    def selftest_division(self, samples, seed=1):
        """Mismatches of the depth kernel's divide-free quotient vs IEEE division."""
        out = ctypes.c_uint64()
        check(lib().mdn_selftest_division(self.h, samples, seed, ctypes.byref(out)))
        return out.value

    def selftest_barrier_timeout(self, limit_cycles, arrive=False):
        """One bounded barrier wait on the device; raises MdnError (TIMEOUT)
        when nothing arrives within limit_cycles."""
        check(lib().mdn_selftest_barrier_timeout(self.h, int(limit_cycles), 1 if arrive else 0))

    def comm_init(self, rank, world, unique_id):
        buf = np.frombuffer(bytes(unique_id), np.uint8).copy()
        check(lib().mdn_comm_init(self.h, rank, world, _ptr(buf)))

    @staticmethod
    def comm_unique_id():
        buf = np.zeros(128, np.uint8)
        check(lib().mdn_comm_unique_id(_ptr(buf)))
        return buf.tobytes()

    def close(self):
        if self.h:
            lib().mdn_comm_destroy(self.h)
            check(lib().mdn_device_close(self.h))
            self.h = _P()


class Sim:
    """Batched environment, the reference Sim (main.mm:516-603)."""

    ACTIVATIONS = {"tanh": 0, "gelu": 1}

    def __init__(self, device, cfg, horizon, raptor=None, physics=None, room=None, actor_hidden=None,
                 actor_layers=None, critic_hidden=None, critic_layers=None, actor_activation=None,
                 critic_activation=None, critic_obs_dim=None):
        """actor_hidden: None/64 for the reference's 12,104-parameter actor, or a
        multiple of 256 (5120 = the 967,688-parameter wide actor) evaluated on
        the tensor cores. actor_layers / critic_hidden / critic_layers /
        actor_activation / critic_activation ("tanh" or "gelu"): layered
        networks (no counterpart in the reference), e.g. a 4 x 480 GELU actor
        with a 2 x 512 critic; any of them selects the layered path for both
        networks. critic_obs_dim=64: the control-state critic of the
        reference's delay-training build (FIXED_PPO_CRITIC_OBS_DIM=64,
        sim.metal:166-180), on the layered path."""
        self.device = device
        self.cfg = np.array(cfg, layouts.CONFIG)
        self.horizon = int(horizon)
        self.raptor = default_raptor() if raptor is None else np.array(raptor, layouts.RAPTOR)
        layered = dict(actor_layers=actor_layers, critic_hidden=critic_hidden, critic_layers=critic_layers,
                       actor_activation=actor_activation, critic_activation=critic_activation,
                       critic_obs_dim=critic_obs_dim)
        shape = None
        if room is not None or actor_hidden is not None or any(v is not None for v in layered.values()):
            shape = np.zeros((), layouts.SHAPE)
            lib().mdn_rollout_shape_default(_ptr(shape))
            if room is not None:
                shape["flags"] = 1
                shape["room_min"] = room[:3]
                shape["room_max"] = room[3:]
            if actor_hidden is not None:
                shape["actor_hidden"] = int(actor_hidden)
            for key, value in layered.items():
                if value is None:
                    continue
                shape[key] = self.ACTIVATIONS[value] if key.endswith("activation") else int(value)
        self.actor_hidden = 64 if actor_hidden is None else int(actor_hidden)
        self.critic_obs_dim = 32 if critic_obs_dim is None else int(critic_obs_dim)
        phys = None if physics is None else np.array(physics, layouts.PARAMS)
        self.h = _P()
        check(lib().mdn_sim_create(device.h, _ptr(self.cfg), None if shape is None else _ptr(shape), self.horizon,
                                   _ptr(self.raptor), None if phys is None else _ptr(phys), ctypes.byref(self.h)))
        self.n = int(self.cfg["n"])
        dims = [_U() for _ in range(4)]
        check(lib().mdn_sim_dims(self.h, *[ctypes.byref(d) for d in dims]))
        self.actor_params = int(dims[2].value)
        self.critic_params = int(dims[3].value)

    def close(self):
        if self.h:
            check(lib().mdn_sim_destroy(self.h))
            self.h = _P()

    def reset(self):
        check(lib().mdn_sim_reset(self.h))

    def set_config(self, cfg):
        c = np.array(cfg, layouts.CONFIG)
        check(lib().mdn_sim_set_config(self.h, _ptr(c)))
        self.cfg = c

    def collect(self, count=0):
        check(lib().mdn_sim_collect(self.h, count))

    def step(self, tick):
        check(lib().mdn_sim_step(self.h, tick))

    def last_collect_ms(self):
        ms = ctypes.c_float()
        check(lib().mdn_sim_last_collect_ms(self.h, ctypes.byref(ms)))
        return ms.value

    def actor_means(self, obs):
        """The current actor's means for observation rows [rows][184] (the
        deployment inference, on the GPU)."""
        x = np.ascontiguousarray(obs, np.float32).reshape(-1, 184)
        out = np.zeros((x.shape[0], 4), np.float32)
        check(lib().mdn_sim_actor_means(self.h, _ptr(x), x.shape[0], _ptr(out)))
        return out

    def profile_step(self, tick):
        """Device ms of (sense, act, advance) for one policy step (CUDA events)."""
        ms = np.zeros(3, np.float32)
        check(lib().mdn_sim_profile_step(self.h, tick, _ptr(ms)))
        return ms

    def upload_raw(self, name, host_ptr, nbytes, offset=0):
        """Upload from a raw host pointer (e.g. pinned memory)."""
        check(lib().mdn_sim_upload(self.h, layouts.BUF[name], _P(host_ptr), offset, nbytes))

    def buffer(self, name):
        """Device pointer and size of a buffer (mdn_sim_buffer)."""
        ptr, nbytes = _P(), ctypes.c_size_t()
        check(lib().mdn_sim_buffer(self.h, layouts.BUF[name], ctypes.byref(ptr), ctypes.byref(nbytes)))
        return ptr.value, nbytes.value

    def download(self, name):
        _, nbytes = self.buffer(name)
        dt = layouts.BUF_DTYPE.get(name, np.dtype(np.float32))
        out = np.zeros(nbytes // dt.itemsize, dt)
        check(lib().mdn_sim_download(self.h, layouts.BUF[name], _ptr(out), 0, nbytes))
        return out

    def upload(self, name, array, offset=0):
        a = np.ascontiguousarray(array)
        check(lib().mdn_sim_upload(self.h, layouts.BUF[name], _ptr(a), offset, a.nbytes))

    def set_contact_audit(self, enabled=True, safety_margin_m=0.04):
        """Per-step mechanical contact audit into buffer 'contact_audit' [T][n]."""
        check(lib().mdn_sim_set_contact_audit(self.h, 1 if enabled else 0, safety_margin_m))

    def set_delay_rehearsal(self, enabled=True):
        """NAV_DELAY_REHEARSAL (sim.metal:14-24) as a run-time switch: under
        mode 22, environments with (global id / 4) even train without delays,
        wind, depth noise or dropout."""
        check(lib().mdn_sim_set_delay_rehearsal(self.h, 1 if enabled else 0))

    def export_policy(self, path, source_checkpoint, max_speed_mps=1.5):
        """Deployable actor file (NAVPOL1, or NAVWID4 for a wide actor)."""
        check(lib().mdn_sim_export_policy(self.h, str(path).encode(), str(source_checkpoint).encode(), max_speed_mps))

    def set_challenge_bank(self, worlds, control=None, horizon=None):
        """Frozen challenge-bank training (mdn_sim_set_challenge_bank).

        worlds: WORLD array of the bank levels; control: a BANK_CONTROL value
        (default: enabled, len(worlds) levels, horizon+1 schedule slots for
        this simulator's horizon). worlds=None switches banks off."""
        if worlds is None:
            check(lib().mdn_sim_set_challenge_bank(self.h, None, None))
            return
        w = np.ascontiguousarray(worlds, layouts.WORLD)
        if control is None:
            h = self.horizon if horizon is None else int(horizon)
            control = (1, len(w), h + 1, h)
        c = np.array(tuple(control) if not isinstance(control, np.ndarray) else control, layouts.BANK_CONTROL)
        check(lib().mdn_sim_set_challenge_bank(self.h, _ptr(w) if len(w) else None, _ptr(c)))

    def set_bank_schedule(self, schedule):
        """Upload this simulator's schedule rows: uint32 [n][schedule_stride]."""
        self.upload("bank_schedule", np.ascontiguousarray(schedule, np.uint32))

    def set_runtime(self, runtime=None):
        """Per-episode plant variation (mdn_sim_set_runtime); None switches it off."""
        if runtime is None:
            check(lib().mdn_sim_set_runtime(self.h, None))
            return
        r = np.array(runtime, layouts.RUNTIME_CONFIG)
        check(lib().mdn_sim_set_runtime(self.h, _ptr(r)))

    def configure_tasks(self, control, domain_amplitude=0.0):
        """navigation_training::configure: enable goal-arrival tasks and reset."""
        ctl = np.array(control, layouts.TASK_CONTROL)
        check(lib().mdn_sim_configure_tasks(self.h, _ptr(ctl), domain_amplitude))

    def validate_tasks(self):
        """navigation_training::validate_rollout."""
        check(lib().mdn_sim_validate_tasks(self.h))

    def report(self):
        out = np.zeros(10, np.float64)
        check(lib().mdn_sim_report(self.h, _ptr(out)))
        keys = ("episodes", "successes", "collisions", "timeouts", "success_time", "total_path", "total_elapsed",
                "final_progress", "min_clearance", "peak_speed")
        return dict(zip(keys, out.tolist()))


class PPOTrainer:
    """The reference PPOTrainer (main.mm:1110-1476)."""

    def __init__(self, sim, epochs=2, minibatch=0):
        self.sim = sim
        self.h = _P()
        check(lib().mdn_ppo_create(sim.h, epochs, minibatch, ctypes.byref(self.h)))
        rows = int(sim.cfg["n"]) * sim.horizon
        self.minibatch = min(minibatch or 256, rows)
        self.updates = epochs * (-(-rows // self.minibatch))
        self.tensor_cores = False

    def close(self):
        if self.h:
            check(lib().mdn_ppo_destroy(self.h))
            self.h = _P()

    def rollout_update(self, rollout_index):
        check(lib().mdn_ppo_rollout_update(self.h, rollout_index))

    @property
    def metric_mean(self):
        out = np.zeros(4, np.float32)
        check(lib().mdn_ppo_metrics(self.h, _ptr(out)))
        return out

    def state(self):
        step, done = ctypes.c_uint64(), _U()
        check(lib().mdn_ppo_state(self.h, ctypes.byref(step), ctypes.byref(done)))
        return step.value, done.value

    @property
    def optimizer_step(self):
        return self.state()[0]

    def set_state(self, optimizer_step, completed_rollouts):
        check(lib().mdn_ppo_set_state(self.h, optimizer_step, completed_rollouts))

    def moments(self, which):
        n = self.sim.actor_params if which < 2 else self.sim.critic_params
        out = np.zeros(n, np.float32)
        check(lib().mdn_ppo_moments(self.h, which, _ptr(out), n, 0))
        return out

    def set_moments(self, which, values):
        v = np.ascontiguousarray(values, np.float32)
        check(lib().mdn_ppo_moments(self.h, which, _ptr(v), v.size, 1))

    def grad_norms(self, updates):
        out = np.zeros(2 * updates, np.float32)
        check(lib().mdn_ppo_grad_norms(self.h, _ptr(out), out.size))
        return out.reshape(updates, 2)

    def minibatch_order(self, rollout_index, updates):
        out = np.zeros(updates, np.uint32)
        check(lib().mdn_ppo_minibatch_order(self.h, rollout_index, _ptr(out), out.size))
        return out

    def launch_counts(self):
        a, b = _U(), _U()
        check(lib().mdn_launch_counts(self.sim.h, self.h, ctypes.byref(a), ctypes.byref(b)))
        return a.value, b.value

    def set_tensor_cores(self, enabled=True):
        """Minibatch products of the 64-unit networks on the tcgen05 tensor
        cores in TF32 (enabled) or in fp32 on the CUDA cores in the
        reference's summation order (the default)."""
        check(lib().mdn_ppo_set_tensor_cores(self.h, 1 if enabled else 0))
        self.tensor_cores = bool(enabled)

    def profile_minibatch(self, update=0):
        """Device ms of one launch of the minibatch gradient kernels."""
        ms = ctypes.c_float()
        check(lib().mdn_ppo_profile_minibatch(self.h, update, ctypes.byref(ms)))
        return ms.value

    def last_update_ms(self):
        ms = ctypes.c_float()
        check(lib().mdn_ppo_last_update_ms(self.h, ctypes.byref(ms)))
        return ms.value

    def save_checkpoint(self, path, family, seed, completed_rollouts):
        check(lib().mdn_ppo_checkpoint_save(self.h, str(path).encode(), family, seed, completed_rollouts))

    def load_checkpoint(self, path, family, horizon, n, seed):
        check(lib().mdn_ppo_checkpoint_load(self.h, str(path).encode(), family, horizon, n, seed))


def write_policy(path, actor, hidden, source_checkpoint, max_speed_mps=1.5):
    """mdn_policy_write: a deployable actor file from host parameters (no device needed)."""
    a = np.ascontiguousarray(actor, np.float32)
    check(lib().mdn_policy_write(str(path).encode(), _ptr(a), int(hidden), str(source_checkpoint).encode(),
                                 max_speed_mps))


def checkpoint_inspect(path):
    """Header, runtime config and task control of a PPOFIX1 file (mdn_checkpoint_inspect)."""
    h = np.zeros((), layouts.CHECKPOINT_HEADER)
    rt = np.zeros((), layouts.RUNTIME_CONFIG)
    tc = np.zeros((), layouts.TASK_CONTROL)
    check(lib().mdn_checkpoint_inspect(str(path).encode(), _ptr(h), _ptr(rt), _ptr(tc)))
    return h, rt, tc


def runtime_config(domain_amplitude, domain_seed=0x3F84D5B5, enabled=1, domain_range=None):
    """NavigationRuntimeConfig with the stress range (rl_physics_domain_stress_range)
    unless a DOMAIN_RANGE value is given; the defaults are navigation_training::configure's."""
    r = np.zeros((), layouts.RUNTIME_CONFIG)
    r["enabled"], r["domain_amplitude"], r["domain_seed"] = enabled, domain_amplitude, domain_seed
    if domain_range is None:
        rng = np.zeros((), layouts.DOMAIN_RANGE)
        lib().mdn_domain_stress_range(_ptr(rng))
        r["domain_range"] = rng
    else:
        r["domain_range"] = np.array(domain_range, layouts.DOMAIN_RANGE)
    return r


def sha256_file(path):
    """SHA-256 hex digest of a file (mdn_sha256_file)."""
    out = ctypes.create_string_buffer(65)
    check(lib().mdn_sha256_file(str(path).encode(), out))
    return out.value.decode()


class ChallengeBank:
    """One split of a frozen challenge-bank JSONL file (challenge_evaluation::
    load_split, challenge_evaluation.hpp:282-313), validated record by record."""

    def __init__(self, path=None, split="train", world_sha256=None, _handle=None, _owner=None):
        self._owner = _owner
        if _handle is not None:
            self.h, self._owns = _handle, False
        else:
            h = _P()
            check(lib().mdn_bank_load(str(path).encode(), split.encode(),
                                      None if world_sha256 is None else world_sha256.encode(), ctypes.byref(h)))
            self.h, self._owns = h, True
        count = _U()
        digest = ctypes.create_string_buffer(65)
        check(lib().mdn_bank_info(self.h, ctypes.byref(count), digest))
        self.count, self.bank_sha256 = count.value, digest.value.decode()

    def __len__(self):
        return self.count

    def close(self):
        if self.h and self._owns:
            lib().mdn_bank_free(self.h)
        self.h = None

    def worlds(self):
        out = np.zeros(self.count, layouts.WORLD)
        check(lib().mdn_bank_worlds(self.h, _ptr(out), self.count))
        return out

    def level(self, index):
        """Numeric fields, text fields and the witness route of one level."""
        info = np.zeros((), layouts.BANK_LEVEL)
        check(lib().mdn_bank_level_get(self.h, index, _ptr(info), None))
        rec = {k: info[k].item() for k in layouts.BANK_LEVEL.names}
        for i, name in enumerate(layouts.BANK_TEXT):
            rec[name] = lib().mdn_bank_level_text(self.h, index, i).decode()
        count = _U()
        check(lib().mdn_bank_witness_route(self.h, index, None, 0, ctypes.byref(count)))
        route = np.zeros((count.value, 3), np.float32)
        check(lib().mdn_bank_witness_route(self.h, index, _ptr(route), count.value, ctypes.byref(count)))
        rec["witness_route"] = route
        return rec


def challenge_settings(**overrides):
    """challenge_training::Settings defaults (challenge_training.hpp:40-49) with overrides."""
    s = np.zeros((), layouts.CHALLENGE_SETTINGS)
    lib().mdn_challenge_settings_default(_ptr(s))
    for k, v in overrides.items():
        s[k] = v
    return s


class ChallengeSampler:
    """challenge_training::ChallengeTraining (challenge_training.hpp:53-427): the
    train-split level sampler with failure scores and its CHTRN1 sidecar."""

    def __init__(self, bank_path, world_sha256, settings=None, **overrides):
        s = challenge_settings() if settings is None else np.array(settings, layouts.CHALLENGE_SETTINGS)
        for k, v in overrides.items():
            s[k] = v
        self.settings = s
        h = _P()
        check(lib().mdn_challenge_create(str(bank_path).encode(), world_sha256.encode(), _ptr(s), ctypes.byref(h)))
        self.h = h
        self.envs, self.horizon = int(s["environment_count"]), int(s["horizon"])
        bank = _P()
        check(lib().mdn_challenge_bank(self.h, ctypes.byref(bank)))
        self.bank = ChallengeBank(_handle=bank, _owner=self)

    def close(self):
        if self.h:
            lib().mdn_challenge_destroy(self.h)
        self.h = None

    def control(self):
        c = np.zeros((), layouts.BANK_CONTROL)
        check(lib().mdn_challenge_control(self.h, _ptr(c)))
        return c

    def _schedule(self):
        return np.zeros((self.envs, self.horizon + 1), np.uint32)

    def initial_schedule(self):
        out = self._schedule()
        check(lib().mdn_challenge_initial_schedule(self.h, _ptr(out)))
        return out

    def next_schedule(self, active_ids, rollout_index):
        a = np.ascontiguousarray(active_ids, np.uint32)
        if a.size != self.envs:
            raise MdnError(ERR["INVALID"], "challenge active-level id count differs from environment count")
        out = self._schedule()
        check(lib().mdn_challenge_next_schedule(self.h, _ptr(a), rollout_index, _ptr(out)))
        return out

    def active_ids(self):
        out = np.zeros(self.envs, np.uint32)
        check(lib().mdn_challenge_active_ids(self.h, _ptr(out)))
        return out

    def observe_raw_gae(self, raw_gae, terminated, truncated, transition_ids, rollout_index):
        rows = self.envs * self.horizon
        arrays = [np.ascontiguousarray(raw_gae, np.float32), np.ascontiguousarray(terminated, np.uint8),
                  np.ascontiguousarray(truncated, np.uint8), np.ascontiguousarray(transition_ids, np.uint32)]
        if any(a.size != rows for a in arrays):
            raise MdnError(ERR["INVALID"], f"rollout evidence must hold horizon x environments = {rows} rows")
        check(lib().mdn_challenge_observe_raw_gae(self.h, *[_ptr(a) for a in arrays], rollout_index))

    def level_stats(self, level):
        score, done, visit = ctypes.c_float(), ctypes.c_uint64(), ctypes.c_uint64()
        check(lib().mdn_challenge_level_stats(self.h, level, ctypes.byref(score), ctypes.byref(done),
                                              ctypes.byref(visit)))
        return score.value, done.value, visit.value

    def save_state(self, path, checkpoint_sha256, completed_rollouts, active_ids):
        a = np.ascontiguousarray(active_ids, np.uint32)
        if a.size != self.envs:
            raise MdnError(ERR["INVALID"], "challenge active-level id count differs from environment count")
        check(lib().mdn_challenge_save_state(self.h, str(path).encode(), checkpoint_sha256.encode(),
                                             completed_rollouts, _ptr(a)))

    def load_state(self, path, checkpoint_sha256, completed_rollouts):
        out = np.zeros(self.envs, np.uint32)
        check(lib().mdn_challenge_load_state(self.h, str(path).encode(), checkpoint_sha256.encode(),
                                             completed_rollouts, _ptr(out)))
        return out


def evaluate_bank(device, checkpoint, bank_path, split, world_sha256, output_csv, mode=17, speed=1.5, max_steps=400,
                  raptor=None):
    """challenge_evaluation::run (mdn_bank_evaluate): one CSV row per level of
    `split` and the aggregate BankScore as a dict."""
    r = np.array(default_raptor() if raptor is None else raptor, layouts.RAPTOR)
    score = np.zeros((), layouts.BANK_SCORE)
    check(lib().mdn_bank_evaluate(device.h, _ptr(r), str(checkpoint).encode(), str(bank_path).encode(),
                                  split.encode(), world_sha256.encode(), str(output_csv).encode(), mode, speed,
                                  max_steps, _ptr(score)))
    out = {k: score[k].item() if score[k].ndim == 0 else score[k].tolist() for k in layouts.BANK_SCORE.names}
    out["success_rate"] = out["successes"] / out["episodes"] if out["episodes"] else 0.0
    return out


def gather_rollout_evidence(raw_gae, terminated, truncated, transition_ids):
    """Under several ranks (torch.distributed initialised, environments sharded
    evenly and in rank order), assemble every rank's [T][n_local] rollout
    evidence into the [T][n_total] arrays that ChallengeSampler.observe_raw_gae
    takes, on every rank, so that all ranks keep identical sampler state."""
    import torch
    import torch.distributed as dist
    device = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" \
        else torch.device("cpu")
    out = []
    for array, dtype in ((raw_gae, np.float32), (terminated, np.uint8), (truncated, np.uint8),
                         (transition_ids, np.uint32)):
        a = np.ascontiguousarray(array, dtype)
        if a.ndim != 2:
            raise MdnError(ERR["INVALID"], "rollout evidence must be [horizon][local environments]")
        wire = a.view(np.int32) if a.dtype == np.uint32 else a.astype(np.int32) if a.dtype == np.uint8 else a
        local = torch.from_numpy(np.ascontiguousarray(wire)).to(device)
        parts = [torch.empty_like(local) for _ in range(dist.get_world_size())]
        dist.all_gather(parts, local)
        full = np.concatenate([p.cpu().numpy() for p in parts], axis=1)
        out.append(full.view(np.uint32) if dtype == np.uint32 else full.astype(dtype))
    return tuple(out)
