"""TEST INFRASTRUCTURE ONLY: ctypes bindings for the CPU checkers.

  liboracle.so           C restatement of the reference path (mdn_oracle.c)
  _ref/libref_oracle.so  the reference's own CPU path compiled unmodified
                         (cpu_reference.hpp + shared headers, see Makefile)

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs may import this module. The product never does.
"""
import ctypes
import os
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libref_oracle.so"


def reference_root(override=None):
    """The reference checkout: `override`, else $MDN_REFERENCE, else a folder
    named `reference` beside this repository (the layout the build used)."""
    return pathlib.Path(override or os.environ.get("MDN_REFERENCE") or HERE.parents[1] / "reference")

_P = ctypes.c_void_p
_F = ctypes.c_float
_U = ctypes.c_uint32


def ptr(a):
    return a.ctypes.data_as(_P) if a is not None else None


def build(reference_root_override=None):
    """Compile liboracle.so, and oracle/_ref when the reference sources exist."""
    subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)
    ref = reference_root(reference_root_override)
    if (ref / "cpu_reference.hpp").exists():
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={ref}"], check=True)


def _declare(lib, name, restype, *argtypes):
    fn = getattr(lib, name)
    fn.restype = restype
    fn.argtypes = list(argtypes)
    return fn


def load_oracle():
    if not ORACLE_SO.exists():
        build()
    lib = ctypes.CDLL(str(ORACLE_SO))
    d = lambda n, r, *a: _declare(lib, n, r, *a)
    d("o_wray_sphere", _F, _P, _P, _P, _F)
    d("o_wray_box", _F, _P, _P, _P, _P)
    d("o_wray_cylinder", _F, _P, _P, _P, _F, _F)
    d("o_wc", None, _P, _F, _P)
    d("o_wray", _F, _P, _P, _P, _P, _F)
    d("o_wclearance", _F, _P, _P, _P, _F, _P)
    d("o_wgenerate", None, _P, _U, _U, _F)
    d("o_wtraining_family", _U, _U, _P)
    d("o_mixed_lane_family", _U, _U)
    d("o_set_argument_order", None, ctypes.c_int)
    d("o_wrng", _U, _P)
    d("o_pixel_ray", None, _F, _F, _U, _P)
    d("o_nav_guidance", None, _P, _P, _P, _F, _P, _F, _F, _P)
    d("o_nav_guidance_memory", None, _P, _P, _P, _F, _P, _F, _F, _P, _P, _P, _U, _U, _P, _F)
    d("o_physics_step", None, _P, _P, _P, _P, _P)
    d("o_physics_default", None, _P)
    d("o_raptor_forward", None, _P, _P, _P, _P)
    d("o_compute_gae", None, _U, _U, _P, _P, _P, _P, _P, _F, _F, _P, _P)
    d("o_normalize_advantages", None, _P, ctypes.c_size_t)
    d("o_sample_loss_and_grad", None, _P, _P, _P, _F, _F, _F, _F, _F, _F, _F, _F, _P, _P, _P, _P)
    d("o_adam_update", None, _P, _P, _P, _P, ctypes.c_size_t, _F, _F, _F)
    d("o_pow_correction", _F, _F, ctypes.c_uint64)
    d("o_sim_create", _P, _P, _U, _P, _P, _P)
    d("o_sim_create_shard", _P, _P, _U, _P, _P, _P, _U)
    d("o_sim_rows_grad", None, _P, _P, _U, _F, _P)
    d("o_sim_destroy", None, _P)
    d("o_sim_buffer", _P, _P, ctypes.c_int, ctypes.POINTER(ctypes.c_size_t))
    d("o_sim_reset", None, _P)
    d("o_sim_set_config", None, _P, _P)
    for n in ("o_sim_observe", "o_sim_act", "o_sim_advance", "o_sim_step"):
        d(n, None, _P, _U)
    d("o_sim_gae_normalize", None, _P, ctypes.c_int)
    d("o_critic_obs_rows", None, _P, _P, _P, _P, _U, _U, _P)
    d("o_sim_train_rollout", None, _P, _U, _U, _P, _U, _P, _P, _P, _P)
    d("o_set_threads", None, ctypes.c_int)
    d("o_sim_set_task_control", None, _P, _P)
    d("o_sim_set_challenge_bank", None, _P, _P, _P)
    d("o_sim_set_runtime", None, _P, _P)
    d("o_sim_set_delay_rehearsal", None, _P, ctypes.c_int)
    d("o_physics_sample_domain", ctypes.c_int, _P, _P, _F, _P, _P, _P)
    d("o_domain_episode_seed", _U, _P, _U, _U, _U)
    d("o_generate_task", _U, _P, _P, _P, _P, _P)
    d("o_task_apply_start", None, _P, _P)
    d("o_task_step", None, _P, _P, _P, _P, _P, _U, _U, _P)
    d("o_task_segment_clearance", _F, _P, _P, _P, _P)
    d("o_wide_param_count", _U, _U)
    d("o_wide_init", None, _U, _P, _P)
    d("o_wide_actor_forward", None, _U, _P, _P, _P, _P)
    return lib


def load_ref_wide():
    """ppo.hpp compiled at the wide actor's shape (oracle/_ref/libref_wide.so),
    or None when it was never built (no reference sources)."""
    so = HERE / "_ref" / "libref_wide.so"
    if not so.exists():
        return None
    lib = ctypes.CDLL(str(so))
    d = lambda n, r, *a: _declare(lib, n, r, *a)
    d("refw_hidden", _U)
    d("refw_actor_param_count", _U)
    d("refw_actor_forward", None, _P, _P, _U, _P, _P)
    return lib


def load_ref_deploy():
    """The reference's deployment readers/writer (oracle/_ref/libref_deploy.so),
    or None when it was never built (no reference sources)."""
    so = HERE / "_ref" / "libref_deploy.so"
    if not so.exists():
        return None
    lib = ctypes.CDLL(str(so))
    d = lambda n, r, *a: _declare(lib, n, r, *a)
    d("refd_write_navpol", ctypes.c_int, ctypes.c_char_p, _P, _F, ctypes.c_char_p)
    d("refd_load_navpol", ctypes.c_int, ctypes.c_char_p, _P, _P, _P)
    d("refd_wide_eval", _U, ctypes.c_char_p, _P, _U, _P, _P, _P)
    d("refd_navpol_eval", ctypes.c_int, ctypes.c_char_p, _P, _U, _P)
    return lib


def load_ref_bank():
    """The reference's challenge-bank sampler (oracle/_ref/libref_bank.so), or
    None when it was never built (no reference sources)."""
    so = HERE / "_ref" / "libref_bank.so"
    if not so.exists():
        return None
    lib = ctypes.CDLL(str(so))
    d = lambda n, r, *a: _declare(lib, n, r, *a)
    d("refb_error", ctypes.c_char_p)
    d("refb_create", ctypes.c_int, ctypes.c_char_p, ctypes.c_char_p, _P, _F, _F, ctypes.POINTER(_P))
    d("refb_destroy", None, _P)
    d("refb_control", ctypes.c_int, _P, _P)
    d("refb_initial_schedule", ctypes.c_int, _P, _P)
    d("refb_next_schedule", ctypes.c_int, _P, _P, _U, ctypes.c_uint64, _P)
    d("refb_observe", ctypes.c_int, _P, _P, _P, _P, _P, ctypes.c_uint64)
    d("refb_level", ctypes.c_int, _P, _U, _P, _P)
    d("refb_save", ctypes.c_int, _P, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_uint64, _P, _U)
    d("refb_load", ctypes.c_int, _P, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_uint64, _P)
    return lib


def load_ref(rehearsal=False):
    """The compiled reference, or None when it was never built (no sources).
    rehearsal=True: the same CPU path built with NAV_DELAY_REHEARSAL=1, the
    switch of the reference's delay-training target (CMakeLists.txt:72-76)."""
    so = HERE / "_ref" / "libref_rehearsal.so" if rehearsal else REF_SO
    if not so.exists():
        return None
    lib = ctypes.CDLL(str(so))
    d = lambda n, r, *a: _declare(lib, n, r, *a)
    d("ref_trainer_create", _P, _P, _U, _P, _P)
    d("ref_trainer_destroy", None, _P)
    d("ref_trainer_buffer", _P, _P, ctypes.c_int, ctypes.POINTER(ctypes.c_size_t))
    d("ref_trainer_optimizer_step", ctypes.POINTER(ctypes.c_uint64), _P)
    d("ref_trainer_reset_env", None, _P, _U, ctypes.c_int)
    for n in ("ref_step_observe", "ref_step_act", "ref_step_advance", "ref_step"):
        d(n, None, _P, _U)
    d("ref_collect_rollout", None, _P)
    d("ref_gae_normalize", None, _P)
    d("ref_gae_only", None, _P)
    d("ref_train_rollout", None, _P, _U, _P)
    d("ref_run", None, _P, _U, _P)
    d("ref_validate_batched_forward", ctypes.c_int, _P)
    d("ref_minibatch_order", None, _U, _U, _U, _U, _P)
    d("ref_set_threads", None, ctypes.c_int)
    d("ref_max_threads", ctypes.c_int)
    d("ref_raptor_load", ctypes.c_int, ctypes.c_char_p, _P)
    d("ref_raptor_forward", None, _P, _P, _P, _P)
    d("ref_physics_step", None, _P, _P, _P, _P, _P)
    d("ref_physics_default", None, _P)
    d("ref_wray", _F, _P, _P, _P, _F)
    d("ref_wray_box", _F, _P, _P, _P, _P)
    d("ref_wray_sphere", _F, _P, _P, _P, _F)
    d("ref_wray_cylinder", _F, _P, _P, _P, _F, _F)
    d("ref_wclearance", _F, _P, _P, _F)
    d("ref_wc", None, _P, _F, _P)
    d("ref_wgenerate", None, _P, _U, _U, _F)
    d("ref_wtraining_family", _U, _U, _P)
    d("ref_pixel_ray", None, _F, _F, _U, _P)
    d("ref_nav_guidance", None, _P, _P, _P, _F, _P, _F, _F, _P)
    d("ref_nav_guidance_memory", None, _P, _P, _P, _F, _P, _F, _F, _P, _P, _P, _U, _U, _P, _F)
    d("ref_compute_gae", None, _U, _U, _P, _P, _P, _P, _P, _F, _F, _P, _P)
    d("ref_normalize_advantages", None, _P, ctypes.c_size_t)
    d("ref_sample_loss_and_grad", None, _P, _P, _P, _F, _F, _F, _F, _F, _F, _F, _F, _P, _P, _P, _P)
    d("ref_actor_forward", None, _P, _P, _P, _P)
    d("ref_critic_forward", _F, _P, _P, _P)
    d("ref_adam_update", None, _P, _P, _P, _P, ctypes.c_size_t, ctypes.c_uint64, _F)
    d("ref_run_cpu_self_tests", ctypes.c_int)
    d("ref_task_default_config", ctypes.c_int, _U, _U, _F, _P)
    d("ref_generate_task", _U, _P, _P, _P, _P)
    d("ref_task_apply_start", None, _P, _P)
    d("ref_task_step", None, _P, _P, _P, _P, _P, _U, _U, _P)
    d("ref_task_segment_clearance", _F, _P, _P, _P)
    d("ref_vg_world_contact", None, _P, _P, _P, _F, _F, _P)
    d("ref_physics_sample_domain", ctypes.c_int, _P, _P, _F, _P, _P, _P)
    d("ref_domain_stress_range", None, _P)
    return lib


class _Buffers:
    """Typed numpy views over a checker's buffers (ids follow MDN_BUF_*)."""

    def _view(self, lib_fn, handle, name):
        from_layouts = self.layouts
        bid = from_layouts.BUF[name] if isinstance(name, str) else name
        nbytes = ctypes.c_size_t()
        addr = lib_fn(handle, bid, ctypes.byref(nbytes))
        if not addr:
            raise KeyError(name)
        dt = from_layouts.BUF_DTYPE.get(name, np.dtype(np.float32)) if isinstance(name, str) else np.dtype(np.float32)
        count = nbytes.value // dt.itemsize
        buf = (ctypes.c_char * nbytes.value).from_address(addr)
        return np.frombuffer(buf, dt, count)


class OracleSim(_Buffers):
    """The C restatement driven like the product Sim (same buffer ids)."""

    def __init__(self, layouts, cfg, horizon, raptor, physics=None, room=None, lib=None, env_base=0):
        self.layouts = layouts
        self.lib = lib or load_oracle()
        self.cfg = np.array(cfg, layouts.CONFIG)
        if physics is None:
            physics = np.zeros((), layouts.PARAMS)
            self.lib.o_physics_default(ptr(physics))
        self.physics = np.array(physics, layouts.PARAMS)
        self.raptor = np.array(raptor, layouts.RAPTOR)
        self.room = None if room is None else np.asarray(room, np.float32)
        self.horizon = horizon
        self.h = self.lib.o_sim_create_shard(ptr(self.cfg), horizon, ptr(self.raptor), ptr(self.physics),
                                             ptr(self.room), env_base)

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.o_sim_destroy(self.h)
            self.h = None

    def buf(self, name):
        return self._view(self.lib.o_sim_buffer, self.h, name)

    def reset(self):
        self.lib.o_sim_reset(self.h)

    def set_config(self, cfg):
        self.cfg = np.array(cfg, self.layouts.CONFIG)
        self.lib.o_sim_set_config(self.h, ptr(self.cfg))

    def set_task_control(self, control):
        """navigation_training::configure without the reset (call reset())."""
        self.task_control = np.array(control, self.layouts.TASK_CONTROL)
        self.lib.o_sim_set_task_control(self.h, ptr(self.task_control))

    def set_challenge_bank(self, worlds, control):
        """Bank worlds + control; the schedule buffer starts zeroed."""
        self.bank_worlds = np.ascontiguousarray(worlds, self.layouts.WORLD)
        self.bank_control = np.array(tuple(control), self.layouts.BANK_CONTROL)
        self.lib.o_sim_set_challenge_bank(self.h, ptr(self.bank_worlds), ptr(self.bank_control))

    def set_runtime(self, runtime):
        """Sim.runtime_control; takes effect at the next reset."""
        self.runtime = np.array(runtime, self.layouts.RUNTIME_CONFIG)
        self.lib.o_sim_set_runtime(self.h, ptr(self.runtime))

    def set_delay_rehearsal(self, enabled=True):
        """NAV_DELAY_REHEARSAL as a switch; takes effect at the next reset / step."""
        self.lib.o_sim_set_delay_rehearsal(self.h, 1 if enabled else 0)

    def step(self, tick):
        self.lib.o_sim_step(self.h, tick)

    def observe(self, tick):
        self.lib.o_sim_observe(self.h, tick)

    def act(self, tick):
        self.lib.o_sim_act(self.h, tick)

    def advance(self, tick):
        self.lib.o_sim_advance(self.h, tick)

    def gae(self, normalize=True):
        self.lib.o_sim_gae_normalize(self.h, int(normalize))

    def critic_obs_rows(self, states, worlds, runs, dim=32):
        """sim_critic_obs (sim.metal:159-180) of the given environments' state
        in this simulator's room: [count][dim], dim 64 = the control-state
        critic's observation."""
        states = np.ascontiguousarray(states, self.layouts.STATE)
        worlds = np.ascontiguousarray(worlds, self.layouts.WORLD)
        runs = np.ascontiguousarray(runs, self.layouts.RUN)
        out = np.zeros((states.size, dim), np.float32)
        self.lib.o_critic_obs_rows(self.h, ptr(states), ptr(worlds), ptr(runs), states.size, dim, ptr(out))
        return out

    def rows_grad(self, rows, batch):
        """Raw [actor | critic] gradient over explicit rollout rows, loss scale 1/batch."""
        rows = np.ascontiguousarray(rows, np.uint32)
        out = np.zeros(self.layouts.ACTOR_PARAMS + self.layouts.CRITIC_PARAMS, np.float32)
        self.lib.o_sim_rows_grad(self.h, ptr(rows), rows.size, float(batch), ptr(out))
        return out

    def train_rollout(self, minibatch, epochs, order, b1corr, b2corr):
        order = np.ascontiguousarray(order, np.uint32)
        chunks = order.size // epochs
        out = np.zeros(4, np.float32)
        norms = np.zeros(2 * order.size, np.float32)
        self.lib.o_sim_train_rollout(self.h, minibatch, epochs, ptr(order), chunks,
                                     ptr(np.ascontiguousarray(b1corr, np.float32)),
                                     ptr(np.ascontiguousarray(b2corr, np.float32)), ptr(out), ptr(norms))
        return out, norms


class RefTrainer(_Buffers):
    """cpu_reference::Trainer (compiled unmodified) with step-level access."""

    def __init__(self, layouts, cfg, horizon, raptor, physics=None, lib=None):
        self.layouts = layouts
        self.lib = lib or load_ref()
        if self.lib is None:
            raise RuntimeError("oracle/_ref was not built (reference sources absent)")
        self.cfg = np.array(cfg, layouts.CONFIG)
        if physics is None:
            physics = np.zeros((), layouts.PARAMS)
            self.lib.ref_physics_default(ptr(physics))
        self.physics = np.array(physics, layouts.PARAMS)
        self.raptor = np.array(raptor, layouts.RAPTOR)
        self.h = self.lib.ref_trainer_create(ptr(self.cfg), horizon, ptr(self.raptor), ptr(self.physics))

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.ref_trainer_destroy(self.h)
            self.h = None

    def buf(self, name):
        return self._view(self.lib.ref_trainer_buffer, self.h, name)

    def step(self, tick):
        self.lib.ref_step(self.h, tick)

    @property
    def optimizer_step(self):
        return self.lib.ref_trainer_optimizer_step(self.h)[0]
