"""numpy views of the byte-identical POD layouts declared in include/mdn.h.

These are the reference's own on-disk and device layouts:
RLPhysicsState / RLPhysicsParams (physics.hpp:12-38), WObstacle / WWorld
(world.hpp:28-29), SimRun / SimConfig (sim.metal:2-12, main.mm:454-465),
RaptorWeights (raptor.hpp:11-21) and the PPOFIX1 header (main.mm:984-991).
"""
import numpy as np

STATE = np.dtype([
    ("position", "<f4", 3), ("orientation_wxyz", "<f4", 4), ("linear_velocity", "<f4", 3),
    ("angular_velocity_body", "<f4", 3), ("rpm", "<f4", 4)])
PARAMS = np.dtype([
    ("rotor_positions", "<f4", 12), ("rotor_thrust_directions", "<f4", 12),
    ("rotor_torque_directions", "<f4", 12), ("rotor_thrust_coefficients", "<f4", 12),
    ("rotor_torque_constants", "<f4", 4), ("rotor_time_constants_rising", "<f4", 4),
    ("rotor_time_constants_falling", "<f4", 4), ("inertia", "<f4", 9), ("inertia_inverse", "<f4", 9),
    ("gravity_world", "<f4", 3), ("mass", "<f4"), ("action_min", "<f4"), ("action_max", "<f4"),
    ("dt", "<f4"), ("position_limit", "<f4"), ("velocity_limit", "<f4"), ("angular_velocity_limit", "<f4")])
OBSTACLE = np.dtype([("kind", "<u4"), ("center", "<f4", 3), ("size", "<f4", 3), ("velocity", "<f4", 3)])
WORLD = np.dtype([("obstacles", OBSTACLE, 16), ("count", "<u4"), ("seed", "<u4"), ("family", "<u4"),
                  ("goal", "<f4", 3), ("wind", "<f4", 3)])
RUN = np.dtype([
    ("hidden", "<f4", 16), ("motors", "<f4", 4), ("previous_nav", "<f4", 4), ("desired_velocity", "<f4", 3),
    ("yaw", "<f4"), ("rng", "<u4"), ("steps", "<u4"), ("path", "<f4"), ("elapsed", "<f4"),
    ("peak_speed", "<f4"), ("min_clearance", "<f4"), ("initial_distance", "<f4"), ("successes", "<u4"),
    ("collisions", "<u4"), ("timeouts", "<u4"), ("episodes", "<u4"), ("success_time", "<f4"),
    ("total_path", "<f4"), ("total_elapsed", "<f4"), ("final_progress", "<f4"),
    ("reference_position", "<f4", 3)])
CONFIG = np.dtype([
    ("n", "<u4"), ("tick", "<u4"), ("mode", "<u4"), ("family", "<u4"), ("substeps", "<u4"),
    ("sensor_period", "<u4"), ("sensor_delay", "<u4"), ("command_delay", "<u4"), ("max_steps", "<u4"),
    ("seed", "<u4"), ("eval", "<u4"), ("speed", "<f4"), ("distance", "<f4"), ("wind", "<f4"),
    ("depth_noise", "<f4"), ("dropout", "<f4"), ("risk_coef", "<f4"), ("entropy_coef", "<f4"),
    ("learning_rate", "<f4"), ("velocity_contract", "<u4"), ("geometry_memory", "<u4")])
RAPTOR = np.dtype([
    ("input_weights", "<f4", 16 * 22), ("input_bias", "<f4", 16), ("gru_input_weights", "<f4", 48 * 16),
    ("gru_hidden_weights", "<f4", 48 * 16), ("gru_input_bias", "<f4", 48), ("gru_hidden_bias", "<f4", 48),
    ("initial_hidden_state", "<f4", 16), ("output_weights", "<f4", 4 * 16), ("output_bias", "<f4", 4)])
SHAPE = np.dtype([
    ("actor_obs_dim", "<u4"), ("critic_obs_dim", "<u4"), ("actor_hidden", "<u4"), ("critic_hidden", "<u4"),
    ("flags", "<u4"), ("room_min", "<f4", 3), ("room_max", "<f4", 3),
    ("actor_layers", "<u4"), ("critic_layers", "<u4"), ("actor_activation", "<u4"), ("critic_activation", "<u4")])
TASK_CONFIG = np.dtype([
    ("family", "<u4"), ("stage", "<u4"), ("objective", "<u4"), ("require_detour", "<u4"),
    ("max_generation_attempts", "<u4"), ("max_nav_steps", "<u4"), ("scene_distance_m", "<f4"),
    ("difficulty", "<f4"), ("goal_distance_min_m", "<f4"), ("goal_distance_max_m", "<f4"),
    ("minimum_endpoint_clearance_m", "<f4"), ("minimum_witness_clearance_m", "<f4"), ("goal_radius_m", "<f4"),
    ("stable_speed_mps", "<f4"), ("stable_hold_s", "<f4"), ("nav_period_s", "<f4"), ("initial_speed_min_mps", "<f4"),
    ("initial_speed_max_mps", "<f4"), ("progress_reward_per_m", "<f4"), ("time_cost_per_s", "<f4"),
    ("contact_penalty", "<f4"), ("stable_arrival_bonus", "<f4"), ("command_smoothness_weight", "<f4"),
    ("start_min_xyz", "<f4", 3), ("start_max_xyz", "<f4", 3), ("goal_min_xyz", "<f4", 3), ("goal_max_xyz", "<f4", 3),
    ("generation_version", "<u4")])
TASK_CONTROL = np.dtype([("enabled", "<u4"), ("config", TASK_CONFIG)])
TASK_STATE = np.dtype([
    ("generation_status", "<u4"), ("valid", "<u4"), ("generation_attempts", "<u4"), ("family", "<u4"),
    ("stage", "<u4"), ("objective", "<u4"), ("max_nav_steps", "<u4"), ("step_count", "<u4"),
    ("stable_ticks", "<u4"), ("was_inside_goal", "<u4"), ("waypoint_event_latched", "<u4"), ("terminal", "<u4"),
    ("start_position", "<f4", 3), ("start_yaw_rad", "<f4"), ("start_velocity_world", "<f4", 3),
    ("goal_position", "<f4", 3), ("initial_distance_m", "<f4"), ("previous_distance_m", "<f4"), ("difficulty", "<f4"),
    ("start_clearance_m", "<f4"), ("goal_clearance_m", "<f4"), ("direct_segment_clearance_m", "<f4"),
    ("witness_min_clearance_m", "<f4"), ("witness_length_m", "<f4"), ("stable_time_s", "<f4"),
    ("last_executed_world_command", "<f4", 4), ("witness_point_count", "<u4"), ("witness_points", "<f4", (4, 3))])
CHECKPOINT_HEADER = np.dtype([
    ("magic", "S8"), ("version", "<u4"), ("actor_count", "<u4"), ("critic_count", "<u4"), ("horizon", "<u4"),
    ("n", "<u4"), ("family", "<u4"), ("base_seed", "<u4"), ("completed_rollouts", "<u4"),
    ("optimizer_step", "<u8"), ("config", CONFIG)], align=True)

assert STATE.itemsize == 68 and PARAMS.itemsize == 352 and OBSTACLE.itemsize == 40
assert WORLD.itemsize == 676 and RUN.itemsize == 184 and CONFIG.itemsize == 84
assert RAPTOR.itemsize == 8336 and SHAPE.itemsize == 60 and CHECKPOINT_HEADER.itemsize == 136
assert TASK_CONFIG.itemsize == 144 and TASK_CONTROL.itemsize == 148 and TASK_STATE.itemsize == 192

# Buffer ids (mdn.h MDN_BUF_*) with their element dtype and per-row shape.
BUF = {
    "states": 0, "runs": 1, "worlds": 2, "sensors": 3, "poses": 4, "commands": 5, "actor": 6, "critic": 7,
    "obs": 8, "co": 9, "actions": 10, "logp": 11, "values": 12, "rewards": 13, "next_values": 14,
    "terminated": 15, "truncated": 16, "advantages": 17, "returns": 18, "raptor": 19, "physics": 20,
    "contact_id": 21, "task_states": 22, "contact_audit": 23, "bank_worlds": 24, "bank_schedule": 25,
    "bank_active_ids": 26, "bank_transition_ids": 27, "raw_advantages": 28, "env_physics": 29,
}
CONTACT_AUDIT = np.dtype([("physical_clearance_m", "<f4"), ("safety_clearance_m", "<f4"), ("contact", "<u4"),
                          ("ambiguous", "<u4")])
BUF_DTYPE = {
    "states": STATE, "runs": RUN, "worlds": WORLD, "raptor": RAPTOR, "physics": PARAMS,
    "terminated": np.dtype(np.uint8), "truncated": np.dtype(np.uint8), "contact_id": np.dtype(np.int32),
    "task_states": TASK_STATE, "contact_audit": CONTACT_AUDIT, "bank_worlds": WORLD,
    "bank_schedule": np.dtype(np.uint32), "bank_active_ids": np.dtype(np.uint32),
    "bank_transition_ids": np.dtype(np.uint32), "env_physics": PARAMS,
}
# RLPhysicsDomainRange (physics_domain.hpp:17-24), NavigationRuntimeConfig
# (navigation_runtime.hpp:9-14).
DOMAIN_RANGE = np.dtype([(k, "<f4") for k in (
    "mass_scale_min", "mass_scale_max", "inertia_axis_scale_min", "inertia_axis_scale_max", "thrust_gain_min",
    "thrust_gain_max", "rising_lag_scale_min", "rising_lag_scale_max", "falling_lag_scale_min",
    "falling_lag_scale_max", "minimum_thrust_to_weight")])
RUNTIME_CONFIG = np.dtype([("enabled", "<u4"), ("domain_amplitude", "<f4"), ("domain_seed", "<u4"),
                           ("domain_range", DOMAIN_RANGE)])
assert DOMAIN_RANGE.itemsize == 44 and RUNTIME_CONFIG.itemsize == 56
# ChallengeBankControl (sim.metal:13) and challenge_training::Settings
# (challenge_training.hpp:40-49); mdn_bank_level = the numeric fields of
# challenge_evaluation::Level (challenge_evaluation.hpp:36-45).
BANK_CONTROL = np.dtype([("enabled", "<u4"), ("bank_count", "<u4"), ("schedule_stride", "<u4"), ("horizon", "<u4")])
CHALLENGE_SETTINGS = np.dtype([
    ("environment_count", "<u4"), ("horizon", "<u4"), ("sampler_seed", "<u4"), ("rehearsal_environments", "<u4"),
    ("selection", "<u4"), ("uniform_floor", "<f4"), ("score_staleness_mix", "<f4"), ("focus_family", "<u4")])
BANK_LEVEL = np.dtype([
    ("family", "<u4"), ("seed", "<u4"), ("base_seed", "<u4"), ("environment_index", "<u4"), ("distance", "<f4"),
    ("difficulty", "<f4"), ("direct_route_clearance_m", "<f4"), ("witness_min_clearance_m", "<f4"),
    ("witness_sample_count", "<u4"), ("witness_point_count", "<u4"), ("mirrored", "<u4"), ("line_number", "<u4")])
BANK_TEXT = ("failure_id", "split", "family_name", "geometry_contract", "difficulty_band", "scene_sha256",
             "world_source_sha256")
INVALID_LEVEL = 0xFFFFFFFF
# challenge_evaluation::BankScore (challenge_evaluation.hpp:53-66).
BANK_SCORE = np.dtype([("episodes", "<u8"), ("successes", "<u8"), ("collisions", "<u8"), ("timeouts", "<u8"),
                       ("family_episodes", "<u8", 3), ("family_successes", "<u8", 3), ("successful_time_s", "<f8")])

# Fixed PPO parameter offsets for the 184/64/4 actor and 32/64/1 critic (ppo.hpp:35-45).
ACTOR_OBS, CRITIC_OBS, HIDDEN, ACTIONS = 184, 32, 64, 4
ACTOR_B1 = HIDDEN * ACTOR_OBS
ACTOR_W2 = ACTOR_B1 + HIDDEN
ACTOR_B2 = ACTOR_W2 + ACTIONS * HIDDEN
ACTOR_LOG_STD = ACTOR_B2 + ACTIONS
ACTOR_PARAMS = ACTOR_LOG_STD + ACTIONS
CRITIC_B1 = HIDDEN * CRITIC_OBS
CRITIC_W2 = CRITIC_B1 + HIDDEN
CRITIC_B2 = CRITIC_W2 + HIDDEN
CRITIC_PARAMS = CRITIC_B2 + 1
assert ACTOR_PARAMS == 12104 and CRITIC_PARAMS == 2177


def default_config(**overrides):
    """SimConfig{} defaults (main.mm:462-463) with field overrides."""
    c = np.zeros((), CONFIG)
    defaults = dict(n=128, tick=0, mode=0, family=0, substeps=5, sensor_period=1, sensor_delay=0, command_delay=0,
                    max_steps=200, seed=42, eval=0, speed=2.0, distance=4.0, wind=0.0, depth_noise=0.0, dropout=0.0,
                    risk_coef=0.0, entropy_coef=0.005, learning_rate=0.0003, velocity_contract=1, geometry_memory=0)
    defaults.update(overrides)
    for k, v in defaults.items():
        c[k] = v
    return c


def load_raptor_file(path):
    """Parse a RAPTOR1 file (raptor.hpp:25-40): 16-byte header then 2,084 floats."""
    raw = open(path, "rb").read()
    if raw[:8] != b"RAPTOR1\x00":
        raise ValueError(f"{path}: not a RAPTOR1 file")
    version, count = np.frombuffer(raw, "<u4", 2, 8)
    if version != 1 or count != 2084:
        raise ValueError(f"{path}: RAPTOR1 version/count mismatch")
    return np.frombuffer(raw, RAPTOR, 1, 16).copy().reshape(())
