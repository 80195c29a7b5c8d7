// Goal-arrival task contract on the device (navigation_tasks.hpp:196-548):
// bounded task generation with a validated witness path, the physical start,
// and the stable-hold step reward. Generation runs at episode resets on a whole
// converged warp per environment (the witness checks' samples are split over
// the lanes); the step runs once per env-step, thread per environment.
#pragma once
#include "world_gen.cuh"

namespace mdn {

constexpr uint32_t kTaskOpen = 0u, kTaskHold = 1u, kTaskClutter = 2u;
constexpr uint32_t kTaskWaypoint = 0u, kTaskFinalHold = 1u;
constexpr uint32_t kTaskInvalidConfig = 1u, kTaskUnsupportedDynamic = 2u, kTaskExhausted = 3u, kTaskReady = 4u,
                   kTaskUnsupportedFamily = 5u;
constexpr uint32_t kTaskMaxWitness = 4u, kTaskMaxAttempts = 64u, kTaskMaxDirections = 64u;

__device__ __forceinline__ float task_clamp(float v, float lo, float hi) { return fminf(fmaxf(v, lo), hi); }

__device__ __forceinline__ void task_random_direction(uint32_t& rng, float out[3]) {  // :212-217
    const float z = 2.0f * wurand(rng) - 1.0f;
    const float angle = 6.28318530718f * wurand(rng);
    const float radial = sqrtf(fmaxf(0.0f, 1.0f - z * z));
    out[0] = radial * cosf(angle);
    out[1] = radial * sinf(angle);
    out[2] = z;
}
// :218-222; the three draws of the reference's wv(...) argument list are
// taken left to right, the order of its platforms (Apple clang, Metal).
__device__ __forceinline__ void task_random_point(uint32_t& rng, const float* low, const float* high, float out[3]) {
    out[0] = low[0] + (high[0] - low[0]) * wurand(rng);
    out[1] = low[1] + (high[1] - low[1]) * wurand(rng);
    out[2] = low[2] + (high[2] - low[2]) * wurand(rng);
}
__device__ __forceinline__ bool task_inside(const float p[3], const float* low, const float* high) {
    return p[0] >= low[0] && p[0] <= high[0] && p[1] >= low[1] && p[1] <= high[1] && p[2] >= low[2] && p[2] <= high[2];
}
// Minimum clearance of the samples every 5 cm along a segment (:240-252), by a
// whole converged warp: lane l takes samples l, l+32, ... and the lanes' minima
// are combined by shuffles. A minimum does not depend on the order of its
// terms, so the value equals the serial loop's. With `stop_at` above -inf the
// scan ends after the first round of 32 samples whose minimum is <= stop_at
// and returns that partial minimum: the caller only needs to know that the
// path fails its clearance test then.
__device__ __forceinline__ float warp_min(float v) {
    for (int m = 16; m > 0; m >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, m));
    return v;
}
__device__ float task_segment_clearance(const SimArgs& a, const mdn_world& w, const float* p0, const float* p1,
                                        float stop_at) {
    const float d[3] = {p1[0] - p0[0], p1[1] - p0[1], p1[2] - p0[2]};
    const float distance = len3(d[0], d[1], d[2]);
    uint32_t count = uint32_t(ceilf(distance / 0.05f));
    if (count < 1u) count = 1u;
    if (count > 512u) return -1e6f;
    const uint32_t lane = threadIdx.x & 31u;
    float minimum = 1e20f;
    for (uint32_t base = 0; base <= count; base += 32u) {
        const uint32_t sample = base + lane;
        if (sample <= count) {
            const float t = float(sample) / float(count);
            const float pt[3] = {p0[0] + d[0] * t, p0[1] + d[1] * t, p0[2] + d[2] * t};
            minimum = fminf(minimum, world_clearance(a, w, pt, 0.0f, nullptr));
        }
        if (stop_at > -INFINITY && warp_min(minimum) <= stop_at) break;
    }
    return warp_min(minimum);
}
struct TaskWitness {
    float p[kTaskMaxWitness][3];
    uint32_t count;
    float min_clearance, length;
};
// :253-259. `stop_at` as for task_segment_clearance: a path whose minimum is
// known to be <= stop_at skips its remaining segments.
__device__ float task_test_path(const SimArgs& a, const mdn_world& w, const float (*pts)[3], uint32_t count,
                                float stop_at = -INFINITY) {
    if (count < 2u || count > kTaskMaxWitness) return -1e6f;
    float minimum = 1e20f;
    for (uint32_t k = 0; k + 1u < count; k++) {
        minimum = fminf(minimum, task_segment_clearance(a, w, pts[k], pts[k + 1], stop_at));
        if (minimum <= stop_at) break;
    }
    return minimum;
}
__device__ void task_save(TaskWitness& out, const float (*pts)[3], uint32_t count, float clearance) {  // :260-273
    out.count = count;
    out.min_clearance = clearance;
    float total = 0;
    for (uint32_t k = 0; k + 1u < count; k++)
        total += len3(pts[k + 1][0] - pts[k][0], pts[k + 1][1] - pts[k][1], pts[k + 1][2] - pts[k][2]);
    out.length = total;
    for (uint32_t i = 0; i < kTaskMaxWitness; i++)
        for (int j = 0; j < 3; j++) out.p[i][j] = i < count ? pts[i][j] : 0.0f;
}
// :276-333: the direct line, or one of a bounded set of doglegs. The direct
// line's clearance is recorded in the task, so it is always scanned in full; a
// dogleg's is recorded only when it passes, so a failing dogleg stops early.
__device__ bool task_find_witness(const SimArgs& a, const mdn_world& w, const float st[3], const float gl[3],
                                  const mdn_task_config& c, TaskWitness& wit, float& direct_clearance) {
    const float direct[2][3] = {{st[0], st[1], st[2]}, {gl[0], gl[1], gl[2]}};
    direct_clearance = task_test_path(a, w, direct, 2u);
    if (direct_clearance > c.minimum_witness_clearance_m && c.require_detour == 0u) {
        task_save(wit, direct, 2u, direct_clearance);
        return true;
    }
    if (direct_clearance > c.minimum_witness_clearance_m) return false;
    const float delta[3] = {gl[0] - st[0], gl[1] - st[1], gl[2] - st[2]};
    const float x_fraction[5] = {0.10f, 0.25f, 0.50f, 0.75f, 0.90f};
    const float side_y[2] = {-4.60f, 4.60f};
    for (uint32_t side = 0; side < 2u; side++)
        for (uint32_t i = 0; i < 5u; i++) {
            const float t = x_fraction[i];
            const float path[3][3] = {{st[0], st[1], st[2]}, {st[0] + t * delta[0], side_y[side], st[2] + t * delta[2]},
                                      {gl[0], gl[1], gl[2]}};
            const float cl = task_test_path(a, w, path, 3u, c.minimum_witness_clearance_m);
            if (cl > c.minimum_witness_clearance_m) {
                task_save(wit, path, 3u, cl);
                return true;
            }
        }
    const float side_offset[4] = {-2.4f, -1.2f, 1.2f, 2.4f};
    for (uint32_t i = 0; i < 4u; i++) {
        const float t = 0.5f;
        const float path[3][3] = {{st[0], st[1], st[2]},
                                  {st[0] + t * delta[0], task_clamp((st[1] + gl[1]) * 0.5f + side_offset[i], -4.60f, 4.60f),
                                   st[2] + t * delta[2]},
                                  {gl[0], gl[1], gl[2]}};
        const float cl = task_test_path(a, w, path, 3u, c.minimum_witness_clearance_m);
        if (cl > c.minimum_witness_clearance_m) {
            task_save(wit, path, 3u, cl);
            return true;
        }
    }
    const float detour_z[2] = {0.55f, 4.45f};
    for (uint32_t i = 0; i < 2u; i++) {
        const float path[3][3] = {{st[0], st[1], st[2]}, {st[0] + 0.5f * delta[0], st[1] + 0.5f * delta[1], detour_z[i]},
                                  {gl[0], gl[1], gl[2]}};
        const float cl = task_test_path(a, w, path, 3u, c.minimum_witness_clearance_m);
        if (cl > c.minimum_witness_clearance_m) {
            task_save(wit, path, 3u, cl);
            return true;
        }
    }
    for (uint32_t side = 0; side < 2u; side++) {
        const float y = side_y[side];
        const float path[4][3] = {{st[0], st[1], st[2]},
                                  {st[0] + 0.20f * delta[0], y, st[2] + 0.20f * delta[2]},
                                  {st[0] + 0.80f * delta[0], y, st[2] + 0.80f * delta[2]},
                                  {gl[0], gl[1], gl[2]}};
        const float cl = task_test_path(a, w, path, 4u, c.minimum_witness_clearance_m);
        if (cl > c.minimum_witness_clearance_m) {
            task_save(wit, path, 4u, cl);
            return true;
        }
    }
    return false;
}

// navigation_generate_task, :343-482.
__device__ uint32_t task_generate(const SimArgs& a, mdn_world& w, mdn_task_state& task, uint32_t& rng) {
    const mdn_task_config& c = a.task_ctl.config;
    task.generation_status = kTaskInvalidConfig;
    task.generation_attempts = 0;
    task.valid = 0;
    // :347-379: configuration, stage/family and bounds checks, evaluated once
    // on the host; a rejected configuration leaves every env at status 1.
    if (!a.task_config_ok) return kTaskInvalidConfig;
    uint32_t attempts = c.max_generation_attempts;
    if (attempts > kTaskMaxAttempts) attempts = kTaskMaxAttempts;
    for (uint32_t attempt = 0; attempt < attempts; attempt++) {
        __syncwarp();  // no lane still stores the previous attempt's fields (run by a whole warp)
        task.generation_attempts = attempt + 1u;
        const uint32_t scene_seed = wrng(rng);
        uint32_t scene_family = c.family;
        if (c.family == 12u) {
            const uint32_t sel = wrng(rng) % 4u;
            scene_family = sel == 0u ? 1u : (sel == 1u ? 2u : (sel == 2u ? 4u : 5u));
        }
        generate_world(w, scene_seed, scene_family, c.scene_distance_m);
        if (c.stage == kTaskClutter) {
            bool moving = false;
            for (uint32_t o = 0; o < w.count; o++)
                for (int ax = 0; ax < 3; ax++) moving = moving || fabsf(w.obstacles[o].velocity[ax]) > 1e-8f;
            if (moving) {
                task.generation_status = kTaskUnsupportedDynamic;
                return task.generation_status;
            }
        }
        float dir[3];
        task_random_direction(rng, dir);
        const float span = c.goal_distance_max_m - c.goal_distance_min_m;  // :234-239
        const float center = c.goal_distance_min_m + c.difficulty * span;
        const float jitter = (wurand(rng) - 0.5f) * 0.20f * span;
        const float distance = task_clamp(center + jitter, c.goal_distance_min_m, c.goal_distance_max_m);
        float st[3], gl[3];
        if (c.stage == kTaskHold) {
            task_random_point(rng, c.goal_min_xyz, c.goal_max_xyz, gl);
            for (int j = 0; j < 3; j++) st[j] = gl[j] - dir[j] * distance;
        } else {
            task_random_point(rng, c.start_min_xyz, c.start_max_xyz, st);
            for (int j = 0; j < 3; j++) gl[j] = st[j] + dir[j] * distance;
            if (c.stage == kTaskClutter) {
                bool in_bounds = task_inside(gl, c.goal_min_xyz, c.goal_max_xyz);
                for (uint32_t da = 1u; !in_bounds && da < kTaskMaxDirections; da++) {
                    task_random_direction(rng, dir);
                    for (int j = 0; j < 3; j++) gl[j] = st[j] + dir[j] * distance;
                    in_bounds = task_inside(gl, c.goal_min_xyz, c.goal_max_xyz);
                }
                if (!in_bounds) continue;
            }
        }
        if (!isfinite(gl[0]) || !isfinite(gl[1]) || !isfinite(gl[2])) continue;
        if (!task_inside(st, c.start_min_xyz, c.start_max_xyz) || !task_inside(gl, c.goal_min_xyz, c.goal_max_xyz)) continue;
        const float start_clear = world_clearance(a, w, st, 0.0f, nullptr);
        const float goal_clear = world_clearance(a, w, gl, 0.0f, nullptr);
        if (start_clear <= c.minimum_endpoint_clearance_m || goal_clear <= c.minimum_endpoint_clearance_m) continue;
        const float actual = len3(gl[0] - st[0], gl[1] - st[1], gl[2] - st[2]);
        if (actual < c.goal_distance_min_m || actual > c.goal_distance_max_m) continue;
        TaskWitness wit;
        float direct_clearance = 0.0f;
        if (!task_find_witness(a, w, st, gl, c, wit, direct_clearance)) continue;
        for (int j = 0; j < 3; j++) w.goal[j] = gl[j];
        task.family = scene_family;
        task.stage = c.stage;
        task.objective = c.objective;
        task.max_nav_steps = c.max_nav_steps;
        task.step_count = 0;
        task.stable_ticks = 0;
        task.was_inside_goal = 0;
        task.waypoint_event_latched = 0;
        task.terminal = 0;
        for (int j = 0; j < 3; j++) task.start_position[j] = st[j];
        task.start_yaw_rad = (wurand(rng) * 2.0f - 1.0f) * 3.14159265359f;
        const float speed = c.initial_speed_min_mps + (c.initial_speed_max_mps - c.initial_speed_min_mps) * wurand(rng);
        for (int j = 0; j < 3; j++) task.start_velocity_world[j] = dir[j] * speed;
        for (int j = 0; j < 3; j++) task.goal_position[j] = gl[j];
        task.initial_distance_m = actual;
        task.previous_distance_m = actual;
        task.difficulty = c.difficulty;
        task.start_clearance_m = start_clear;
        task.goal_clearance_m = goal_clear;
        task.direct_segment_clearance_m = direct_clearance;
        task.witness_min_clearance_m = wit.min_clearance;
        task.witness_length_m = wit.length;
        task.stable_time_s = 0.0f;
        for (int j = 0; j < 3; j++) task.last_executed_world_command[j] = task.start_velocity_world[j];
        task.last_executed_world_command[3] = 0.0f;
        task.witness_point_count = wit.count;
        for (uint32_t k = 0; k < kTaskMaxWitness; k++)
            for (int j = 0; j < 3; j++) task.witness_points[k][j] = k < wit.count ? wit.p[k][j] : 0.0f;
        task.valid = 1;
        task.generation_status = kTaskReady;
        return task.generation_status;
    }
    task.generation_status = kTaskExhausted;
    return task.generation_status;
}

struct TaskStep {
    float reward;
    uint32_t stable_success, timeout;
};

// navigation_task_step, :499-548 (reward, stable-hold success, timeout).
__device__ TaskStep task_step(mdn_task_state& task, const mdn_task_config& c, const float* pos, const float* vel,
                              const float cmd[4], bool contact, bool forced_timeout) {
    TaskStep r{0.0f, 0u, 0u};
    if (task.generation_status != kTaskReady || task.terminal != 0u) return r;
    const float dx = task.goal_position[0] - pos[0], dy = task.goal_position[1] - pos[1], dz = task.goal_position[2] - pos[2];
    const float distance = sqrtf(dx * dx + dy * dy + dz * dz);
    const float speed = sqrtf(vel[0] * vel[0] + vel[1] * vel[1] + vel[2] * vel[2]);
    if (!isfinite(distance) || !isfinite(speed)) {
        task.terminal = 1u;
        return r;
    }
    task.step_count++;
    const float progress = task.previous_distance_m - distance;
    float reward = c.progress_reward_per_m * progress - c.time_cost_per_s * c.nav_period_s;
    task.previous_distance_m = distance;
    const uint32_t inside = distance <= c.goal_radius_m ? 1u : 0u;
    if (task.objective == kTaskWaypoint && inside != 0u && task.waypoint_event_latched == 0u) task.waypoint_event_latched = 1u;
    const uint32_t stable_now = (inside != 0u && speed <= c.stable_speed_mps) ? 1u : 0u;
    if (task.objective == kTaskFinalHold && stable_now != 0u) task.stable_time_s += c.nav_period_s;
    else task.stable_time_s = 0.0f;
    task.stable_ticks = uint32_t(ceilf(task.stable_time_s / fmaxf(c.nav_period_s, 1e-6f) - 1e-5f));
    const uint32_t stable = (task.objective == kTaskFinalHold && stable_now != 0u &&
                             task.stable_time_s + 1e-6f >= c.stable_hold_s) ? 1u : 0u;
    const uint32_t collision = contact ? 1u : 0u;
    const uint32_t timeout = (forced_timeout || task.step_count >= task.max_nav_steps) ? 1u : 0u;
    if (c.command_smoothness_weight > 0.0f) {
        float difference = 0.0f;
        for (int ax = 0; ax < 4; ax++) {
            const float delta = cmd[ax] - task.last_executed_world_command[ax];
            difference += delta * delta;
            task.last_executed_world_command[ax] = cmd[ax];
        }
        reward -= c.command_smoothness_weight * difference * c.nav_period_s;
    }
    if (collision) reward -= c.contact_penalty;
    if (stable && !collision) reward += c.stable_arrival_bonus;
    task.terminal = (collision || stable || timeout) ? 1u : 0u;
    r.reward = reward;
    r.stable_success = stable;
    r.timeout = timeout;
    return r;
}

// Episode reset with the task contract: sim_reset_one, the challenge-bank
// world of schedule slot `slot` (sim.metal:143,330), then
// sim_reset_navigation_task (sim.metal:125-141), then the SoA world mirror.
// Run by a whole converged warp. The task's scene is generated and its witness
// checked in the warp's shared-memory world, then stored once. Returns true
// (the caller refills the env's range ring).
__device__ __noinline__ bool episode_reset(const SimArgs& a, uint32_t i, bool first, uint32_t slot,
                                           mdn_world& scratch) {
    reset_env(a, i, first, scratch);
    if (a.bank_enabled) apply_challenge_world(a, i, slot);
    else a.bank_active[i] = 0xffffffffu;
    mdn_task_state& task = a.tasks[i];
    task = mdn_task_state{};
    if (a.task_ctl.enabled) {
        const uint32_t gid = a.env_base + i;
        mdn_sim_run& run = a.runs[i];
        mdn_physics_state& s = a.states[i];
        mdn_world& w = scratch;
        __syncwarp();
        copy_world_warp(w, a.worlds[i]);  // the bank may have replaced the reset's world
        uint32_t rng = a.cfg.seed ^ ((gid + 1u) * 0x27d4eb2du) ^ ((run.episodes + 1u) * 0x165667b1u);
        task_generate(a, w, task, rng);
        if (task.valid) {  // navigation_task_apply_start, navigation_tasks.hpp:486-495
            for (int ax = 0; ax < 3; ax++) {
                s.position[ax] = task.start_position[ax];
                s.linear_velocity[ax] = task.start_velocity_world[ax];
                s.angular_velocity_body[ax] = 0.0f;
            }
            const float half_yaw = task.start_yaw_rad * 0.5f;
            s.orientation_wxyz[0] = cosf(half_yaw);
            s.orientation_wxyz[1] = 0.0f;
            s.orientation_wxyz[2] = 0.0f;
            s.orientation_wxyz[3] = sinf(half_yaw);
            run.yaw = task.start_yaw_rad;
            run.initial_distance = task.initial_distance_m;
            for (int ax = 0; ax < 3; ax++) {
                run.reference_position[ax] = s.position[ax];
                run.desired_velocity[ax] = s.linear_velocity[ax];
            }
            w.wind[0] = clean_env(a, gid) ? 0.0f : a.cfg.wind;
            w.wind[1] = 0;
            w.wind[2] = 0;
        }
        __syncwarp();
        copy_world_warp(a.worlds[i], w);
    }
    __syncwarp();
    mirror_world_warp(a, i);
    return true;
}

}  // namespace mdn
