// Device math for the rollout kernels (sm_100a).
//
// Compiled with --fmad=false: every `a*b+c` written here rounds the product and
// the sum separately, exactly like the reference's CPU path (x86-64 SSE, no
// contraction), so the geometry (world.hpp), L2F integrator (physics.hpp) and
// observation arithmetic reproduce the reference's float results bit for bit
// on the same inputs. Division and sqrt are IEEE round-to-nearest
// (-prec-div/-prec-sqrt defaults). Dot products of the learned networks (RAPTOR
// GRU, actor, critic) use explicit fmaf: their outputs pass through
// transcendental functions whose last-ulp results differ between CUDA and libm
// anyway, and they are compared with tolerances.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "mdn_shared.h"

namespace mdn {

__device__ __forceinline__ float smin(float a, float b) { return b < a ? b : a; }  // std::min
__device__ __forceinline__ float smax(float a, float b) { return a < b ? b : a; }  // std::max
__device__ __forceinline__ float clampf(float x, float lo, float hi) { return smax(lo, smin(hi, x)); }
__device__ __forceinline__ float len3(float x, float y, float z) { return sqrtf(x * x + y * y + z * z); }

// xorshift32, world.hpp:30-31
__device__ __forceinline__ uint32_t wrng(uint32_t& s) {
    s ^= s << 13;
    s ^= s >> 17;
    s ^= s << 5;
    return s;
}
__device__ __forceinline__ float wurand(uint32_t& s) { return float(wrng(s) >> 8) * (1.0f / 16777216.0f); }
// Box-Muller draw, sim.metal:49
__device__ __forceinline__ float sim_normal(uint32_t& rng) {
    const float u = smax(wurand(rng), 1e-7f), v = wurand(rng);
    return sqrtf(-2.0f * logf(u)) * cosf(6.28318530718f * v);
}

// Obstacle centre at time t, world.hpp:32-41.
__device__ __forceinline__ void obstacle_center(uint32_t kind, const float* c, const float* size, const float* v,
                                                float t, float out[3]) {
    if (kind == 3) {
        const float speed = len3(v[0], v[1], v[2]), amplitude = size[1];
        if (speed <= 1e-8f || amplitude <= 1e-8f) {
            out[0] = c[0]; out[1] = c[1]; out[2] = c[2];
            return;
        }
        const float offset = amplitude * sinf(t * speed / amplitude + size[2]) / speed;
        out[0] = c[0] + v[0] * offset;
        out[1] = c[1] + v[1] * offset;
        out[2] = c[2] + v[2] * offset;
        return;
    }
    out[0] = c[0] + t * v[0];
    out[1] = c[1] + t * v[1];
    out[2] = c[2] + t * v[2];
}

// a / d rounded to nearest, from y = RN(1/d) and no divide instruction:
// q0 = a*y, then two residual corrections with fused multiply-adds. Markstein
// ("Computation of elementary functions on the IBM RISC System/6000 processor",
// IBM J. Res. Dev. 34(1), 1990) shows that when y is the correctly rounded
// reciprocal and q is faithful, RN(q + (a - d*q)*y) = RN(a/d), the residual
// being exact; the first correction makes q0 faithful, the second rounds.
// Used where d is a ray direction component with |d| >= 1e-8 and |a| is a
// room-scale distance, so no intermediate overflows or becomes subnormal.
// mdn_selftest_division compares it with IEEE division on the GPU.
__device__ __forceinline__ float div_by_rcp(float a, float d, float y) {
    const float q0 = a * y;
    const float q1 = fmaf(fmaf(-d, q0, a), y, q0);
    return fmaf(fmaf(-d, q1, a), y, q1);
}

// Slab test with the ray's reciprocal direction components (rcp[j] =
// __frcp_rn(d[j]) where |d[j]| >= 1e-8): ray_box below, bit for bit.
__device__ __forceinline__ float ray_box_rcp(float px, float py, float pz, const float dd[3], const float rcp[3],
                                             float cx, float cy, float cz, float ex, float ey, float ez) {
    float lo = -1e20f, hi = 1e20f;
    const float pp[3] = {px - cx, py - cy, pz - cz}, ee[3] = {ex, ey, ez};
#pragma unroll
    for (int j = 0; j < 3; j++) {
        if (fabsf(dd[j]) < 1e-8f) {
            if (fabsf(pp[j]) > ee[j]) return 1000.0f;
        } else {
            const float a = div_by_rcp(-ee[j] - pp[j], dd[j], rcp[j]), b = div_by_rcp(ee[j] - pp[j], dd[j], rcp[j]);
            lo = fmaxf(lo, fminf(a, b));
            hi = fminf(hi, fmaxf(a, b));
        }
    }
    if (hi < fmaxf(lo, 0.0f)) return 1000.0f;
    return lo >= 0 ? lo : hi;
}

// Slab test, world.hpp:48-57 (same operation order; IEEE division).
__device__ __forceinline__ float ray_box(float px, float py, float pz, float dx, float dy, float dz, float cx, float cy,
                                         float cz, float ex, float ey, float ez) {
    float lo = -1e20f, hi = 1e20f;
    const float pp[3] = {px - cx, py - cy, pz - cz}, dd[3] = {dx, dy, dz}, ee[3] = {ex, ey, ez};
#pragma unroll
    for (int j = 0; j < 3; j++) {
        if (fabsf(dd[j]) < 1e-8f) {
            if (fabsf(pp[j]) > ee[j]) return 1000.0f;
        } else {
            const float a = (-ee[j] - pp[j]) / dd[j], b = (ee[j] - pp[j]) / dd[j];
            lo = fmaxf(lo, fminf(a, b));
            hi = fminf(hi, fmaxf(a, b));
        }
    }
    if (hi < fmaxf(lo, 0.0f)) return 1000.0f;
    return lo >= 0 ? lo : hi;
}
// world.hpp:42-47
__device__ __forceinline__ float ray_sphere(float px, float py, float pz, float dx, float dy, float dz, float cx,
                                            float cy, float cz, float r) {
    const float qx = px - cx, qy = py - cy, qz = pz - cz;
    const float b = qx * dx + qy * dy + qz * dz;
    const float k = (qx * qx + qy * qy + qz * qz) - r * r;
    const float disc = b * b - k;
    if (disc < 0) return 1000.0f;
    const float s = sqrtf(disc);
    const float lo = -b - s, hi = -b + s;
    return lo >= 0 ? lo : (hi >= 0 ? hi : 1000.0f);
}
// world.hpp:58-70
__device__ __forceinline__ float ray_cylinder(float px, float py, float pz, float dx, float dy, float dz, float cx,
                                              float cy, float cz, float r, float h) {
    const float qx = px - cx, qy = py - cy, qz = pz - cz;
    const float a = dx * dx + dy * dy, b = qx * dx + qy * dy, k = qx * qx + qy * qy - r * r;
    float best = 1000.0f;
    const float disc = b * b - a * k;
    if (a > 1e-10f && disc >= 0) {
        const float s = sqrtf(disc);
        const float r0 = (-b - s) / a, r1 = (-b + s) / a;
        if (r0 >= 0 && fabsf(qz + r0 * dz) <= h) best = fminf(best, r0);
        if (r1 >= 0 && fabsf(qz + r1 * dz) <= h) best = fminf(best, r1);
    }
    if (fabsf(dz) > 1e-8f) {
#pragma unroll
        for (int sign = -1; sign <= 1; sign += 2) {
            const float t = (float(sign) * h - qz) / dz;
            const float x = qx + t * dx, y = qy + t * dy;
            if (t >= 0 && x * x + y * y <= r * r) best = fminf(best, t);
        }
    }
    return best;
}

// Signed distance from a point (offset q from the centre) to a box of half
// extents e, world.hpp:93-94.
__device__ __forceinline__ float box_distance(const float* e, float qx, float qy, float qz) {
    const float kx = fabsf(qx) - e[0], ky = fabsf(qy) - e[1], kz = fabsf(qz) - e[2];
    return len3(fmaxf(kx, 0.0f), fmaxf(ky, 0.0f), fmaxf(kz, 0.0f)) + fminf(fmaxf(kx, fmaxf(ky, kz)), 0.0f);
}

// Signed distance minus the 0.18 m drone radius to one obstacle, world.hpp:86-96.
__device__ __forceinline__ float obstacle_clearance(uint32_t kind, const float* size, float qx, float qy, float qz) {
    float distance;
    if (kind == 1 || kind == 3) {
        distance = len3(qx, qy, qz) - size[0];
    } else if (kind == 2) {
        const float a = sqrtf(qx * qx + qy * qy) - size[0], b = fabsf(qz) - size[2];
        distance = sqrtf(fmaxf(a, 0.0f) * fmaxf(a, 0.0f) + fmaxf(b, 0.0f) * fmaxf(b, 0.0f)) + fminf(fmaxf(a, b), 0.0f);
    } else {
        distance = box_distance(size, qx, qy, qz);
    }
    return distance - 0.18f;
}

// Input 32 + j of the control-state critic's observation (sim.metal:166-180,
// built with FIXED_PPO_CRITIC_OBS_DIM=64 and NAV_CRITIC_CONTROL_STATE):
// j 0-15 the RAPTOR hidden state, 16-19 the rotor speeds, 20-21 sine and cosine
// of the run's yaw minus the body's yaw, 22-25 the last policy command, 26-28
// the desired velocity / 2, 29 the goal-closing speed / 4, 30 the goal
// distance / 10, 31 the speed / 4. The arguments describe the state the
// observation is of: hidden, rpm, dvel (desired velocity) may live in
// registers when j is a compile-time index, or in device memory.
__device__ __forceinline__ float control_state_input(int j, const float* hidden, const float* rpm, const float q[4],
                                                     const float pos[3], const float vel[3], const float* dvel,
                                                     const mdn_sim_run& run, const mdn_world& w) {
    if (j < 16) return hidden[j];
    if (j < 20) return rpm[j - 16];
    if (j < 22) {
        const float body_yaw =
            atan2f(2.0f * (q[0] * q[3] + q[1] * q[2]), 1.0f - 2.0f * (q[2] * q[2] + q[3] * q[3]));
        return j == 20 ? sinf(run.yaw - body_yaw) : cosf(run.yaw - body_yaw);
    }
    if (j < 26) return run.previous_nav[j - 22];
    if (j < 29) return dvel[j - 26] / 2.0f;
    const float g0 = w.goal[0] - pos[0], g1 = w.goal[1] - pos[1], g2 = w.goal[2] - pos[2];
    const float distance = len3(g0, g1, g2);
    if (j == 29) return (g0 * vel[0] + g1 * vel[1] + g2 * vel[2]) / fmaxf(distance, 1e-6f) / 4.0f;
    if (j == 30) return distance / 10.0f;
    return len3(vel[0], vel[1], vel[2]) / 4.0f;
}

// Room term of wclearance, world.hpp:85 (p - lo == p + 2 etc. for the reference room).
__device__ __forceinline__ float room_clearance(const SimArgs& a, const float p[3]) {
    return fminf(fminf(p[0] - a.room_lo[0], a.room_hi[0] - p[0]),
                 fminf(fminf(p[1] - a.room_lo[1], a.room_hi[1] - p[1]), fminf(p[2] - a.room_lo[2], a.room_hi[2] - p[2]))) -
           0.18f;
}

// Whole wclearance for one thread, with the id of the first minimising term
// (-1 = room walls).
__device__ __forceinline__ float world_clearance(const SimArgs& a, const mdn_world& w, const float p[3], float t,
                                                 int32_t* argmin) {
    float best = room_clearance(a, p);
    int32_t id = -1;
    const uint32_t count = w.count < 16u ? w.count : 16u;
    for (uint32_t i = 0; i < count; i++) {
        const mdn_obstacle& o = w.obstacles[i];
        float c[3];
        obstacle_center(o.kind, o.center, o.size, o.velocity, t, c);
        const float cand = obstacle_clearance(o.kind, o.size, p[0] - c[0], p[1] - c[1], p[2] - c[2]);
        if (cand < best) id = int32_t(i);
        best = fminf(best, cand);
    }
    if (argmin) *argmin = id;
    return best;
}

// wclearance (world.hpp:84-99) reading the structure-of-arrays mirror: thread
// i's loads of word w across a warp are contiguous.
__device__ __forceinline__ float world_clearance_soa(const SimArgs& a, uint32_t i, const float p[3], float t,
                                                     int32_t* argmin) {
    const float* soa = a.world_soa;
    const size_t n = a.n;
    float best = room_clearance(a, p);
    int32_t id = -1;
    uint32_t count = __float_as_uint(__ldg(&soa[160 * n + i]));
    count = count < 16u ? count : 16u;
    for (uint32_t o = 0; o < count; o++) {
        const float* f = soa + size_t(o) * 10 * n + i;
        const uint32_t kind = __float_as_uint(__ldg(f));
        const float c[3] = {__ldg(f + n), __ldg(f + 2 * n), __ldg(f + 3 * n)};
        const float size[3] = {__ldg(f + 4 * n), __ldg(f + 5 * n), __ldg(f + 6 * n)};
        const float v[3] = {__ldg(f + 7 * n), __ldg(f + 8 * n), __ldg(f + 9 * n)};
        float cc[3];
        obstacle_center(kind, c, size, v, t, cc);
        const float cand = obstacle_clearance(kind, size, p[0] - cc[0], p[1] - cc[1], p[2] - cc[2]);
        if (cand < best) id = int32_t(o);
        best = fminf(best, cand);
    }
    if (argmin) *argmin = id;
    return best;
}

// world_clearance_soa on a group of G lanes that share environment i (lane r
// of the group takes obstacles r, r + G, ...). Each lane keeps the smallest
// clearance of its obstacles and the first index that reached it below the
// room's; the group then keeps the smallest value, and on a tie the smaller
// index (equal values are either both the room's, index -1, or both below
// it). That is the value and index of the sequential scan.
template <int G>
__device__ __forceinline__ float world_clearance_lanes(const SimArgs& a, uint32_t i, const float p[3], float t,
                                                       int32_t* argmin, int r, unsigned mask) {
    if constexpr (G == 1) {
        return world_clearance_soa(a, i, p, t, argmin);
    } else {
        const float* soa = a.world_soa;
        const size_t n = a.n;
        float best = room_clearance(a, p);
        int32_t id = -1;
        uint32_t count = __float_as_uint(__ldg(&soa[160 * n + i]));
        count = count < 16u ? count : 16u;
        for (uint32_t o = uint32_t(r); o < count; o += G) {
            const float* f = soa + size_t(o) * 10 * n + i;
            const uint32_t kind = __float_as_uint(__ldg(f));
            const float c[3] = {__ldg(f + n), __ldg(f + 2 * n), __ldg(f + 3 * n)};
            const float size[3] = {__ldg(f + 4 * n), __ldg(f + 5 * n), __ldg(f + 6 * n)};
            const float v[3] = {__ldg(f + 7 * n), __ldg(f + 8 * n), __ldg(f + 9 * n)};
            float cc[3];
            obstacle_center(kind, c, size, v, t, cc);
            const float cand = obstacle_clearance(kind, size, p[0] - cc[0], p[1] - cc[1], p[2] - cc[2]);
            if (cand < best) id = int32_t(o);
            best = fminf(best, cand);
        }
#pragma unroll
        for (int off = G / 2; off > 0; off >>= 1) {
            const float ob = __shfl_xor_sync(mask, best, off);
            const int32_t oi = __shfl_xor_sync(mask, id, off);
            if (ob < best || (ob == best && oi < id)) {
                best = ob;
                id = oi;
            }
        }
        if (argmin) *argmin = id;
        return best;
    }
}

// Body-to-world rotation from a wxyz quaternion, sim.metal:43-48.
__device__ __forceinline__ void rotation(const float q[4], float r[9]) {
    const float w = q[0], x = q[1], y = q[2], z = q[3];
    r[0] = 1 - 2 * (y * y + z * z); r[1] = 2 * (x * y - w * z); r[2] = 2 * (x * z + w * y);
    r[3] = 2 * (x * y + w * z); r[4] = 1 - 2 * (x * x + z * z); r[5] = 2 * (y * z - w * x);
    r[6] = 2 * (x * z - w * y); r[7] = 2 * (y * z + w * x); r[8] = 1 - 2 * (x * x + y * y);
}

// ---------------------------------------------------------------- physics
// L2F rigid body + motor lag, physics.hpp:60-179. State as 17 floats.
struct Phys17 {
    float v[17];
};
__device__ __forceinline__ void l2f_derivative(const mdn_physics_params& p, const float* s, const float sp[4],
                                               const float wind[3], float* d) {
    float thrust[3] = {0, 0, 0}, torque[3] = {0, 0, 0};
    const float* rpm = s + 13;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const float speed = rpm[r];
        const float* c = &p.rotor_thrust_coefficients[3 * r];
        const float magnitude = c[0] + c[1] * speed + c[2] * speed * speed;
        float rt[3];
#pragma unroll
        for (int i = 0; i < 3; ++i) {
            rt[i] = p.rotor_thrust_directions[3 * r + i] * magnitude;
            thrust[i] += rt[i];
            torque[i] += p.rotor_torque_directions[3 * r + i] * magnitude * p.rotor_torque_constants[r];
        }
        const float* pos = &p.rotor_positions[3 * r];
        const float arm0 = pos[1] * rt[2] - pos[2] * rt[1];
        const float arm1 = pos[2] * rt[0] - pos[0] * rt[2];
        const float arm2 = pos[0] * rt[1] - pos[1] * rt[0];
        torque[0] += arm0;
        torque[1] += arm1;
        torque[2] += arm2;
    }
#pragma unroll
    for (int i = 0; i < 3; ++i) d[i] = s[7 + i];
    const float* q = s + 3;
    const float* w = s + 10;
    d[3] = -q[1] * w[0] - q[2] * w[1] - q[3] * w[2];
    d[4] = q[0] * w[0] + q[2] * w[2] - q[3] * w[1];
    d[5] = q[0] * w[1] + q[3] * w[0] - q[1] * w[2];
    d[6] = q[0] * w[2] + q[1] * w[1] - q[2] * w[0];
#pragma unroll
    for (int i = 3; i < 7; ++i) d[i] *= 0.5f;
    // rotate_body_to_world, physics.hpp:51-58
    const float tx = 2.0f * (q[2] * thrust[2] - q[3] * thrust[1]);
    const float ty = 2.0f * (q[3] * thrust[0] - q[1] * thrust[2]);
    const float tz = 2.0f * (q[1] * thrust[1] - q[2] * thrust[0]);
    const float lv0 = thrust[0] + q[0] * tx + q[2] * tz - q[3] * ty;
    const float lv1 = thrust[1] + q[0] * ty + q[3] * tx - q[1] * tz;
    const float lv2 = thrust[2] + q[0] * tz + q[1] * ty - q[2] * tx;
    d[7] = lv0 / p.mass + p.gravity_world[0] + wind[0] / p.mass;
    d[8] = lv1 / p.mass + p.gravity_world[1] + wind[1] / p.mass;
    d[9] = lv2 / p.mass + p.gravity_world[2] + wind[2] / p.mass;
    float am[3] = {0, 0, 0};
#pragma unroll
    for (int row = 0; row < 3; ++row)
#pragma unroll
        for (int col = 0; col < 3; ++col) am[row] += p.inertia[3 * row + col] * w[col];
    const float g0 = w[1] * am[2] - w[2] * am[1];
    const float g1 = w[2] * am[0] - w[0] * am[2];
    const float g2 = w[0] * am[1] - w[1] * am[0];
    am[0] = torque[0] - g0;
    am[1] = torque[1] - g1;
    am[2] = torque[2] - g2;
#pragma unroll
    for (int row = 0; row < 3; ++row) {
        float acc = 0.0f;
#pragma unroll
        for (int col = 0; col < 3; ++col) acc += p.inertia_inverse[3 * row + col] * am[col];
        d[10 + row] = acc;
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const float tau = sp[r] >= rpm[r] ? p.rotor_time_constants_rising[r] : p.rotor_time_constants_falling[r];
        d[13 + r] = (sp[r] - rpm[r]) / tau;
    }
}

// rl_physics_step, physics.hpp:149-179.
__device__ __forceinline__ void l2f_step(const mdn_physics_params& p, const float* s, const float action[4],
                                         const float wind[3], float* out) {
    float sp[4];
    const float half_range = (p.action_max - p.action_min) * 0.5f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float a = action[i];
        if (a < -1.0f) a = -1.0f;
        if (a > 1.0f) a = 1.0f;
        sp[i] = a * half_range + p.action_min + half_range;
    }
    // k1 + 2 k2 + 2 k3 + k4 accumulated left to right, the reference's order.
    float k[17], acc[17], tmp[17];
    l2f_derivative(p, s, sp, wind, k);
    const float hdt = 0.5f * p.dt;
#pragma unroll
    for (int i = 0; i < 17; ++i) {
        acc[i] = k[i];
        tmp[i] = s[i] + hdt * k[i];
    }
    l2f_derivative(p, tmp, sp, wind, k);
#pragma unroll
    for (int i = 0; i < 17; ++i) {
        acc[i] = acc[i] + 2.0f * k[i];
        tmp[i] = s[i] + hdt * k[i];
    }
    l2f_derivative(p, tmp, sp, wind, k);
#pragma unroll
    for (int i = 0; i < 17; ++i) {
        acc[i] = acc[i] + 2.0f * k[i];
        tmp[i] = s[i] + p.dt * k[i];
    }
    l2f_derivative(p, tmp, sp, wind, k);
#pragma unroll
    for (int i = 0; i < 17; ++i) out[i] = s[i] + p.dt * (acc[i] + k[i]) / 6.0f;
    const float norm = sqrtf(out[3] * out[3] + out[4] * out[4] + out[5] * out[5] + out[6] * out[6]);
#pragma unroll
    for (int i = 3; i < 7; ++i) out[i] /= norm;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        if (out[i] < -p.position_limit) out[i] = -p.position_limit;
        if (out[i] > p.position_limit) out[i] = p.position_limit;
        if (out[7 + i] < -p.velocity_limit) out[7 + i] = -p.velocity_limit;
        if (out[7 + i] > p.velocity_limit) out[7 + i] = p.velocity_limit;
        if (out[10 + i] < -p.angular_velocity_limit) out[10 + i] = -p.angular_velocity_limit;
        if (out[10 + i] > p.angular_velocity_limit) out[10 + i] = p.angular_velocity_limit;
    }
#pragma unroll
    for (int i = 13; i < 17; ++i) {
        if (out[i] < p.action_min) out[i] = p.action_min;
        if (out[i] > p.action_max) out[i] = p.action_max;
    }
}

// ----------------------------------------------------------------- RAPTOR
// Dense(22,16)-ReLU -> GRU(16) -> Dense(16,4), raptor.hpp:52-92. `w` points to
// the 2,084-float RaptorWeights block (shared memory in the advance kernel).
__device__ __forceinline__ void raptor_forward(const float* __restrict__ w, const float obs[22], float h[16],
                                               float action[4]) {
    const float* in_w = w;
    const float* in_b = w + 352;
    const float* gi_w = w + 368;
    const float* gh_w = w + 1136;
    const float* gi_b = w + 1904;
    const float* gh_b = w + 1952;
    const float* out_w = w + 2016;
    const float* out_b = w + 2080;
    float x[16];
#pragma unroll
    for (int row = 0; row < 16; ++row) {
        float value = in_b[row];
#pragma unroll
        for (int col = 0; col < 22; ++col) value = fmaf(in_w[row * 22 + col], obs[col], value);
        x[row] = smax(value, 0.0f);
    }
    float nh[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float ir = gi_b[i], hr = gh_b[i], iz = gi_b[16 + i], hz = gh_b[16 + i], in_ = gi_b[32 + i], hn = gh_b[32 + i];
#pragma unroll
        for (int col = 0; col < 16; ++col) {
            ir = fmaf(gi_w[i * 16 + col], x[col], ir);
            hr = fmaf(gh_w[i * 16 + col], h[col], hr);
            iz = fmaf(gi_w[(16 + i) * 16 + col], x[col], iz);
            hz = fmaf(gh_w[(16 + i) * 16 + col], h[col], hz);
            in_ = fmaf(gi_w[(32 + i) * 16 + col], x[col], in_);
            hn = fmaf(gh_w[(32 + i) * 16 + col], h[col], hn);
        }
        const float reset = 1.0f / (1.0f + expf(-(ir + hr)));
        const float update = 1.0f / (1.0f + expf(-(iz + hz)));
        const float cand = tanhf(in_ + reset * hn);
        nh[i] = (1.0f - update) * cand + update * h[i];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) h[i] = nh[i];
#pragma unroll
    for (int row = 0; row < 4; ++row) {
        float value = out_b[row];
#pragma unroll
        for (int col = 0; col < 16; ++col) value = fmaf(out_w[row * 16 + col], h[col], value);
        action[row] = value;
    }
}

}  // namespace mdn
