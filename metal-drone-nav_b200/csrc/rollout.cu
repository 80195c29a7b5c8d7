// Rollout kernels for sm_100a: reset, sense (depth + observation), act (actor
// + critic + sampling), advance (5 RAPTOR/L2F substeps, reward, next value,
// in-kernel reset). One policy step = sense -> act -> advance; a rollout of T
// steps is captured once into a CUDA graph by the host (host.cpp).
//
// Reference kernels restated: sim_reset/sim_depth/sim_observe/sim_act/
// sim_advance (sim.metal:142-332) with the CPU path's semantics
// (cpu_reference.hpp:240-513).
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>

#include "contact.cuh"
#include "mdn_device.cuh"
#include "task.cuh"
#include "mlp.h"
#include "wide.h"
#include "world_gen.cuh"

namespace mdn {

// Camera tables in global memory, read through the L1: lanes index them with
// different pixels, which the constant cache would serialise.
__device__ float4 g_pixel_ray[kPixels];  // nav_sensor_pixel_ray(1, 0.75, k) as (x, y, z, 0), sensor_profile.hpp:89-91
__device__ float g_pool_ray[80 * 3];      // nav_ray(row, col, 0.75), guidance.hpp:22-26
// Cone around each 4x8 pixel tile's rays (camera frame): unit axis and the
// cosine / sine of a half-angle that covers all 32 rays with a margin.
__device__ float4 g_tile_cone[kPixels / 32];  // (axis, cos)
__device__ float g_tile_sin[kPixels / 32];
#define c_pool_ray_at(i) __ldg(&g_pool_ray[(i)])

// ------------------------------------------------------------------ reset
// Range ring of environment i refilled with 12 m by the whole warp.
__device__ __forceinline__ void refill_ring_warp(const SimArgs& a, uint32_t i) {
    const float4 twelve = make_float4(12.0f, 12.0f, 12.0f, 12.0f);
    float4* ring = reinterpret_cast<float4*>(a.sensors + size_t(i) * kFrames * kPixels);
    for (int j = threadIdx.x & 31; j < kFrames * kPixels / 4; j += 32) ring[j] = twelve;
}

// sim_reset: one warp per environment (episode_reset is warp-cooperative).
__global__ void __launch_bounds__(128) k_reset(SimArgs a, int first) {
    __shared__ mdn_world scratch[4];  // one world per warp of the 128-thread block
    const uint32_t i = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (i >= a.n) return;  // warp-uniform
    episode_reset(a, i, first != 0, 0, scratch[threadIdx.x >> 5]);
    refill_ring_warp(a, i);
    if ((threadIdx.x & 31) == 0) a.reset_pending[i] = 0;
}

// In-step episode resets (sim.metal:330) of the environments k_advance listed,
// one warp per listed environment (episode_reset is warp-cooperative), so a
// reset neither holds up an advance warp nor runs its generator's checks on
// one lane. Schedule slot tick + 1 as in the advance. This is the flush that
// ends a step whose state the host may read (a single step, the last step of
// a collected rollout); inside a collected rollout the next step's
// k_reset_sense runs the listed resets instead. Clears each environment's
// pending flag.
__global__ void __launch_bounds__(128) k_reset_list(SimArgs a) {
    __shared__ mdn_world scratch[4];  // one world per warp of the 128-thread block
    const uint32_t listed = a.reset_count[a.phase];
    const uint32_t count = listed < a.n ? listed : a.n;
    const uint32_t warps = gridDim.x * (blockDim.x / 32);
    for (uint32_t k = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); k < count; k += warps) {
        const uint32_t i = a.reset_list[k];
        episode_reset(a, i, false, a.tick + 1, scratch[threadIdx.x >> 5]);
        refill_ring_warp(a, i);
        if ((threadIdx.x & 31) == 0) a.reset_pending[i] = 0;
    }
}

// Refresh the structure-of-arrays mirror from the AoS worlds (after an upload
// or a checkpoint load replaced them).
__global__ void k_world_mirror(SimArgs a) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < a.n) mirror_world(a, i);
}

// ------------------------------------------------------------------ sense
// One warp per environment. Lanes cast 10 of the 320 rays each (world.hpp:71-83)
// against the room and the env's obstacles staged in shared memory, write the
// range ring frame and camera pose (sim.metal:145-158), then build the 184-float
// actor observation with the 2x2 min pool, 21 context features and the
// geometry-prior hint (sim.metal:182-228, guidance.hpp:39-90) and the 32-float
// critic observation (sim.metal:159-165).
constexpr int kSenseWarps = 8;

struct WarpScene {
    // Obstacles that can be seen this step, compacted and packed for 128-bit
    // loads in the ray loop: cull = (centre relative to the camera, inflated
    // bounding radius), cull2 = (squared distance, radius squared, kind bits),
    // geom = (centre, size x), geom2 = (size y, size z).
    float4 cull[16], cull2[16], geom[16], geom2[16];
    uint32_t tile_mask[kPixels / 32];  // candidates that can reach each pixel tile
    float cx[16], cy[16], cz[16];   // obstacle centres at the step's time
    float sx[16], sy[16], sz[16];   // sizes
    uint32_t kind[16];
    float cur[80], prev[80];        // pooled ranges (metres, obs*12 as the reference re-derives them)
    float risk_term[80];            // guidance.hpp:59-66 contribution of each cell as a neighbour
    float ctx[24];
};

__device__ __forceinline__ void warp_argmax_first(float& score, int& index) {
    // Max score; equal scores keep the smaller index, matching a sequential
    // scan that replaces only on a strictly greater score.
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float os = __shfl_xor_sync(0xffffffffu, score, off);
        const int oi = __shfl_xor_sync(0xffffffffu, index, off);
        if (os > score || (os == score && oi < index)) {
            score = os;
            index = oi;
        }
    }
}

__device__ __forceinline__ float pooled_min3x3(const float* range, int row, int col) {  // guidance.hpp:27-34
    float nearest = 12.0f;
#pragma unroll
    for (int dr = -1; dr <= 1; dr++)
#pragma unroll
        for (int dc = -1; dc <= 1; dc++) {
            const int r = row + dr, c = col + dc;
            if (r >= 0 && r < 8 && c >= 0 && c < 10) nearest = fminf(nearest, range[r * 10 + c]);
        }
    return nearest;
}

// Contribution of cell k to the temporal risk of the cells around it
// (guidance.hpp:59-66): the per-neighbour term depends only on the neighbour.
__device__ __forceinline__ float neighbour_risk(const WarpScene& ws, int k, const float vel[3], float sensor_dt) {
    const float old = ws.prev[k], now = ws.cur[k];
    if (!(old < 11.9f && now < 11.9f)) return 0.0f;
    const float unexpected = (old - now) / fmaxf(sensor_dt, 1e-3f) -
                             (vel[0] * c_pool_ray_at(3 * k) + vel[1] * c_pool_ray_at(3 * k + 1) +
                              vel[2] * c_pool_ray_at(3 * k + 2));
    return unexpected > 0.5f ? fminf(0.20f * unexpected, 1.0f) : 0.0f;
}

// risk = max(0, max over in-grid 3x3 neighbours of their terms): the same
// fmaxf chain as the reference's loop, in any order (fmaxf is exact).
__device__ __forceinline__ float cell_risk(const WarpScene& ws, int row, int col, float sensor_dt) {
    float risk = 0.0f;
    if (sensor_dt > 1e-4f) {
#pragma unroll
        for (int dr = -1; dr <= 1; dr++)
#pragma unroll
            for (int dc = -1; dc <= 1; dc++) {
                const int r = row + dr, c = col + dc;
                if (r < 0 || r >= 8 || c < 0 || c >= 10) continue;
                risk = fmaxf(risk, ws.risk_term[r * 10 + c]);
            }
    }
    return risk;
}

// sim_depth + sim_observe + sim_critic_obs of environment i, by one warp.
__device__ __forceinline__ void sense_env(const SimArgs& a, uint32_t i, WarpScene& ws) {
    const int lane = threadIdx.x & 31;
    const mdn_sim_config& c = a.cfg;
    const mdn_sim_run& run = a.runs[i];
    const uint32_t episodes = run.episodes, steps = run.steps;
    if (c.eval && episodes) return;
    const uint32_t gid = a.env_base + i;
    const mdn_physics_state& st = a.states[i];
    const float pos[3] = {st.position[0], st.position[1], st.position[2]};
    const float q[4] = {st.orientation_wxyz[0], st.orientation_wxyz[1], st.orientation_wxyz[2], st.orientation_wxyz[3]};
    float r[9];
    rotation(q, r);
    const float elapsed = run.elapsed;
    const mdn_world& w = a.worlds[i];
    const uint32_t count = w.count < 16u ? w.count : 16u;
    if (lane < int(count)) {
        const mdn_obstacle& o = w.obstacles[lane];
        float cc[3];
        obstacle_center(o.kind, o.center, o.size, o.velocity, elapsed, cc);
        ws.cx[lane] = cc[0]; ws.cy[lane] = cc[1]; ws.cz[lane] = cc[2];
        ws.sx[lane] = o.size[0]; ws.sy[lane] = o.size[1]; ws.sz[lane] = o.size[2];
        ws.kind[lane] = o.kind;
    }
    __syncwarp();
    float* ring = a.sensors + size_t(i) * kFrames * kPixels;

    // ---- depth (sim_depth): only on sensor ticks
    if (steps % c.sensor_period == 0) {
        const uint32_t frame = (steps / c.sensor_period) % kFrames;
        const float ox = pos[0] + 0.0f * r[0], oy = pos[1] + 0.0f * r[3], oz = pos[2] + 0.0f * r[6];  // mount 0
        const float noise = clean_env(a, gid) ? 0.0f : c.depth_noise;
        const float dropout = clean_env(a, gid) ? 0.0f : c.dropout;
        // Visibility cull, one obstacle per lane: the obstacle's bounding sphere
        // (inflated by 0.01% + 1 mm, far above the float error of the exact
        // tests) must reach into the camera frustum |y| <= x, |z| <= 0.75 x
        // (a superset of every pixel ray, sensor_profile.hpp:81-85) and lie
        // nearer than the 12 m range cap. A culled obstacle cannot lower any
        // ray's minimum, so the ranges stay bit-identical to testing all.
        int ncand = 0;
        {
            bool visible = false;
            float qx = 0.0f, qy = 0.0f, qz = 0.0f, q2 = 0.0f, rbi = 0.0f;
            if (lane < int(count)) {
                const uint32_t kind = ws.kind[lane];
                const float e0 = ws.sx[lane], e1 = ws.sy[lane], e2 = ws.sz[lane];
                const float bound = kind == 0 ? sqrtf(e0 * e0 + e1 * e1 + e2 * e2)
                                  : (kind == 2 ? sqrtf(e0 * e0 + e2 * e2) : e0);
                rbi = bound * 1.0001f + 1e-3f;
                qx = ws.cx[lane] - ox;
                qy = ws.cy[lane] - oy;
                qz = ws.cz[lane] - oz;
                q2 = qx * qx + qy * qy + qz * qz;
                const float bx = r[0] * qx + r[3] * qy + r[6] * qz;  // body frame = R^T q
                const float by = r[1] * qx + r[4] * qy + r[7] * qz;
                const float bz = r[2] * qx + r[5] * qy + r[8] * qz;
                visible = (bx - by) * 0.70710678f >= -rbi && (bx + by) * 0.70710678f >= -rbi &&
                          (0.75f * bx - bz) * 0.8f >= -rbi && (0.75f * bx + bz) * 0.8f >= -rbi &&
                          sqrtf(q2) - rbi < 12.0f;
            }
            const unsigned vis = __ballot_sync(0xffffffffu, visible);
            if (visible) {
                const int slot = __popc(vis & ((1u << lane) - 1u));
                ws.cull[slot] = make_float4(qx, qy, qz, rbi);
                ws.cull2[slot] = make_float4(q2, rbi * rbi, __uint_as_float(ws.kind[lane]), 0.0f);
                ws.geom[slot] = make_float4(ws.cx[lane], ws.cy[lane], ws.cz[lane], ws.sx[lane]);
                ws.geom2[slot] = make_float4(ws.sy[lane], ws.sz[lane], 0.0f, 0.0f);
            }
            ncand = __popc(vis);
            __syncwarp();
        }
        // Tile cull: lanes 0-15 test candidate `lane` against tile u, lanes
        // 16-31 candidate `lane - 16` against tile u + 5. A candidate is kept
        // for a tile when its bounding sphere may meet the tile's ray cone:
        // the camera is inside the sphere, or the angle between the cone axis
        // and the centre is at most the cone half-angle plus the sphere's
        // angular radius (with 1 mm per metre of slack). A dropped candidate
        // cannot lower any of the tile's ranges, so they stay bit-identical.
        {
            const int jc = lane & 15;
            const bool live = jc < ncand;
            float4 cu = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            float qn = 0.0f, sb = 0.0f, cb = 1.0f;
            bool inside = false;
            if (live) {
                cu = ws.cull[jc];
                const float q2 = ws.cull2[jc].x;
                inside = q2 <= cu.w * cu.w;
                qn = sqrtf(q2);
                sb = inside ? 1.0f : cu.w / qn;
                cb = sqrtf(fmaxf(0.0f, 1.0f - sb * sb));
            }
#pragma unroll
            for (int u = 0; u < kPixels / 64; u++) {
                const int t = u + (lane >> 4) * (kPixels / 64);
                const float4 cone = __ldg(&g_tile_cone[t]);
                const float sa = __ldg(&g_tile_sin[t]);
                const float ax = r[0] * cone.x + r[1] * cone.y + r[2] * cone.z;
                const float ay = r[3] * cone.x + r[4] * cone.y + r[5] * cone.z;
                const float az = r[6] * cone.x + r[7] * cone.y + r[8] * cone.z;
                const float qa = cu.x * ax + cu.y * ay + cu.z * az;
                const bool keep = live && (inside || qa >= qn * (cone.w * cb - sa * sb) - 1e-3f * qn);
                const unsigned b = __ballot_sync(0xffffffffu, keep);
                if (lane == 0) {
                    ws.tile_mask[u] = b & 0xffffu;
                    ws.tile_mask[u + kPixels / 64] = b >> 16;
                }
            }
            __syncwarp();
        }
        const float rp[3] = {ox - a.room_c[0], oy - a.room_c[1], oz - a.room_c[2]};
        const float re[3] = {a.room_e[0], a.room_e[1], a.room_e[2]};
        const bool inside_room = fabsf(rp[0]) < re[0] && fabsf(rp[1]) < re[1] && fabsf(rp[2]) < re[2];
        // Each pass covers one 4-column x 8-row pixel tile (10 tiles = 20x16),
        // so a warp's rays are angular neighbours and share their culls.
        for (int tile = 0; tile < kPixels / 32; tile++) {
            const int col = (tile % 5) * 4 + (lane & 3), prow = (tile / 5) * 8 + (lane >> 2);
            const int k = prow * 20 + col;
            const float4 pr = __ldg(&g_pixel_ray[k]);
            const float rx = pr.x, ry = pr.y, rz = pr.z;
            const float dx = r[0] * rx + r[1] * ry + r[2] * rz;
            const float dy = r[3] * rx + r[4] * ry + r[5] * rz;
            const float dz = r[6] * rx + r[7] * ry + r[8] * rz;
            const float dd[3] = {dx, dy, dz};
            float rcp[3];
#pragma unroll
            for (int j = 0; j < 3; j++) rcp[j] = fabsf(dd[j]) < 1e-8f ? 0.0f : __frcp_rn(dd[j]);
            float best = 12.0f;
            if (inside_room) {
                // Origin strictly inside the room box: on every axis the two slab
                // distances have opposite signs, lo < 0, and ray_box returns
                // hi = min over axes of the non-negative one. Computing only that
                // division gives the same float as world.hpp:48-57.
                float hi = 1e20f;
#pragma unroll
                for (int j = 0; j < 3; j++)
                    if (!(fabsf(dd[j]) < 1e-8f))
                        hi = fminf(hi, div_by_rcp((dd[j] > 0.0f ? re[j] : -re[j]) - rp[j], dd[j], rcp[j]));
                best = fminf(best, hi);
            } else {
                best = fminf(best, ray_box_rcp(ox, oy, oz, dd, rcp, a.room_c[0], a.room_c[1], a.room_c[2],
                                               a.room_e[0], a.room_e[1], a.room_e[2]));
            }
            for (unsigned m = ws.tile_mask[tile]; m; m &= m - 1) {
                const int j = __ffs(m) - 1;
                // Per-ray bounding-sphere test: behind the camera, beyond the
                // current nearest hit, or passing outside the sphere -> the
                // exact test could only return a miss or a larger range.
                const float4 cu = ws.cull[j];
                const float tc = cu.x * dx + cu.y * dy + cu.z * dz;
                if (tc + cu.w < 0.0f || tc - cu.w >= best) continue;
                const float4 cu2 = ws.cull2[j];
                if (cu2.x - tc * tc > cu2.y) continue;
                const uint32_t kind = __float_as_uint(cu2.z);
                const float4 g = ws.geom[j];
                float t = 1000.0f;
                if (kind == 0) {
                    const float4 g2 = ws.geom2[j];
                    t = ray_box_rcp(ox, oy, oz, dd, rcp, g.x, g.y, g.z, g.w, g2.x, g2.y);
                } else if (kind == 1 || kind == 3) {
                    t = ray_sphere(ox, oy, oz, dx, dy, dz, g.x, g.y, g.z, g.w);
                } else if (kind == 2) {
                    t = ray_cylinder(ox, oy, oz, dx, dy, dz, g.x, g.y, g.z, g.w, ws.geom2[j].y);
                }
                best = fminf(best, t);
            }
            float depth = fmaxf(0.0f, best);
            if (noise != 0.0f || dropout != 0.0f) {
                uint32_t rng = run.rng + uint32_t(k) * 1664525u + steps * 1013904223u;
                depth = clampf(depth + noise * sim_normal(rng), 0.0f, 12.0f);
                if (wurand(rng) < dropout) depth = 12.0f;
            }
            ring[frame * kPixels + k] = depth;
        }
        float* pose = a.poses + (size_t(i) * kFrames + frame) * 12;
        if (lane < 3) pose[lane] = lane == 0 ? ox : (lane == 1 ? oy : oz);
        else if (lane < 12) pose[lane] = r[lane - 3];
        __syncwarp();
    }

    // ---- observation (sim_observe)
    const uint32_t delay = clean_env(a, gid) ? 0u : c.sensor_delay;
    const uint32_t available = steps / c.sensor_period;
    const uint32_t frame = available > delay ? available - delay : 0;
    const uint32_t prevf = frame > 0 ? frame - 1 : 0;
    const bool have = available >= delay;
    const size_t row = size_t(a.tick) * a.n + i;
    float* obs = a.obs + row * kActorObs;
    const float* cur_frame = ring + (frame % kFrames) * kPixels;
    const float* prev_frame = ring + (prevf % kFrames) * kPixels;
    for (int k = lane; k < 80; k += 32) {
        const int y = (k / 10) * 2, x = (k % 10) * 2;
        float cur = 12.0f, pre = 12.0f;
#pragma unroll
        for (int dy = 0; dy < 2; dy++)
#pragma unroll
            for (int dx = 0; dx < 2; dx++) {
                const int px = (y + dy) * 20 + x + dx;
                cur = smin(cur, cur_frame[px]);
                pre = smin(pre, prev_frame[px]);
            }
        const float oc = have ? cur / 12.0f : 1.0f;
        float op = have ? pre / 12.0f : 1.0f;
        if (c.mode == 18) op = oc;
        obs[k] = oc;
        obs[80 + k] = op;
        ws.cur[k] = oc * 12.0f;
        ws.prev[k] = op * 12.0f;
    }
    // Context features (every lane computes the shared scalars; lane j writes feature j).
    const float vel[3] = {st.linear_velocity[0], st.linear_velocity[1], st.linear_velocity[2]};
    const float delta[3] = {w.goal[0] - pos[0], w.goal[1] - pos[1], w.goal[2] - pos[2]};
    const float distance = smax(len3(delta[0], delta[1], delta[2]), 1.0e-6f);
    if (lane < 21) {
        float v;
        const int j = lane;
        if (j < 3) v = (r[j] * delta[0] + r[3 + j] * delta[1] + r[6 + j] * delta[2]) / distance;
        else if (j == 3) v = smin(distance / 10.0f, 1.5f);
        else if (j < 7) v = (r[j - 4] * vel[0] + r[3 + j - 4] * vel[1] + r[6 + j - 4] * vel[2]) / 4.0f;
        else if (j < 10) v = st.angular_velocity_body[j - 7] / 4.0f;
        else if (j < 13) v = r[6 + j - 10];
        else if (j < 17) v = run.previous_nav[j - 13];
        else if (j == 17) v = float(steps - frame * c.sensor_period) * a.physics->dt * float(c.substeps);
        else {
            const int k = j - 18;
            const float ref0 = run.reference_position[0] - pos[0], ref1 = run.reference_position[1] - pos[1],
                        ref2 = run.reference_position[2] - pos[2];
            v = clampf((r[k] * ref0 + r[3 + k] * ref1 + r[6 + k] * ref2) * 2.0f, -1.0f, 1.0f);
        }
        obs[160 + j] = v;
        ws.ctx[j] = v;
    }
    __syncwarp();
    // Geometry-prior hint, nav_guidance (guidance.hpp:39-90), 80 cells over the lanes.
    {
        const float g0 = ws.ctx[0], g1 = ws.ctx[1], g2 = ws.ctx[2];
        const float gvel[3] = {ws.ctx[4] * 4.0f, ws.ctx[5] * 4.0f, ws.ctx[6] * 4.0f};
        const float sensor_dt = float(c.sensor_period) * a.physics->dt * float(c.substeps);
        const float gnorm = sqrtf(g0 * g0 + g1 * g1 + g2 * g2);
        float hint[3] = {0, 0, 0};
        if (!(gnorm < 1e-6f || distance < 0.05f)) {
            const float goal[3] = {g0 / gnorm, g1 / gnorm, g2 / gnorm};
            const float speed = sqrtf(gvel[0] * gvel[0] + gvel[1] * gvel[1] + gvel[2] * gvel[2]);
            const float stop_margin = 0.28f + speed * fmaxf(sensor_dt, 0.0f) + 0.25f * speed * speed;
            float best_score = -1e20f, goal_dot = -1e20f;
            int best_cell = 1 << 20, goal_cell = 1 << 20;
            float best_range_lane = 0.0f;
            for (int k = lane; k < 80; k += 32) ws.risk_term[k] = neighbour_risk(ws, k, gvel, sensor_dt);
            __syncwarp();
            for (int k = lane; k < 80; k += 32) {
                const int row_ = k / 10, col = k % 10;
                const float d[3] = {c_pool_ray_at(3 * k), c_pool_ray_at(3 * k + 1), c_pool_ray_at(3 * k + 2)};
                const float alignment = d[0] * goal[0] + d[1] * goal[1] + d[2] * goal[2];
                const float nearby = pooled_min3x3(ws.cur, row_, col);
                const float risk = cell_risk(ws, row_, col, sensor_dt);
                const float safe_range = fmaxf(nearby - risk, 0.0f);
                const float score = 1.4f * alignment + 0.12f * fminf(safe_range, 6.0f);
                if (score > best_score) {
                    best_score = score;
                    best_cell = k;
                    best_range_lane = safe_range;
                }
                if (alignment > goal_dot) {
                    goal_dot = alignment;
                    goal_cell = k;
                }
            }
            const int my_best = best_cell;
            warp_argmax_first(best_score, best_cell);
            warp_argmax_first(goal_dot, goal_cell);
            // the lane that owns the winning cell holds its safe range
            const int owner = best_cell < 80 ? (best_cell & 31) : 0;
            const float best_range = best_cell < 80 ? __shfl_sync(0xffffffffu, best_range_lane, owner) : 0.0f;
            (void)my_best;
            float best_dir[3] = {1, 0, 0};
            if (best_cell < 80) {
                best_dir[0] = c_pool_ray_at(3 * best_cell);
                best_dir[1] = c_pool_ray_at(3 * best_cell + 1);
                best_dir[2] = c_pool_ray_at(3 * best_cell + 2);
            }
            const int grow = goal_cell < 80 ? goal_cell / 10 : 0, gcol = goal_cell < 80 ? goal_cell % 10 : 0;
            const float desired_speed = fminf(1.6f, sqrtf(4.0f * fmaxf(distance - 0.28f, 0.0f)));
            const float direct_range = fmaxf(pooled_min3x3(ws.cur, grow, gcol), 0.0f);
            float dir[3] = {best_dir[0], best_dir[1], best_dir[2]}, available_range = best_range;
            if (goal[0] > 0.0f && direct_range > stop_margin + 0.25f * desired_speed * desired_speed) {
                dir[0] = goal[0]; dir[1] = goal[1]; dir[2] = goal[2];
                available_range = direct_range;
            }
            const float after_stop = fmaxf(available_range - stop_margin - 0.15f, 0.0f);
            const float command_speed = fminf(desired_speed, sqrtf(4.0f * after_stop));
            const float fraction = fminf(0.8f, command_speed * 0.5f);
            if (direct_range < 1.2f && available_range > direct_range + 0.25f) {
                const float advance = fmaxf(0.05f, fminf(1.0f, (direct_range - 0.25f) / 0.95f));
                dir[0] *= advance;
                const float norm = sqrtf(dir[0] * dir[0] + dir[1] * dir[1] + dir[2] * dir[2]);
                for (int j = 0; j < 3; j++) dir[j] /= fmaxf(norm, 1e-6f);
            }
            for (int j = 0; j < 3; j++) {
                const float x = fraction * dir[j];
                hint[j] = 0.5f * logf((1.0f + x) / (1.0f - x));  // guidance.hpp:35
            }
        }
        if (lane < 3) obs[181 + lane] = hint[lane];
    }
    // Critic observation (sim_critic_obs, sim.metal:159-165): clearance over lanes.
    {
        float cand = 3.0e38f;
        if (lane < int(count)) {
            const float size[3] = {ws.sx[lane], ws.sy[lane], ws.sz[lane]};
            cand = obstacle_clearance(ws.kind[lane], size, pos[0] - ws.cx[lane], pos[1] - ws.cy[lane], pos[2] - ws.cz[lane]);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) cand = fminf(cand, __shfl_xor_sync(0xffffffffu, cand, off));
        const float clearance = count ? fminf(room_clearance(a, pos), cand) : room_clearance(a, pos);
        float* co = a.co + row * a.co_dim;
        float v = 0.0f;
        const int j = lane;
        if (j < 3) v = (w.goal[j] - pos[j]) / 10.0f;
        else if (j < 6) v = vel[j - 3] / 4.0f;
        else if (j < 9) v = st.angular_velocity_body[j - 6] / 4.0f;
        else if (j < 13) v = q[j - 9];
        else if (j < 16) v = pos[j - 13] / 10.0f;
        else if (j < 19) v = (run.reference_position[j - 16] - pos[j - 16]) * 2.0f;
        else if (j == 19) v = clearance / 5.0f;
        else if (j == 20) v = float(steps) / 200.0f;
        else if (j < 30) {
            const int o = (j - 21) / 3, axis = (j - 21) % 3;
            if (o < int(count < 3u ? count : 3u)) {
                const float cc = axis == 0 ? ws.cx[o] : (axis == 1 ? ws.cy[o] : ws.cz[o]);
                v = (cc - pos[axis]) / 10.0f;
            }
        } else if (j == 30) v = w.wind[0];
        else v = w.wind[1];
        co[j] = v;  // inputs 32..63 of the control-state critic: k_control_state
    }
}

// Inputs 32..63 of the control-state critic's observation (sim.metal:166-180),
// one warp per environment, lane j writing input 32 + j, from the state in
// device memory. Launched after the sensing kernels into this step's critic
// observation rows (the state sim_observe sees), and after k_advance into
// next_co_full, whose first 32 inputs it copies from the rows k_advance left
// in next_co (the post-step state of the bootstrap value, sim.metal:327): the
// episode resets of the step run later in both cases. Environments the
// sensing skips in evaluation mode are skipped here too.
constexpr int kControlWarps = 8;
__global__ void __launch_bounds__(kControlWarps * 32) k_control_state(SimArgs a, int post_step) {
    const int lane = threadIdx.x & 31;
    const uint32_t i = blockIdx.x * kControlWarps + (threadIdx.x >> 5);
    if (i >= a.n) return;  // warp-uniform
    const mdn_sim_run& run = a.runs[i];
    if (!post_step && a.cfg.eval && run.episodes) return;
    const mdn_physics_state& st = a.states[i];
    const float q[4] = {st.orientation_wxyz[0], st.orientation_wxyz[1], st.orientation_wxyz[2], st.orientation_wxyz[3]};
    const float pos[3] = {st.position[0], st.position[1], st.position[2]};
    const float vel[3] = {st.linear_velocity[0], st.linear_velocity[1], st.linear_velocity[2]};
    float* row = post_step ? a.next_co_full + size_t(i) * a.co_dim : a.co + (size_t(a.tick) * a.n + i) * a.co_dim;
    if (post_step) row[lane] = a.next_co[size_t(i) * kCriticObs + lane];
    row[kCriticObs + lane] = control_state_input(lane, run.hidden, st.rpm, q, pos, vel, run.desired_velocity, run,
                                                 a.worlds[i]);
}

// One policy step's sensing, one warp per environment. Environments whose
// episode ended in the previous step of a collected rollout (reset_pending)
// are left to k_reset_sense, which runs beside this kernel.
__global__ void __launch_bounds__(kSenseWarps * 32, 4) k_sense(SimArgs a) {
    __shared__ WarpScene scenes[kSenseWarps];
    if (blockIdx.x == 0 && threadIdx.x == 0) a.reset_count[a.phase] = 0;  // this step's reset list starts empty
    const int wid = threadIdx.x >> 5;
    const uint32_t i = blockIdx.x * kSenseWarps + wid;
    if (i >= a.n || a.reset_pending[i]) return;  // warp-uniform
    sense_env(a, i, scenes[wid]);
}

// A warp's shared memory in k_reset_sense: the world that an episode reset
// generates, then the scene of the environment it senses.
union SenseSmem {
    WarpScene scene;
    mdn_world world;
};

// The episode resets of the previous step of a collected rollout (sim.metal:330,
// schedule slot = this tick), each followed by that environment's sensing:
// one warp per environment that k_advance listed. Launched on a forked branch
// of the rollout graph beside k_sense (which skips these environments), with
// a higher priority, so that the long world generations overlap the other
// environments' sensing instead of running as a kernel of their own between
// the advance and the next sense. A reset and the sensing after it are the
// same per-environment computations as k_reset_list + k_sense, so the results
// are unchanged.
__global__ void __launch_bounds__(kSenseWarps * 32) k_reset_sense(SimArgs a) {
    __shared__ SenseSmem smem[kSenseWarps];
    const int wid = threadIdx.x >> 5;
    const uint32_t listed = a.reset_count[a.phase ^ 1u];
    const uint32_t count = listed < a.n ? listed : a.n;
    for (uint32_t k = blockIdx.x * kSenseWarps + wid; k < count; k += gridDim.x * kSenseWarps) {
        const uint32_t i = a.reset_list[k];
        // An entry whose flag is clear was reset already (a list that a
        // k_reset_list flush consumed).
        if (i >= a.n || !a.reset_pending[i]) continue;
        episode_reset(a, i, false, a.tick, smem[wid].world);
        refill_ring_warp(a, i);
        __syncwarp();
        sense_env(a, i, smem[wid].scene);
        __syncwarp();
    }
}

// ------------------------------------------------------- geometry memory
// Memory-guided geometry prior (sim.metal:216-218 with geometry_memory = 1;
// nav_guidance_memory, guidance.hpp:106-194), one warp per environment, run
// after k_sense has written the pooled ranges and the context features. The
// up to 8 x 80 remembered obstacle points (each pooled cell's nearest pixel
// in an older range frame, moved into the current body frame through the
// pose ring) are built once into shared memory; lanes then own the 85
// candidate directions and sweep every point. Only fminf/fmaxf combine the
// points, so the split over lanes keeps the reference's values exactly.
constexpr int kMemWarps = 4;
constexpr int kMemPoints = kFrames * 80;

struct MemScene {
    float px[kMemPoints], py[kMemPoints], pz[kMemPoints], pr2[kMemPoints];  // point, |point|^2
    float rad[kMemPoints], rad2[kMemPoints];                                  // memory radius and its square
    float cur[80], prev[80], risk_term[80];
};

__global__ void __launch_bounds__(kMemWarps * 32) k_memory_hint(SimArgs a) {
    extern __shared__ float mem_sm[];
    MemScene& ms = reinterpret_cast<MemScene*>(mem_sm)[threadIdx.x >> 5];
    const int lane = threadIdx.x & 31;
    const uint32_t i = blockIdx.x * kMemWarps + (threadIdx.x >> 5);
    if (i >= a.n) return;
    const mdn_sim_config& c = a.cfg;
    const mdn_sim_run& run = a.runs[i];
    if (c.eval && run.episodes) return;
    const uint32_t steps = run.steps, gid = a.env_base + i;
    const mdn_physics_state& st = a.states[i];
    const mdn_world& w = a.worlds[i];
    const float pos[3] = {st.position[0], st.position[1], st.position[2]};
    const float q[4] = {st.orientation_wxyz[0], st.orientation_wxyz[1], st.orientation_wxyz[2], st.orientation_wxyz[3]};
    float r[9];
    rotation(q, r);
    const size_t row = size_t(a.tick) * a.n + i;
    float* obs = a.obs + row * kActorObs;
    const uint32_t delay = clean_env(a, gid) ? 0u : c.sensor_delay;
    const uint32_t available = steps / c.sensor_period;
    const uint32_t frame = available > delay ? available - delay : 0;
    const uint32_t valid = available >= delay ? min(frame + 1u, uint32_t(kFrames) - delay) : 0u;
    const float sensor_dt = float(c.sensor_period) * a.physics->dt * float(c.substeps);
    const float tan_v = 0.75f;
    const float gvel[3] = {obs[164] * 4.0f, obs[165] * 4.0f, obs[166] * 4.0f};
    for (int k = lane; k < 80; k += 32) {
        ms.cur[k] = obs[k] * 12.0f;
        ms.prev[k] = obs[80 + k] * 12.0f;
    }
    __syncwarp();
    for (int k = lane; k < 80; k += 32) {
        const float old = ms.prev[k], now = ms.cur[k];
        float term = 0.0f;
        if (old < 11.9f && now < 11.9f) {
            const float unexpected = (old - now) / fmaxf(sensor_dt, 1e-3f) -
                                     (gvel[0] * c_pool_ray_at(3 * k) + gvel[1] * c_pool_ray_at(3 * k + 1) +
                                      gvel[2] * c_pool_ray_at(3 * k + 2));
            if (unexpected > 0.5f) term = fminf(0.20f * unexpected, 1.0f);
        }
        ms.risk_term[k] = term;
    }
    // remembered points, compacted (nav_memory_clearance's loops, :106-140)
    const float* ring = a.sensors + size_t(i) * kFrames * kPixels;
    const float* poses = a.poses + size_t(i) * kFrames * 12;
    const float cur_pose[12] = {pos[0], pos[1], pos[2], r[0], r[1], r[2], r[3], r[4], r[5], r[6], r[7], r[8]};
    int npoints = 0;
    for (int base = 0; base < int(valid) * 80; base += 32) {
        const int p = base + lane;
        bool keep = false;
        float x = 0, y = 0, z = 0, radius = 0;
        if (p < int(valid) * 80) {
            const uint32_t back = uint32_t(p / 80), cell = uint32_t(p % 80);
            const uint32_t f = (frame + 8u - back) % 8u;
            const float* old_pose = poses + f * 12;
            const float* ranges = ring + f * kPixels;
            const float age = float(back) * fmaxf(sensor_dt, 0.0f);
            const uint32_t px = (cell / 10u) * 2u * 20u + (cell % 10u) * 2u;
            uint32_t hit = px;
            float range = ranges[px];
            const uint32_t others[3] = {px + 1u, px + 20u, px + 21u};
            for (int j = 0; j < 3; j++)
                if (ranges[others[j]] < range) {
                    range = ranges[others[j]];
                    hit = others[j];
                }
            if (!(range <= 0.01f || range >= 11.9f)) {
                keep = true;
                const float ry = 1.0f - (float(hit % 20u) + 0.5f) / 10.0f;
                const float rz = tan_v * (1.0f - (float(hit / 20u) + 0.5f) / 8.0f);
                const float inv = 1.0f / sqrtf(1.0f + ry * ry + rz * rz);
                const float ray[3] = {inv, ry * inv, rz * inv};
                const float wx = old_pose[3] * ray[0] + old_pose[4] * ray[1] + old_pose[5] * ray[2];
                const float wy = old_pose[6] * ray[0] + old_pose[7] * ray[1] + old_pose[8] * ray[2];
                const float wz = old_pose[9] * ray[0] + old_pose[10] * ray[1] + old_pose[11] * ray[2];
                const float dx = old_pose[0] + range * wx - cur_pose[0];
                const float dy = old_pose[1] + range * wy - cur_pose[1];
                const float dz = old_pose[2] + range * wz - cur_pose[2];
                x = cur_pose[3] * dx + cur_pose[6] * dy + cur_pose[9] * dz;
                y = cur_pose[4] * dx + cur_pose[7] * dy + cur_pose[10] * dz;
                z = cur_pose[5] * dx + cur_pose[8] * dy + cur_pose[11] * dz;
                radius = 0.20f + 0.015f * range + 0.15f * age;  // memory_point_radius, :96-100
            }
        }
        const unsigned kept = __ballot_sync(0xffffffffu, keep);
        if (keep) {
            const int slot = npoints + __popc(kept & ((1u << lane) - 1u));
            ms.px[slot] = x;
            ms.py[slot] = y;
            ms.pz[slot] = z;
            ms.pr2[slot] = x * x + y * y + z * z;
            ms.rad[slot] = radius;
            ms.rad2[slot] = radius * radius;
        }
        npoints += __popc(kept);
    }
    __syncwarp();
    const float delta[3] = {w.goal[0] - pos[0], w.goal[1] - pos[1], w.goal[2] - pos[2]};
    const float distance = smax(len3(delta[0], delta[1], delta[2]), 1.0e-6f);
    const float g0 = obs[160], g1 = obs[161], g2 = obs[162];
    const float gnorm = sqrtf(g0 * g0 + g1 * g1 + g2 * g2);
    float hint[3] = {0, 0, 0};
    if (!(gnorm < 1e-6f || distance < 0.05f)) {
        const float goal[3] = {g0 / gnorm, g1 / gnorm, g2 / gnorm};
        const float speed = sqrtf(gvel[0] * gvel[0] + gvel[1] * gvel[1] + gvel[2] * gvel[2]);
        const float stop_margin = 0.28f + speed * fmaxf(sensor_dt, 0.0f) + 0.25f * speed * speed;
        float goal_dot = -1e20f;
        int goal_cell = 1 << 20;
        for (int k = lane; k < 80; k += 32) {
            const float al = c_pool_ray_at(3 * k) * goal[0] + c_pool_ray_at(3 * k + 1) * goal[1] +
                             c_pool_ray_at(3 * k + 2) * goal[2];
            if (al > goal_dot) {
                goal_dot = al;
                goal_cell = k;
            }
        }
        warp_argmax_first(goal_dot, goal_cell);
        const int grow = goal_cell < 80 ? goal_cell / 10 : 0, gcol = goal_cell < 80 ? goal_cell % 10 : 0;
        const float desired_speed = fminf(1.6f, sqrtf(4.0f * fmaxf(distance - 0.28f, 0.0f)));
        const float required = stop_margin + 0.15f + desired_speed * desired_speed * 0.25f;
        float best_score = -1e20f, best_free = 0.0f;
        int best = 1 << 20;
        for (int cand = lane; cand < 85; cand += 32) {
            float d[3];
            int crow = grow, ccol = gcol;
            if (cand < 80) {
                crow = cand / 10;
                ccol = cand % 10;
                d[0] = c_pool_ray_at(3 * cand);
                d[1] = c_pool_ray_at(3 * cand + 1);
                d[2] = c_pool_ray_at(3 * cand + 2);
            } else if (cand == 80) {
                d[0] = goal[0]; d[1] = goal[1]; d[2] = goal[2];
            } else {
                d[0] = 0.0f;
                d[1] = cand >= 83 ? (cand == 83 ? 1.0f : -1.0f) : 0.0f;
                d[2] = cand < 83 ? (cand == 81 ? 1.0f : -1.0f) : 0.0f;
            }
            float sweep[3] = {1.2f * d[0] + 0.35f * gvel[0], 1.2f * d[1] + 0.35f * gvel[1], 1.2f * d[2] + 0.35f * gvel[2]};
            const float sweep_norm = sqrtf(sweep[0] * sweep[0] + sweep[1] * sweep[1] + sweep[2] * sweep[2]);
            for (int j = 0; j < 3; j++) sweep[j] /= fmaxf(sweep_norm, 1e-6f);
            float nearest = 3.0f;
            for (int p = 0; p < npoints; p++) {
                const float along = ms.px[p] * sweep[0] + ms.py[p] * sweep[1] + ms.pz[p] * sweep[2];
                if (along <= 0.0f || along > 3.0f + ms.rad[p]) continue;
                const float lateral2 = fmaxf(ms.pr2[p] - along * along, 0.0f);
                const float radius2 = ms.rad2[p];
                if (lateral2 < radius2) nearest = fminf(nearest, fmaxf(along - sqrtf(radius2 - lateral2), 0.0f));
            }
            float free_ = nearest;
            if (cand < 81) free_ = fminf(free_, pooled_min3x3(ms.cur, crow, ccol));
            float risk = 0.0f;
            if (sensor_dt > 1e-4f)
                for (int dr = -1; dr <= 1; dr++)
                    for (int dc = -1; dc <= 1; dc++) {
                        const int rr = crow + dr, cc = ccol + dc;
                        if (rr < 0 || rr >= 8 || cc < 0 || cc >= 10) continue;
                        risk = fmaxf(risk, ms.risk_term[rr * 10 + cc]);
                    }
            free_ = fmaxf(free_ - risk, 0.0f);
            const float alignment = d[0] * goal[0] + d[1] * goal[1] + d[2] * goal[2];
            const float score = 1.4f * alignment + 0.20f * fminf(free_, 3.0f) -
                                (free_ < required ? 3.0f * (required - free_) / required : 0.0f);
            if (score > best_score) {
                best_score = score;
                best_free = free_;
                best = cand;
            }
        }
        const float lane_free = best_free;
        const int lane_best = best;
        warp_argmax_first(best_score, best);
        const unsigned owner_mask = __ballot_sync(0xffffffffu, lane_best == best);
        const float chosen_free = __shfl_sync(0xffffffffu, lane_free, owner_mask ? __ffs(owner_mask) - 1 : 0);
        float dir[3] = {1.0f, 0.0f, 0.0f};
        if (best < 80) {
            dir[0] = c_pool_ray_at(3 * best);
            dir[1] = c_pool_ray_at(3 * best + 1);
            dir[2] = c_pool_ray_at(3 * best + 2);
        } else if (best == 80) {
            dir[0] = goal[0]; dir[1] = goal[1]; dir[2] = goal[2];
        } else if (best < 85) {
            dir[0] = 0.0f;
            dir[1] = best >= 83 ? (best == 83 ? 1.0f : -1.0f) : 0.0f;
            dir[2] = best < 83 ? (best == 81 ? 1.0f : -1.0f) : 0.0f;
        }
        const float chosen = best < 85 ? chosen_free : 0.0f;
        const bool goal_in_fov = goal[0] > 0.0f && fabsf(goal[1]) <= goal[0] && fabsf(goal[2]) <= tan_v * goal[0];
        const float after_stop = fmaxf(chosen - stop_margin - 0.15f, 0.0f);
        float command_speed = fminf(desired_speed, sqrtf(4.0f * after_stop));
        if (!goal_in_fov) command_speed = fminf(command_speed, 0.25f);
        const float fraction = fminf(0.8f, command_speed * 0.5f);
        for (int j = 0; j < 3; j++) {
            const float x = fraction * dir[j];
            hint[j] = 0.5f * logf((1.0f + x) / (1.0f - x));  // guidance.hpp:35
        }
    }
    if (lane < 3) obs[181 + lane] = hint[lane];
}

// -------------------------------------------------------------------- act
// Actor mean (tanh MLP 184->64->4 plus geometry prior, ppo.hpp:65-80), critic
// value (32->64->1, ppo.hpp:82-93), Gaussian sample, log-prob, command ring,
// command delay and desired velocity (sim.metal:229-271). A warp handles four
// environments per pass: lanes own hidden units (lane, lane+32), so every
// weight loaded from shared memory feeds four environments; lanes 0-3 then
// sample the four environments' actions in parallel. The CTA keeps W1 in
// shared memory as rows padded to 185 words, so lane h reading row h and the
// row-order fill from global memory are both free of bank conflicts, and loops
// over the environments.
constexpr int kActWarps = 8;
constexpr int kActEnvs = 4;
constexpr int kActW1Pitch = kActorObs + 1;   // padded rows: lane h reads row h, bank (25 h + k) % 32
constexpr int kActCw1Pitch = kCriticObs + 1;
constexpr int kActSmemFloats = kHidden * kActW1Pitch + kHidden + kActions * kHidden + 2 * kActions +
                               kHidden * kActCw1Pitch + kHidden + kHidden + 1 +
                               kActWarps * kActEnvs * (kActorObs + kCriticObs);

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// Share of the 20 overhead cells whose range exceeds 2.5 m, mapped to the
// mode-17 blend scale .25 + .75 * share (sim.metal:233, 235-240).
__device__ __forceinline__ float overhead_scale(const float* ob) {
    float overhead = 0.0f;
    for (int k = 0; k < 20; k++) overhead += ob[k] * 12.0f > 2.5f ? 1.0f : 0.0f;
    return 0.25f + 0.75f * (overhead / 20.0f);
}

// The rest of sim_act for env i at `row` once its actor mean and critic value
// are known (sim.metal:229-271): mode blends, sampling, log-prob, command ring
// and delay, desired velocity and yaw. `ob` is the env's observation row.
__device__ __forceinline__ void act_finish_body(const SimArgs& a, uint32_t i, size_t row, const float* ob,
                                                const float* mean_in, float value, const float* log_std) {
    const mdn_sim_config& c = a.cfg;
    mdn_sim_run& run = a.runs[i];
    a.values[row] = value;
    const float* prior = ob + kActorObs - 3;
    const uint32_t mode = c.mode;
    float mean[4] = {mean_in[0], mean_in[1], mean_in[2], mean_in[3]};
    // Geometry-prior blends of the evaluation modes 9-21 (sim.metal:233).
    if (mode >= 9u && mode <= 21u) {
        float scale = (mode == 9u || mode == 13u) ? 0.0f
                    : ((mode == 10u || mode == 14u || mode == 16u) ? 0.25f : (mode == 15u ? 1.0f : 0.5f));
        if (mode >= 17u) scale = overhead_scale(ob);
        if (mode == 12u) {
            float near_ = 12.0f;
            for (int k = 0; k < 80; k++) near_ = smin(near_, ob[k] * 12.0f);
            scale = clampf((near_ - 0.3f) / 2.0f, 0.2f, 1.0f);
        }
        for (int j = 0; j < 3; j++) mean[j] = prior[j] + scale * (mean[j] - prior[j]);
        mean[3] *= scale;
        if (mode == 16u) {
            const float yaw = atan2f(ob[161], ob[160]);
            const float x = clampf(yaw * 1.5f, -0.85f, 0.85f);
            mean[3] += 0.5f * logf((1.0f + x) / (1.0f - x));  // nav_atanh, guidance.hpp:35
        }
    }
    // Mode 22 trains the deployed mode-17 action map (sim.metal:235-256).
    const float deployed = mode == 22u ? overhead_scale(ob) : 1.0f;
    uint32_t rng = run.rng;
    const uint32_t steps = run.steps;
    float act[4];
    float* cmd = a.commands + size_t(i) * kFrames * kActions;
    for (int j = 0; j < 4; j++) {
        act[j] = mean[j] + ((mode == 0u || mode == 22u) ? expf(log_std[j]) * sim_normal(rng) : 0.0f);
        if (mode == 1u) act[j] = sim_normal(rng);
        a.actions[row * kActions + j] = act[j];
        float executed = act[j];
        if (mode == 22u) executed = j < 3 ? prior[j] + deployed * (act[j] - prior[j]) : deployed * act[j];
        cmd[(steps % kFrames) * kActions + j] = tanhf(executed);
    }
    float lp = 0.0f;  // gaussian_log_prob, ppo.hpp:95-103
    for (int j = 0; j < 4; j++) {
        const float inv_std = expf(-log_std[j]);
        const float d = (act[j] - mean[j]) * inv_std;
        lp += -0.5f * (d * d + 2.0f * log_std[j] + kLogTwoPi);
    }
    a.logp[row] = lp;
    run.rng = rng;
    const mdn_physics_state& st = a.states[i];
    const float q[4] = {st.orientation_wxyz[0], st.orientation_wxyz[1], st.orientation_wxyz[2],
                        st.orientation_wxyz[3]};
    float r[9];
    rotation(q, r);
    if (mode == 2u || mode == 3u || mode == 20u) {  // scripted goal pursuit, sim.metal:257-263
        const mdn_world& w = a.worlds[i];
        float d[3] = {w.goal[0] - st.position[0], w.goal[1] - st.position[1], w.goal[2] - st.position[2]};
        const float len = len3(d[0], d[1], d[2]);
        const float inv = 1.0f / len, keep = smin(len, c.speed);
        for (int j = 0; j < 3; j++) d[j] = d[j] * inv * keep;
        float* slot = cmd + (steps % kFrames) * kActions;
        slot[0] = (r[0] * d[0] + r[3] * d[1] + r[6] * d[2]) / c.speed;
        slot[1] = (r[1] * d[0] + r[4] * d[1] + r[7] * d[2]) / c.speed;
        slot[2] = (r[2] * d[0] + r[5] * d[1] + r[8] * d[2]) / c.speed;
        slot[3] = 0.0f;
    }
    const uint32_t gid = a.env_base + i;
    const uint32_t delay = clean_env(a, gid) ? 0u : c.command_delay;
    const uint32_t applied = steps > delay ? steps - delay : 0;
    float pn[4];
    for (int j = 0; j < 4; j++) {
        pn[j] = steps < delay ? 0.0f : cmd[(applied % kFrames) * kActions + j];
        run.previous_nav[j] = pn[j];
    }
    float v[3] = {pn[0] * c.speed, pn[1] * c.speed, pn[2] * c.speed * (c.velocity_contract == 0 ? 0.5f : 1.0f)};
    if (c.velocity_contract == 1) {
        const float scale = smin(1.0f, c.speed / smax(len3(v[0], v[1], v[2]), 1e-8f));
        for (int j = 0; j < 3; j++) v[j] *= scale;
    }
    if (mode == 19u) {  // fixed-speed command, sim.metal:269
        const float magnitude = len3(v[0], v[1], v[2]);
        if (magnitude > 1e-8f) {
            const float scale = c.speed / magnitude;
            for (int j = 0; j < 3; j++) v[j] *= scale;
        }
    }
    for (int j = 0; j < 3; j++) run.desired_velocity[j] = r[j * 3] * v[0] + r[j * 3 + 1] * v[1] + r[j * 3 + 2] * v[2];
    run.yaw += pn[3] * a.physics->dt * float(c.substeps) * 0.5f;
}

// Out of line for the thread-per-environment actor, whose 128 registers are
// better spent on the dot products; the quad actor inlines the body (8,192
// envs: 0.037 vs 0.039 ms).
__device__ __noinline__ void act_finish(const SimArgs& a, uint32_t i, size_t row, const float* ob,
                                        const float* mean_in, float value, const float* log_std) {
    act_finish_body(a, i, row, ob, mean_in, value, log_std);
}

// The 64-unit actor and the critic with one thread per environment: every
// thread keeps its environment's 64 pre-activations in registers and the warp
// reads one broadcast 128-bit word of W1 (4 inputs of one unit) per 4 FMAs.
// Pre-activations are in-order fmaf chains from zero, then the bias; the heads
// sum the hidden units in order (cpu_reference.hpp:437-458).
constexpr int kRowThreads = 256;
constexpr int kW1Pitch = kActorObs + 4;    // padded W1 rows: 16-byte aligned, rows 1..3 apart on other banks
constexpr int kCw1Pitch = kCriticObs + 4;
constexpr int kRowSmemFloats = kHidden * kW1Pitch + kHidden * kCw1Pitch + kHidden + kActions * kHidden + kHidden +
                               kHidden + 4 + 4 + 4;

// The 64-unit actor's and the critic's weights in shared memory, W1 in its
// own row-major layout (unit h's inputs at w1[h * kW1Pitch + k]): the fill is
// a straight, coalesced 128-bit copy, and a thread reads 4 inputs of one unit
// per 128-bit word (a broadcast when the warp's threads share the unit).
struct ActSmem {
    float *w1, *cw1, *b1, *w2, *cb1, *cw2, *b2, *log_std, *cb2;
};
__device__ __forceinline__ ActSmem act_weights_fill(const SimArgs& a, float* base) {
    ActSmem m;
    m.w1 = base;                               // [64][188]
    m.cw1 = m.w1 + kHidden * kW1Pitch;         // [64][36]
    m.b1 = m.cw1 + kHidden * kCw1Pitch;        // [64]
    m.w2 = m.b1 + kHidden;                     // [4][64]
    m.cb1 = m.w2 + kActions * kHidden;         // [64]
    m.cw2 = m.cb1 + kHidden;                   // [64]
    m.b2 = m.cw2 + kHidden;                    // [4]
    m.log_std = m.b2 + 4;                      // [4]
    m.cb2 = m.log_std + 4;                     // [1]
    const int tid = threadIdx.x;
    const float4* actor4 = reinterpret_cast<const float4*>(a.actor);
    const float4* critic4 = reinterpret_cast<const float4*>(a.critic);
    for (int k = tid; k < kHidden * (kActorObs / 4); k += blockDim.x) {
        const int h = k / (kActorObs / 4), c4 = k % (kActorObs / 4);
        *reinterpret_cast<float4*>(m.w1 + h * kW1Pitch + 4 * c4) = __ldg(actor4 + k);
    }
    for (int k = tid; k < kHidden * (kCriticObs / 4); k += blockDim.x) {
        const int h = k / (kCriticObs / 4), c4 = k % (kCriticObs / 4);
        *reinterpret_cast<float4*>(m.cw1 + h * kCw1Pitch + 4 * c4) = __ldg(critic4 + k);
    }
    for (int k = tid; k < kHidden; k += blockDim.x) {
        m.b1[k] = a.actor[kActorB1 + k];
        m.cb1[k] = a.critic[kCriticB1 + k];
        m.cw2[k] = a.critic[kCriticW2 + k];
    }
    for (int k = tid; k < kActions * kHidden; k += blockDim.x) m.w2[k] = a.actor[kActorW2 + k];
    if (tid < kActions) {
        m.b2[tid] = a.actor[a.actor_b2 + tid];
        m.log_std[tid] = a.actor[a.actor_log_std + tid];
    }
    if (tid == 0) m.cb2[0] = a.critic[kCriticB2];
    __syncthreads();
    return m;
}

__global__ void __launch_bounds__(kRowThreads, 2) k_act_rows(SimArgs a) {
    extern __shared__ float4 smem4[];
    const ActSmem m = act_weights_fill(a, reinterpret_cast<float*>(smem4));
    const float *w1 = m.w1, *cw1 = m.cw1, *b1 = m.b1, *w2 = m.w2, *cb1 = m.cb1, *cw2 = m.cw2, *b2 = m.b2,
                *log_std = m.log_std, *cb2 = m.cb2;
    const int tid = threadIdx.x;
    const mdn_sim_config& c = a.cfg;
    for (uint32_t i = blockIdx.x * blockDim.x + tid; i < a.n; i += gridDim.x * blockDim.x) {
        if (c.eval && a.runs[i].episodes) continue;
        const size_t row = size_t(a.tick) * a.n + i;
        const float* ob = a.obs + row * kActorObs;
        float z[kHidden];
#pragma unroll
        for (int h = 0; h < kHidden; h++) z[h] = 0.0f;
        const float4* ob4 = reinterpret_cast<const float4*>(ob);
#pragma unroll 1
        for (int k4 = 0; k4 < kActorObs / 4; k4++) {
            const float4 o4 = __ldg(ob4 + k4);
#pragma unroll
            for (int h = 0; h < kHidden; h++) {  // inputs 4k4..4k4+3 of unit h, in order
                const float4 w = *reinterpret_cast<const float4*>(w1 + h * kW1Pitch + 4 * k4);
                z[h] = fmaf(o4.x, w.x, z[h]);
                z[h] = fmaf(o4.y, w.y, z[h]);
                z[h] = fmaf(o4.z, w.z, z[h]);
                z[h] = fmaf(o4.w, w.w, z[h]);
            }
        }
#pragma unroll
        for (int h = 0; h < kHidden; h++) z[h] = tanhf(z[h] + b1[h]);
        float mean[4];
#pragma unroll
        for (int j = 0; j < kActions; j++) {
            float m = 0.0f;
#pragma unroll
            for (int h = 0; h < kHidden; h++) m = fmaf(z[h], w2[j * kHidden + h], m);
            mean[j] = m + b2[j];
        }
        const float4 pr = make_float4(__ldg(ob + kActorObs - 3), __ldg(ob + kActorObs - 2), __ldg(ob + kActorObs - 1), 0.0f);
        mean[0] += pr.x;  // geometry prior, ppo.hpp:77
        mean[1] += pr.y;
        mean[2] += pr.z;
        const float4* co4 = reinterpret_cast<const float4*>(a.co + row * kCriticObs);
#pragma unroll
        for (int h = 0; h < kHidden; h++) z[h] = 0.0f;
#pragma unroll 1
        for (int k4 = 0; k4 < kCriticObs / 4; k4++) {
            const float4 o4 = __ldg(co4 + k4);
#pragma unroll
            for (int h = 0; h < kHidden; h++) {
                const float4 w = *reinterpret_cast<const float4*>(cw1 + h * kCw1Pitch + 4 * k4);
                z[h] = fmaf(o4.x, w.x, z[h]);
                z[h] = fmaf(o4.y, w.y, z[h]);
                z[h] = fmaf(o4.z, w.z, z[h]);
                z[h] = fmaf(o4.w, w.w, z[h]);
            }
        }
        float value = 0.0f;
#pragma unroll
        for (int h = 0; h < kHidden; h++) value = fmaf(tanhf(z[h] + cb1[h]), cw2[h], value);
        value += cb2[0];
        act_finish(a, i, row, ob, mean, value, log_std);
    }
}

// k_act_rows with four threads per environment, for shards too small to
// fill the GPU with one thread per environment: thread `part` of a quad owns
// the 16 hidden units part, part + 4, ... (its four rows of W1 are 1 row
// apart, so the quad's 128-bit reads fall on different banks), the four
// partial head sums are combined in a fixed tree, and the first thread of the
// quad finishes sim_act.
constexpr int kQuadSplit = 4;
constexpr int kQuadUnits = kHidden / kQuadSplit;
constexpr int kQuadEnvs = kRowThreads / kQuadSplit;  // environments per block pass
static_assert(kRowSmemFloats % 4 == 0, "the staged observations start on a 16-byte boundary");

__device__ __forceinline__ float quad_sum(float v) {  // ((t0 + t1) + (t2 + t3)) on every lane of the quad
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    return v + __shfl_xor_sync(0xffffffffu, v, 2);
}

__global__ void __launch_bounds__(kRowThreads) k_act_quads(SimArgs a) {
    extern __shared__ float4 smem4[];
    const ActSmem m = act_weights_fill(a, reinterpret_cast<float*>(smem4));
    const float *w1 = m.w1, *cw1 = m.cw1, *b1 = m.b1, *w2 = m.w2, *cb1 = m.cb1, *cw2 = m.cw2, *b2 = m.b2,
                *log_std = m.log_std, *cb2 = m.cb2;
    const int tid = threadIdx.x;
    const mdn_sim_config& c = a.cfg;
    const int part = tid % kQuadSplit;  // this thread's units: part, part + 4, ..., part + 60
    const uint32_t per_block = kQuadEnvs;
    // The pass's observation rows (contiguous in HBM) staged in shared memory by
    // the whole block, so the dot products wait on one load round trip.
    float4* obs_s = smem4 + kRowSmemFloats / 4;  // [kQuadEnvs][46]
    // Every lane of a quad runs the loop the same number of times (the
    // shuffles need the whole quad); `live` masks the tail.
    for (uint32_t base = blockIdx.x * per_block; base < a.n; base += gridDim.x * per_block) {
        const uint32_t i = base + uint32_t(tid / kQuadSplit);
        const bool live = i < a.n && !(c.eval && a.runs[i].episodes);
        const size_t row = size_t(a.tick) * a.n + (live ? i : 0);
        const float* ob = a.obs + row * kActorObs;
        {
            const uint32_t rows = min(per_block, a.n - base);
            const float4* src = reinterpret_cast<const float4*>(a.obs + (size_t(a.tick) * a.n + base) * kActorObs);
            __syncthreads();  // the previous pass is done with the staged rows
            for (uint32_t k = tid; k < rows * (kActorObs / 4); k += kRowThreads) obs_s[k] = __ldg(src + k);
            __syncthreads();
        }
        float z[kQuadUnits];
#pragma unroll
        for (int h = 0; h < kQuadUnits; h++) z[h] = 0.0f;
        const float4* ob4 = obs_s + (tid / kQuadSplit) * (kActorObs / 4);
#pragma unroll 2
        for (int k4 = 0; k4 < kActorObs / 4; k4++) {
            const float4 o4 = ob4[k4];
#pragma unroll
            for (int u = 0; u < kQuadUnits; u++) {  // unit part + 4u
                const float4 w = *reinterpret_cast<const float4*>(w1 + (part + kQuadSplit * u) * kW1Pitch + 4 * k4);
                z[u] = fmaf(o4.x, w.x, z[u]);
                z[u] = fmaf(o4.y, w.y, z[u]);
                z[u] = fmaf(o4.z, w.z, z[u]);
                z[u] = fmaf(o4.w, w.w, z[u]);
            }
        }
#pragma unroll
        for (int h = 0; h < kQuadUnits; h++) z[h] = tanhf(z[h] + b1[part + kQuadSplit * h]);
        float mean[4];
#pragma unroll
        for (int j = 0; j < kActions; j++) {
            float m = 0.0f;
#pragma unroll
            for (int h = 0; h < kQuadUnits; h++) m = fmaf(z[h], w2[j * kHidden + part + kQuadSplit * h], m);
            mean[j] = quad_sum(m) + b2[j];
        }
        mean[0] += __ldg(ob + kActorObs - 3);  // geometry prior, ppo.hpp:77
        mean[1] += __ldg(ob + kActorObs - 2);
        mean[2] += __ldg(ob + kActorObs - 1);
        const float4* co4 = reinterpret_cast<const float4*>(a.co + row * kCriticObs);
#pragma unroll
        for (int h = 0; h < kQuadUnits; h++) z[h] = 0.0f;
#pragma unroll 2
        for (int k4 = 0; k4 < kCriticObs / 4; k4++) {
            const float4 o4 = __ldg(co4 + k4);
#pragma unroll
            for (int u = 0; u < kQuadUnits; u++) {
                const float4 w = *reinterpret_cast<const float4*>(cw1 + (part + kQuadSplit * u) * kCw1Pitch + 4 * k4);
                z[u] = fmaf(o4.x, w.x, z[u]);
                z[u] = fmaf(o4.y, w.y, z[u]);
                z[u] = fmaf(o4.z, w.z, z[u]);
                z[u] = fmaf(o4.w, w.w, z[u]);
            }
        }
        float value = 0.0f;
#pragma unroll
        for (int h = 0; h < kQuadUnits; h++) value = fmaf(tanhf(z[h] + cb1[part + kQuadSplit * h]), cw2[part + kQuadSplit * h], value);
        value = quad_sum(value) + cb2[0];
        if (live && part == 0) act_finish_body(a, i, row, ob, mean, value, log_std);
    }
}

// kWide: the actor mean comes from the tensor-core forward's slice sums.
template <bool kWide>
__global__ void __launch_bounds__(kActWarps * 32) k_act(SimArgs a) {
    extern __shared__ float sm[];
    float* w1p = sm;                                  // [64][185] actor W1, row-major, padded
    float* b1 = w1p + kHidden * kActW1Pitch;          // [64]
    float* w2 = b1 + kHidden;                         // [4][64]
    float* b2 = w2 + kActions * kHidden;              // [4]
    float* log_std = b2 + kActions;                   // [4]
    float* cw1p = log_std + kActions;                 // [64][33] critic W1, row-major, padded
    float* cb1 = cw1p + kHidden * kActCw1Pitch;       // [64]
    float* cw2 = cb1 + kHidden;                       // [64]
    float* cb2 = cw2 + kHidden;                       // [1]
    float* rows = cb2 + 1;                            // per warp: obs[4][184], co[4][32]
    const int tid = threadIdx.x;
    constexpr bool wide = kWide;
    if (!wide)
        for (int k = tid; k < kActorObs * kHidden; k += blockDim.x) {
            const int h = k / kActorObs, col = k % kActorObs;
            w1p[h * kActW1Pitch + col] = a.actor[k];
        }
    const bool own_critic = a.critic_values == nullptr;  // else the layered critic's values
    if (own_critic)
        for (int k = tid; k < kCriticObs * kHidden; k += blockDim.x) {
            const int h = k / kCriticObs, col = k % kCriticObs;
            cw1p[h * kActCw1Pitch + col] = a.critic[k];
        }
    for (int k = tid; k < kHidden; k += blockDim.x) {
        if (!wide) b1[k] = a.actor[kActorB1 + k];
        cb1[k] = own_critic ? a.critic[kCriticB1 + k] : 0.0f;
        cw2[k] = own_critic ? a.critic[kCriticW2 + k] : 0.0f;
    }
    if (!wide)
        for (int k = tid; k < kActions * kHidden; k += blockDim.x) w2[k] = a.actor[kActorW2 + k];
    if (tid < kActions) {
        b2[tid] = a.actor[a.actor_b2 + tid];
        log_std[tid] = a.actor[a.actor_log_std + tid];
    }
    if (tid == 0) cb2[0] = own_critic ? a.critic[kCriticB2] : 0.0f;
    __syncthreads();
    const int lane = tid & 31, wid = tid >> 5;
    float* my_obs = rows + wid * kActEnvs * (kActorObs + kCriticObs);  // [4][184]
    float* my_co = my_obs + kActEnvs * kActorObs;                        // [4][32]
    const mdn_sim_config& c = a.cfg;
    const uint32_t stride = gridDim.x * kActWarps * kActEnvs;
    for (uint32_t base = (blockIdx.x * kActWarps + wid) * kActEnvs; base < a.n; base += stride) {
        const size_t row0 = size_t(a.tick) * a.n + base;
        const int envs = int(min(uint32_t(kActEnvs), a.n - base));
        for (int e = 0; e < kActEnvs; e++) {
            const float* og = a.obs + (row0 + e) * kActorObs;
            for (int k = lane; k < kActorObs; k += 32) my_obs[e * kActorObs + k] = e < envs ? og[k] : 0.0f;
            if (own_critic) my_co[e * kCriticObs + lane] = e < envs ? a.co[(row0 + e) * kCriticObs + lane] : 0.0f;
        }
        __syncwarp();
        // actor pre-activations, in-order dot from zero then the bias (cpu_reference.hpp:437-442)
        float z0[kActEnvs], z1[kActEnvs];
#pragma unroll
        for (int e = 0; e < kActEnvs; e++) z0[e] = z1[e] = 0.0f;
#pragma unroll 4
        for (int k = 0; k < (wide ? 0 : kActorObs); k++) {
            const float wa = w1p[lane * kActW1Pitch + k], wb = w1p[(lane + 32) * kActW1Pitch + k];
#pragma unroll
            for (int e = 0; e < kActEnvs; e++) {
                const float o = my_obs[e * kActorObs + k];
                z0[e] = fmaf(o, wa, z0[e]);
                z1[e] = fmaf(o, wb, z1[e]);
            }
        }
        float y0[kActEnvs], y1[kActEnvs];
#pragma unroll
        for (int e = 0; e < kActEnvs; e++) y0[e] = y1[e] = 0.0f;
#pragma unroll 4
        for (int k = 0; k < kCriticObs; k++) {
            const float wa = cw1p[lane * kActCw1Pitch + k], wb = cw1p[(lane + 32) * kActCw1Pitch + k];
#pragma unroll
            for (int e = 0; e < kActEnvs; e++) {
                const float o = my_co[e * kCriticObs + k];
                y0[e] = fmaf(o, wa, y0[e]);
                y1[e] = fmaf(o, wb, y1[e]);
            }
        }
        // heads: lane e ends with environment e's means and value
        float mean_mine[4] = {0, 0, 0, 0}, value_mine = 0.0f;
        if (wide) {
            // Wide actor: lanes 8e..8e+7 add environment e's slice sums (slice
            // q, q+8, ... on lane 8e+q), then a fixed three-level tree.
            const int e = lane >> 3, q = lane & 7;
            float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (e < envs)
                for (uint32_t sl = q; sl < a.wide_slices; sl += 8) {
                    const float4 v = __ldg(reinterpret_cast<const float4*>(a.wide_partials) + size_t(sl) * a.n + base + e);
                    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
                }
#pragma unroll
            for (int off = 4; off > 0; off >>= 1) {
                acc.x += __shfl_xor_sync(0xffffffffu, acc.x, off);
                acc.y += __shfl_xor_sync(0xffffffffu, acc.y, off);
                acc.z += __shfl_xor_sync(0xffffffffu, acc.z, off);
                acc.w += __shfl_xor_sync(0xffffffffu, acc.w, off);
            }
            const int src = (lane & 3) * 8;  // lane e < 4 takes group e's total
            const float s0 = __shfl_sync(0xffffffffu, acc.x, src), s1 = __shfl_sync(0xffffffffu, acc.y, src);
            const float s2 = __shfl_sync(0xffffffffu, acc.z, src), s3 = __shfl_sync(0xffffffffu, acc.w, src);
            if (lane < kActEnvs) {
                const float* pr = my_obs + lane * kActorObs + kActorObs - 3;  // ppo.hpp:77 geometry prior
                mean_mine[0] = s0 + b2[0] + pr[0];
                mean_mine[1] = s1 + b2[1] + pr[1];
                mean_mine[2] = s2 + b2[2] + pr[2];
                mean_mine[3] = s3 + b2[3];
            }
        }
#pragma unroll
        for (int e = 0; e < kActEnvs; e++) {
            if (!wide) {
                const float h0 = tanhf(z0[e] + b1[lane]), h1 = tanhf(z1[e] + b1[lane + 32]);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    float m = warp_sum(fmaf(h0, w2[j * kHidden + lane], h1 * w2[j * kHidden + lane + 32])) + b2[j];
                    if (j < 3) m += my_obs[e * kActorObs + kActorObs - 3 + j];
                    if (lane == e) mean_mine[j] = m;
                }
            }
            if (own_critic) {
                const float v = warp_sum(fmaf(tanhf(y0[e] + cb1[lane]), cw2[lane],
                                              tanhf(y1[e] + cb1[lane + 32]) * cw2[lane + 32])) + cb2[0];
                if (lane == e) value_mine = v;
            } else if (lane == e && e < envs) {
                value_mine = a.critic_values[base + e];
            }
        }
        __syncwarp();
        const uint32_t i = base + uint32_t(lane);
        if (lane < envs && !(c.eval && a.runs[i].episodes))
            act_finish(a, i, row0 + lane, my_obs + lane * kActorObs, mean_mine, value_mine, log_std);
        __syncwarp();
    }
}

// ---------------------------------------------------------------- advance
// 5 substeps of reference integration per policy step (sim.metal:272-332,
// cpu_reference.hpp:460-513): RAPTOR GRU + L2F RK4 with finiteness and
// sphere-contact checks, reward and termination flags, bootstrap value,
// episode statistics and in-kernel reset; also records the id of the obstacle
// nearest at the step's closest approach.
//
// G lanes advance one environment (G = 1 or 2, chosen by the host). The
// serial chain of one environment bounds this kernel when few environments
// share a GPU (one shard of a multi-GPU run), so with G = 2 the RAPTOR layers'
// units (unit u on lane u % 2), its outputs and the bootstrap critic's hidden
// units are split over a lane pair and exchanged with shuffles; the L2F RK4
// step and the clearance scan run on both lanes on the same operands, so the
// state needs no exchange. Every dot product keeps the one-thread order of
// operations (same results bit for bit); only the bootstrap value's final sum
// over hidden units is reassociated. Large shards use G = 1 (more
// environments in flight, no redundant work).
constexpr int kAdvanceThreads = 128;

// Shared-memory layout of the RAPTOR weights for a group of G lanes with
// U = 16 / G units each (unit j on lane j % G, slot j / G): for every weight
// column the U units of one lane are adjacent, so one 16-byte load feeds four
// FMAs and the lanes of a group read adjacent words
// (raptor.hpp:11-21 holds the weights row-major).
template <int G>
struct RaptorSmem {
    static constexpr int U = 16 / G;
    static constexpr int kIn = 0;                 // [22 cols][G][U]   input layer
    static constexpr int kInB = kIn + 22 * 16;    // [G][U]
    static constexpr int kGi = kInB + 16;         // [3 gates][16 cols][G][U]
    static constexpr int kGh = kGi + 3 * 256;     // [3 gates][16 cols][G][U]
    static constexpr int kGiB = kGh + 3 * 256;    // [3 gates][G][U]
    static constexpr int kGhB = kGiB + 48;        // [3 gates][G][U]
    static constexpr int kOut = kGhB + 48;        // [4 rows][16 cols] (row-major)
    static constexpr int kOutB = kOut + 64;       // [4]
    static constexpr int kFloats = kOutB + 4;
    __device__ static int slot(int unit) { return (unit % G) * U + unit / G; }
    __device__ static void fill(float* s, const float* rw, int tid, int threads) {
        for (int k = tid; k < 352; k += threads) s[kIn + (k % 22) * 16 + slot(k / 22)] = rw[k];
        for (int k = tid; k < 16; k += threads) s[kInB + slot(k)] = rw[352 + k];
        for (int k = tid; k < 768; k += threads) {
            const int gate = k / 256, unit = (k / 16) % 16, col = k % 16;
            s[kGi + gate * 256 + col * 16 + slot(unit)] = rw[368 + k];
            s[kGh + gate * 256 + col * 16 + slot(unit)] = rw[1136 + k];
        }
        for (int k = tid; k < 48; k += threads) {
            s[kGiB + (k / 16) * 16 + slot(k % 16)] = rw[1904 + k];
            s[kGhB + (k / 16) * 16 + slot(k % 16)] = rw[1952 + k];
        }
        for (int k = tid; k < 64; k += threads) s[kOut + k] = rw[2016 + k];
        if (tid < 4) s[kOutB + tid] = rw[2080 + tid];
    }
};

// Shared-memory layout of the RAPTOR weights for one lane per environment:
// the reference's row-major order (raptor.hpp:11-21) with the input rows
// padded from 22 to 24 floats, so that every row starts on a 16-byte
// boundary and a unit's weights stream in as float4 loads.
struct RaptorRows {
    static constexpr int kIn = 0;               // [16 units][24]
    static constexpr int kInB = kIn + 16 * 24;  // [16]
    static constexpr int kGi = kInB + 16;       // [3 gates][16 units][16 cols]
    static constexpr int kGh = kGi + 768;       // [3 gates][16 units][16 cols]
    static constexpr int kGiB = kGh + 768;      // [3][16]
    static constexpr int kGhB = kGiB + 48;      // [3][16]
    static constexpr int kOut = kGhB + 48;      // [4 rows][16 cols]
    static constexpr int kOutB = kOut + 64;     // [4]
    static constexpr int kFloats = kOutB + 4;
    __device__ static void fill(float* s, const float* rw, int tid, int threads) {
        for (int k = tid; k < 16 * 24; k += threads) s[kIn + k] = k % 24 < 22 ? rw[(k / 24) * 22 + k % 24] : 0.0f;
        for (int k = tid; k < 16; k += threads) s[kInB + k] = rw[352 + k];
        for (int k = tid; k < 1536; k += threads) s[kGi + k] = rw[368 + k];   // gi then gh
        for (int k = tid; k < 96; k += threads) s[kGiB + k] = rw[1904 + k];   // gi_b then gh_b
        for (int k = tid; k < 68; k += threads) s[kOut + k] = rw[2016 + k];   // out_w then out_b
    }
};

// Dense(22,16)-ReLU -> GRU(16) -> Dense(16,4) (raptor.hpp:52-92) for one
// environment on one lane, unit by unit: only one unit's six gate sums are
// live at a time (column by column, all 96 are, and the kernel spills).
// Every sum starts from its bias and runs over the columns in order.
__device__ __forceinline__ void raptor_forward_rows(const float* __restrict__ w, const float obs[22], float h[16],
                                                    float action[4]) {
    using L = RaptorRows;
    float x[16];
#pragma unroll
    for (int u = 0; u < 16; u++) {
        const float4* row = reinterpret_cast<const float4*>(w + L::kIn + u * 24);
        float acc = w[L::kInB + u];
#pragma unroll
        for (int q = 0; q < 6; q++) {
            const float4 v = row[q];
            acc = fmaf(v.x, obs[4 * q], acc);
            acc = fmaf(v.y, obs[4 * q + 1], acc);
            if (q < 5) {  // columns 22, 23 are padding
                acc = fmaf(v.z, obs[4 * q + 2], acc);
                acc = fmaf(v.w, obs[4 * q + 3], acc);
            }
        }
        x[u] = smax(acc, 0.0f);
    }
    float nh[16];
#pragma unroll
    for (int u = 0; u < 16; u++) {
        float ir = w[L::kGiB + u], hr = w[L::kGhB + u], iz = w[L::kGiB + 16 + u], hz = w[L::kGhB + 16 + u],
              in_ = w[L::kGiB + 32 + u], hn = w[L::kGhB + 32 + u];
        const float4* gi = reinterpret_cast<const float4*>(w + L::kGi + u * 16);
        const float4* gh = reinterpret_cast<const float4*>(w + L::kGh + u * 16);
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float4 a0 = gi[q], a1 = gi[64 + q], a2 = gi[128 + q];  // gates r, z, n (256 floats apart)
            const float4 b0 = gh[q], b1 = gh[64 + q], b2 = gh[128 + q];
            const float ar[4] = {a0.x, a0.y, a0.z, a0.w}, az[4] = {a1.x, a1.y, a1.z, a1.w},
                        an[4] = {a2.x, a2.y, a2.z, a2.w};
            const float br[4] = {b0.x, b0.y, b0.z, b0.w}, bz[4] = {b1.x, b1.y, b1.z, b1.w},
                        bn[4] = {b2.x, b2.y, b2.z, b2.w};
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int col = 4 * q + e;
                ir = fmaf(ar[e], x[col], ir);
                hr = fmaf(br[e], h[col], hr);
                iz = fmaf(az[e], x[col], iz);
                hz = fmaf(bz[e], h[col], hz);
                in_ = fmaf(an[e], x[col], in_);
                hn = fmaf(bn[e], h[col], hn);
            }
        }
        const float reset = 1.0f / (1.0f + expf(-(ir + hr)));
        const float update = 1.0f / (1.0f + expf(-(iz + hz)));
        const float cand = tanhf(in_ + reset * hn);
        nh[u] = (1.0f - update) * cand + update * h[u];
    }
#pragma unroll
    for (int u = 0; u < 16; u++) h[u] = nh[u];
#pragma unroll
    for (int row = 0; row < 4; ++row) {
        float value = w[L::kOutB + row];
#pragma unroll
        for (int col = 0; col < 16; col += 4) {
            const float4 ow = *reinterpret_cast<const float4*>(w + L::kOut + row * 16 + col);
            value = fmaf(ow.x, h[col], value);
            value = fmaf(ow.y, h[col + 1], value);
            value = fmaf(ow.z, h[col + 2], value);
            value = fmaf(ow.w, h[col + 3], value);
        }
        action[row] = value;
    }
}

// U consecutive floats of shared memory (U = 1, 2, 4, 8 or 16; 16-byte
// aligned for U >= 4) into registers.
template <int U>
__device__ __forceinline__ void load_units(const float* p, float (&out)[U]) {
    if constexpr (U >= 4) {
#pragma unroll
        for (int q = 0; q < U / 4; q++) {
            const float4 v = reinterpret_cast<const float4*>(p)[q];
            out[4 * q] = v.x; out[4 * q + 1] = v.y; out[4 * q + 2] = v.z; out[4 * q + 3] = v.w;
        }
    } else if constexpr (U == 2) {
        const float2 v = *reinterpret_cast<const float2*>(p);
        out[0] = v.x; out[1] = v.y;
    } else {
        out[0] = p[0];
    }
}

// Dense(22,16)-ReLU -> GRU(16) -> Dense(16,4) (raptor.hpp:52-92) for one
// environment on a group of G lanes. Each unit's dot products run in the
// reference's column order, starting from the bias, so every unit's result is
// the one a single thread computes.
template <int G>
__device__ __forceinline__ void raptor_forward_group(const float* __restrict__ w, const float obs[22], float h[16],
                                                     float action[4], unsigned mask, int base, int r) {
    using L = RaptorSmem<G>;
    constexpr int U = L::U;
    float xm[U];
    load_units<U>(w + L::kInB + r * U, xm);
#pragma unroll
    for (int col = 0; col < 22; ++col) {
        float wv[U];
        load_units<U>(w + L::kIn + col * 16 + r * U, wv);
#pragma unroll
        for (int u = 0; u < U; u++) xm[u] = fmaf(wv[u], obs[col], xm[u]);
    }
    float x[16];
#pragma unroll
    for (int u = 0; u < U; u++) xm[u] = smax(xm[u], 0.0f);
#pragma unroll
    for (int j = 0; j < 16; j++) {
        if constexpr (G == 1) x[j] = xm[j];
        else x[j] = __shfl_sync(mask, xm[j / G], base + j % G);
    }
    float ir[U], hr[U], iz[U], hz[U], in_[U], hn[U];
    load_units<U>(w + L::kGiB + r * U, ir);
    load_units<U>(w + L::kGhB + r * U, hr);
    load_units<U>(w + L::kGiB + 16 + r * U, iz);
    load_units<U>(w + L::kGhB + 16 + r * U, hz);
    load_units<U>(w + L::kGiB + 32 + r * U, in_);
    load_units<U>(w + L::kGhB + 32 + r * U, hn);
#pragma unroll
    for (int col = 0; col < 16; ++col) {
        float a0[U], a1[U], a2[U], b0[U], b1[U], b2[U];
        load_units<U>(w + L::kGi + col * 16 + r * U, a0);
        load_units<U>(w + L::kGi + 256 + col * 16 + r * U, a1);
        load_units<U>(w + L::kGi + 512 + col * 16 + r * U, a2);
        load_units<U>(w + L::kGh + col * 16 + r * U, b0);
        load_units<U>(w + L::kGh + 256 + col * 16 + r * U, b1);
        load_units<U>(w + L::kGh + 512 + col * 16 + r * U, b2);
#pragma unroll
        for (int u = 0; u < U; u++) {
            ir[u] = fmaf(a0[u], x[col], ir[u]);
            hr[u] = fmaf(b0[u], h[col], hr[u]);
            iz[u] = fmaf(a1[u], x[col], iz[u]);
            hz[u] = fmaf(b1[u], h[col], hz[u]);
            in_[u] = fmaf(a2[u], x[col], in_[u]);
            hn[u] = fmaf(b2[u], h[col], hn[u]);
        }
    }
    float nm[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
        const float reset = 1.0f / (1.0f + expf(-(ir[u] + hr[u])));
        const float update = 1.0f / (1.0f + expf(-(iz[u] + hz[u])));
        const float cand = tanhf(in_[u] + reset * hn[u]);
        nm[u] = (1.0f - update) * cand + update * h[r + G * u];
    }
#pragma unroll
    for (int j = 0; j < 16; j++) {
        if constexpr (G == 1) h[j] = nm[j];
        else h[j] = __shfl_sync(mask, nm[j / G], base + j % G);
    }
    {
#pragma unroll
        for (int row = 0; row < 4; ++row) {
            float value = w[L::kOutB + row];
#pragma unroll
            for (int col = 0; col < 16; col += 4) {
                const float4 ow = *reinterpret_cast<const float4*>(w + L::kOut + row * 16 + col);
                value = fmaf(ow.x, h[col], value);
                value = fmaf(ow.y, h[col + 1], value);
                value = fmaf(ow.z, h[col + 2], value);
                value = fmaf(ow.w, h[col + 3], value);
            }
            action[row] = value;
        }
    }
}

// kEnvPhysics: each env integrates its own episode plant (runtime config on,
// sim.metal:287) instead of the block's shared copy of the nominal one.
// `nominal` is the plant of MDN_BUF_PHYSICS by value: as a kernel argument it
// sits in the constant bank, and every use is an instruction operand, so the
// integrator keeps none of its 88 coefficients in registers.
template <int G, bool kEnvPhysics>
__global__ void __launch_bounds__(kAdvanceThreads, G == 1 ? 4 : 3) k_advance(SimArgs a, mdn_physics_params nominal) {
    using L = std::conditional_t<G == 1, RaptorRows, RaptorSmem<G>>;
    constexpr int kGroups = kAdvanceThreads / G;
    constexpr int V = kHidden / G;             // bootstrap critic hidden units per lane
    __shared__ __align__(16) float raptor_w[L::kFloats];
    __shared__ __align__(16) float cw1p[kCriticObs * kHidden];  // [32 inputs][G][V] critic W1
    __shared__ __align__(16) float cb1p[kHidden], cw2p[kHidden];  // [G][V]
    __shared__ float cb2;
    const int tid = threadIdx.x;
    {
        L::fill(raptor_w, reinterpret_cast<const float*>(a.raptor), tid, blockDim.x);
        if (!a.next_co) {  // the 64-unit critic (a layered critic runs after this kernel)
            for (int k = tid; k < kCriticObs * kHidden; k += blockDim.x) {
                const int hh = k / kCriticObs, col = k % kCriticObs;
                cw1p[col * kHidden + (hh % G) * V + hh / G] = a.critic[k];
            }
            for (int k = tid; k < kHidden; k += blockDim.x) {
                cb1p[(k % G) * V + k / G] = a.critic[kCriticB1 + k];
                cw2p[(k % G) * V + k / G] = a.critic[kCriticW2 + k];
            }
            if (tid == 0) cb2 = a.critic[kCriticB2];
        }
    }
    __syncthreads();

    const int lane = tid & 31, r = lane & (G - 1), base = lane & ~(G - 1);
    const unsigned mask = ((1u << G) - 1u) << base;
    const int group = tid / G;
    const mdn_sim_config& c = a.cfg;
    for (uint32_t tile = blockIdx.x * kGroups; tile < a.n; tile += gridDim.x * kGroups) {
        const uint32_t i = tile + group;
        bool active = i < a.n;
        if (active && c.eval && a.runs[i].episodes) active = false;
        bool refill = false;
        if (active) {
            mdn_sim_run& run = a.runs[i];
            const mdn_world& w = a.worlds[i];
            const size_t row = size_t(a.tick) * a.n + i;
            const uint32_t count = w.count < 16u ? w.count : 16u;
            float s[17];
            {
                const float* sp = reinterpret_cast<const float*>(&a.states[i]);
#pragma unroll
                for (int k = 0; k < 17; k++) s[k] = sp[k];
            }
            float h[16], motors[4];
#pragma unroll
            for (int k = 0; k < 16; k++) h[k] = run.hidden[k];
#pragma unroll
            for (int k = 0; k < 4; k++) motors[k] = run.motors[k];
            const float goal[3] = {w.goal[0], w.goal[1], w.goal[2]};
            const float before = len3(goal[0] - s[0], goal[1] - s[1], goal[2] - s[2]);
            const float yaw = run.yaw, cy = cosf(yaw), sy = sinf(yaw);
            const float ch = cosf(yaw * .5f), sh = sinf(yaw * .5f);
            bool collision = false;
            float step_clearance = 12.0f;
            int32_t contact = -1;
            const mdn_physics_params& plant = kEnvPhysics ? a.env_physics[i] : nominal;
            const float wind[3] = {w.wind[0] * plant.mass, w.wind[1] * plant.mass, w.wind[2] * plant.mass};
            float refp[3] = {run.reference_position[0], run.reference_position[1], run.reference_position[2]};
            const float dv_[3] = {run.desired_velocity[0], run.desired_velocity[1], run.desired_velocity[2]};
            float path = run.path, elapsed = run.elapsed, min_clear = run.min_clearance, peak = run.peak_speed;
            float clear_now = 0.0f;
            bool clear_valid = false;
            for (uint32_t step = 0; step < c.substeps; step++) {
                float mo[22];
                for (int j = 0; j < 3; j++) refp[j] += dv_[j] * nominal.dt;
                const float dp0 = s[0] - refp[0], dp1 = s[1] - refp[1], dp2 = s[2] - refp[2];
                const float dvx = s[7] - dv_[0], dvy = s[8] - dv_[1], dvz = s[9] - dv_[2];
                mo[0] = clampf(cy * dp0 + sy * dp1, -.5f, .5f);
                mo[1] = clampf(-sy * dp0 + cy * dp1, -.5f, .5f);
                mo[2] = clampf(dp2, -.5f, .5f);
                const float qy[4] = {ch * s[3] + sh * s[6], ch * s[4] + sh * s[5], ch * s[5] - sh * s[4],
                                     ch * s[6] - sh * s[3]};
                float rr[9];
                rotation(qy, rr);
#pragma unroll
                for (int j = 0; j < 9; j++) mo[3 + j] = rr[j];
                mo[12] = clampf(cy * dvx + sy * dvy, -1.0f, 1.0f);
                mo[13] = clampf(-sy * dvx + cy * dvy, -1.0f, 1.0f);
                mo[14] = clampf(dvz, -1.0f, 1.0f);
                mo[15] = s[10]; mo[16] = s[11]; mo[17] = s[12];
#pragma unroll
                for (int j = 0; j < 4; j++) mo[18 + j] = motors[j];
                if constexpr (G == 1) raptor_forward_rows(raptor_w, mo, h, motors);
                else raptor_forward_group<G>(raptor_w, mo, h, motors, mask, base, r);
#pragma unroll
                for (int j = 0; j < 4; j++) motors[j] = smax(-1.0f, smin(1.0f, motors[j]));
                float nx[17];
                l2f_step(plant, s, motors, wind, nx);
                bool valid = true;
#pragma unroll
                for (int j = 0; j < 17; j++) valid = valid && isfinite(nx[j]);
                if (!valid) {
                    collision = true;
                    break;
                }
                path += len3(s[0] - nx[0], s[1] - nx[1], s[2] - nx[2]);
#pragma unroll
                for (int j = 0; j < 17; j++) s[j] = nx[j];
                elapsed += nominal.dt;
                int32_t id;
                const float clearance = world_clearance_lanes<G>(a, i, s, elapsed, &id, r, mask);
                clear_now = clearance;  // the clearance at (s, elapsed) from here on
                clear_valid = true;
                if (clearance < step_clearance) contact = id;
                step_clearance = smin(step_clearance, clearance);
                min_clear = smin(min_clear, clearance);
                peak = smax(peak, len3(s[7], s[8], s[9]));
                if (clearance <= 0 || !isfinite(s[0]) || !isfinite(s[1]) || !isfinite(s[2])) {
                    collision = true;
                    break;
                }
            }
            const uint32_t steps = run.steps + 1;
            // Bootstrap value of the post-step critic observation (sim.metal:327),
            // hidden units r, r+G, ... on lane r.
            float value;
            {
                float co[kCriticObs];
                for (int j = 0; j < 3; j++) {
                    co[j] = (goal[j] - s[j]) / 10.0f;
                    co[j + 3] = s[7 + j] / 4.0f;
                    co[j + 6] = s[10 + j] / 4.0f;
                    co[j + 13] = s[j] / 10.0f;
                    co[j + 16] = (refp[j] - s[j]) * 2.0f;
                }
                for (int j = 0; j < 4; j++) co[9 + j] = s[3 + j];
                // wclearance of the final pose: the last substep's value unless
                // the first substep already stopped on an invalid state.
                co[19] = (clear_valid ? clear_now : world_clearance_lanes<G>(a, i, s, elapsed, nullptr, r, mask)) / 5.0f;
                co[20] = float(steps) / 200.0f;
                for (int j = 21; j < 30; j++) co[j] = 0.0f;
                const uint32_t m = count < 3u ? count : 3u;
#pragma unroll
                for (uint32_t o = 0; o < 3; o++) {
                    if (o < m) {
                        float f[10];
#pragma unroll
                        for (int k = 0; k < 10; k++) f[k] = __ldg(a.world_soa + size_t(o * 10 + k) * a.n + i);
                        float cc[3];
                        obstacle_center(__float_as_uint(f[0]), f + 1, f + 4, f + 7, elapsed, cc);
                        co[21 + o * 3] = (cc[0] - s[0]) / 10.0f;
                        co[22 + o * 3] = (cc[1] - s[1]) / 10.0f;
                        co[23 + o * 3] = (cc[2] - s[2]) / 10.0f;
                    }
                }
                co[30] = w.wind[0];
                co[31] = w.wind[1];
                float part = 0.0f;
                if (a.next_co) {  // layered critic: keep the observation for it
                    if (r == 0)  // (inputs 32..63 of the control-state critic: k_control_state)
#pragma unroll
                        for (int k = 0; k < kCriticObs; k++) a.next_co[size_t(i) * kCriticObs + k] = co[k];
                } else
#pragma unroll
                for (int v0 = 0; v0 < V; v0 += 4) {
                    float z[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                    for (int k = 0; k < kCriticObs; k++) {
                        const float4 wv = *reinterpret_cast<const float4*>(cw1p + k * kHidden + r * V + v0);
                        z[0] = fmaf(co[k], wv.x, z[0]);
                        z[1] = fmaf(co[k], wv.y, z[1]);
                        z[2] = fmaf(co[k], wv.z, z[2]);
                        z[3] = fmaf(co[k], wv.w, z[3]);
                    }
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        part = fmaf(tanhf(z[q] + cb1p[r * V + v0 + q]), cw2p[r * V + v0 + q], part);
                }
                if constexpr (G > 1) {
#pragma unroll
                    for (int off = G / 2; off > 0; off >>= 1) part += __shfl_xor_sync(mask, part, off);
                }
                value = part + cb2;
            }
            if (r == 0) {
                run.steps = steps;
                {
                    float* sp = reinterpret_cast<float*>(&a.states[i]);
#pragma unroll
                    for (int k = 0; k < 17; k++) sp[k] = s[k];
                }
#pragma unroll
                for (int k = 0; k < 16; k++) run.hidden[k] = h[k];
#pragma unroll
                for (int k = 0; k < 4; k++) run.motors[k] = motors[k];
                for (int j = 0; j < 3; j++) run.reference_position[j] = refp[j];
                run.path = path;
                run.elapsed = elapsed;
                run.min_clearance = min_clear;
                run.peak_speed = peak;
                const float after = len3(goal[0] - s[0], goal[1] - s[1], goal[2] - s[2]);
                bool success = after < (c.mode == 20 ? .10f : .35f) && !collision;
                bool timeout = steps >= c.max_steps;
                a.rewards[row] = (before - after) * 2.0f - .01f -
                                 c.risk_coef * clampf((0.6f - step_clearance) / 0.6f, 0.0f, 1.0f) +
                                 (success ? 10.0f : 0.0f) - (collision ? 10.0f : 0.0f);
                bool term = collision || success;
                a.terminated[row] = term;
                a.truncated[row] = timeout && !term;
                a.contact[row] = contact;
                if (a.task_ctl.enabled) {  // sim.metal:307-317
                    const float executed[4] = {run.desired_velocity[0], run.desired_velocity[1],
                                               run.desired_velocity[2], run.previous_nav[3] * 0.5f};
                    const float pv[6] = {s[0], s[1], s[2], s[7], s[8], s[9]};  // keeps s out of local memory
                    const TaskStep out =
                        task_step(a.tasks[i], a.task_ctl.config, pv, pv + 3, executed, collision, timeout);
                    success = out.stable_success != 0u && !collision;
                    timeout = out.timeout != 0u;
                    a.rewards[row] = out.reward;
                    term = collision || success;
                    a.terminated[row] = term;
                    a.truncated[row] = timeout && !term;
                }
                if (!a.next_co) a.next_values[row] = value;
                if (a.bank_transition) a.bank_transition[row] = a.bank_enabled ? a.bank_active[i] : 0xffffffffu;
                if (success || collision || timeout) {
                    run.successes += success;
                    run.collisions += collision;
                    run.timeouts += timeout && !term;
                    run.episodes++;
                    run.success_time += success ? elapsed : 0.0f;
                    run.total_path += path;
                    run.total_elapsed += elapsed;
                    run.final_progress += 1.0f - after / smax(run.initial_distance, 1.0e-4f);
                    refill = !c.eval;  // reset by the next k_sense or by the k_reset_list flush
                }
                a.reset_pending[i] = refill ? 1 : 0;
                if (a.audit) {  // mechanical contact audit of the post-integration pose
                    // Called last, with the pose read back from the stores above, so
                    // that little is live across this out-of-line call.
                    const float* sp = reinterpret_cast<const float*>(&a.states[i]);
                    const float pos[3] = {sp[0], sp[1], sp[2]}, orient[4] = {sp[3], sp[4], sp[5], sp[6]};
                    a.audit[row] = contact::world_contact(pos, orient, w, run.elapsed, a.audit_margin);
                }
            }
        }
        // Environments whose episode ended (their leader lanes) join the
        // step's reset list: one atomic per warp, slots in lane order. Every
        // active environment's pending flag says whether it is listed.
        const unsigned m = __ballot_sync(0xffffffffu, refill);
        if (m) {
            const int leader = __ffs(m) - 1;
            uint32_t slot = 0;
            if (lane == leader) slot = atomicAdd(a.reset_count + a.phase, uint32_t(__popc(m)));
            slot = __shfl_sync(0xffffffffu, slot, leader);
            if (refill) a.reset_list[slot + uint32_t(__popc(m & ((1u << lane) - 1u)))] = i;
        }
    }
}

template <int G>
static int advance_blocks_per_sm() {
    int blocks = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, k_advance<G, false>, kAdvanceThreads, 0) != cudaSuccess)
        blocks = 1;
    return blocks > 0 ? blocks : 1;
}

static void launch_reset_list(const SimArgs& a, const StepPlan& plan, cudaStream_t s) {
    k_reset_list<<<plan.reset_grid, 128, 0, s>>>(a);
}

static cudaError_t launch_advance(const SimArgs& a, const StepPlan& plan, const mdn_physics_params& nominal,
                                  cudaStream_t s) {
    const bool own = a.runtime.enabled != 0;
    switch (plan.advance_group) {
        case 8:
            if (own) k_advance<8, true><<<plan.advance_grid, kAdvanceThreads, 0, s>>>(a, nominal);
            else k_advance<8, false><<<plan.advance_grid, kAdvanceThreads, 0, s>>>(a, nominal);
            break;
        case 4:
            if (own) k_advance<4, true><<<plan.advance_grid, kAdvanceThreads, 0, s>>>(a, nominal);
            else k_advance<4, false><<<plan.advance_grid, kAdvanceThreads, 0, s>>>(a, nominal);
            break;
        case 2:
            if (own) k_advance<2, true><<<plan.advance_grid, kAdvanceThreads, 0, s>>>(a, nominal);
            else k_advance<2, false><<<plan.advance_grid, kAdvanceThreads, 0, s>>>(a, nominal);
            break;
        default:
            if (own) k_advance<1, true><<<plan.advance_grid, kAdvanceThreads, 0, s>>>(a, nominal);
            else k_advance<1, false><<<plan.advance_grid, kAdvanceThreads, 0, s>>>(a, nominal);
            break;
    }
    return cudaGetLastError();
}

// ------------------------------------------------------------- launchers
static inline unsigned blocks_for(uint32_t n, int per_block) { return (n + per_block - 1) / per_block; }

cudaError_t upload_camera_tables(const float* pixel_rays, const float* pool_rays) {
    float4 rays[kPixels];
    for (int k = 0; k < kPixels; k++)
        rays[k] = make_float4(pixel_rays[3 * k], pixel_rays[3 * k + 1], pixel_rays[3 * k + 2], 0.0f);
    cudaError_t e = cudaMemcpyToSymbol(g_pixel_ray, rays, sizeof(rays));
    if (e != cudaSuccess) return e;
    // Tile cones, in double: axis = normalised sum of the tile's rays,
    // half-angle = the widest ray's angle + 3 mrad; cosine rounded down and
    // sine rounded up so the float test only errs towards keeping.
    float4 cones[kPixels / 32];
    float sines[kPixels / 32];
    for (int t = 0; t < kPixels / 32; t++) {
        double axis[3] = {0.0, 0.0, 0.0};
        int ks[32];
        for (int l = 0; l < 32; l++) {
            const int col = (t % 5) * 4 + (l & 3), prow = (t / 5) * 8 + (l >> 2);
            ks[l] = prow * 20 + col;
            for (int j = 0; j < 3; j++) axis[j] += pixel_rays[3 * ks[l] + j];
        }
        const double norm = std::sqrt(axis[0] * axis[0] + axis[1] * axis[1] + axis[2] * axis[2]);
        for (int j = 0; j < 3; j++) axis[j] /= norm;
        double widest = 0.0;
        for (int l = 0; l < 32; l++) {
            const float* ray = pixel_rays + 3 * ks[l];
            const double rn = std::sqrt(double(ray[0]) * ray[0] + double(ray[1]) * ray[1] + double(ray[2]) * ray[2]);
            const double dot = (axis[0] * ray[0] + axis[1] * ray[1] + axis[2] * ray[2]) / rn;
            widest = std::max(widest, std::acos(std::min(1.0, dot)));
        }
        const double half = widest + 3e-3;
        cones[t] = make_float4(float(axis[0]), float(axis[1]), float(axis[2]),
                               std::nextafter(float(std::cos(half)), -1.0f));
        sines[t] = std::nextafter(float(std::sin(half)), 2.0f);
    }
    e = cudaMemcpyToSymbol(g_tile_cone, cones, sizeof(cones));
    if (e != cudaSuccess) return e;
    e = cudaMemcpyToSymbol(g_tile_sin, sines, sizeof(sines));
    if (e != cudaSuccess) return e;
    return cudaMemcpyToSymbol(g_pool_ray, pool_rays, sizeof(float) * 80 * 3);
}

// Sim::report's aggregates (main.mm:599-602) over the run records, on the
// GPU: one CTA; thread t adds environments t, t + 1024, ... in order (double
// sums of the counters and float totals), then a fixed tree over the threads.
// Only the ten results leave the device.
constexpr int kReportThreads = 1024;
__global__ void __launch_bounds__(kReportThreads) k_report(SimArgs a, double* out) {
    __shared__ double part[8][kReportThreads / 32];
    __shared__ float lo[kReportThreads / 32], hi[kReportThreads / 32];
    double v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float mn = 12.0f, mx = 0.0f;
    for (uint32_t i = threadIdx.x; i < a.n; i += kReportThreads) {
        const mdn_sim_run& r = a.runs[i];
        v[0] += r.episodes;
        v[1] += r.successes;
        v[2] += r.collisions;
        v[3] += r.timeouts;
        v[4] += r.success_time;
        v[5] += r.total_path;
        v[6] += r.total_elapsed;
        v[7] += r.final_progress;
        mn = fminf(mn, r.min_clearance);
        mx = fmaxf(mx, r.peak_speed);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] += __shfl_xor_sync(0xffffffffu, v[k], off);
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    }
    if (lane == 0) {
#pragma unroll
        for (int k = 0; k < 8; k++) part[k][warp] = v[k];
        lo[warp] = mn;
        hi[warp] = mx;
    }
    __syncthreads();
    if (threadIdx.x < 10) {
        const int k = threadIdx.x;
        double t = k == 8 ? 12.0 : 0.0;
        for (int w = 0; w < kReportThreads / 32; w++) {
            if (k < 8) t += part[k][w];
            else if (k == 8) t = fmin(t, double(lo[w]));
            else t = fmax(t, double(hi[w]));
        }
        out[k] = t;
    }
}

cudaError_t launch_report(const SimArgs& a, double* out, cudaStream_t s) {
    k_report<<<1, kReportThreads, 0, s>>>(a, out);
    return cudaGetLastError();
}

cudaError_t launch_world_mirror(const SimArgs& a, cudaStream_t s) {
    k_world_mirror<<<blocks_for(a.n, 128), 128, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_reset(const SimArgs& a, bool first, cudaStream_t s) {
    k_reset<<<blocks_for(a.n, 4), 128, 0, s>>>(a, first ? 1 : 0);
    return cudaGetLastError();
}

size_t act_smem_bytes() { return sizeof(float) * kActSmemFloats; }
static size_t act_rows_smem_bytes() { return sizeof(float) * kRowSmemFloats; }
static size_t act_quads_smem_bytes() { return sizeof(float) * (kRowSmemFloats + size_t(kQuadEnvs) * kActorObs); }

static void launch_act(const SimArgs& a, const StepPlan& plan, cudaStream_t s) {
    if (a.wide_slices)
        k_act<true><<<plan.act_grid, kActWarps * 32, act_smem_bytes(), s>>>(a);
    else if (plan.act_quads)
        k_act_quads<<<plan.act_rows_grid, kRowThreads, act_quads_smem_bytes(), s>>>(a);
    else
        k_act_rows<<<plan.act_rows_grid, kRowThreads, act_rows_smem_bytes(), s>>>(a);
}

// The wide actor's tensor-core forward over this tick's observation rows.
static cudaError_t launch_wide(const SimArgs& a, const WideStep* wide, cudaStream_t s) {
    if (!wide) return cudaSuccess;
    WideRowsArgs p = wide->args;
    p.row0 = a.tick * a.n;
    return launch_wide_forward(wide->obs_map, wide->w1_map, p, wide->sm_count, s);
}

// The control-state critic's extra inputs (nothing for the 32-input critic).
static void launch_control_state(const SimArgs& a, bool post_step, cudaStream_t s) {
    if (a.co_dim == kCriticObsControl)
        k_control_state<<<blocks_for(a.n, kControlWarps), kControlWarps * 32, 0, s>>>(a, post_step ? 1 : 0);
}

static void launch_sense(const SimArgs& a, cudaStream_t s) {
    k_sense<<<blocks_for(a.n, kSenseWarps), kSenseWarps * 32, 0, s>>>(a);
}

// k_reset_sense on the fork's side stream, between an event recorded on `s`
// and one that `s` waits on before the actor: inside a stream capture this is
// a parallel branch of the graph beside k_sense.
static cudaError_t launch_sense_with_resets(const SimArgs& a, const StepPlan& plan, cudaStream_t s,
                                            const StepFork& fork) {
    cudaError_t e = cudaEventRecord(fork.fork, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(fork.side, fork.fork, 0);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(plan.sense_reset_blocks));
    cfg.blockDim = dim3(kSenseWarps * 32);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = fork.side;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributePriority;
    attr[0].val.priority = fork.priority;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, k_reset_sense, a);
    if (e == cudaSuccess) launch_sense(a, s);
    if (e == cudaSuccess) e = cudaEventRecord(fork.join, fork.side);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, fork.join, 0);
    return e;
}

cudaError_t launch_step(const SimArgs& a, const StepPlan& plan, const mdn_physics_params& nominal, cudaStream_t s,
                        const WideStep* wide, bool flush, const StepFork* fork, const LayeredStep* layered) {
    if (fork) {
        const cudaError_t fe = launch_sense_with_resets(a, plan, s, *fork);
        if (fe != cudaSuccess) return fe;
    } else {
        launch_sense(a, s);
    }
    if (a.cfg.geometry_memory)
        k_memory_hint<<<blocks_for(a.n, kMemWarps), kMemWarps * 32, kMemWarps * sizeof(MemScene), s>>>(a);
    launch_control_state(a, false, s);
    cudaError_t e = launch_wide(a, wide, s);
    if (e == cudaSuccess && layered) e = launch_layered_step_forward(*layered, a.n, a.tick, s);
    if (e != cudaSuccess) return e;
    launch_act(a, plan, s);
    e = launch_advance(a, plan, nominal, s);
    if (e == cudaSuccess) launch_control_state(a, true, s);
    if (e == cudaSuccess && layered) e = launch_layered_bootstrap(*layered, a.n, a.tick, s);
    if (e != cudaSuccess) return e;
    if (flush) launch_reset_list(a, plan, s);
    return cudaGetLastError();
}

cudaError_t launch_step_profiled(const SimArgs& a, const StepPlan& plan, const mdn_physics_params& nominal, cudaStream_t s,
                                 cudaEvent_t ev[4], const WideStep* wide, const LayeredStep* layered) {
    cudaEventRecord(ev[0], s);
    launch_sense(a, s);
    if (a.cfg.geometry_memory)
        k_memory_hint<<<blocks_for(a.n, kMemWarps), kMemWarps * 32, kMemWarps * sizeof(MemScene), s>>>(a);
    launch_control_state(a, false, s);
    cudaEventRecord(ev[1], s);
    cudaError_t we = launch_wide(a, wide, s);
    if (we == cudaSuccess && layered) we = launch_layered_step_forward(*layered, a.n, a.tick, s);
    if (we != cudaSuccess) return we;
    launch_act(a, plan, s);
    cudaEventRecord(ev[2], s);
    cudaError_t e = launch_advance(a, plan, nominal, s);
    if (e == cudaSuccess) launch_control_state(a, true, s);
    if (e == cudaSuccess && layered) e = launch_layered_bootstrap(*layered, a.n, a.tick, s);
    if (e != cudaSuccess) return e;
    launch_reset_list(a, plan, s);
    cudaEventRecord(ev[3], s);
    return cudaGetLastError();
}

// Launch shapes of one policy step for n environments. On small shards the
// per-environment chain of k_advance sets its time, so the RAPTOR units, the
// clearance scan and the bootstrap critic are split over 2 or 4 lanes; on
// large ones occupancy does, and one lane per environment is fastest (65,536:
// 0.272 vs 0.384 ms with 2).
StepPlan plan_step(uint32_t n, int sm_count, int group_override, int act_override) {
    StepPlan p{};
    p.act_grid = int(std::min<size_t>((size_t(n) + 31) / 32, size_t(sm_count) * 2));
    // Four threads per environment when one per environment would leave the
    // SMs with under two warps each (measured: 8,192 envs 0.062 vs 0.073 ms;
    // 16,384 envs 0.094 vs 0.074 ms).
    p.act_quads = size_t(n) <= size_t(sm_count) * 64 ? 1 : 0;
    if (act_override == 1 || act_override == 4) p.act_quads = act_override == 4 ? 1 : 0;
    const size_t per_block = p.act_quads ? kRowThreads / kQuadSplit : kRowThreads;
    p.act_rows_grid = int(std::min<size_t>((size_t(n) + per_block - 1) / per_block, size_t(sm_count) * 2));
    // Lanes per environment for k_advance: 4 on shards of at most 64
    // environments per SM (8,192 envs: 0.151 vs 0.163 ms with 2), 2 while the
    // pairs fit one wave of three 128-thread blocks per SM, 192 environments
    // (16,384: 0.167 vs 0.214 ms with 1; 24,576: 0.179 vs 0.222), else 1
    // (32,768: 0.224 vs 0.263 ms with 2).
    // Eight lanes on shards of at most 32 environments per SM (4,096 envs:
    // 27.6 vs 26.0M env-steps/s with 4; 8,192: 37.5 vs 44.0M).
    int g = size_t(n) <= size_t(sm_count) * 64 ? 4 : (size_t(n) <= size_t(sm_count) * 192 ? 2 : 1);
    if (size_t(n) <= size_t(sm_count) * 32) g = 8;
    if (group_override == 1 || group_override == 2 || group_override == 4 || group_override == 8) g = group_override;
    p.advance_group = g;
    const int per_sm = g == 1 ? advance_blocks_per_sm<1>()
                     : (g == 2 ? advance_blocks_per_sm<2>() : (g == 4 ? advance_blocks_per_sm<4>() : advance_blocks_per_sm<8>()));
    const size_t need = (size_t(n) * g + kAdvanceThreads - 1) / kAdvanceThreads;
    p.advance_grid = int(std::max<size_t>(1, std::min<size_t>(need, size_t(sm_count) * per_sm)));
    p.reset_grid = int(std::max<size_t>(1, std::min<size_t>((size_t(n) + 3) / 4, size_t(sm_count) * 8)));
    // k_reset_sense blocks: one per SM (eight warps), fewer on shards that
    // have fewer sensing blocks.
    p.sense_reset_blocks = int(std::max<size_t>(1, std::min<size_t>(blocks_for(n, kSenseWarps), size_t(sm_count))));
    return p;
}

// div_by_rcp against IEEE division on the ray tests' operand ranges: a is 0
// or of magnitude 2^-24..2^6, d of magnitude 2^-26..2^0 (random signs and
// mantissas from a per-thread hash); counts the mismatched bit patterns.
__global__ void k_division_check(uint64_t samples, uint64_t seed, unsigned long long* mismatches) {
    unsigned long long local = 0;
    for (uint64_t k = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; k < samples;
         k += uint64_t(gridDim.x) * blockDim.x) {
        uint64_t h = (k + 1) * 0x9e3779b97f4a7c15ull ^ seed;
        h ^= h >> 31;
        h *= 0xbf58476d1ce4e5b9ull;
        h ^= h >> 27;
        h *= 0x94d049bb133111ebull;
        h ^= h >> 31;
        const uint32_t u = uint32_t(h), v = uint32_t(h >> 32);
        const uint32_t ea = 127u - 24u + (u >> 24) % 31u, ed = 127u - 26u + (v >> 24) % 27u;
        float a = __uint_as_float((u & 0x80000000u) | (ea << 23) | (u & 0x7fffffu));
        const float d = __uint_as_float((v & 0x80000000u) | (ed << 23) | (v & 0x7fffffu));
        if ((u & 0xff000000u) == 0u) a = 0.0f;
        if (!(fabsf(d) >= 1e-8f)) continue;
        const float q = div_by_rcp(a, d, __frcp_rn(d));
        if (__float_as_uint(q) != __float_as_uint(a / d)) local++;
    }
    if (local) atomicAdd(mismatches, local);
}

cudaError_t division_check(uint64_t samples, uint64_t seed, uint64_t* mismatches, int sm_count) {
    unsigned long long* d = nullptr;
    cudaError_t e = cudaMalloc(&d, sizeof(*d));
    if (e != cudaSuccess) return e;
    e = cudaMemset(d, 0, sizeof(*d));
    if (e == cudaSuccess) {
        k_division_check<<<sm_count * 8, 256>>>(samples, seed, d);
        e = cudaGetLastError();
    }
    unsigned long long h = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&h, d, sizeof(h), cudaMemcpyDeviceToHost);
    cudaFree(d);
    *mismatches = h;
    return e;
}

// Pure FP32 FMA stream: 8 independent chains per thread, `iters` rounds.
__global__ void k_fma_peak(float* out, int iters, float seed) {
    float a[8];
#pragma unroll
    for (int j = 0; j < 8; j++) a[j] = seed + float(threadIdx.x + j);
    const float m = 0.999999f, c = 1e-7f;
    for (int i = 0; i < iters; i++) {
#pragma unroll
        for (int j = 0; j < 8; j++) a[j] = fmaf(a[j], m, c);
    }
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) s += a[j];
    if (s == 12345.678f) out[0] = s;  // keeps the chains live
}

cudaError_t fp32_peak(int sm_count, double* tflops) {
    float* out = nullptr;
    cudaError_t e = cudaMalloc(&out, 16);
    if (e != cudaSuccess) return e;
    const int blocks = sm_count * 8, threads = 256, iters = 4096;
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    k_fma_peak<<<blocks, threads>>>(out, iters, 1.0f);  // warm-up
    float best = 1e30f;
    for (int r = 0; r < 5; r++) {
        cudaEventRecord(a);
        k_fma_peak<<<blocks, threads>>>(out, iters, 1.0f);
        cudaEventRecord(b);
        cudaEventSynchronize(b);
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, a, b);
        best = fminf(best, ms);
    }
    e = cudaGetLastError();
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaFree(out);
    *tflops = 2.0 * 8.0 * double(iters) * double(blocks) * threads / (double(best) * 1e-3) / 1e12;
    return e;
}

// Launches per policy step of a collected rollout: sense, the previous step's
// listed resets (k_reset_sense; the last step's k_reset_list flush instead for
// the first step), act and advance, plus the geometry-memory hint and the
// wide actor's tensor-core forward when they run.
int kernels_per_step(const mdn_sim_config& c, bool wide) { return 4 + (c.geometry_memory ? 1 : 0) + (wide ? 1 : 0); }

cudaError_t configure_kernels() {
    cudaError_t e = cudaFuncSetAttribute(k_act_rows, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(act_rows_smem_bytes()));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_act_quads, cudaFuncAttributeMaxDynamicSharedMemorySize, int(act_quads_smem_bytes()));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_act<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(act_smem_bytes()));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_act<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(act_smem_bytes()));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_memory_hint, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kMemWarps * sizeof(MemScene)));
}

}  // namespace mdn
