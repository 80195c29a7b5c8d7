// Procedural world families and episode reset on the device.
// world.hpp:104-318 (generators) and sim.metal:55-94 (sim_reset_one).
#pragma once
#include "domain.cuh"
#include "mdn_device.cuh"

namespace mdn {

// Run by a whole converged warp (every lane computes and stores the same
// values). Fields that are rewritten and then read back - the obstacle count
// here, the world at each new generation or task attempt - are fenced with
// __syncwarp(), so that a lane that fell behind cannot overwrite a newer value
// with an older one before another lane reads it.
struct WorldBuilder {
    mdn_world& w;
    __device__ void add(uint32_t kind, float cx, float cy, float cz, float ex, float ey, float ez, float vx, float vy,
                        float vz) {  // world.hpp:104-111
        __syncwarp();  // every lane's earlier stores to w are done
        const uint32_t slot = w.count;
        __syncwarp();  // every lane has read the count before it changes
        if (slot >= 16) return;
        w.count = slot + 1;
        mdn_obstacle& o = w.obstacles[slot];
        o.kind = kind;
        o.center[0] = cx; o.center[1] = cy; o.center[2] = cz;
        o.size[0] = ex; o.size[1] = ey; o.size[2] = ez;
        o.velocity[0] = vx; o.velocity[1] = vy; o.velocity[2] = vz;
    }
    __device__ void box(float cx, float cy, float cz, float ex, float ey, float ez) { add(0, cx, cy, cz, ex, ey, ez, 0, 0, 0); }
    __device__ void table(float x, float y, float hx, float hy, float top) {  // world.hpp:115-125
        const float slab = 0.08f, under = top - slab;
        box(x, y, top, hx, hy, slab);
        const float lx = hx - 0.12f, ly = hy - 0.12f, lh = 0.08f, lcz = under * 0.5f, lhz = under * 0.5f;
        box(x - lx, y - ly, lcz, lh, lh, lhz);
        box(x - lx, y + ly, lcz, lh, lh, lhz);
        box(x + lx, y - ly, lcz, lh, lh, lhz);
        box(x + lx, y + ly, lcz, lh, lh, lhz);
    }
    __device__ float route_y(float x, float distance) const { return w.goal[1] * (x / distance); }
    __device__ void doorway(float wall_x, float gap_y, float gap_z, float half_gap, float half_gap_z) {  // :129-137
        const float low_y = gap_y - half_gap, high_y = gap_y + half_gap;
        const float low_z = gap_z - half_gap_z, high_z = gap_z + half_gap_z;
        const float hx = 0.12f;
        box(wall_x, (-5.0f + low_y) * 0.5f, 2.5f, hx, (low_y + 5.0f) * 0.5f, 2.5f);
        box(wall_x, (high_y + 5.0f) * 0.5f, 2.5f, hx, (5.0f - high_y) * 0.5f, 2.5f);
        box(wall_x, 0, low_z * 0.5f, hx, 5.0f, low_z * 0.5f);
        box(wall_x, 0, (high_z + 5.0f) * 0.5f, hx, 5.0f, (5.0f - high_z) * 0.5f);
    }
};

__device__ __forceinline__ float challenge_span(float d) { return fminf(fmaxf(d, 3.0f), 10.0f); }  // world.hpp:225

// Mixed-capability lanes (families 19, 20; no reference generator, IEEE-exact
// operations only, identical to the oracle's restatement). Goal: a random
// horizontal direction (8 rejection tries) at distance dmin + dspan*U,
// clamped into the room.
__device__ __forceinline__ void clutter_goal(mdn_world& w, uint32_t& rng, float dmin, float dspan, float xmax) {
    float dx = 1.0f, dy = 0.0f;
    for (int attempt = 0; attempt < 8; attempt++) {
        const float ux = 2.0f * wurand(rng) - 1.0f, uy = 2.0f * wurand(rng) - 1.0f;
        const float norm = sqrtf(ux * ux + uy * uy);
        if (norm > 0.1f && norm <= 1.0f) {
            dx = ux / norm;
            dy = uy / norm;
            break;
        }
    }
    const float dist = dmin + dspan * wurand(rng);
    w.goal[0] = fminf(fmaxf(dist * dx, -1.5f), xmax);
    w.goal[1] = fminf(fmaxf(dist * dy, -4.5f), 4.5f);
    w.goal[2] = 1.0f + wurand(rng);
}
// Static boxes with centres in x[-2,-2+xspan] y[-5,5] z[0,4], half-extents
// U(0.2,1.0); redrawn (8 tries, else left out) unless 0.5 m clear of start and goal.
__device__ __forceinline__ void clutter_boxes(mdn_world& w, uint32_t& rng, int boxes, float xspan) {
    WorldBuilder b{w};
    for (int i = 0; i < boxes; i++)
        for (int attempt = 0; attempt < 8; attempt++) {
            const float cx = -2.0f + xspan * wurand(rng), cy = -5.0f + 10.0f * wurand(rng), cz = 4.0f * wurand(rng);
            const float ex = 0.2f + 0.8f * wurand(rng), ey = 0.2f + 0.8f * wurand(rng), ez = 0.2f + 0.8f * wurand(rng);
            const float size[3] = {ex, ey, ez};
            const float ds = box_distance(size, 0.0f - cx, 0.0f - cy, 1.5f - cz);
            const float dg = box_distance(size, w.goal[0] - cx, w.goal[1] - cy, w.goal[2] - cz);
            if (ds > 0.5f && dg > 0.5f) {
                b.box(cx, cy, cz, ex, ey, ez);
                break;
            }
        }
}
// Whether a bounded mover (centre c, unit direction d, amplitude) clears its
// whole swept segment (17 samples): the static boxes by radius + 0.05 m, the
// start by radius + 0.5 m and the goal by radius + 0.3 m. Called by a whole
// converged warp with identical arguments: lane l tests the (sample, box)
// pairs l, l + 32, ... (the last "box" of a sample stands for the start and
// goal tests) and the warp ANDs the results, which is the serial answer.
__device__ __forceinline__ bool mover_clear(const mdn_world& w, uint32_t statics, const float c[3], const float d[3],
                                            float radius, float amplitude) {
    const int lane = threadIdx.x & 31;
    const int per_sample = int(statics) + 1;
    bool ok = true;
    for (int q = lane; q < 17 * per_sample; q += 32) {
        const int k = q / per_sample, o = q % per_sample;
        const float f = amplitude * (float(k) / 8.0f - 1.0f);
        const float p[3] = {c[0] + d[0] * f, c[1] + d[1] * f, c[2] + d[2] * f};
        if (o < int(statics)) {
            const mdn_obstacle& ob = w.obstacles[o];
            if (!(box_distance(ob.size, p[0] - ob.center[0], p[1] - ob.center[1], p[2] - ob.center[2]) > radius + 0.05f))
                ok = false;
        } else {
            const float ds = len3(p[0] - 0.0f, p[1] - 0.0f, p[2] - 1.5f);
            const float dg = len3(p[0] - w.goal[0], p[1] - w.goal[1], p[2] - w.goal[2]);
            if (!(ds > radius + 0.5f) || !(dg > radius + 0.3f)) ok = false;
        }
    }
    return __all_sync(0xffffffffu, ok);
}
// Bounded moving spheres (kind 3, world.hpp:32-41) whose whole swept segment
// clears the boxes, start and goal (mover_clear; 8 tries each, else left out).
// Warp-cooperative: see mover_clear.
__device__ __forceinline__ void clutter_movers(mdn_world& w, uint32_t& rng, int movers) {
    const uint32_t statics = w.count;
    for (int i = 0; i < movers && w.count < 16; i++)
        for (int attempt = 0; attempt < 8; attempt++) {
            const float c[3] = {-2.0f + 10.0f * wurand(rng), -5.0f + 10.0f * wurand(rng), 0.5f + 3.0f * wurand(rng)};
            const float radius = 0.2f + 0.3f * wurand(rng);
            const float amplitude = 0.5f + 1.5f * wurand(rng);
            const float speed = 0.5f + 1.5f * wurand(rng);
            const float phase = 6.2831853f * wurand(rng);
            const float ux = 2.0f * wurand(rng) - 1.0f, uy = 2.0f * wurand(rng) - 1.0f, uz = 2.0f * wurand(rng) - 1.0f;
            const float norm = sqrtf(ux * ux + uy * uy + uz * uz);
            if (!(norm > 0.1f && norm <= 1.0f)) continue;
            const float d[3] = {ux / norm, uy / norm, uz / norm};
            if (mover_clear(w, statics, c, d, radius, amplitude)) {
                WorldBuilder{w}.add(3, c[0], c[1], c[2], radius, amplitude, phase, d[0] * speed, d[1] * speed,
                                    d[2] * speed);
                break;
            }
        }
}

// Family 18 (mixed capability, BASELINE configs 2 and 4): the generator family
// of global env gid - 50% static clutter (17), 25% long-goal rooms (19), 25%
// combined courses with movers (20).
__device__ __forceinline__ uint32_t mixed_lane_family(uint32_t gid) {
    return (gid & 3u) < 2u ? 17u : ((gid & 3u) == 2u ? 19u : 20u);
}

// wgenerate, world.hpp:299-318, with every family generator of world.hpp:138-291.
__device__ void generate_world_body(mdn_world& w, uint32_t seed, uint32_t family, float distance) {
    __syncwarp();  // stores of an earlier world or attempt are done before this one's
    uint32_t rng = seed ? seed : 1;
    w.seed = seed;
    w.family = family;
    w.count = family == 0 ? 0 : 8;
    w.goal[0] = distance;
    w.goal[1] = (wurand(rng) - 0.5f) * 2;
    w.goal[2] = 1.5f + (wurand(rng) - 0.5f) * 0.8f;
    w.wind[0] = w.wind[1] = w.wind[2] = 0;
    __syncwarp();  // the families below rewrite the count and goal set above, then read them
    WorldBuilder b{w};
    if (family == 4) {  // single doorway, :138-147
        w.count = 0;
        const float wall_x = distance * (0.42f + 0.16f * wurand(rng));
        const float rf = wall_x / distance;
        const float gap_y = w.goal[1] * rf + (wurand(rng) - 0.5f) * 1.20f;
        const float half_gap = 0.40f + 0.30f * wurand(rng);
        const float route_z = 1.5f + (w.goal[2] - 1.5f) * rf;
        const float gap_z = route_z + (wurand(rng) - 0.5f) * 0.20f;
        const float half_gap_z = 0.65f + 0.25f * wurand(rng);
        b.doorway(wall_x, gap_y, gap_z, half_gap, half_gap_z);
        return;
    }
    if (family == 5) {  // table or counter, :161-176
        w.count = 0;
        const float x = distance * (0.45f + 0.10f * wurand(rng));
        const float y = b.route_y(x, distance) + (wurand(rng) - 0.5f) * 0.20f;
        if (wurand(rng) < 0.5f) {
            const float hx = 0.55f + 0.20f * wurand(rng);
            const float hy = 0.75f + 0.20f * wurand(rng);
            const float top = 1.55f + 0.50f * wurand(rng);
            b.table(x, y, hx, hy, top);
        } else {
            const float hx = 0.60f + 0.20f * wurand(rng);
            const float hy = 0.80f + 0.20f * wurand(rng);
            const float height = 1.35f + 0.80f * wurand(rng);
            b.box(x, y, height * 0.5f, hx, hy, height * 0.5f);
        }
        return;
    }
    if (family == 6) {  // mixed, :177-201; call arguments drawn left to right (Metal/Apple clang order)
        w.count = 0;
        const float tx = distance * (0.46f + 0.08f * wurand(rng));
        const float ty = b.route_y(tx, distance) + (wurand(rng) - 0.5f) * 0.16f;
        const float thx = 0.58f + 0.10f * wurand(rng);
        const float thy = 0.76f + 0.10f * wurand(rng);
        const float ttop = 1.62f + 0.42f * wurand(rng);
        b.table(tx, ty, thx, thy, ttop);
        const float cx = distance * 0.22f;
        const float cy = b.route_y(cx, distance) - 1.30f;
        const float ch = 1.55f + 0.45f * wurand(rng);
        b.box(cx, cy, ch * 0.5f, 0.30f, 0.50f, ch * 0.5f);
        const float sx = distance * 0.72f;
        const float sy = b.route_y(sx, distance) + 1.35f;
        const float sr = 0.34f + 0.10f * wurand(rng);
        const float sz = 1.05f + 1.10f * wurand(rng);
        const float sign = wurand(rng) < 0.5f ? -1.0f : 1.0f;
        const float svy = sign * (0.18f + 0.16f * wurand(rng));
        b.add(1, sx, sy, sz, sr, sr, sr, 0, svy, 0);
        const float r0 = 0.20f + 0.08f * wurand(rng), r1 = 0.20f + 0.08f * wurand(rng);
        b.add(2, distance * 0.34f, b.route_y(distance * 0.34f, distance) + 2.05f, 2.5f, r0, r0, 2.5f, 0, 0, 0);
        b.add(2, distance * 0.82f, b.route_y(distance * 0.82f, distance) - 2.05f, 2.5f, r1, r1, 2.5f, 0, 0, 0);
        const float lx = distance * 0.74f;
        const float ly = b.route_y(lx, distance) - 0.88f;
        b.box(lx, ly, 0.48f, 0.34f, 0.30f, 0.48f);
        return;
    }
    if (family == 8) {  // two doorways, :148-160
        w.count = 0;
        for (uint32_t door = 0; door < 2; door++) {
            const float fraction = door == 0 ? 0.33f + 0.02f * (wurand(rng) - 0.5f) : 0.67f + 0.02f * (wurand(rng) - 0.5f);
            const float wall_x = distance * fraction;
            const float rf = wall_x / distance;
            const float gap_y = b.route_y(wall_x, distance) + (wurand(rng) - 0.5f) * 1.00f;
            const float route_z = 1.5f + (w.goal[2] - 1.5f) * rf;
            const float gap_z = route_z + (wurand(rng) - 0.5f) * 0.24f;
            const float half_gap = 0.40f + 0.30f * wurand(rng);
            const float half_gap_z = 0.65f + 0.25f * wurand(rng);
            b.doorway(wall_x, gap_y, gap_z, half_gap, half_gap_z);
        }
        return;
    }
    if (family == 10 || family == 11) {  // flying threat sphere, :202-222
        w.count = 0;
        const float drone_speed = 1.5f;
        uint32_t r2 = seed ^ 0x9e3779b9u;
        if (r2 == 0) r2 = 1;
        const float lateral = (wurand(r2) - 0.5f) * 0.20f;
        const float vertical = (wurand(r2) - 0.5f) * 0.16f;
        const uint32_t choice = wrng(r2) % 3;
        const float ts = choice == 0 ? 0.5f : (choice == 1 ? 1.0f : 2.0f);
        const float ttc = 0.7f + 0.8f * wurand(r2);
        const float combined = 0.18f + 0.35f;
        w.goal[0] = 4.0f; w.goal[1] = 0.0f; w.goal[2] = 1.5f;
        if (family == 10)
            b.add(1, (drone_speed + ts) * ttc + combined, lateral, 1.5f + vertical, 0.35f, 0.35f, 0.35f, -ts, 0, 0);
        else
            b.add(1, drone_speed * ttc, -ts * ttc + lateral, 1.5f + vertical, 0.35f, 0.35f, 0.35f, 0, ts, 0);
        return;
    }
    if (family == 14 || family == 15 || family == 16) {  // challenge layouts, :226-291
        w.count = 0;
        const float difficulty = wurand(rng);
        const float span = challenge_span(distance);
        w.goal[0] = span * (0.90f + 0.10f * wurand(rng));
        w.goal[1] = (wurand(rng) - 0.5f) * 1.20f;
        w.goal[2] = 1.10f + 0.80f * wurand(rng);
        if (family == 14) {
            const float wall_x = w.goal[0] * (0.24f + 0.04f * wurand(rng));
            const float gap_x = w.goal[0] * (0.70f + 0.08f * difficulty);
            const float lane_width = 1.80f - 0.80f * difficulty;
            const float lane_edge = 5.0f - lane_width;
            const float wall_y = (-5.0f + lane_edge) * 0.5f;
            const float wall_half_y = (lane_edge + 5.0f) * 0.5f;
            b.box(wall_x, wall_y, 2.5f, 0.15f, wall_half_y, 2.5f);
            b.box((wall_x + gap_x) * 0.5f, lane_edge + 0.03f, 2.5f, (gap_x - wall_x) * 0.5f + 0.15f, 0.15f, 2.5f);
        } else if (family == 15) {
            const float wall_1 = w.goal[0] * (0.16f + 0.02f * wurand(rng));
            const float wall_2 = w.goal[0] * 0.85f;
            const float gap_1 = -(0.60f + 0.80f * difficulty);
            const float gap_2 = +(0.60f + 0.80f * difficulty);
            const float gap_half = 0.85f - 0.30f * difficulty;
            const float gap_z = 1.50f;
            const float gap_half_z = 0.85f - 0.10f * difficulty;
            b.doorway(wall_1, gap_1, gap_z, gap_half, gap_half_z);
            b.doorway(wall_2, gap_2, gap_z, gap_half, gap_half_z);
            const float table_x = w.goal[0] * 0.50f;
            const float table_y = (wurand(rng) - 0.5f) * 0.20f;
            const float thx = fminf(0.45f, w.goal[0] * 0.06f);
            const float thy = 0.60f + 0.20f * difficulty;
            const float ttop = 1.45f + 0.25f * difficulty;
            b.table(table_x, table_y, thx, thy, ttop);
            b.box(w.goal[0] * 0.38f, 3.75f, 0.55f, 0.22f, 0.35f, 0.55f);
            b.box(w.goal[0] * 0.50f, -3.80f, 0.80f, 0.25f, 0.35f, 0.80f);
            b.box(w.goal[0] * 0.62f, 3.70f, 0.50f, 0.22f, 0.40f, 0.50f);
        } else {
            const float low_x = w.goal[0] * (0.14f + 0.02f * (1.0f - difficulty));
            const float overhead_x = w.goal[0] * (0.46f + 0.02f * difficulty);
            const float choice_x = w.goal[0] * (0.76f + 0.02f * difficulty);
            const float low_top = 1.50f + 0.25f * difficulty;
            const float overhead_bottom = 2.80f - 0.20f * difficulty;
            const float choice_half_z = 0.10f + 0.05f * difficulty;
            b.box(low_x, 0, low_top * 0.5f, 0.12f, 5.0f, low_top * 0.5f);
            const float ohz = (5.0f - overhead_bottom) * 0.5f;
            b.box(overhead_x, 0, overhead_bottom + ohz, 0.12f, 5.0f, ohz);
            b.box(choice_x, 0, 2.0f + choice_half_z, 0.10f, 5.0f, choice_half_z);
        }
        return;
    }
    if (family == 17) {  // baseline clutter (no reference generator; see oracle/mdn_oracle.c)
        w.count = 0;
        float dx = 1.0f, dy = 0.0f;
        for (int attempt = 0; attempt < 8; attempt++) {
            const float ux = 2.0f * wurand(rng) - 1.0f, uy = 2.0f * wurand(rng) - 1.0f;
            const float norm = sqrtf(ux * ux + uy * uy);
            if (norm > 0.1f && norm <= 1.0f) {
                dx = ux / norm;
                dy = uy / norm;
                break;
            }
        }
        const float dist = 2.0f + 6.0f * wurand(rng);
        w.goal[0] = fminf(fmaxf(dist * dx, -1.5f), 7.5f);
        w.goal[1] = fminf(fmaxf(dist * dy, -4.5f), 4.5f);
        w.goal[2] = 1.0f + wurand(rng);
        for (int i = 0; i < 16; i++)
            for (int attempt = 0; attempt < 8; attempt++) {
                const float cx = -2.0f + 10.0f * wurand(rng), cy = -5.0f + 10.0f * wurand(rng), cz = 4.0f * wurand(rng);
                const float ex = 0.2f + 0.8f * wurand(rng), ey = 0.2f + 0.8f * wurand(rng), ez = 0.2f + 0.8f * wurand(rng);
                const float size[3] = {ex, ey, ez};
                const float ds = box_distance(size, 0.0f - cx, 0.0f - cy, 1.5f - cz);
                const float dg = box_distance(size, w.goal[0] - cx, w.goal[1] - cy, w.goal[2] - cz);
                if (ds > 0.5f && dg > 0.5f) {
                    b.box(cx, cy, cz, ex, ey, ez);
                    break;
                }
            }
        return;
    }
    if (family == 19) {  // long-goal room (see clutter_goal)
        w.count = 0;
        clutter_goal(w, rng, 2.0f, 10.0f, 13.5f);
        clutter_boxes(w, rng, 16, 16.0f);
        return;
    }
    if (family == 20) {  // combined course: 12 static boxes + 4 movers
        w.count = 0;
        clutter_goal(w, rng, 2.0f, 6.0f, 7.5f);
        clutter_boxes(w, rng, 12, 10.0f);
        clutter_movers(w, rng, 4);
        return;
    }
    // Families 0-3 (and any other id): 16 random primitives, :311-317.
    for (int i = 0; i < 16; i++) {
        mdn_obstacle& o = w.obstacles[i];
        o.kind = family == 2 ? 2 : (family == 3 ? 1 : 0);
        o.center[0] = 1.2f + wurand(rng) * fmaxf(0.1f, distance - 2.2f);
        o.center[1] = (wurand(rng) - 0.5f) * 7;
        o.center[2] = family == 2 ? 2.5f : 0.6f + wurand(rng) * 3;
        o.size[0] = 0.2f + wurand(rng) * 0.35f;
        o.size[1] = 0.3f + wurand(rng) * 0.55f;
        o.size[2] = family == 2 ? 2.5f : 0.2f + wurand(rng) * 0.75f;
        o.velocity[0] = 0;
        o.velocity[1] = family == 3 ? (wurand(rng) - 0.5f) * 0.8f : 0;
        o.velocity[2] = 0;
    }
}

// The generator with a warp barrier on exit (see WorldBuilder).
__device__ void generate_world(mdn_world& w, uint32_t seed, uint32_t family, float distance) {
    generate_world_body(w, seed, family, distance);
    __syncwarp();  // the new world is complete for every lane before anything reads it
}

// Training-only family mixture, world.hpp:293-298.
__device__ __forceinline__ uint32_t training_family(uint32_t family, uint32_t& rng) {
    if (family == 7) return wrng(rng) % 7;
    if (family == 9 || family == 12) {
        const uint32_t c = wrng(rng) % 4;
        return c < 2 ? 4 : (c == 2 ? 5 : wrng(rng) % 7);
    }
    if (family == 13) {
        const uint32_t c = wrng(rng) % 6;
        if (c < 2) return 4;
        if (c == 2) return 5;
        if (c == 3) return wrng(rng) % 7;
        return c == 4 ? 10 : 11;
    }
    return family;
}

// Clean-sensing training environments (sim.metal:17-21): the even
// environments of families 12 and 13 and, with delay rehearsal on, mode-22
// environments of even four-environment groups. Never in evaluation.
__device__ __forceinline__ bool clean_env(const SimArgs& a, uint32_t gid) {
    const mdn_sim_config& c = a.cfg;
    if (c.eval != 0) return false;
    const bool clean_family = (c.family == 12 || c.family == 13) && gid % 2 == 0;
    const bool rehearsal = a.delay_rehearsal != 0 && c.mode == 22 && (gid / 4) % 2 == 0;
    return clean_family || rehearsal;
}

// Copy env i's obstacle block into the structure-of-arrays mirror.
__device__ __forceinline__ void mirror_world(const SimArgs& a, uint32_t i) {
    const mdn_world& w = a.worlds[i];
    const float* words = reinterpret_cast<const float*>(w.obstacles);
    for (int k = 0; k < 160; k++) a.world_soa[size_t(k) * a.n + i] = words[k];
    a.world_soa[size_t(160) * a.n + i] = __uint_as_float(w.count);
}
// The same from a whole warp, words split over the lanes (word 160 = count).
__device__ __forceinline__ void mirror_world_warp(const SimArgs& a, uint32_t i) {
    const float* words = reinterpret_cast<const float*>(&a.worlds[i]);
    static_assert(offsetof(mdn_world, count) == 160 * sizeof(float), "count follows the 16 obstacles");
    for (int k = threadIdx.x & 31; k < 161; k += 32) a.world_soa[size_t(k) * a.n + i] = words[k];
}
// Whole-warp copy of one world (169 words), then a warp barrier, so that
// every lane sees the copy.
__device__ __forceinline__ void copy_world_warp(mdn_world& dst, const mdn_world& src) {
    constexpr int kWords = int(sizeof(mdn_world) / sizeof(uint32_t));
    const uint32_t* s = reinterpret_cast<const uint32_t*>(&src);
    uint32_t* d = reinterpret_cast<uint32_t*>(&dst);
    for (int k = threadIdx.x & 31; k < kWords; k += 32) d[k] = s[k];
    __syncwarp();
}

// sim_reset_one (sim.metal:55-94) for one environment, except the 8x320 range
// ring refill, which the caller performs cooperatively (returns true when the
// ring must be refilled with 12 m). Run by a whole converged warp for the same
// environment: every lane computes the same values and stores them (identical
// stores to one address), and the generators' heavy checks are split over the
// lanes (mover_clear). The world is generated in `w`, the warp's copy in shared
// memory (the generators read back what they wrote, which in global memory
// would cost an L2 round trip each time), and then stored to a.worlds[i].
__device__ bool reset_env(const SimArgs& a, uint32_t i, bool first, mdn_world& w) {
    const mdn_sim_config& c = a.cfg;
    const uint32_t gid = a.env_base + i;
    mdn_sim_run& run = a.runs[i];
    mdn_physics_state& s = a.states[i];
    copy_world_warp(w, a.worlds[i]);  // fields a generator leaves alone keep their bytes
    uint32_t rng = first ? (c.seed + gid * 747796405u + 2891336453u) : run.rng;
    const uint32_t family = c.family == 18u ? mixed_lane_family(gid) : training_family(c.family, rng);
    generate_world(w, wrng(rng), family, c.distance);
    w.wind[0] = clean_env(a, gid) ? 0.0f : c.wind;
    w.wind[1] = 0;
    w.wind[2] = 0;
    for (int j = 0; j < 3; j++) {
        s.position[j] = j == 2 ? 1.5f : 0;
        s.linear_velocity[j] = 0;
        s.angular_velocity_body[j] = 0;
        run.desired_velocity[j] = 0;
        run.reference_position[j] = s.position[j];
    }
    s.orientation_wxyz[0] = 1;
    s.orientation_wxyz[1] = s.orientation_wxyz[2] = s.orientation_wxyz[3] = 0;
    const mdn_physics_params& p = *a.physics;
    float hover[4];
    if (!a.runtime.enabled) {
        const float target = p.mass * 9.81f / 4;
        const float c0 = p.rotor_thrust_coefficients[0], c1 = p.rotor_thrust_coefficients[1],
                    c2 = p.rotor_thrust_coefficients[2];
        const float h = clampf((-c1 + sqrtf(c1 * c1 - 4 * c2 * (c0 - target))) / (2 * c2), p.action_min, p.action_max);
        for (int j = 0; j < 4; j++) hover[j] = h;
    } else {
        // The episode's own plant (sim.metal:62-69), then per-rotor hover at
        // its thrust curve (sim.metal:75-80).
        mdn_physics_params& ep = a.env_physics[i];
        ep = p;
        if (a.runtime.domain_amplitude > 0.0f) {
            uint32_t drng = domain_episode_seed(a.runtime, c.seed, gid, first ? 0u : run.episodes);
            mdn_physics_params varied;
            if (sample_domain(p, drng, a.runtime.domain_amplitude, a.runtime.domain_range, varied)) ep = varied;
            else ep.mass = __int_as_float(0x7fc00000);
        }
        const float target = ep.mass * 9.81f / 4;
        for (int rotor = 0; rotor < 4; rotor++) {
            const float c0 = ep.rotor_thrust_coefficients[3 * rotor], c1 = ep.rotor_thrust_coefficients[3 * rotor + 1],
                        c2 = ep.rotor_thrust_coefficients[3 * rotor + 2];
            const float disc = c1 * c1 - 4 * c2 * (c0 - target);
            hover[rotor] = disc >= 0.0f ? clampf((-c1 + sqrtf(disc)) / (2 * c2), ep.action_min, ep.action_max)
                                        : ep.action_max;
        }
    }
    for (int j = 0; j < 16; j++) run.hidden[j] = a.raptor->initial_hidden_state[j];
    for (int j = 0; j < 4; j++) {
        s.rpm[j] = hover[j];
        run.motors[j] = 0;
        run.previous_nav[j] = 0;
    }
    if (family == 10 || family == 11) {
        s.linear_velocity[0] = c.speed;
        run.desired_velocity[0] = c.speed;
        run.previous_nav[0] = 1.0f;
    }
    float* cmd = a.commands + size_t(i) * kFrames * kActions;
    for (int j = 0; j < kFrames * kActions; j++) cmd[j] = 0;
    run.yaw = 0;
    run.rng = rng;
    run.steps = 0;
    run.path = run.elapsed = run.peak_speed = 0;
    run.min_clearance = 12;
    run.initial_distance = len3(w.goal[0], w.goal[1], w.goal[2] - 1.5f);
    if (first) {
        run.successes = run.collisions = run.timeouts = run.episodes = 0;
        run.success_time = run.total_path = run.total_elapsed = run.final_progress = 0;
        float* pose = a.poses + size_t(i) * kFrames * 12;
        for (int j = 0; j < kFrames * 12; j++) pose[j] = 0;
    }
    __syncwarp();
    copy_world_warp(a.worlds[i], w);
    return true;
}

// sim_apply_challenge_world (sim.metal:95-122): after the procedural reset,
// replace env i's world by the frozen bank level that its schedule names for
// `slot` (0 at sim_reset, tick + 1 for a reset inside step `tick`), or, for the
// level id 0xffffffff, by a rehearsal world of the short-task mixture (training
// family 12 on even, 13 on odd environments, 4 m goals). A slot beyond the
// schedule or an unknown level id keeps the procedural world and leaves the
// env's active id unchanged, as the reference does.
__device__ __forceinline__ void apply_challenge_world(const SimArgs& a, uint32_t i, uint32_t slot) {
    if (a.bank_count == 0 || slot >= a.bank_stride) return;
    const uint32_t gid = a.env_base + i;
    const uint32_t level = a.bank_schedule[size_t(i) * a.bank_stride + slot];
    mdn_sim_run& run = a.runs[i];
    mdn_world& w = a.worlds[i];
    if (level == 0xffffffffu) {
        uint32_t rng = run.rng;
        const uint32_t family = training_family(gid % 2 == 0 ? 12u : 13u, rng);
        generate_world(w, wrng(rng), family, 4.0f);
        run.rng = rng;
    } else {
        if (level >= a.bank_count) return;
        w = a.bank_worlds[level];
        __syncwarp();  // the bank world's wind is stored by every lane before it is overwritten
    }
    w.wind[0] = clean_env(a, gid) ? 0.0f : a.cfg.wind;
    w.wind[1] = 0;
    w.wind[2] = 0;
    run.initial_distance = len3(w.goal[0], w.goal[1], w.goal[2] - 1.5f);
    if (w.family == 10 || w.family == 11) {
        a.states[i].linear_velocity[0] = a.cfg.speed;
        run.desired_velocity[0] = a.cfg.speed;
        run.previous_nav[0] = 1.0f;
    }
    a.bank_active[i] = level;
}

}  // namespace mdn
