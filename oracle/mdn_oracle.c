/*
 * TEST INFRASTRUCTURE ONLY - the CPU checker for the CUDA path. Never linked
 * into the product; only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg load it.
 *
 * A scalar C restatement of the reference algorithm on the rollout/PPO path.
 * Every function cites the reference file:line it restates. Expressions keep
 * the reference's evaluation order and are compiled without FMA contraction
 * (oracle/Makefile), so the +,-,*,/,sqrt parts reproduce the reference's
 * float results bit for bit; transcendental calls use the C library's float
 * functions, as the reference CPU path does (std::exp(float) == expf etc.).
 *
 * Pinned by tests/test_oracle_pin.py against the reference compiled unmodified
 * (oracle/_ref) and against the reference's golden fixtures.
 */
#include "mdn_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define NPIX 320u
#define NFRAMES 8u
#define AOBS 184u
#define COBS 32u
#define HID 64u
#define ACT 4u
#define LOG_TWO_PI 1.8378770664093453f
/* fixed_ppo offsets, ppo.hpp:35-45, for the 184/64/4 actor and 32/64/1 critic */
#define A_B1 (HID * AOBS)
#define A_W2 (A_B1 + HID)
#define A_B2 (A_W2 + ACT * HID)
#define A_LS (A_B2 + ACT)
#define A_P (A_LS + ACT)
#define C_B1 (HID * COBS)
#define C_W2 (C_B1 + HID)
#define C_B2 (C_W2 + HID)
#define C_P (C_B2 + 1)

static const float REF_ROOM[6] = {-2.0f, -5.0f, 0.0f, 14.0f, 5.0f, 5.0f};

/* std::min / std::max semantics (cpu_reference.hpp uses them): b<a?b:a, a<b?b:a */
static inline float smin(float a, float b) { return b < a ? b : a; }
static inline float smax(float a, float b) { return a < b ? b : a; }
static inline float clampf_(float x, float lo, float hi) { return smax(lo, smin(hi, x)); } /* cpu_reference.hpp:72-74 */
static inline float len3(float x, float y, float z) { return sqrtf(x * x + y * y + z * z); } /* world.hpp:23-24 */

/* ------------------------------------------------------------------ world */
uint32_t o_wrng(uint32_t* s) { /* world.hpp:30 */
    *s ^= *s << 13;
    *s ^= *s >> 17;
    *s ^= *s << 5;
    return *s;
}
float o_wurand(uint32_t* s) { return (float)(o_wrng(s) >> 8) * (1.0f / 16777216.0f); } /* world.hpp:31 */

void o_wc(const mdn_obstacle* o, float t, float out[3]) { /* world.hpp:32-41 */
    if (o->kind == 3) {
        const float speed = len3(o->velocity[0], o->velocity[1], o->velocity[2]), amplitude = o->size[1];
        if (speed <= 1e-8f || amplitude <= 1e-8f) {
            out[0] = o->center[0]; out[1] = o->center[1]; out[2] = o->center[2];
            return;
        }
        const float offset = amplitude * sinf(t * speed / amplitude + o->size[2]) / speed;
        out[0] = o->center[0] + o->velocity[0] * offset;
        out[1] = o->center[1] + o->velocity[1] * offset;
        out[2] = o->center[2] + o->velocity[2] * offset;
        return;
    }
    out[0] = o->center[0] + t * o->velocity[0];
    out[1] = o->center[1] + t * o->velocity[1];
    out[2] = o->center[2] + t * o->velocity[2];
}

float o_wray_sphere(const float p[3], const float d[3], const float c[3], float r) { /* world.hpp:42-47 */
    const float q[3] = {p[0] - c[0], p[1] - c[1], p[2] - c[2]};
    const float b = q[0] * d[0] + q[1] * d[1] + q[2] * d[2];
    const float k = (q[0] * q[0] + q[1] * q[1] + q[2] * q[2]) - r * r;
    const float disc = b * b - k;
    if (disc < 0) return 1000;
    const float lo = -b - sqrtf(disc), hi = -b + sqrtf(disc);
    return lo >= 0 ? lo : (hi >= 0 ? hi : 1000);
}

float o_wray_box(const float p[3], const float d[3], const float c[3], const float e[3]) { /* world.hpp:48-57 */
    float lo = -1e20f, hi = 1e20f;
    const float pp[3] = {p[0] - c[0], p[1] - c[1], p[2] - c[2]};
    for (int j = 0; j < 3; j++) {
        if (fabsf(d[j]) < 1e-8f) {
            if (fabsf(pp[j]) > e[j]) return 1000;
        } else {
            const float a = (-e[j] - pp[j]) / d[j], b = (e[j] - pp[j]) / d[j];
            lo = fmaxf(lo, fminf(a, b));
            hi = fminf(hi, fmaxf(a, b));
        }
    }
    if (hi < fmaxf(lo, 0.0f)) return 1000;
    return lo >= 0 ? lo : hi;
}

float o_wray_cylinder(const float p[3], const float d[3], const float c[3], float r, float h) { /* world.hpp:58-70 */
    const float q[3] = {p[0] - c[0], p[1] - c[1], p[2] - c[2]};
    const float a = d[0] * d[0] + d[1] * d[1], b = q[0] * d[0] + q[1] * d[1], k = q[0] * q[0] + q[1] * q[1] - r * r;
    float best = 1000;
    const float disc = b * b - a * k;
    if (a > 1e-10f && disc >= 0) {
        const float roots[2] = {(-b - sqrtf(disc)) / a, (-b + sqrtf(disc)) / a};
        for (int j = 0; j < 2; j++) {
            const float t = roots[j];
            if (t >= 0 && fabsf(q[2] + t * d[2]) <= h) best = fminf(best, t);
        }
    }
    if (fabsf(d[2]) > 1e-8f)
        for (int sign = -1; sign <= 1; sign += 2) {
            const float t = ((float)sign * h - q[2]) / d[2];
            const float x = q[0] + t * d[0], y = q[1] + t * d[1];
            if (t >= 0 && x * x + y * y <= r * r) best = fminf(best, t);
        }
    return best;
}

/* Room as a box: centre and half extents computed in float from the bounds.
 * For the reference room this is exactly (6,0,2.5) / (8,5,2.5) (world.hpp:74). */
static void room_box(const float* room, float c[3], float e[3]) {
    if (!room) room = REF_ROOM;
    for (int j = 0; j < 3; j++) {
        c[j] = (room[j] + room[3 + j]) * 0.5f;
        e[j] = (room[3 + j] - room[j]) * 0.5f;
    }
}

float o_wray(const mdn_world* w, const float* room, const float p[3], const float d[3], float t) { /* world.hpp:71-83 */
    float best = 12;
    float rc[3], re[3];
    room_box(room, rc, re);
    best = fminf(best, o_wray_box(p, d, rc, re));
    for (uint32_t i = 0; i < w->count; i++) {
        const mdn_obstacle* o = &w->obstacles[i];
        float c[3];
        o_wc(o, t, c);
        float hit = 1000;
        if (o->kind == 0) hit = o_wray_box(p, d, c, o->size);
        if (o->kind == 1 || o->kind == 3) hit = o_wray_sphere(p, d, c, o->size[0]);
        if (o->kind == 2) hit = o_wray_cylinder(p, d, c, o->size[0], o->size[2]);
        best = fminf(best, hit);
    }
    return fmaxf(0.0f, best);
}

/* world.hpp:84-99. argmin (optional): index of the first term attaining the
 * minimum, -1 for the room walls. */
float o_wclearance(const mdn_world* w, const float* room, const float p[3], float t, int32_t* argmin) {
    if (!room) room = REF_ROOM;
    float best = fminf(fminf(p[0] - room[0], room[3] - p[0]), fminf(fminf(p[1] - room[1], room[4] - p[1]),
                                                                     fminf(p[2] - room[2], room[5] - p[2]))) - 0.18f;
    int32_t id = -1;
    for (uint32_t i = 0; i < w->count; i++) {
        const mdn_obstacle* o = &w->obstacles[i];
        float c[3];
        o_wc(o, t, c);
        const float q[3] = {p[0] - c[0], p[1] - c[1], p[2] - c[2]};
        float distance;
        if (o->kind == 1 || o->kind == 3) {
            distance = len3(q[0], q[1], q[2]) - o->size[0];
        } else if (o->kind == 2) {
            const float a = sqrtf(q[0] * q[0] + q[1] * q[1]) - o->size[0], b = fabsf(q[2]) - o->size[2];
            distance = sqrtf(fmaxf(a, 0.0f) * fmaxf(a, 0.0f) + fmaxf(b, 0.0f) * fmaxf(b, 0.0f)) + fminf(fmaxf(a, b), 0.0f);
        } else {
            const float k[3] = {fabsf(q[0]) - o->size[0], fabsf(q[1]) - o->size[1], fabsf(q[2]) - o->size[2]};
            distance = len3(fmaxf(k[0], 0.0f), fmaxf(k[1], 0.0f), fmaxf(k[2], 0.0f)) +
                       fminf(fmaxf(k[0], fmaxf(k[1], k[2])), 0.0f);
        }
        const float cand = distance - 0.18f;
        if (cand < best) id = (int32_t)i;
        best = fminf(best, cand);
    }
    if (argmin) *argmin = id;
    return best;
}

/* The reference room constant in wclearance is p.x+2, 14-p.x ... (world.hpp:85):
 * p - (-2) == p + 2 exactly in float, so the generic bounds form above is the
 * same arithmetic for the reference room. */

static void wadd(mdn_world* w, uint32_t kind, float cx, float cy, float cz, float ex, float ey, float ez, float vx,
                 float vy, float vz) { /* world.hpp:104-111 */
    if (w->count >= 16) return;
    mdn_obstacle* o = &w->obstacles[w->count++];
    o->kind = kind;
    o->center[0] = cx; o->center[1] = cy; o->center[2] = cz;
    o->size[0] = ex; o->size[1] = ey; o->size[2] = ez;
    o->velocity[0] = vx; o->velocity[1] = vy; o->velocity[2] = vz;
}
static void wadd_box(mdn_world* w, float cx, float cy, float cz, float ex, float ey, float ez) { /* world.hpp:112-114 */
    wadd(w, 0, cx, cy, cz, ex, ey, ez, 0, 0, 0);
}
static void wadd_table(mdn_world* w, float x, float y, float half_x, float half_y, float top_z) { /* world.hpp:115-125 */
    const float slab_half_z = 0.08f;
    const float underside = top_z - slab_half_z;
    wadd_box(w, x, y, top_z, half_x, half_y, slab_half_z);
    const float leg_x = half_x - 0.12f, leg_y = half_y - 0.12f, leg_half = 0.08f;
    const float leg_center_z = underside * 0.5f, leg_half_z = underside * 0.5f;
    wadd_box(w, x - leg_x, y - leg_y, leg_center_z, leg_half, leg_half, leg_half_z);
    wadd_box(w, x - leg_x, y + leg_y, leg_center_z, leg_half, leg_half, leg_half_z);
    wadd_box(w, x + leg_x, y - leg_y, leg_center_z, leg_half, leg_half, leg_half_z);
    wadd_box(w, x + leg_x, y + leg_y, leg_center_z, leg_half, leg_half, leg_half_z);
}
static int g_args_right_to_left = 0;
void o_set_argument_order(int right_to_left) { g_args_right_to_left = right_to_left; }
static float wroute_y(const mdn_world* w, float x, float distance) { return w->goal[1] * (x / distance); } /* world.hpp:126-128 */
static void wadd_doorway(mdn_world* w, float wall_x, float gap_y, float gap_z, float half_gap, float half_gap_z) {
    /* world.hpp:129-137 */
    const float low_y = gap_y - half_gap, high_y = gap_y + half_gap;
    const float low_z = gap_z - half_gap_z, high_z = gap_z + half_gap_z;
    const float wall_half_x = 0.12f;
    wadd_box(w, wall_x, (-5.0f + low_y) * 0.5f, 2.5f, wall_half_x, (low_y + 5.0f) * 0.5f, 2.5f);
    wadd_box(w, wall_x, (high_y + 5.0f) * 0.5f, 2.5f, wall_half_x, (5.0f - high_y) * 0.5f, 2.5f);
    wadd_box(w, wall_x, 0, low_z * 0.5f, wall_half_x, 5.0f, low_z * 0.5f);
    wadd_box(w, wall_x, 0, (high_z + 5.0f) * 0.5f, wall_half_x, 5.0f, (5.0f - high_z) * 0.5f);
}
static void wgenerate_doorway(mdn_world* w, uint32_t* rng, float distance) { /* world.hpp:138-147 */
    const float wall_x = distance * (0.42f + 0.16f * o_wurand(rng));
    const float route_fraction = wall_x / distance;
    const float gap_y = w->goal[1] * route_fraction + (o_wurand(rng) - 0.5f) * 1.20f;
    const float half_gap = 0.40f + 0.30f * o_wurand(rng);
    const float route_z = 1.5f + (w->goal[2] - 1.5f) * route_fraction;
    const float gap_z = route_z + (o_wurand(rng) - 0.5f) * 0.20f;
    const float half_gap_z = 0.65f + 0.25f * o_wurand(rng);
    wadd_doorway(w, wall_x, gap_y, gap_z, half_gap, half_gap_z);
}
static void wgenerate_two_doorways(mdn_world* w, uint32_t* rng, float distance) { /* world.hpp:148-160 */
    for (uint32_t door = 0; door < 2; door++) {
        const float fraction = door == 0 ? 0.33f + 0.02f * (o_wurand(rng) - 0.5f) : 0.67f + 0.02f * (o_wurand(rng) - 0.5f);
        const float wall_x = distance * fraction;
        const float route_fraction = wall_x / distance;
        const float gap_y = wroute_y(w, wall_x, distance) + (o_wurand(rng) - 0.5f) * 1.00f;
        const float route_z = 1.5f + (w->goal[2] - 1.5f) * route_fraction;
        const float gap_z = route_z + (o_wurand(rng) - 0.5f) * 0.24f;
        const float half_gap = 0.40f + 0.30f * o_wurand(rng);
        const float half_gap_z = 0.65f + 0.25f * o_wurand(rng);
        wadd_doorway(w, wall_x, gap_y, gap_z, half_gap, half_gap_z);
    }
}
static void wgenerate_table_or_counter(mdn_world* w, uint32_t* rng, float distance) { /* world.hpp:161-176 */
    const float x = distance * (0.45f + 0.10f * o_wurand(rng));
    const float y = wroute_y(w, x, distance) + (o_wurand(rng) - 0.5f) * 0.20f;
    if (o_wurand(rng) < 0.5f) {
        const float half_x = 0.55f + 0.20f * o_wurand(rng);
        const float half_y = 0.75f + 0.20f * o_wurand(rng);
        const float top_z = 1.55f + 0.50f * o_wurand(rng);
        wadd_table(w, x, y, half_x, half_y, top_z);
    } else {
        const float half_x = 0.60f + 0.20f * o_wurand(rng);
        const float half_y = 0.80f + 0.20f * o_wurand(rng);
        const float height = 1.35f + 0.80f * o_wurand(rng);
        wadd_box(w, x, y, height * 0.5f, half_x, half_y, height * 0.5f);
    }
}
static void wgenerate_mixed(mdn_world* w, uint32_t* rng, float distance) { /* world.hpp:177-201 */
    const float table_x = distance * (0.46f + 0.08f * o_wurand(rng));
    const float table_y = wroute_y(w, table_x, distance) + (o_wurand(rng) - 0.5f) * 0.16f;
    /* The reference draws these three inside one call's argument list, whose
     * evaluation order C++ leaves unspecified. The reference platforms (Apple
     * clang for the CPU path, Metal for the GPU path) evaluate left to right,
     * which is the order used here and by the CUDA kernels. g++ evaluates right
     * to left; o_set_argument_order(1) reproduces a g++ build of the reference
     * so the pin test can compare against oracle/_ref. */
    float t_hx, t_hy, t_top;
    if (g_args_right_to_left) {
        t_top = 1.62f + 0.42f * o_wurand(rng);
        t_hy = 0.76f + 0.10f * o_wurand(rng);
        t_hx = 0.58f + 0.10f * o_wurand(rng);
    } else {
        t_hx = 0.58f + 0.10f * o_wurand(rng);
        t_hy = 0.76f + 0.10f * o_wurand(rng);
        t_top = 1.62f + 0.42f * o_wurand(rng);
    }
    wadd_table(w, table_x, table_y, t_hx, t_hy, t_top);
    const float counter_x = distance * 0.22f;
    const float counter_y = wroute_y(w, counter_x, distance) - 1.30f;
    const float counter_h = 1.55f + 0.45f * o_wurand(rng);
    wadd_box(w, counter_x, counter_y, counter_h * 0.5f, 0.30f, 0.50f, counter_h * 0.5f);
    const float sphere_x = distance * 0.72f;
    const float sphere_y = wroute_y(w, sphere_x, distance) + 1.35f;
    const float sphere_r = 0.34f + 0.10f * o_wurand(rng);
    const float sphere_z = 1.05f + 1.10f * o_wurand(rng);
    const float sign = o_wurand(rng) < 0.5f ? -1.0f : 1.0f;
    const float sphere_vy = sign * (0.18f + 0.16f * o_wurand(rng));
    wadd(w, 1, sphere_x, sphere_y, sphere_z, sphere_r, sphere_r, sphere_r, 0, sphere_vy, 0);
    const float pole_r0 = 0.20f + 0.08f * o_wurand(rng), pole_r1 = 0.20f + 0.08f * o_wurand(rng);
    wadd(w, 2, distance * 0.34f, wroute_y(w, distance * 0.34f, distance) + 2.05f, 2.5f, pole_r0, pole_r0, 2.5f, 0, 0, 0);
    wadd(w, 2, distance * 0.82f, wroute_y(w, distance * 0.82f, distance) - 2.05f, 2.5f, pole_r1, pole_r1, 2.5f, 0, 0, 0);
    const float low_box_x = distance * 0.74f;
    const float low_box_y = wroute_y(w, low_box_x, distance) - 0.88f;
    wadd_box(w, low_box_x, low_box_y, 0.48f, 0.34f, 0.30f, 0.48f);
}
static void wgenerate_threat_sphere(mdn_world* w, uint32_t seed, uint32_t family) { /* world.hpp:202-222 */
    const float drone_speed = 1.5f;
    uint32_t rng = seed ^ 0x9e3779b9u;
    if (rng == 0) rng = 1;
    const float lateral = (o_wurand(&rng) - 0.5f) * 0.20f;
    const float vertical = (o_wurand(&rng) - 0.5f) * 0.16f;
    const uint32_t speed_choice = o_wrng(&rng) % 3;
    const float threat_speed = speed_choice == 0 ? 0.5f : (speed_choice == 1 ? 1.0f : 2.0f);
    const float nominal_ttc = 0.7f + 0.8f * o_wurand(&rng);
    const float combined_radius = 0.18f + 0.35f;
    float cx, cy, cz, vx = 0, vy = 0;
    if (family == 10) {
        cx = (drone_speed + threat_speed) * nominal_ttc + combined_radius; cy = lateral; cz = 1.5f + vertical;
        vx = -threat_speed;
    } else {
        cx = drone_speed * nominal_ttc; cy = -threat_speed * nominal_ttc + lateral; cz = 1.5f + vertical;
        vy = threat_speed;
    }
    w->goal[0] = 4.0f; w->goal[1] = 0.0f; w->goal[2] = 1.5f;
    wadd(w, 1, cx, cy, cz, 0.35f, 0.35f, 0.35f, vx, vy, 0);
}
static float wchallenge_distance(float d) { return fminf(fmaxf(d, 3.0f), 10.0f); } /* world.hpp:225 */
static void wgenerate_bent_hallway(mdn_world* w, uint32_t* rng, float distance) { /* world.hpp:226-241 */
    const float difficulty = o_wurand(rng);
    const float span = wchallenge_distance(distance);
    w->goal[0] = span * (0.90f + 0.10f * o_wurand(rng));
    w->goal[1] = (o_wurand(rng) - 0.5f) * 1.20f;
    w->goal[2] = 1.10f + 0.80f * o_wurand(rng);
    const float wall_x = w->goal[0] * (0.24f + 0.04f * o_wurand(rng));
    const float gap_x = w->goal[0] * (0.70f + 0.08f * difficulty);
    const float lane_width = 1.80f - 0.80f * difficulty;
    const float lane_edge = 5.0f - lane_width;
    const float wall_y = (-5.0f + lane_edge) * 0.5f;
    const float wall_half_y = (lane_edge + 5.0f) * 0.5f;
    wadd_box(w, wall_x, wall_y, 2.5f, 0.15f, wall_half_y, 2.5f);
    wadd_box(w, (wall_x + gap_x) * 0.5f, lane_edge + 0.03f, 2.5f, (gap_x - wall_x) * 0.5f + 0.15f, 0.15f, 2.5f);
}
static void wgenerate_connected_rooms(mdn_world* w, uint32_t* rng, float distance) { /* world.hpp:242-269 */
    const float difficulty = o_wurand(rng);
    const float span = wchallenge_distance(distance);
    w->goal[0] = span * (0.90f + 0.10f * o_wurand(rng));
    w->goal[1] = (o_wurand(rng) - 0.5f) * 1.20f;
    w->goal[2] = 1.10f + 0.80f * o_wurand(rng);
    const float wall_1 = w->goal[0] * (0.16f + 0.02f * o_wurand(rng));
    const float wall_2 = w->goal[0] * 0.85f;
    const float gap_1 = -(0.60f + 0.80f * difficulty);
    const float gap_2 = +(0.60f + 0.80f * difficulty);
    const float gap_half = 0.85f - 0.30f * difficulty;
    const float gap_z = 1.50f;
    const float gap_half_z = 0.85f - 0.10f * difficulty;
    wadd_doorway(w, wall_1, gap_1, gap_z, gap_half, gap_half_z);
    wadd_doorway(w, wall_2, gap_2, gap_z, gap_half, gap_half_z);
    const float table_x = w->goal[0] * 0.50f;
    const float table_y = (o_wurand(rng) - 0.5f) * 0.20f;
    const float table_half_x = fminf(0.45f, w->goal[0] * 0.06f);
    const float table_half_y = 0.60f + 0.20f * difficulty;
    const float table_top = 1.45f + 0.25f * difficulty;
    wadd_table(w, table_x, table_y, table_half_x, table_half_y, table_top);
    wadd_box(w, w->goal[0] * 0.38f, 3.75f, 0.55f, 0.22f, 0.35f, 0.55f);
    wadd_box(w, w->goal[0] * 0.50f, -3.80f, 0.80f, 0.25f, 0.35f, 0.80f);
    wadd_box(w, w->goal[0] * 0.62f, 3.70f, 0.50f, 0.22f, 0.40f, 0.50f);
}
static void wgenerate_vertical_choices(mdn_world* w, uint32_t* rng, float distance) { /* world.hpp:270-291 */
    const float difficulty = o_wurand(rng);
    const float span = wchallenge_distance(distance);
    w->goal[0] = span * (0.90f + 0.10f * o_wurand(rng));
    w->goal[1] = (o_wurand(rng) - 0.5f) * 1.20f;
    w->goal[2] = 1.10f + 0.80f * o_wurand(rng);
    const float low_x = w->goal[0] * (0.14f + 0.02f * (1.0f - difficulty));
    const float overhead_x = w->goal[0] * (0.46f + 0.02f * difficulty);
    const float choice_x = w->goal[0] * (0.76f + 0.02f * difficulty);
    const float low_top = 1.50f + 0.25f * difficulty;
    const float overhead_bottom = 2.80f - 0.20f * difficulty;
    const float choice_half_z = 0.10f + 0.05f * difficulty;
    wadd_box(w, low_x, 0, low_top * 0.5f, 0.12f, 5.0f, low_top * 0.5f);
    const float overhead_half_z = (5.0f - overhead_bottom) * 0.5f;
    wadd_box(w, overhead_x, 0, overhead_bottom + overhead_half_z, 0.12f, 5.0f, overhead_half_z);
    wadd_box(w, choice_x, 0, 2.0f + choice_half_z, 0.10f, 5.0f, choice_half_z);
}
/* Family 17, "baseline clutter": the scene of the benchmark configuration
 * (16 static boxes, centres uniform in x[-2,8] y[-5,5] z[0,4], half-extents
 * U(0.2,1.0) per axis, goal 2-8 m from the (0,0,1.5) start). No reference
 * generator exists for it; it uses only IEEE-exact operations so the CUDA
 * generator reproduces it bit for bit. Boxes whose surface lies within 0.5 m
 * of the start or the goal are redrawn (8 tries), else left out. */
static float box_sdf(const float p[3], const float c[3], const float e[3]) {
    const float k[3] = {fabsf(p[0] - c[0]) - e[0], fabsf(p[1] - c[1]) - e[1], fabsf(p[2] - c[2]) - e[2]};
    return len3(fmaxf(k[0], 0.0f), fmaxf(k[1], 0.0f), fmaxf(k[2], 0.0f)) + fminf(fmaxf(k[0], fmaxf(k[1], k[2])), 0.0f);
}
static void wgenerate_baseline_clutter(mdn_world* w, uint32_t* rng) {
    w->count = 0;
    float dx = 1.0f, dy = 0.0f;
    for (int attempt = 0; attempt < 8; attempt++) {
        const float ux = 2.0f * o_wurand(rng) - 1.0f, uy = 2.0f * o_wurand(rng) - 1.0f;
        const float norm = sqrtf(ux * ux + uy * uy);
        if (norm > 0.1f && norm <= 1.0f) {
            dx = ux / norm;
            dy = uy / norm;
            break;
        }
    }
    const float dist = 2.0f + 6.0f * o_wurand(rng);
    w->goal[0] = fminf(fmaxf(dist * dx, -1.5f), 7.5f);
    w->goal[1] = fminf(fmaxf(dist * dy, -4.5f), 4.5f);
    w->goal[2] = 1.0f + o_wurand(rng);
    const float start[3] = {0.0f, 0.0f, 1.5f};
    for (int i = 0; i < 16; i++)
        for (int attempt = 0; attempt < 8; attempt++) {
            const float c[3] = {-2.0f + 10.0f * o_wurand(rng), -5.0f + 10.0f * o_wurand(rng), 4.0f * o_wurand(rng)};
            const float e[3] = {0.2f + 0.8f * o_wurand(rng), 0.2f + 0.8f * o_wurand(rng), 0.2f + 0.8f * o_wurand(rng)};
            if (box_sdf(start, c, e) > 0.5f && box_sdf(w->goal, c, e) > 0.5f) {
                wadd_box(w, c[0], c[1], c[2], e[0], e[1], e[2]);
                break;
            }
        }
}

/* Families 19 and 20: the long-goal and combined-course lanes of the
 * mixed-capability distribution (family 18). No reference generator exists
 * (the reference's course runners are outside its tracked tree); IEEE-exact
 * operations only, so the CUDA generator reproduces them bit for bit.
 *   19: 16 static boxes over the reference room x[-2,14] y[-5,5] z[0,4],
 *       half-extents U(0.2,1.0), goal 2-12 m from the start.
 *   20: 12 static boxes as family 17, then 4 bounded moving spheres (kind 3,
 *       world.hpp:32-41): centre uniform in x[-2,8] y[-5,5] z[0.5,3.5], radius
 *       U(0.2,0.5), amplitude U(0.5,2.0) m, peak speed U(0.5,2.0) m/s, phase
 *       U(0,2pi), random unit direction; a mover is redrawn (8 tries, else left
 *       out) unless its whole swept segment, sampled at 17 points, stays
 *       radius + 0.05 m clear of every static box and radius + 0.5 m clear of
 *       the start, radius + 0.3 m clear of the goal. */
static void wgenerate_clutter_goal(mdn_world* w, uint32_t* rng, float dmin, float dspan, float xmax) {
    float dx = 1.0f, dy = 0.0f;
    for (int attempt = 0; attempt < 8; attempt++) {
        const float ux = 2.0f * o_wurand(rng) - 1.0f, uy = 2.0f * o_wurand(rng) - 1.0f;
        const float norm = sqrtf(ux * ux + uy * uy);
        if (norm > 0.1f && norm <= 1.0f) {
            dx = ux / norm;
            dy = uy / norm;
            break;
        }
    }
    const float dist = dmin + dspan * o_wurand(rng);
    w->goal[0] = fminf(fmaxf(dist * dx, -1.5f), xmax);
    w->goal[1] = fminf(fmaxf(dist * dy, -4.5f), 4.5f);
    w->goal[2] = 1.0f + o_wurand(rng);
}
static void wgenerate_clutter_boxes(mdn_world* w, uint32_t* rng, int boxes, float xspan) {
    const float start[3] = {0.0f, 0.0f, 1.5f};
    for (int i = 0; i < boxes; i++)
        for (int attempt = 0; attempt < 8; attempt++) {
            const float c[3] = {-2.0f + xspan * o_wurand(rng), -5.0f + 10.0f * o_wurand(rng), 4.0f * o_wurand(rng)};
            const float e[3] = {0.2f + 0.8f * o_wurand(rng), 0.2f + 0.8f * o_wurand(rng), 0.2f + 0.8f * o_wurand(rng)};
            if (box_sdf(start, c, e) > 0.5f && box_sdf(w->goal, c, e) > 0.5f) {
                wadd_box(w, c[0], c[1], c[2], e[0], e[1], e[2]);
                break;
            }
        }
}
static void wgenerate_movers(mdn_world* w, uint32_t* rng, int movers) {
    const float start[3] = {0.0f, 0.0f, 1.5f};
    const uint32_t statics = w->count;
    for (int i = 0; i < movers && w->count < 16; i++)
        for (int attempt = 0; attempt < 8; attempt++) {
            const float c[3] = {-2.0f + 10.0f * o_wurand(rng), -5.0f + 10.0f * o_wurand(rng), 0.5f + 3.0f * o_wurand(rng)};
            const float radius = 0.2f + 0.3f * o_wurand(rng);
            const float amplitude = 0.5f + 1.5f * o_wurand(rng);
            const float speed = 0.5f + 1.5f * o_wurand(rng);
            const float phase = 6.2831853f * o_wurand(rng);
            const float ux = 2.0f * o_wurand(rng) - 1.0f, uy = 2.0f * o_wurand(rng) - 1.0f, uz = 2.0f * o_wurand(rng) - 1.0f;
            const float norm = sqrtf(ux * ux + uy * uy + uz * uz);
            if (!(norm > 0.1f && norm <= 1.0f)) continue;
            const float d[3] = {ux / norm, uy / norm, uz / norm};
            int ok = 1;
            for (int k = 0; k <= 16 && ok; k++) {
                const float f = amplitude * ((float)k / 8.0f - 1.0f);
                const float p[3] = {c[0] + d[0] * f, c[1] + d[1] * f, c[2] + d[2] * f};
                for (uint32_t b = 0; b < statics && ok; b++)
                    if (!(box_sdf(p, w->obstacles[b].center, w->obstacles[b].size) > radius + 0.05f)) ok = 0;
                const float ds = len3(p[0] - start[0], p[1] - start[1], p[2] - start[2]);
                const float dg = len3(p[0] - w->goal[0], p[1] - w->goal[1], p[2] - w->goal[2]);
                if (!(ds > radius + 0.5f) || !(dg > radius + 0.3f)) ok = 0;
            }
            if (ok) {
                mdn_obstacle* o = &w->obstacles[w->count++];
                o->kind = 3;
                o->center[0] = c[0]; o->center[1] = c[1]; o->center[2] = c[2];
                o->size[0] = radius; o->size[1] = amplitude; o->size[2] = phase;
                o->velocity[0] = d[0] * speed; o->velocity[1] = d[1] * speed; o->velocity[2] = d[2] * speed;
                break;
            }
        }
}
/* Family 18, mixed capability (BASELINE configs 2 and 4): environments
 * alternate by global id, 50% static clutter (17), 25% long-goal rooms (19),
 * 25% combined courses with movers (20). */
uint32_t o_mixed_lane_family(uint32_t gid) { return (gid & 3u) < 2u ? 17u : ((gid & 3u) == 2u ? 19u : 20u); }

uint32_t o_wtraining_family(uint32_t family, uint32_t* rng) { /* world.hpp:293-298 */
    if (family == 7) return o_wrng(rng) % 7;
    if (family == 9 || family == 12) {
        const uint32_t choice = o_wrng(rng) % 4;
        return choice < 2 ? 4 : (choice == 2 ? 5 : o_wrng(rng) % 7);
    }
    if (family == 13) {
        const uint32_t choice = o_wrng(rng) % 6;
        if (choice < 2) return 4;
        if (choice == 2) return 5;
        if (choice == 3) return o_wrng(rng) % 7;
        return choice == 4 ? 10 : 11;
    }
    return family;
}
void o_wgenerate(mdn_world* w, uint32_t seed, uint32_t family, float distance) { /* world.hpp:299-318 */
    uint32_t rng = seed ? seed : 1;
    w->seed = seed;
    w->family = family;
    w->count = family == 0 ? 0 : 8;
    w->goal[0] = distance;
    w->goal[1] = (o_wurand(&rng) - 0.5f) * 2;
    w->goal[2] = 1.5f + (o_wurand(&rng) - 0.5f) * 0.8f;
    for (int j = 0; j < 3; j++) w->wind[j] = 0;
    switch (family) {
        case 4: w->count = 0; wgenerate_doorway(w, &rng, distance); return;
        case 5: w->count = 0; wgenerate_table_or_counter(w, &rng, distance); return;
        case 6: w->count = 0; wgenerate_mixed(w, &rng, distance); return;
        case 8: w->count = 0; wgenerate_two_doorways(w, &rng, distance); return;
        case 10: case 11: w->count = 0; wgenerate_threat_sphere(w, seed, family); return;
        case 14: w->count = 0; wgenerate_bent_hallway(w, &rng, distance); return;
        case 15: w->count = 0; wgenerate_connected_rooms(w, &rng, distance); return;
        case 16: w->count = 0; wgenerate_vertical_choices(w, &rng, distance); return;
        case 17: wgenerate_baseline_clutter(w, &rng); return;
        case 19:
            w->count = 0;
            wgenerate_clutter_goal(w, &rng, 2.0f, 10.0f, 13.5f);
            wgenerate_clutter_boxes(w, &rng, 16, 16.0f);
            return;
        case 20:
            w->count = 0;
            wgenerate_clutter_goal(w, &rng, 2.0f, 6.0f, 7.5f);
            wgenerate_clutter_boxes(w, &rng, 12, 10.0f);
            wgenerate_movers(w, &rng, 4);
            return;
        default: break;
    }
    for (int i = 0; i < 16; i++) {
        mdn_obstacle* o = &w->obstacles[i];
        o->kind = family == 2 ? 2 : (family == 3 ? 1 : 0);
        o->center[0] = 1.2f + o_wurand(&rng) * fmaxf(0.1f, distance - 2.2f);
        o->center[1] = (o_wurand(&rng) - 0.5f) * 7;
        o->center[2] = family == 2 ? 2.5f : 0.6f + o_wurand(&rng) * 3;
        o->size[0] = 0.2f + o_wurand(&rng) * 0.35f;
        o->size[1] = 0.3f + o_wurand(&rng) * 0.55f;
        o->size[2] = family == 2 ? 2.5f : 0.2f + o_wurand(&rng) * 0.75f;
        o->velocity[0] = 0;
        o->velocity[1] = family == 3 ? (o_wurand(&rng) - 0.5f) * 0.8f : 0;
        o->velocity[2] = 0;
    }
}


/* ------------------------------------------- goal-arrival task contract */
/* navigation_tasks.hpp:21-48 constants */
#define NT_STAGE_OPEN 0u
#define NT_STAGE_HOLD 1u
#define NT_STAGE_CLUTTER 2u
#define NT_OBJ_WAYPOINT 0u
#define NT_OBJ_FINAL_HOLD 1u
#define NT_INVALID_CONFIG 1u
#define NT_UNSUPPORTED_DYNAMIC 2u
#define NT_EXHAUSTED 3u
#define NT_READY 4u
#define NT_UNSUPPORTED_FAMILY 5u
#define NT_MAX_WITNESS 4u
#define NT_MAX_ATTEMPTS 64u
#define NT_MAX_DIRECTIONS 64u

typedef struct { float p[NT_MAX_WITNESS][3]; uint32_t count; float min_clearance, length; } nt_witness;

static float nt_clamp(float v, float lo, float hi) { return fminf(fmaxf(v, lo), hi); } /* :208-210 */
static void nt_random_direction(uint32_t* rng, float out[3]) { /* :212-217 */
    const float z = 2.0f * o_wurand(rng) - 1.0f;
    const float angle = 6.28318530718f * o_wurand(rng);
    const float radial = sqrtf(fmaxf(0.0f, 1.0f - z * z));
    out[0] = radial * cosf(angle);
    out[1] = radial * sinf(angle);
    out[2] = z;
}
static void nt_random_point(uint32_t* rng, const float* low, const float* high, float out[3]) { /* :218-222 */
    /* three draws inside one wv(...) argument list: reference platforms left
     * to right, g++ right to left (see wgenerate_mixed) */
    if (g_args_right_to_left) {
        out[2] = low[2] + (high[2] - low[2]) * o_wurand(rng);
        out[1] = low[1] + (high[1] - low[1]) * o_wurand(rng);
        out[0] = low[0] + (high[0] - low[0]) * o_wurand(rng);
    } else {
        out[0] = low[0] + (high[0] - low[0]) * o_wurand(rng);
        out[1] = low[1] + (high[1] - low[1]) * o_wurand(rng);
        out[2] = low[2] + (high[2] - low[2]) * o_wurand(rng);
    }
}
static int nt_inside(const float p[3], const float* low, const float* high) { /* :229-232 */
    return p[0] >= low[0] && p[0] <= high[0] && p[1] >= low[1] && p[1] <= high[1] && p[2] >= low[2] && p[2] <= high[2];
}
static float nt_goal_distance(uint32_t* rng, const mdn_task_config* c) { /* :234-239 */
    const float span = c->goal_distance_max_m - c->goal_distance_min_m;
    const float center = c->goal_distance_min_m + c->difficulty * span;
    const float jitter = (o_wurand(rng) - 0.5f) * 0.20f * span;
    return nt_clamp(center + jitter, c->goal_distance_min_m, c->goal_distance_max_m);
}
float o_task_segment_clearance(const mdn_world* w, const float* room, const float a[3], const float b[3]) { /* :240-252 */
    const float d[3] = {b[0] - a[0], b[1] - a[1], b[2] - a[2]};
    const float distance = len3(d[0], d[1], d[2]);
    uint32_t count = (uint32_t)ceilf(distance / 0.05f);
    if (count < 1u) count = 1u;
    if (count > 512u) return -1e6f;
    float minimum = 1e20f;
    for (uint32_t sample = 0; sample <= count; sample++) {
        const float t = (float)sample / (float)count;
        const float pt[3] = {a[0] + d[0] * t, a[1] + d[1] * t, a[2] + d[2] * t};
        minimum = fminf(minimum, o_wclearance(w, room, pt, 0.0f, NULL));
    }
    return minimum;
}
static float nt_test_path(const mdn_world* w, const float* room, const float (*pts)[3], uint32_t count) { /* :253-259 */
    if (count < 2u || count > NT_MAX_WITNESS) return -1e6f;
    float minimum = 1e20f;
    for (uint32_t k = 0; k + 1u < count; k++) minimum = fminf(minimum, o_task_segment_clearance(w, room, pts[k], pts[k + 1]));
    return minimum;
}
static void nt_save(nt_witness* out, const float (*pts)[3], uint32_t count, float clearance) { /* :260-273 */
    out->count = count;
    out->min_clearance = clearance;
    float total = 0;
    for (uint32_t k = 0; k + 1u < count; k++)
        total += len3(pts[k + 1][0] - pts[k][0], pts[k + 1][1] - pts[k][1], pts[k + 1][2] - pts[k][2]);
    out->length = total;
    for (uint32_t i = 0; i < NT_MAX_WITNESS; i++)
        for (int j = 0; j < 3; j++) out->p[i][j] = i < count ? pts[i][j] : 0.0f;
}
static int nt_find_witness(const mdn_world* w, const float* room, const float st[3], const float gl[3],
                           const mdn_task_config* c, nt_witness* wit, float* direct_clearance) { /* :276-333 */
    const float direct[2][3] = {{st[0], st[1], st[2]}, {gl[0], gl[1], gl[2]}};
    *direct_clearance = nt_test_path(w, room, direct, 2u);
    if (*direct_clearance > c->minimum_witness_clearance_m && c->require_detour == 0u) {
        nt_save(wit, direct, 2u, *direct_clearance);
        return 1;
    }
    if (*direct_clearance > c->minimum_witness_clearance_m) return 0;
    const float delta[3] = {gl[0] - st[0], gl[1] - st[1], gl[2] - st[2]};
    const float x_fraction[5] = {0.10f, 0.25f, 0.50f, 0.75f, 0.90f};
    const float side_y[2] = {-4.60f, 4.60f};
    for (uint32_t side = 0; side < 2u; side++)
        for (uint32_t i = 0; i < 5u; i++) {
            const float t = x_fraction[i];
            const float path[3][3] = {{st[0], st[1], st[2]}, {st[0] + t * delta[0], side_y[side], st[2] + t * delta[2]},
                                      {gl[0], gl[1], gl[2]}};
            const float cl = nt_test_path(w, room, path, 3u);
            if (cl > c->minimum_witness_clearance_m) {
                nt_save(wit, path, 3u, cl);
                return 1;
            }
        }
    const float side_offset[4] = {-2.4f, -1.2f, 1.2f, 2.4f};
    for (uint32_t i = 0; i < 4u; i++) {
        const float t = 0.5f;
        const float path[3][3] = {{st[0], st[1], st[2]},
                                  {st[0] + t * delta[0], nt_clamp((st[1] + gl[1]) * 0.5f + side_offset[i], -4.60f, 4.60f),
                                   st[2] + t * delta[2]},
                                  {gl[0], gl[1], gl[2]}};
        const float cl = nt_test_path(w, room, path, 3u);
        if (cl > c->minimum_witness_clearance_m) {
            nt_save(wit, path, 3u, cl);
            return 1;
        }
    }
    const float detour_z[2] = {0.55f, 4.45f};
    for (uint32_t i = 0; i < 2u; i++) {
        const float path[3][3] = {{st[0], st[1], st[2]},
                                  {st[0] + 0.5f * delta[0], st[1] + 0.5f * delta[1], detour_z[i]},
                                  {gl[0], gl[1], gl[2]}};
        const float cl = nt_test_path(w, room, path, 3u);
        if (cl > c->minimum_witness_clearance_m) {
            nt_save(wit, path, 3u, cl);
            return 1;
        }
    }
    for (uint32_t side = 0; side < 2u; side++) {
        const float y = side_y[side];
        const float path[4][3] = {{st[0], st[1], st[2]},
                                  {st[0] + 0.20f * delta[0], y, st[2] + 0.20f * delta[2]},
                                  {st[0] + 0.80f * delta[0], y, st[2] + 0.80f * delta[2]},
                                  {gl[0], gl[1], gl[2]}};
        const float cl = nt_test_path(w, room, path, 4u);
        if (cl > c->minimum_witness_clearance_m) {
            nt_save(wit, path, 4u, cl);
            return 1;
        }
    }
    return 0;
}
static int nt_static_world(const mdn_world* w) { /* :335-339 */
    for (uint32_t o = 0; o < w->count; o++)
        for (int a = 0; a < 3; a++)
            if (fabsf(w->obstacles[o].velocity[a]) > 1e-8f) return 0;
    return 1;
}
static int nt_config_valid(const mdn_task_config* c) { /* :347-369 */
    const int valid_stage = c->stage <= NT_STAGE_CLUTTER, valid_objective = c->objective <= NT_OBJ_FINAL_HOLD;
    if (c->generation_version != 1u || !valid_stage || !valid_objective || c->family > 16u || c->require_detour > 1u ||
        !isfinite(c->scene_distance_m) || c->scene_distance_m < 3.0f || c->scene_distance_m > 10.0f ||
        !isfinite(c->difficulty) || c->difficulty < 0.0f || c->difficulty > 1.0f ||
        !isfinite(c->goal_distance_min_m) || !isfinite(c->goal_distance_max_m) ||
        c->goal_distance_min_m <= c->goal_radius_m || c->goal_distance_max_m < c->goal_distance_min_m ||
        !isfinite(c->minimum_endpoint_clearance_m) || c->minimum_endpoint_clearance_m < 0.30f ||
        !isfinite(c->minimum_witness_clearance_m) || c->minimum_witness_clearance_m < 0.02f ||
        !isfinite(c->goal_radius_m) || c->goal_radius_m <= 0.0f || !isfinite(c->stable_speed_mps) ||
        c->stable_speed_mps < 0.0f || !isfinite(c->stable_hold_s) || c->stable_hold_s < 0.0f ||
        !isfinite(c->nav_period_s) || c->nav_period_s <= 0.0f || !isfinite(c->initial_speed_min_mps) ||
        !isfinite(c->initial_speed_max_mps) || c->initial_speed_min_mps < 0.0f ||
        c->initial_speed_max_mps < c->initial_speed_min_mps || !isfinite(c->progress_reward_per_m) ||
        c->progress_reward_per_m < 0.0f || !isfinite(c->time_cost_per_s) || c->time_cost_per_s < 0.0f ||
        !isfinite(c->contact_penalty) || c->contact_penalty < 0.0f || !isfinite(c->stable_arrival_bonus) ||
        c->stable_arrival_bonus < 0.0f || !isfinite(c->command_smoothness_weight) ||
        c->command_smoothness_weight < 0.0f || c->max_nav_steps == 0u || c->max_generation_attempts == 0u)
        return 0;
    return 1;
}
uint32_t o_generate_task(mdn_world* w, mdn_task_state* task, uint32_t* rng, const mdn_task_config* c,
                         const float* room) { /* :343-482 */
    task->generation_status = NT_INVALID_CONFIG;
    task->generation_attempts = 0;
    task->valid = 0;
    if (!nt_config_valid(c)) return NT_INVALID_CONFIG;
    if ((c->stage == NT_STAGE_OPEN || c->stage == NT_STAGE_HOLD) && c->family != 0u) return NT_INVALID_CONFIG;
    if (c->stage == NT_STAGE_CLUTTER &&
        !(c->family == 1u || c->family == 2u || c->family == 4u || c->family == 5u || c->family == 12u))
        return NT_UNSUPPORTED_FAMILY;
    for (int axis = 0; axis < 3; axis++) {
        const float room_min = axis == 0 ? -2.0f : (axis == 1 ? -5.0f : 0.0f);
        const float room_max = axis == 0 ? 14.0f : 5.0f;
        if (!isfinite(c->start_min_xyz[axis]) || !isfinite(c->start_max_xyz[axis]) || !isfinite(c->goal_min_xyz[axis]) ||
            !isfinite(c->goal_max_xyz[axis]) || c->start_min_xyz[axis] >= c->start_max_xyz[axis] ||
            c->goal_min_xyz[axis] >= c->goal_max_xyz[axis] ||
            c->start_min_xyz[axis] < room_min + c->minimum_endpoint_clearance_m ||
            c->start_max_xyz[axis] > room_max - c->minimum_endpoint_clearance_m ||
            c->goal_min_xyz[axis] < room_min + c->minimum_endpoint_clearance_m ||
            c->goal_max_xyz[axis] > room_max - c->minimum_endpoint_clearance_m)
            return NT_INVALID_CONFIG;
    }
    uint32_t attempts = c->max_generation_attempts;
    if (attempts > NT_MAX_ATTEMPTS) attempts = NT_MAX_ATTEMPTS;
    for (uint32_t attempt = 0; attempt < attempts; attempt++) {
        task->generation_attempts = attempt + 1u;
        const uint32_t scene_seed = o_wrng(rng);
        uint32_t scene_family = c->family;
        if (c->family == 12u) {
            const uint32_t sel = o_wrng(rng) % 4u;
            scene_family = sel == 0u ? 1u : (sel == 1u ? 2u : (sel == 2u ? 4u : 5u));
        }
        o_wgenerate(w, scene_seed, scene_family, c->scene_distance_m);
        if (c->stage == NT_STAGE_CLUTTER && !nt_static_world(w)) {
            task->generation_status = NT_UNSUPPORTED_DYNAMIC;
            return task->generation_status;
        }
        float dir[3];
        nt_random_direction(rng, dir);
        const float distance = nt_goal_distance(rng, c);
        float st[3], gl[3];
        if (c->stage == NT_STAGE_HOLD) {
            nt_random_point(rng, c->goal_min_xyz, c->goal_max_xyz, gl);
            for (int j = 0; j < 3; j++) st[j] = gl[j] - dir[j] * distance;
        } else {
            nt_random_point(rng, c->start_min_xyz, c->start_max_xyz, st);
            for (int j = 0; j < 3; j++) gl[j] = st[j] + dir[j] * distance;
            if (c->stage == NT_STAGE_CLUTTER) {
                int in_bounds = nt_inside(gl, c->goal_min_xyz, c->goal_max_xyz);
                for (uint32_t da = 1u; !in_bounds && da < NT_MAX_DIRECTIONS; da++) {
                    nt_random_direction(rng, dir);
                    for (int j = 0; j < 3; j++) gl[j] = st[j] + dir[j] * distance;
                    in_bounds = nt_inside(gl, c->goal_min_xyz, c->goal_max_xyz);
                }
                if (!in_bounds) continue;
            }
        }
        if (!isfinite(gl[0]) || !isfinite(gl[1]) || !isfinite(gl[2])) continue;
        if (!nt_inside(st, c->start_min_xyz, c->start_max_xyz) || !nt_inside(gl, c->goal_min_xyz, c->goal_max_xyz)) continue;
        const float start_clear = o_wclearance(w, room, st, 0.0f, NULL);
        const float goal_clear = o_wclearance(w, room, gl, 0.0f, NULL);
        if (start_clear <= c->minimum_endpoint_clearance_m || goal_clear <= c->minimum_endpoint_clearance_m) continue;
        const float actual = len3(gl[0] - st[0], gl[1] - st[1], gl[2] - st[2]);
        if (actual < c->goal_distance_min_m || actual > c->goal_distance_max_m) continue;
        nt_witness wit;
        memset(&wit, 0, sizeof(wit));
        float direct_clearance = 0.0f;
        if (!nt_find_witness(w, room, st, gl, c, &wit, &direct_clearance)) continue;
        for (int j = 0; j < 3; j++) w->goal[j] = gl[j];
        task->family = scene_family;
        task->stage = c->stage;
        task->objective = c->objective;
        task->max_nav_steps = c->max_nav_steps;
        task->step_count = 0;
        task->stable_ticks = 0;
        task->was_inside_goal = 0;
        task->waypoint_event_latched = 0;
        task->terminal = 0;
        for (int j = 0; j < 3; j++) task->start_position[j] = st[j];
        task->start_yaw_rad = (o_wurand(rng) * 2.0f - 1.0f) * 3.14159265359f;
        const float speed = c->initial_speed_min_mps + (c->initial_speed_max_mps - c->initial_speed_min_mps) * o_wurand(rng);
        for (int j = 0; j < 3; j++) task->start_velocity_world[j] = dir[j] * speed;
        for (int j = 0; j < 3; j++) task->goal_position[j] = gl[j];
        task->initial_distance_m = actual;
        task->previous_distance_m = actual;
        task->difficulty = c->difficulty;
        task->start_clearance_m = start_clear;
        task->goal_clearance_m = goal_clear;
        task->direct_segment_clearance_m = direct_clearance;
        task->witness_min_clearance_m = wit.min_clearance;
        task->witness_length_m = wit.length;
        task->stable_time_s = 0.0f;
        for (int j = 0; j < 3; j++) task->last_executed_world_command[j] = task->start_velocity_world[j];
        task->last_executed_world_command[3] = 0.0f;
        task->witness_point_count = wit.count;
        for (uint32_t k = 0; k < NT_MAX_WITNESS; k++)
            for (int j = 0; j < 3; j++) task->witness_points[k][j] = k < wit.count ? wit.p[k][j] : 0.0f;
        task->valid = 1;
        task->generation_status = NT_READY;
        return task->generation_status;
    }
    task->generation_status = NT_EXHAUSTED;
    return task->generation_status;
}
void o_task_apply_start(const mdn_task_state* task, mdn_physics_state* s) { /* :486-495 */
    for (int a = 0; a < 3; a++) {
        s->position[a] = task->start_position[a];
        s->linear_velocity[a] = task->start_velocity_world[a];
        s->angular_velocity_body[a] = 0.0f;
    }
    const float half_yaw = task->start_yaw_rad * 0.5f;
    s->orientation_wxyz[0] = cosf(half_yaw);
    s->orientation_wxyz[1] = 0.0f;
    s->orientation_wxyz[2] = 0.0f;
    s->orientation_wxyz[3] = sinf(half_yaw);
}
/* out: reward, goal_distance, actual_speed as floats then waypoint, stable,
 * collision, timeout, done as uint32 (NavigationTaskStep, :179-188) */
void o_task_step(mdn_task_state* task, const mdn_task_config* c, const float* pos, const float* vel, const float* cmd,
                 uint32_t contact, uint32_t forced_timeout, void* out) { /* :499-548 */
    float r_reward = 0, r_dist = 0, r_speed = 0;
    uint32_t waypoint = 0, stable = 0, collision = 0, timeout = 0, done = 0;
    if (task->generation_status != NT_READY || task->terminal != 0u) {
        done = 1u;
    } else {
        const float dx = task->goal_position[0] - pos[0], dy = task->goal_position[1] - pos[1], dz = task->goal_position[2] - pos[2];
        const float distance = sqrtf(dx * dx + dy * dy + dz * dz);
        const float speed = sqrtf(vel[0] * vel[0] + vel[1] * vel[1] + vel[2] * vel[2]);
        if (!isfinite(distance) || !isfinite(speed)) {
            collision = 1u;
            done = 1u;
            task->terminal = 1u;
        } else {
            task->step_count++;
            r_dist = distance;
            r_speed = speed;
            const float progress = task->previous_distance_m - distance;
            r_reward = c->progress_reward_per_m * progress - c->time_cost_per_s * c->nav_period_s;
            task->previous_distance_m = distance;
            const uint32_t inside = distance <= c->goal_radius_m ? 1u : 0u;
            waypoint = (task->objective == NT_OBJ_WAYPOINT && inside != 0u && task->waypoint_event_latched == 0u) ? 1u : 0u;
            if (waypoint) task->waypoint_event_latched = 1u;
            const uint32_t stable_now = (inside != 0u && speed <= c->stable_speed_mps) ? 1u : 0u;
            if (task->objective == NT_OBJ_FINAL_HOLD && stable_now != 0u) task->stable_time_s += c->nav_period_s;
            else task->stable_time_s = 0.0f;
            task->stable_ticks = (uint32_t)ceilf(task->stable_time_s / fmaxf(c->nav_period_s, 1e-6f) - 1e-5f);
            stable = (task->objective == NT_OBJ_FINAL_HOLD && stable_now != 0u &&
                      task->stable_time_s + 1e-6f >= c->stable_hold_s) ? 1u : 0u;
            collision = contact ? 1u : 0u;
            timeout = (forced_timeout || task->step_count >= task->max_nav_steps) ? 1u : 0u;
            if (c->command_smoothness_weight > 0.0f) {
                float difference = 0.0f;
                for (int a = 0; a < 4; a++) {
                    const float delta = cmd[a] - task->last_executed_world_command[a];
                    difference += delta * delta;
                    task->last_executed_world_command[a] = cmd[a];
                }
                r_reward -= c->command_smoothness_weight * difference * c->nav_period_s;
            }
            if (collision) r_reward -= c->contact_penalty;
            if (stable && !collision) r_reward += c->stable_arrival_bonus;
            done = (collision || stable || timeout) ? 1u : 0u;
            task->terminal = done;
        }
    }
    float* f = (float*)out;
    uint32_t* u = (uint32_t*)out;
    f[0] = r_reward; f[1] = r_dist; f[2] = r_speed;
    u[3] = waypoint; u[4] = stable; u[5] = collision; u[6] = timeout; u[7] = done;
}

/* ------------------------------------------------------------- sensor */
void o_pixel_ray(float tan_h, float tan_v, uint32_t pixel, float out[3]) { /* sensor_profile.hpp:81-91, world.hpp:25 */
    const uint32_t row = pixel / 20u, col = pixel % 20u;
    const float y = (((float)col + 0.5f) / 20.0f * 2.0f - 1.0f) * tan_h;
    const float z = (((float)row + 0.5f) / 16.0f * 2.0f - 1.0f) * tan_v;
    const float d[3] = {1.0f, -y, -z};
    const float inv = 1.0f / fmaxf(len3(d[0], d[1], d[2]), 1e-8f);
    out[0] = d[0] * inv; out[1] = d[1] * inv; out[2] = d[2] * inv;
}

/* ------------------------------------------------------------ guidance */
static void nav_ray(uint32_t row, uint32_t col, float tan_v, float* d) { /* guidance.hpp:22-26 */
    const float y = 0.9f - 0.2f * (float)col, z = (0.875f - 0.25f * (float)row) * tan_v;
    const float inv = 1.0f / sqrtf(1.0f + y * y + z * z);
    d[0] = inv; d[1] = y * inv; d[2] = z * inv;
}
static float nav_min3x3(const float* range, uint32_t row, uint32_t col) { /* guidance.hpp:27-34 */
    float nearest = 12.0f;
    for (int dr = -1; dr <= 1; dr++)
        for (int dc = -1; dc <= 1; dc++) {
            const int r = (int)row + dr, c = (int)col + dc;
            if (r >= 0 && r < 8 && c >= 0 && c < 10) nearest = fminf(nearest, range[r * 10 + c]);
        }
    return nearest;
}
static float nav_atanh(float x) { return 0.5f * logf((1.0f + x) / (1.0f - x)); } /* guidance.hpp:35 */
static float temporal_risk(const float* cur, const float* prev, uint32_t row, uint32_t col, const float* vel,
                           float sensor_dt, float tan_v) { /* guidance.hpp:58-67 and 175-179 */
    float risk = 0.0f;
    if (sensor_dt > 1e-4f)
        for (int dr = -1; dr <= 1; dr++)
            for (int dc = -1; dc <= 1; dc++) {
                const int r = (int)row + dr, c = (int)col + dc;
                if (r < 0 || r >= 8 || c < 0 || c >= 10) continue;
                const uint32_t k = (uint32_t)(r * 10 + c);
                const float old = prev[k], now = cur[k];
                if (old < 11.9f && now < 11.9f) {
                    float ray[3];
                    nav_ray((uint32_t)r, (uint32_t)c, tan_v, ray);
                    const float unexpected = (old - now) / fmaxf(sensor_dt, 1e-3f) -
                                             (vel[0] * ray[0] + vel[1] * ray[1] + vel[2] * ray[2]);
                    if (unexpected > 0.5f) risk = fmaxf(risk, fminf(0.20f * unexpected, 1.0f));
                }
            }
    return risk;
}
void o_nav_guidance(const float* cur, const float* prev, const float* goal_body, float goal_distance, const float* vel,
                    float sensor_dt, float tan_v, float* hint) { /* guidance.hpp:39-90 */
    const float gnorm = sqrtf(goal_body[0] * goal_body[0] + goal_body[1] * goal_body[1] + goal_body[2] * goal_body[2]);
    if (gnorm < 1e-6f || goal_distance < 0.05f) {
        hint[0] = hint[1] = hint[2] = 0;
        return;
    }
    const float goal[3] = {goal_body[0] / gnorm, goal_body[1] / gnorm, goal_body[2] / gnorm};
    const float speed = sqrtf(vel[0] * vel[0] + vel[1] * vel[1] + vel[2] * vel[2]);
    const float stop_margin = 0.28f + speed * fmaxf(sensor_dt, 0.0f) + 0.25f * speed * speed;
    float best_score = -1e20f, best_dir[3] = {1, 0, 0}, best_range = 0;
    float goal_cell_dot = -1e20f;
    uint32_t goal_row = 0, goal_col = 0;
    for (uint32_t row = 0; row < 8; row++)
        for (uint32_t col = 0; col < 10; col++) {
            float d[3];
            nav_ray(row, col, tan_v, d);
            const float alignment = d[0] * goal[0] + d[1] * goal[1] + d[2] * goal[2];
            const float nearby = nav_min3x3(cur, row, col);
            const float risk = temporal_risk(cur, prev, row, col, vel, sensor_dt, tan_v);
            const float safe_range = fmaxf(nearby - risk, 0.0f);
            const float score = 1.4f * alignment + 0.12f * fminf(safe_range, 6.0f);
            if (score > best_score) {
                best_score = score;
                best_dir[0] = d[0]; best_dir[1] = d[1]; best_dir[2] = d[2];
                best_range = safe_range;
            }
            if (alignment > goal_cell_dot) {
                goal_cell_dot = alignment;
                goal_row = row;
                goal_col = col;
            }
        }
    const float max_speed = 1.6f;
    const float desired_speed = fminf(max_speed, sqrtf(4.0f * fmaxf(goal_distance - 0.28f, 0.0f)));
    const float direct_range = fmaxf(nav_min3x3(cur, goal_row, goal_col), 0.0f);
    float direction[3] = {best_dir[0], best_dir[1], best_dir[2]}, available = best_range;
    if (goal[0] > 0.0f && direct_range > stop_margin + 0.25f * desired_speed * desired_speed) {
        direction[0] = goal[0]; direction[1] = goal[1]; direction[2] = goal[2];
        available = direct_range;
    }
    const float after_stop = fmaxf(available - stop_margin - 0.15f, 0.0f);
    const float command_speed = fminf(desired_speed, sqrtf(4.0f * after_stop));
    const float fraction = fminf(0.8f, command_speed * 0.5f);
    if (direct_range < 1.2f && available > direct_range + 0.25f) {
        const float advance = fmaxf(0.05f, fminf(1.0f, (direct_range - 0.25f) / 0.95f));
        direction[0] *= advance;
        const float norm = sqrtf(direction[0] * direction[0] + direction[1] * direction[1] + direction[2] * direction[2]);
        for (int i = 0; i < 3; i++) direction[i] /= fmaxf(norm, 1e-6f);
    }
    for (int i = 0; i < 3; i++) hint[i] = nav_atanh(fraction * direction[i]);
}

static float memory_point_radius(float range, float history_age) { /* guidance.hpp:96-100, capture age off */
    const float age = fmaxf(history_age, 0.0f) + 0.0f;
    return 0.20f + 0.015f * range + 0.15f * age;
}
static float nav_memory_clearance(const float* direction, const float* range_ring, const float* pose_ring,
                                  const float* cur_pose, uint32_t latest_frame, uint32_t valid_frames,
                                  float sensor_dt, float tan_v) { /* guidance.hpp:106-140 */
    float nearest = 3.0f;
    for (uint32_t back = 0; back < valid_frames && back < 8; back++) {
        const uint32_t frame = (latest_frame + 8u - back) % 8u;
        const float* old_pose = pose_ring + frame * 12;
        const float* ranges = range_ring + frame * 320;
        const float age = (float)back * fmaxf(sensor_dt, 0.0f);
        for (uint32_t row = 0; row < 8; row++)
            for (uint32_t col = 0; col < 10; col++) {
                const uint32_t px = row * 2 * 20 + col * 2;
                uint32_t hit = px;
                float range = ranges[px];
                const uint32_t pixels[3] = {px + 1, px + 20, px + 21};
                for (int j = 0; j < 3; j++)
                    if (ranges[pixels[j]] < range) {
                        range = ranges[pixels[j]];
                        hit = pixels[j];
                    }
                if (range <= 0.01f || range >= 11.9f) continue;
                const float ry = 1.0f - ((float)(hit % 20) + .5f) / 10.0f;
                const float rz = tan_v * (1.0f - ((float)(hit / 20) + .5f) / 8.0f);
                const float inv = 1.0f / sqrtf(1 + ry * ry + rz * rz);
                const float ray[3] = {inv, ry * inv, rz * inv};
                const float wx = old_pose[3] * ray[0] + old_pose[4] * ray[1] + old_pose[5] * ray[2];
                const float wy = old_pose[6] * ray[0] + old_pose[7] * ray[1] + old_pose[8] * ray[2];
                const float wz = old_pose[9] * ray[0] + old_pose[10] * ray[1] + old_pose[11] * ray[2];
                const float dx = old_pose[0] + range * wx - cur_pose[0];
                const float dy = old_pose[1] + range * wy - cur_pose[1];
                const float dz = old_pose[2] + range * wz - cur_pose[2];
                const float x = cur_pose[3] * dx + cur_pose[6] * dy + cur_pose[9] * dz;
                const float y = cur_pose[4] * dx + cur_pose[7] * dy + cur_pose[10] * dz;
                const float z = cur_pose[5] * dx + cur_pose[8] * dy + cur_pose[11] * dz;
                const float along = x * direction[0] + y * direction[1] + z * direction[2];
                const float radius = memory_point_radius(range, age);
                if (along <= 0.0f || along > 3.0f + radius) continue;
                const float lateral2 = fmaxf(x * x + y * y + z * z - along * along, 0.0f);
                const float radius2 = radius * radius;
                if (lateral2 < radius2) nearest = fminf(nearest, fmaxf(along - sqrtf(radius2 - lateral2), 0.0f));
            }
    }
    return nearest;
}
void o_nav_guidance_memory(const float* cur, const float* prev, const float* goal_body, float goal_distance,
                           const float* vel, float sensor_dt, float tan_v, const float* range_ring,
                           const float* pose_ring, const float* cur_pose, uint32_t latest_frame,
                           uint32_t valid_frames, float* hint, float latest_capture_age) { /* guidance.hpp:145-194 */
    (void)latest_capture_age; /* NAV_MEMORY_USE_CAPTURE_AGE == 0 (guidance.hpp:93-95) */
    const float gnorm = sqrtf(goal_body[0] * goal_body[0] + goal_body[1] * goal_body[1] + goal_body[2] * goal_body[2]);
    if (gnorm < 1e-6f || goal_distance < 0.05f) {
        hint[0] = hint[1] = hint[2] = 0;
        return;
    }
    const float goal[3] = {goal_body[0] / gnorm, goal_body[1] / gnorm, goal_body[2] / gnorm};
    const float speed = sqrtf(vel[0] * vel[0] + vel[1] * vel[1] + vel[2] * vel[2]);
    const float stop_margin = 0.28f + speed * fmaxf(sensor_dt, 0.0f) + 0.25f * speed * speed;
    float goal_cell_dot = -1e20f;
    uint32_t goal_row = 0, goal_col = 0;
    for (uint32_t row = 0; row < 8; row++)
        for (uint32_t col = 0; col < 10; col++) {
            float d[3];
            nav_ray(row, col, tan_v, d);
            const float a = d[0] * goal[0] + d[1] * goal[1] + d[2] * goal[2];
            if (a > goal_cell_dot) {
                goal_cell_dot = a;
                goal_row = row;
                goal_col = col;
            }
        }
    const float desired_speed = fminf(1.6f, sqrtf(4.0f * fmaxf(goal_distance - 0.28f, 0.0f)));
    float best_score = -1e20f, best_free = 0.0f, best_dir[3] = {1, 0, 0};
    for (uint32_t candidate = 0; candidate < 85; candidate++) {
        float d[3];
        uint32_t row = goal_row, col = goal_col;
        if (candidate < 80) {
            row = candidate / 10;
            col = candidate % 10;
            nav_ray(row, col, tan_v, d);
        } else if (candidate == 80) {
            d[0] = goal[0]; d[1] = goal[1]; d[2] = goal[2];
        } else {
            d[0] = 0;
            d[1] = candidate >= 83 ? (candidate == 83 ? 1.0f : -1.0f) : 0;
            d[2] = candidate < 83 ? (candidate == 81 ? 1.0f : -1.0f) : 0;
        }
        float sweep[3] = {1.2f * d[0] + 0.35f * vel[0], 1.2f * d[1] + 0.35f * vel[1], 1.2f * d[2] + 0.35f * vel[2]};
        const float sweep_norm = sqrtf(sweep[0] * sweep[0] + sweep[1] * sweep[1] + sweep[2] * sweep[2]);
        for (int j = 0; j < 3; j++) sweep[j] /= fmaxf(sweep_norm, 1e-6f);
        float free = nav_memory_clearance(sweep, range_ring, pose_ring, cur_pose, latest_frame, valid_frames, sensor_dt,
                                          tan_v);
        const float observed = nav_min3x3(cur, row, col);
        if (candidate < 81) free = fminf(free, observed);
        const float risk = temporal_risk(cur, prev, row, col, vel, sensor_dt, tan_v);
        free = fmaxf(free - risk, 0.0f);
        const float alignment = d[0] * goal[0] + d[1] * goal[1] + d[2] * goal[2];
        const float required = stop_margin + 0.15f + desired_speed * desired_speed * .25f;
        const float score = 1.4f * alignment + 0.20f * fminf(free, 3.0f) -
                            (free < required ? 3.0f * (required - free) / required : 0.0f);
        if (score > best_score) {
            best_score = score;
            best_free = free;
            best_dir[0] = d[0]; best_dir[1] = d[1]; best_dir[2] = d[2];
        }
    }
    const int goal_in_fov = goal[0] > 0.0f && fabsf(goal[1]) <= goal[0] && fabsf(goal[2]) <= tan_v * goal[0];
    const float after_stop = fmaxf(best_free - stop_margin - 0.15f, 0.0f);
    float command_speed = fminf(desired_speed, sqrtf(4.0f * after_stop));
    if (!goal_in_fov) command_speed = fminf(command_speed, 0.25f);
    const float fraction = fminf(0.8f, command_speed * 0.5f);
    for (int i = 0; i < 3; i++) hint[i] = nav_atanh(fraction * best_dir[i]);
}

/* ------------------------------------------------------------ physics */
static void cross3(const float a[3], const float b[3], float out[3]) { /* physics.hpp:44-48 */
    out[0] = a[1] * b[2] - a[2] * b[1];
    out[1] = a[2] * b[0] - a[0] * b[2];
    out[2] = a[0] * b[1] - a[1] * b[0];
}
static void rotate_b2w(const float q[4], const float v[3], float out[3]) { /* physics.hpp:51-58 */
    const float tx = 2.0f * (q[2] * v[2] - q[3] * v[1]);
    const float ty = 2.0f * (q[3] * v[0] - q[1] * v[2]);
    const float tz = 2.0f * (q[1] * v[1] - q[2] * v[0]);
    out[0] = v[0] + q[0] * tx + q[2] * tz - q[3] * ty;
    out[1] = v[1] + q[0] * ty + q[3] * tx - q[1] * tz;
    out[2] = v[2] + q[0] * tz + q[1] * ty - q[2] * tx;
}
static void derivative(const mdn_physics_params* p, const mdn_physics_state* s, const float sp[4],
                       const float wind[3], mdn_physics_state* d) { /* physics.hpp:60-112 */
    float thrust[3] = {0, 0, 0}, torque[3] = {0, 0, 0};
    for (int r = 0; r < 4; ++r) {
        const float speed = s->rpm[r];
        const float* c = &p->rotor_thrust_coefficients[3 * r];
        const float magnitude = c[0] + c[1] * speed + c[2] * speed * speed;
        float rt[3];
        const float* dir = &p->rotor_thrust_directions[3 * r];
        for (int i = 0; i < 3; ++i) {
            rt[i] = dir[i] * magnitude;
            thrust[i] += rt[i];
            torque[i] += p->rotor_torque_directions[3 * r + i] * magnitude * p->rotor_torque_constants[r];
        }
        float arm[3];
        cross3(&p->rotor_positions[3 * r], rt, arm);
        for (int i = 0; i < 3; ++i) torque[i] += arm[i];
    }
    for (int i = 0; i < 3; ++i) d->position[i] = s->linear_velocity[i];
    const float* q = s->orientation_wxyz;
    const float* w = s->angular_velocity_body;
    d->orientation_wxyz[0] = -q[1] * w[0] - q[2] * w[1] - q[3] * w[2];
    d->orientation_wxyz[1] = q[0] * w[0] + q[2] * w[2] - q[3] * w[1];
    d->orientation_wxyz[2] = q[0] * w[1] + q[3] * w[0] - q[1] * w[2];
    d->orientation_wxyz[3] = q[0] * w[2] + q[1] * w[1] - q[2] * w[0];
    for (int i = 0; i < 4; ++i) d->orientation_wxyz[i] *= 0.5f;
    rotate_b2w(q, thrust, d->linear_velocity);
    for (int i = 0; i < 3; ++i)
        d->linear_velocity[i] = d->linear_velocity[i] / p->mass + p->gravity_world[i] + wind[i] / p->mass;
    float am[3] = {0, 0, 0};
    for (int row = 0; row < 3; ++row)
        for (int col = 0; col < 3; ++col) am[row] += p->inertia[3 * row + col] * w[col];
    float gyro[3];
    cross3(w, am, gyro);
    for (int i = 0; i < 3; ++i) am[i] = torque[i] - gyro[i];
    for (int row = 0; row < 3; ++row) {
        d->angular_velocity_body[row] = 0.0f;
        for (int col = 0; col < 3; ++col) d->angular_velocity_body[row] += p->inertia_inverse[3 * row + col] * am[col];
    }
    for (int r = 0; r < 4; ++r) {
        const float tau = sp[r] >= s->rpm[r] ? p->rotor_time_constants_rising[r] : p->rotor_time_constants_falling[r];
        d->rpm[r] = (sp[r] - s->rpm[r]) / tau;
    }
}
static void add_scaled(const mdn_physics_state* s, const mdn_physics_state* d, float scale, mdn_physics_state* out) {
    const float* a = (const float*)s; /* physics.hpp:114-120: fields are 17 consecutive floats */
    const float* b = (const float*)d;
    float* o = (float*)out;
    for (int i = 0; i < 17; ++i) o[i] = a[i] + scale * b[i];
}
void o_physics_step(const mdn_physics_state* state, const float action[4], const float wind[3],
                    const mdn_physics_params* p, mdn_physics_state* next) { /* physics.hpp:122-179 */
    float sp[4];
    const float half_range = (p->action_max - p->action_min) * 0.5f;
    for (int i = 0; i < 4; ++i) {
        float a = action[i];
        if (a < -1.0f) a = -1.0f;
        if (a > 1.0f) a = 1.0f;
        sp[i] = a * half_range + p->action_min + half_range;
    }
    mdn_physics_state k1, k2, k3, k4, temp;
    derivative(p, state, sp, wind, &k1);
    add_scaled(state, &k1, 0.5f * p->dt, &temp);
    derivative(p, &temp, sp, wind, &k2);
    add_scaled(state, &k2, 0.5f * p->dt, &temp);
    derivative(p, &temp, sp, wind, &k3);
    add_scaled(state, &k3, p->dt, &temp);
    derivative(p, &temp, sp, wind, &k4);
    const float* s = (const float*)state;
    const float *a1 = (const float*)&k1, *a2 = (const float*)&k2, *a3 = (const float*)&k3, *a4 = (const float*)&k4;
    float* o = (float*)next;
    for (int i = 0; i < 17; ++i) o[i] = s[i] + p->dt * (a1[i] + 2.0f * a2[i] + 2.0f * a3[i] + a4[i]) / 6.0f;
    float* q = next->orientation_wxyz;
    const float norm = sqrtf(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]);
    for (int i = 0; i < 4; ++i) q[i] /= norm;
    for (int i = 0; i < 3; ++i) {
        if (next->position[i] < -p->position_limit) next->position[i] = -p->position_limit;
        if (next->position[i] > p->position_limit) next->position[i] = p->position_limit;
        if (next->linear_velocity[i] < -p->velocity_limit) next->linear_velocity[i] = -p->velocity_limit;
        if (next->linear_velocity[i] > p->velocity_limit) next->linear_velocity[i] = p->velocity_limit;
        if (next->angular_velocity_body[i] < -p->angular_velocity_limit)
            next->angular_velocity_body[i] = -p->angular_velocity_limit;
        if (next->angular_velocity_body[i] > p->angular_velocity_limit)
            next->angular_velocity_body[i] = p->angular_velocity_limit;
    }
    for (int i = 0; i < 4; ++i) {
        if (next->rpm[i] < p->action_min) next->rpm[i] = p->action_min;
        if (next->rpm[i] > p->action_max) next->rpm[i] = p->action_max;
    }
}
void o_physics_default(mdn_physics_params* p) { /* physics.hpp:184-219 */
    memset(p, 0, sizeof(*p));
    const float positions[12] = {.028f, -.028f, 0, -.028f, -.028f, 0, -.028f, .028f, 0, .028f, .028f, 0};
    const float torque_z[4] = {-1, 1, -1, 1};
    const float inertia_diag[3] = {9.416556729130406e-6f, 9.644051701582312e-6f, 1.745951732253285e-5f};
    const float inertia_inv_diag[3] = {106195.93007988465f, 103690.85846314249f, 57275.35197719487f};
    for (int r = 0; r < 4; ++r) {
        const int i = 3 * r;
        p->rotor_positions[i] = positions[i];
        p->rotor_positions[i + 1] = positions[i + 1];
        p->rotor_thrust_directions[i + 2] = 1.0f;
        p->rotor_torque_directions[i + 2] = torque_z[r];
        p->rotor_thrust_coefficients[i] = 0.00352526f;
        p->rotor_thrust_coefficients[i + 1] = 0.01437313f;
        p->rotor_thrust_coefficients[i + 2] = 0.09223048f;
        p->rotor_torque_constants[r] = 4.665e-3f;
        p->rotor_time_constants_rising[r] = 0.05545454545454546f;
        p->rotor_time_constants_falling[r] = 0.24939393939393945f;
    }
    for (int i = 0; i < 3; ++i) {
        p->inertia[4 * i] = inertia_diag[i];
        p->inertia_inverse[4 * i] = inertia_inv_diag[i];
    }
    p->gravity_world[2] = -9.81f;
    p->mass = 0.027f + 0.0017f + 0.0003f + 0.0016f;
    p->action_min = 0.0f;
    p->action_max = 1.0f;
    p->dt = 0.01f;
    p->position_limit = 100000.0f;
    p->velocity_limit = 100000.0f;
    p->angular_velocity_limit = 100000.0f;
}

/* ------------------------------------------------------------- RAPTOR */
static float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); } /* raptor.hpp:46-48 */
void o_raptor_forward(const mdn_raptor_weights* w, const float obs[22], float hidden[16], float action[4]) {
    /* raptor.hpp:52-92 */
    float x[16];
    for (int row = 0; row < 16; ++row) {
        float value = w->input_bias[row];
        for (int col = 0; col < 22; ++col) value += w->input_weights[row * 22 + col] * obs[col];
        x[row] = smax(value, 0.0f);
    }
    float ig[48], hg[48];
    for (int row = 0; row < 48; ++row) {
        float iv = w->gru_input_bias[row], hv = w->gru_hidden_bias[row];
        for (int col = 0; col < 16; ++col) {
            iv += w->gru_input_weights[row * 16 + col] * x[col];
            hv += w->gru_hidden_weights[row * 16 + col] * hidden[col];
        }
        ig[row] = iv;
        hg[row] = hv;
    }
    float nh[16];
    for (int i = 0; i < 16; ++i) {
        const float reset = sigmoidf_(ig[i] + hg[i]);
        const float update = sigmoidf_(ig[16 + i] + hg[16 + i]);
        const float cand = tanhf(ig[32 + i] + reset * hg[32 + i]);
        nh[i] = (1.0f - update) * cand + update * hidden[i];
    }
    memcpy(hidden, nh, sizeof(nh));
    for (int row = 0; row < 4; ++row) {
        float value = w->output_bias[row];
        for (int col = 0; col < 16; ++col) value += w->output_weights[row * 16 + col] * hidden[col];
        action[row] = value;
    }
}

/* ----------------------------------------------------------------- PPO */
void o_compute_gae(uint32_t horizon, uint32_t envs, const float* rewards, const float* values, const float* next_values,
                   const uint8_t* term, const uint8_t* trunc, float gamma, float lambda, float* adv, float* ret) {
    /* ppo.hpp:108-126 */
    for (uint32_t env = 0; env < envs; ++env) {
        float carry = 0.0f;
        for (uint32_t rev = 0; rev < horizon; ++rev) {
            const uint32_t t = horizon - 1 - rev;
            const size_t k = (size_t)t * envs + env;
            const int te = term[k] != 0;
            const int boundary = te || trunc[k] != 0;
            const float bootstrap = te ? 0.0f : next_values[k];
            const float delta = rewards[k] + gamma * bootstrap - values[k];
            carry = delta + (boundary ? 0.0f : gamma * lambda * carry);
            adv[k] = carry;
            ret[k] = carry + values[k];
        }
    }
}
void o_normalize_advantages(float* adv, size_t count) { /* ppo.hpp:128-140 */
    if (count == 0) return;
    double sum = 0.0;
    for (size_t i = 0; i < count; ++i) sum += adv[i];
    const float mean = (float)(sum / (double)count);
    double sq = 0.0;
    for (size_t i = 0; i < count; ++i) {
        const double d = (double)(adv[i] - mean);
        sq += d * d;
    }
    const float inv = 1.0f / sqrtf((float)(sq / (double)count) + 1.0e-8f);
    for (size_t i = 0; i < count; ++i) adv[i] = (adv[i] - mean) * inv;
}
static float gaussian_log_prob(const float* action, const float* mean, const float* log_std) { /* ppo.hpp:95-103 */
    float result = 0.0f;
    for (int a = 0; a < 4; ++a) {
        const float inv_std = expf(-log_std[a]);
        const float d = (action[a] - mean[a]) * inv_std;
        result += -0.5f * (d * d + 2.0f * log_std[a] + LOG_TWO_PI);
    }
    return result;
}
void o_sample_loss_and_grad(const float* action, const float* mean, const float* log_std, float old_logp, float value,
                            float advantage, float target, float batch, float clip, float vcoef, float ecoef,
                            float* d_mean, float* d_log_std, float* d_value, float losses[4]) { /* ppo.hpp:144-181 */
    const float logp = gaussian_log_prob(action, mean, log_std);
    const float raw = logp - old_logp;
    const float log_ratio = clampf_(raw, -20.0f, 20.0f);
    const float ratio = expf(log_ratio);
    const float clipped = clampf_(ratio, 1.0f - clip, 1.0f + clip);
    const float chosen = smin(ratio * advantage, clipped * advantage);
    const int in_range = raw >= -20.0f && raw <= 20.0f;
    const int active = in_range && (advantage >= 0.0f ? ratio <= 1.0f + clip : ratio >= 1.0f - clip);
    const float scale = 1.0f / smax(batch, 1.0f);
    float entropy = 0.0f;
    for (int a = 0; a < 4; ++a) {
        const float inv_var = expf(-2.0f * log_std[a]);
        const float diff = action[a] - mean[a];
        if (active) {
            const float dlogp = -ratio * advantage * scale;
            d_mean[a] = dlogp * diff * inv_var;
            d_log_std[a] = dlogp * (diff * diff * inv_var - 1.0f);
        } else {
            d_mean[a] = 0.0f;
            d_log_std[a] = 0.0f;
        }
        d_log_std[a] -= ecoef * scale;
        entropy += -ecoef * (log_std[a] + 0.5f * (1.0f + LOG_TWO_PI)) * scale;
    }
    *d_value = vcoef * (value - target) * scale;
    losses[0] = -chosen * scale;
    losses[1] = 0.5f * vcoef * (value - target) * (value - target) * scale;
    losses[2] = entropy;
    losses[3] = ratio;
}
float o_pow_correction(float beta, uint64_t step) { return 1.0f - powf(beta, (float)step); } /* cpu_reference.hpp:558-559 */
void o_adam_update(float* params, const float* grad, float* m, float* v, size_t count, float b1corr, float b2corr,
                   float lr) { /* cpu_reference.hpp:561-566, ppo.hpp:316-323 */
    for (size_t i = 0; i < count; i++) {
        m[i] = 0.9f * m[i] + (1.0f - 0.9f) * grad[i];
        v[i] = 0.999f * v[i] + (1.0f - 0.999f) * grad[i] * grad[i];
        const float mh = m[i] / b1corr, vh = v[i] / b2corr;
        params[i] -= lr * mh / (sqrtf(vh) + 1.0e-8f);
    }
}

/* ----------------------------------------------------------- simulator */
struct o_sim {
    mdn_sim_config cfg;
    uint32_t horizon;
    uint32_t env_base; /* global id of local env 0 (a rank's shard) */
    int delay_rehearsal; /* NAV_DELAY_REHEARSAL, off by default */
    mdn_raptor_weights raptor;
    mdn_physics_params physics;
    float room[6];
    mdn_physics_state* states;
    mdn_sim_run* runs;
    mdn_world* worlds;
    float *sensors, *poses, *commands;
    float *actor, *critic, *actor_m, *actor_v, *critic_m, *critic_v;
    float *obs, *co, *actions, *logp, *values, *rewards, *next_values, *adv, *ret;
    uint8_t *term, *trunc;
    int32_t* contact;
    float* pixel_rays; /* [320][3] */
    mdn_task_control task_ctl; /* goal-arrival tasks (navigation_training::configure) */
    mdn_task_state* tasks;
    /* per-episode plants (NavigationRuntimeConfig, navigation_runtime.hpp:9-14) */
    mdn_runtime_config runtime;
    mdn_physics_params* env_physics;
    /* frozen challenge bank (ChallengeBankControl, sim.metal:13) */
    mdn_bank_control bank;
    mdn_world* bank_worlds;
    uint32_t *bank_schedule, *bank_active, *bank_transition;
};

uint32_t o_actor_param_count(void) { return A_P; }
void o_sim_set_delay_rehearsal(o_sim* s, int enabled) { s->delay_rehearsal = enabled != 0; }
uint32_t o_critic_param_count(void) { return C_P; }
void o_set_threads(int n) {
#ifdef _OPENMP
    extern void omp_set_num_threads(int);
    omp_set_num_threads(n > 0 ? n : 1);
#else
    (void)n;
#endif
}

static void* zalloc(size_t bytes) { return calloc(bytes ? bytes : 1, 1); }

o_sim* o_sim_create(const mdn_sim_config* cfg, uint32_t horizon, const mdn_raptor_weights* raptor,
                    const mdn_physics_params* physics, const float* room) {
    return o_sim_create_shard(cfg, horizon, raptor, physics, room, 0);
}
o_sim* o_sim_create_shard(const mdn_sim_config* cfg, uint32_t horizon, const mdn_raptor_weights* raptor,
                          const mdn_physics_params* physics, const float* room, uint32_t env_base) {
    o_sim* s = (o_sim*)zalloc(sizeof(o_sim));
    s->env_base = env_base;
    s->cfg = *cfg;
    s->horizon = horizon;
    s->raptor = *raptor;
    s->physics = *physics;
    memcpy(s->room, room ? room : REF_ROOM, sizeof(s->room));
    const size_t n = cfg->n, rows = n * horizon;
    s->states = zalloc(n * sizeof(mdn_physics_state));
    s->runs = zalloc(n * sizeof(mdn_sim_run));
    s->worlds = zalloc(n * sizeof(mdn_world));
    s->sensors = zalloc(n * NFRAMES * NPIX * 4);
    s->poses = zalloc(n * NFRAMES * 12 * 4);
    s->commands = zalloc(n * NFRAMES * ACT * 4);
    s->actor = zalloc(A_P * 4); s->actor_m = zalloc(A_P * 4); s->actor_v = zalloc(A_P * 4);
    s->critic = zalloc(C_P * 4); s->critic_m = zalloc(C_P * 4); s->critic_v = zalloc(C_P * 4);
    s->obs = zalloc(rows * AOBS * 4);
    s->co = zalloc(rows * COBS * 4);
    s->actions = zalloc(rows * ACT * 4);
    s->logp = zalloc(rows * 4); s->values = zalloc(rows * 4); s->rewards = zalloc(rows * 4);
    s->next_values = zalloc(rows * 4); s->adv = zalloc(rows * 4); s->ret = zalloc(rows * 4);
    s->term = zalloc(rows); s->trunc = zalloc(rows);
    s->contact = zalloc(rows * 4);
    s->pixel_rays = zalloc(NPIX * 3 * 4);
    s->tasks = zalloc(n * sizeof(mdn_task_state));
    s->env_physics = zalloc(n * sizeof(mdn_physics_params));
    s->bank_active = zalloc(n * 4);
    s->bank_transition = zalloc(rows * 4);
    for (size_t k = 0; k < n; k++) s->bank_active[k] = 0xffffffffu;
    for (size_t k = 0; k < rows; k++) s->bank_transition[k] = 0xffffffffu;
    for (uint32_t k = 0; k < NPIX; k++) o_pixel_ray(1.0f, 0.75f, k, s->pixel_rays + 3 * k);
    /* Policy initialisation, cpu_reference.hpp:89-103 (== main.mm:548-555). */
    uint32_t seed = 1789;
#define NORMAL_DRAW(out)                                                  \
    do {                                                                  \
        const float u_ = smax(o_wurand(&seed), 1.0e-7f);                  \
        const float a_ = sqrtf(-2.0f * logf(u_));                         \
        (out) = a_ * cosf(6.2831853f * o_wurand(&seed));                  \
    } while (0)
    for (size_t i = 0; i < A_B1; i++) { float z; NORMAL_DRAW(z); s->actor[i] = z * 0.04f; }
    for (size_t i = A_W2; i < A_B2; i++) { float z; NORMAL_DRAW(z); s->actor[i] = z * 0.01f; }
    for (size_t i = 0; i < ACT; i++) s->actor[A_LS + i] = -1.0f;
    for (size_t i = 0; i < C_B1; i++) { float z; NORMAL_DRAW(z); s->critic[i] = z * 0.15f; }
    for (size_t i = C_W2; i < C_B2; i++) { float z; NORMAL_DRAW(z); s->critic[i] = z * 0.1f; }
#undef NORMAL_DRAW
    o_sim_reset(s);
    return s;
}
void o_sim_destroy(o_sim* s) {
    if (!s) return;
    void* bufs[] = {s->states, s->runs, s->worlds, s->sensors, s->poses, s->commands, s->actor, s->critic,
                    s->actor_m, s->actor_v, s->critic_m, s->critic_v, s->obs, s->co, s->actions, s->logp,
                    s->values, s->rewards, s->next_values, s->adv, s->ret, s->term, s->trunc, s->contact,
                    s->pixel_rays, s->tasks, s->bank_worlds, s->bank_schedule, s->bank_active,
                    s->bank_transition, s->env_physics};
    for (size_t i = 0; i < sizeof(bufs) / sizeof(bufs[0]); i++) free(bufs[i]);
    free(s);
}
void o_sim_set_config(o_sim* s, const mdn_sim_config* cfg) { s->cfg = *cfg; }
void o_sim_set_task_control(o_sim* s, const mdn_task_control* ctl) { s->task_ctl = *ctl; }
void o_sim_set_runtime(o_sim* s, const mdn_runtime_config* rt) {
    memset(&s->runtime, 0, sizeof(s->runtime));
    if (rt && rt->enabled) s->runtime = *rt;
}
/* Bank worlds and a zeroed env-major schedule [n][stride] (main.mm:543-547,
 * 2351-2353); enabled == 0 switches banks off. */
void o_sim_set_challenge_bank(o_sim* s, const mdn_world* worlds, const mdn_bank_control* ctl) {
    free(s->bank_worlds);
    free(s->bank_schedule);
    s->bank_worlds = NULL;
    s->bank_schedule = NULL;
    memset(&s->bank, 0, sizeof(s->bank));
    if (!ctl || !ctl->enabled) return;
    s->bank = *ctl;
    s->bank_worlds = zalloc((size_t)ctl->bank_count * sizeof(mdn_world));
    if (ctl->bank_count) memcpy(s->bank_worlds, worlds, (size_t)ctl->bank_count * sizeof(mdn_world));
    s->bank_schedule = zalloc((size_t)s->cfg.n * ctl->schedule_stride * 4);
}
void* o_sim_buffer(o_sim* s, int id, size_t* bytes) {
    const size_t n = s->cfg.n, rows = n * s->horizon;
    switch (id) {
        case MDN_BUF_STATES: *bytes = n * sizeof(mdn_physics_state); return s->states;
        case MDN_BUF_RUNS: *bytes = n * sizeof(mdn_sim_run); return s->runs;
        case MDN_BUF_WORLDS: *bytes = n * sizeof(mdn_world); return s->worlds;
        case MDN_BUF_SENSORS: *bytes = n * NFRAMES * NPIX * 4; return s->sensors;
        case MDN_BUF_POSES: *bytes = n * NFRAMES * 12 * 4; return s->poses;
        case MDN_BUF_COMMANDS: *bytes = n * NFRAMES * ACT * 4; return s->commands;
        case MDN_BUF_ACTOR: *bytes = A_P * 4; return s->actor;
        case MDN_BUF_CRITIC: *bytes = C_P * 4; return s->critic;
        case MDN_BUF_OBS: *bytes = rows * AOBS * 4; return s->obs;
        case MDN_BUF_CO: *bytes = rows * COBS * 4; return s->co;
        case MDN_BUF_ACTIONS: *bytes = rows * ACT * 4; return s->actions;
        case MDN_BUF_LOGP: *bytes = rows * 4; return s->logp;
        case MDN_BUF_VALUES: *bytes = rows * 4; return s->values;
        case MDN_BUF_REWARDS: *bytes = rows * 4; return s->rewards;
        case MDN_BUF_NEXT_VALUES: *bytes = rows * 4; return s->next_values;
        case MDN_BUF_TERMINATED: *bytes = rows; return s->term;
        case MDN_BUF_TRUNCATED: *bytes = rows; return s->trunc;
        case MDN_BUF_ADVANTAGES: *bytes = rows * 4; return s->adv;
        case MDN_BUF_RETURNS: *bytes = rows * 4; return s->ret;
        case MDN_BUF_RAPTOR: *bytes = sizeof(mdn_raptor_weights); return &s->raptor;
        case MDN_BUF_PHYSICS: *bytes = sizeof(mdn_physics_params); return &s->physics;
        case MDN_BUF_CONTACT_ID: *bytes = rows * 4; return s->contact;
        case MDN_BUF_TASK_STATES: *bytes = n * sizeof(mdn_task_state); return s->tasks;
        case MDN_BUF_BANK_WORLDS: *bytes = (size_t)s->bank.bank_count * sizeof(mdn_world); return s->bank_worlds;
        case MDN_BUF_BANK_SCHEDULE: *bytes = s->bank_schedule ? n * s->bank.schedule_stride * 4 : 0; return s->bank_schedule;
        case MDN_BUF_BANK_ACTIVE_IDS: *bytes = n * 4; return s->bank_active;
        case MDN_BUF_BANK_TRANSITION_IDS: *bytes = rows * 4; return s->bank_transition;
        case MDN_BUF_ENV_PHYSICS: *bytes = n * sizeof(mdn_physics_params); return s->env_physics;
        case 100: *bytes = A_P * 4; return s->actor_m;
        case 101: *bytes = A_P * 4; return s->actor_v;
        case 102: *bytes = C_P * 4; return s->critic_m;
        case 103: *bytes = C_P * 4; return s->critic_v;
        default: *bytes = 0; return NULL;
    }
}

/* sim.metal:14-36 (cpu_reference.hpp:1-3,219-238); delay_rehearsal stands for
 * the NAV_DELAY_REHEARSAL build switch. */
static int clean_env(const o_sim* s, uint32_t n) {
    const mdn_sim_config* c = &s->cfg;
    return c->eval == 0 && (((c->family == 12 || c->family == 13) && n % 2 == 0) ||
                            (s->delay_rehearsal && c->mode == 22 && (n / 4) % 2 == 0));
}
static void rotation(const float q[4], float r[9]) { /* sim.metal:43-48, cpu_reference.hpp:82-87 */
    const float w = q[0], x = q[1], y = q[2], z = q[3];
    r[0] = 1 - 2 * (y * y + z * z); r[1] = 2 * (x * y - w * z); r[2] = 2 * (x * z + w * y);
    r[3] = 2 * (x * y + w * z); r[4] = 1 - 2 * (x * x + z * z); r[5] = 2 * (y * z - w * x);
    r[6] = 2 * (x * z - w * y); r[7] = 2 * (y * z + w * x); r[8] = 1 - 2 * (x * x + y * y);
}
static float sim_normal(uint32_t* rng) { /* sim.metal:49, cpu_reference.hpp:76-80 */
    const float u = smax(o_wurand(rng), 1e-7f), v = o_wurand(rng);
    return sqrtf(-2.0f * logf(u)) * cosf(6.28318530718f * v);
}

/* ---- per-episode plant variation, physics_domain.hpp:43-157 ---- */
static uint32_t domain_next(uint32_t* state) { /* :43-48 */
    uint32_t v = *state ? *state : 1u;
    v ^= v << 13;
    v ^= v >> 17;
    v ^= v << 5;
    *state = v ? v : 1u;
    return *state;
}
static float domain_scale(uint32_t* state, float low, float high, float amplitude) { /* :50-58 */
    const float u = (float)(domain_next(state) >> 8) * (1.0f / 16777216.0f);
    const float draw = low + (high - low) * u;
    return 1.0f + amplitude * (draw - 1.0f);
}
static int domain_inverse3(const float* m, float* inv) { /* :60-83 */
    const float a = m[0], b = m[1], c = m[2], d = m[3], e = m[4], f = m[5], g = m[6], h = m[7], i = m[8];
    for (int j = 0; j < 9; j++)
        if (!isfinite(m[j])) return 0;
    if (fabsf(b - d) > 1.0e-6f || fabsf(c - g) > 1.0e-6f || fabsf(f - h) > 1.0e-6f) return 0;
    const float minor2 = a * e - b * d;
    const float det = a * (e * i - f * h) - b * (d * i - f * g) + c * (d * h - e * g);
    if (!(a > 0.0f) || !(minor2 > 0.0f) || !(det > 0.0f) || !isfinite(det)) return 0;
    const float rcp = 1.0f / det;
    inv[0] = (e * i - f * h) * rcp; inv[1] = (c * h - b * i) * rcp; inv[2] = (b * f - c * e) * rcp;
    inv[3] = (f * g - d * i) * rcp; inv[4] = (a * i - c * g) * rcp; inv[5] = (c * d - a * f) * rcp;
    inv[6] = (d * h - e * g) * rcp; inv[7] = (b * g - a * h) * rcp; inv[8] = (a * e - b * d) * rcp;
    for (int j = 0; j < 9; j++)
        if (!isfinite(inv[j])) return 0;
    return 1;
}
static float domain_thrust_to_weight(const mdn_physics_params* p) { /* :85-95 */
    float thrust = 0.0f;
    const float action = p->action_max;
    for (int r = 0; r < 4; r++) {
        const float* k = p->rotor_thrust_coefficients + 3 * r;
        const float magnitude = k[0] + k[1] * action + k[2] * action * action;
        thrust += p->rotor_thrust_directions[3 * r + 2] * magnitude;
    }
    const float weight = p->mass * fabsf(p->gravity_world[2]);
    return weight > 0.0f ? thrust / weight : 0.0f;
}
/* rl_physics_sample_domain (:100-157). sample_out (may be NULL) receives the
 * 17 floats of RLPhysicsDomainSample. */
int o_physics_sample_domain(const mdn_physics_params* nominal, uint32_t* rng, float amplitude,
                            const mdn_domain_range* r, mdn_physics_params* varied, float* sample_out) {
    if (!isfinite(amplitude) || amplitude < 0.0f || amplitude > 1.0f || !isfinite(r->minimum_thrust_to_weight) ||
        r->minimum_thrust_to_weight < 1.0f || !isfinite(r->mass_scale_min) || !isfinite(r->mass_scale_max) ||
        !isfinite(r->inertia_axis_scale_min) || !isfinite(r->inertia_axis_scale_max) ||
        !isfinite(r->thrust_gain_min) || !isfinite(r->thrust_gain_max) || !isfinite(r->rising_lag_scale_min) ||
        !isfinite(r->rising_lag_scale_max) || !isfinite(r->falling_lag_scale_min) ||
        !isfinite(r->falling_lag_scale_max) || !(r->mass_scale_min > 0.0f && r->mass_scale_min <= r->mass_scale_max) ||
        !(r->inertia_axis_scale_min > 0.0f && r->inertia_axis_scale_min <= r->inertia_axis_scale_max) ||
        !(r->thrust_gain_min > 0.0f && r->thrust_gain_min <= r->thrust_gain_max) ||
        !(r->rising_lag_scale_min > 0.0f && r->rising_lag_scale_min <= r->rising_lag_scale_max) ||
        !(r->falling_lag_scale_min > 0.0f && r->falling_lag_scale_min <= r->falling_lag_scale_max))
        return 0;
    float sm[17]; /* mass, inertia axes[3], gain[4], rising[4], falling[4], thrust-to-weight */
    for (int k = 0; k < 16; k++) sm[k] = 1.0f;
    sm[16] = 0.0f;
    *varied = *nominal;
    if (amplitude > 0.0f) {
        sm[0] = domain_scale(rng, r->mass_scale_min, r->mass_scale_max, amplitude);
        for (int k = 0; k < 3; k++) sm[1 + k] = domain_scale(rng, r->inertia_axis_scale_min, r->inertia_axis_scale_max, amplitude);
        for (int k = 0; k < 4; k++) {
            sm[4 + k] = domain_scale(rng, r->thrust_gain_min, r->thrust_gain_max, amplitude);
            sm[8 + k] = domain_scale(rng, r->rising_lag_scale_min, r->rising_lag_scale_max, amplitude);
            sm[12 + k] = domain_scale(rng, r->falling_lag_scale_min, r->falling_lag_scale_max, amplitude);
        }
        varied->mass = nominal->mass * sm[0];
        float root[3];
        for (int k = 0; k < 3; k++) root[k] = sqrtf(sm[1 + k]);
        for (int row = 0; row < 3; row++)
            for (int col = 0; col < 3; col++)
                varied->inertia[3 * row + col] = nominal->inertia[3 * row + col] * sm[0] * root[row] * root[col];
        if (!domain_inverse3(varied->inertia, varied->inertia_inverse)) {
            if (sample_out) memcpy(sample_out, sm, sizeof(sm));
            return 0;
        }
        for (int k = 0; k < 4; k++) {
            for (int j = 0; j < 3; j++)
                varied->rotor_thrust_coefficients[3 * k + j] = nominal->rotor_thrust_coefficients[3 * k + j] * sm[4 + k];
            varied->rotor_time_constants_rising[k] = nominal->rotor_time_constants_rising[k] * sm[8 + k];
            varied->rotor_time_constants_falling[k] = nominal->rotor_time_constants_falling[k] * sm[12 + k];
        }
    }
    sm[16] = domain_thrust_to_weight(varied);
    if (sample_out) memcpy(sample_out, sm, sizeof(sm));
    return sm[16] >= r->minimum_thrust_to_weight;
}
/* sim_domain_episode_seed, sim.metal:50-54. */
uint32_t o_domain_episode_seed(const mdn_runtime_config* rt, uint32_t cfg_seed, uint32_t env, uint32_t episode) {
    uint32_t seed = rt->domain_seed ^ cfg_seed ^ ((env + 1u) * 0x9e3779b9u) ^ ((episode + 1u) * 0x85ebca6bu);
    seed ^= seed >> 16;
    seed *= 0x7feb352du;
    seed ^= seed >> 15;
    seed *= 0x846ca68bu;
    seed ^= seed >> 16;
    return seed ? seed : 1u;
}

/* sim_apply_challenge_world, sim.metal:95-122. */
static void apply_challenge_world(o_sim* s, uint32_t n, uint32_t slot) {
    const mdn_bank_control* b = &s->bank;
    if (b->enabled == 0 || b->bank_count == 0 || n >= s->cfg.n || slot >= b->schedule_stride) return;
    const uint32_t gid = s->env_base + n;
    const uint32_t level = s->bank_schedule[(size_t)n * b->schedule_stride + slot];
    mdn_sim_run* run = &s->runs[n];
    mdn_world* w = &s->worlds[n];
    if (level == 0xffffffffu) {
        uint32_t rng = run->rng;
        const uint32_t family = o_wtraining_family(gid % 2 == 0 ? 12u : 13u, &rng);
        o_wgenerate(w, o_wrng(&rng), family, 4.0f);
        run->rng = rng;
    } else {
        if (level >= b->bank_count) return;
        *w = s->bank_worlds[level];
    }
    w->wind[0] = clean_env(s, gid) ? 0.0f : s->cfg.wind;
    w->wind[1] = 0;
    w->wind[2] = 0;
    run->initial_distance = len3(w->goal[0], w->goal[1], w->goal[2] - 1.5f);
    if (w->family == 10 || w->family == 11) {
        s->states[n].linear_velocity[0] = s->cfg.speed;
        run->desired_velocity[0] = s->cfg.speed;
        run->previous_nav[0] = 1.0f;
    }
    s->bank_active[n] = level;
}

/* sim.metal:55-94 (cpu_reference.hpp:240-273); runtime domain randomisation off;
 * then the challenge-bank world of schedule slot `slot` (sim.metal:143,330). */
static void reset_one(o_sim* s, uint32_t n, int first, uint32_t slot) {
    const mdn_sim_config* c = &s->cfg;
    mdn_physics_state* st = &s->states[n];
    mdn_sim_run* run = &s->runs[n];
    mdn_world* w = &s->worlds[n];
    const uint32_t gid = s->env_base + n;
    uint32_t rng = first ? (c->seed + gid * 747796405u + 2891336453u) : run->rng;
    const uint32_t family = c->family == 18u ? o_mixed_lane_family(gid) : o_wtraining_family(c->family, &rng);
    o_wgenerate(w, o_wrng(&rng), family, c->distance);
    w->wind[0] = clean_env(s, gid) ? 0.0f : c->wind;
    w->wind[1] = 0;
    w->wind[2] = 0;
    for (int j = 0; j < 3; j++) {
        st->position[j] = j == 2 ? 1.5f : 0;
        st->linear_velocity[j] = 0;
        st->angular_velocity_body[j] = 0;
        run->desired_velocity[j] = 0;
        run->reference_position[j] = st->position[j];
    }
    st->orientation_wxyz[0] = 1;
    for (int j = 1; j < 4; j++) st->orientation_wxyz[j] = 0;
    const mdn_physics_params* p = &s->physics;
    float hover[4];
    /* sim.metal:62-82: the episode's plant, then hover at its thrust curve */
    mdn_physics_params* ep = &s->env_physics[n];
    *ep = *p;
    if (s->runtime.enabled && s->runtime.domain_amplitude > 0.0f) {
        uint32_t drng = o_domain_episode_seed(&s->runtime, c->seed, gid, first ? 0u : run->episodes);
        mdn_physics_params varied;
        if (o_physics_sample_domain(p, &drng, s->runtime.domain_amplitude, &s->runtime.domain_range, &varied, NULL))
            *ep = varied;
        else {
            const uint32_t qnan = 0x7fc00000u;
            memcpy(&ep->mass, &qnan, 4);
        }
    }
    if (!s->runtime.enabled) {
        const float target = p->mass * 9.81f / 4;
        const float c0 = p->rotor_thrust_coefficients[0], c1 = p->rotor_thrust_coefficients[1],
                    c2 = p->rotor_thrust_coefficients[2];
        const float h = clampf_((-c1 + sqrtf(c1 * c1 - 4 * c2 * (c0 - target))) / (2 * c2), p->action_min, p->action_max);
        for (int j = 0; j < 4; j++) hover[j] = h;
    } else {
        const float target = ep->mass * 9.81f / 4;
        for (int r = 0; r < 4; r++) {
            const float c0 = ep->rotor_thrust_coefficients[3 * r], c1 = ep->rotor_thrust_coefficients[3 * r + 1],
                        c2 = ep->rotor_thrust_coefficients[3 * r + 2];
            const float disc = c1 * c1 - 4 * c2 * (c0 - target);
            hover[r] = disc >= 0.0f ? clampf_((-c1 + sqrtf(disc)) / (2 * c2), ep->action_min, ep->action_max)
                                    : ep->action_max;
        }
    }
    memcpy(run->hidden, s->raptor.initial_hidden_state, sizeof(run->hidden));
    for (int j = 0; j < 4; j++) {
        st->rpm[j] = hover[j];
        run->motors[j] = 0;
        run->previous_nav[j] = 0;
    }
    if (family == 10 || family == 11) {
        st->linear_velocity[0] = c->speed;
        run->desired_velocity[0] = c->speed;
        run->previous_nav[0] = 1.0f;
    }
    for (uint32_t j = 0; j < NFRAMES * NPIX; j++) s->sensors[(size_t)n * NFRAMES * NPIX + j] = 12;
    for (uint32_t j = 0; j < NFRAMES * ACT; j++) s->commands[(size_t)n * NFRAMES * ACT + j] = 0;
    run->yaw = 0;
    run->rng = rng;
    run->steps = 0;
    run->path = run->elapsed = run->peak_speed = 0;
    run->min_clearance = 12;
    run->initial_distance = len3(w->goal[0], w->goal[1], w->goal[2] - 1.5f);
    if (first) {
        run->successes = run->collisions = run->timeouts = run->episodes = 0;
        run->success_time = run->total_path = run->total_elapsed = run->final_progress = 0;
        for (uint32_t j = 0; j < NFRAMES * 12; j++) s->poses[(size_t)n * NFRAMES * 12 + j] = 0;
    }
    if (s->bank.enabled) apply_challenge_world(s, n, slot);
    else s->bank_active[n] = 0xffffffffu;
    /* sim_reset_navigation_task, sim.metal:125-141 */
    mdn_task_state* task = &s->tasks[n];
    memset(task, 0, sizeof(*task));
    if (s->task_ctl.enabled) {
        uint32_t task_rng = c->seed ^ ((gid + 1u) * 0x27d4eb2du) ^ ((run->episodes + 1u) * 0x165667b1u);
        o_generate_task(w, task, &task_rng, &s->task_ctl.config, s->room);
        if (task->valid) {
            o_task_apply_start(task, st);
            run->yaw = task->start_yaw_rad;
            run->initial_distance = task->initial_distance_m;
            for (int a = 0; a < 3; a++) {
                run->reference_position[a] = st->position[a];
                run->desired_velocity[a] = st->linear_velocity[a];
            }
            w->wind[0] = clean_env(s, gid) ? 0.0f : c->wind;
            w->wind[1] = 0;
            w->wind[2] = 0;
        }
    }
}
void o_sim_reset(o_sim* s) {
    for (uint32_t n = 0; n < s->cfg.n; n++) reset_one(s, n, 1, 0);
}

/* sim.metal:145-158 (cpu_reference.hpp:278-302) */
static void depth_env(o_sim* s, uint32_t n) {
    const mdn_sim_config* c = &s->cfg;
    const mdn_sim_run* run = &s->runs[n];
    if ((c->eval && run->episodes) || run->steps % c->sensor_period != 0) return;
    const mdn_physics_state* st = &s->states[n];
    float r[9];
    rotation(st->orientation_wxyz, r);
    const float mx = 0.0f; /* legacy camera mount, sensor_profile.hpp:46 */
    const float origin[3] = {st->position[0] + mx * r[0], st->position[1] + mx * r[3], st->position[2] + mx * r[6]};
    const uint32_t frame = (run->steps / c->sensor_period) % NFRAMES;
    float* pose = s->poses + ((size_t)n * NFRAMES + frame) * 12;
    pose[0] = origin[0]; pose[1] = origin[1]; pose[2] = origin[2];
    for (int j = 0; j < 9; j++) pose[3 + j] = r[j];
    const uint32_t gid = s->env_base + n;
    const float noise = clean_env(s, gid) ? 0.0f : c->depth_noise, dropout = clean_env(s, gid) ? 0.0f : c->dropout;
    for (uint32_t k = 0; k < NPIX; k++) {
        const float* ray = s->pixel_rays + 3 * k;
        const float d[3] = {r[0] * ray[0] + r[1] * ray[1] + r[2] * ray[2], r[3] * ray[0] + r[4] * ray[1] + r[5] * ray[2],
                            r[6] * ray[0] + r[7] * ray[1] + r[8] * ray[2]};
        float depth = o_wray(&s->worlds[n], s->room, origin, d, run->elapsed);
        if (noise != 0 || dropout != 0) {
            uint32_t rng = run->rng + k * 1664525u + run->steps * 1013904223u;
            depth = clampf_(depth + noise * sim_normal(&rng), 0.0f, 12.0f);
            if (o_wurand(&rng) < dropout) depth = 12.0f;
        }
        s->sensors[((size_t)n * NFRAMES + frame) * NPIX + k] = depth;
    }
}

/* sim.metal:159-165 (cpu_reference.hpp:379-394) */
static void critic_obs(const o_sim* s, const mdn_physics_state* st, const mdn_world* w, const mdn_sim_run* run,
                       float* o) {
    memset(o, 0, COBS * 4);
    for (int j = 0; j < 3; j++) {
        o[j] = (w->goal[j] - st->position[j]) / 10.0f;
        o[j + 3] = st->linear_velocity[j] / 4.0f;
        o[j + 6] = st->angular_velocity_body[j] / 4.0f;
        o[j + 13] = st->position[j] / 10.0f;
        o[j + 16] = (run->reference_position[j] - st->position[j]) * 2.0f;
    }
    for (int j = 0; j < 4; j++) o[9 + j] = st->orientation_wxyz[j];
    o[30] = w->wind[0];
    o[31] = w->wind[1];
    o[19] = o_wclearance(w, s->room, st->position, run->elapsed, NULL) / 5.0f;
    o[20] = (float)run->steps / 200.0f;
    const uint32_t m = w->count < 3 ? w->count : 3;
    for (uint32_t j = 0; j < m; j++) {
        float c[3];
        o_wc(&w->obstacles[j], run->elapsed, c);
        o[21 + j * 3] = (c[0] - st->position[0]) / 10.0f;
        o[22 + j * 3] = (c[1] - st->position[1]) / 10.0f;
        o[23 + j * 3] = (c[2] - st->position[2]) / 10.0f;
    }
}

/* sim.metal:166-180, the control-state inputs 32..63 of the delay-training
 * build's critic (FIXED_PPO_CRITIC_OBS_DIM=64, NAV_CRITIC_CONTROL_STATE=1;
 * the reference has this only in its Metal kernel, so this restatement is the
 * check). o points at input 32. */
static void critic_control_state(const mdn_physics_state* st, const mdn_world* w, const mdn_sim_run* run, float* o) {
    for (int j = 0; j < 16; j++) o[j] = run->hidden[j];
    for (int j = 0; j < 4; j++) {
        o[16 + j] = st->rpm[j];
        o[22 + j] = run->previous_nav[j];
    }
    const float* q = st->orientation_wxyz;
    const float yaw = atan2f(2.0f * (q[0] * q[3] + q[1] * q[2]), 1.0f - 2.0f * (q[2] * q[2] + q[3] * q[3]));
    o[20] = sinf(run->yaw - yaw);
    o[21] = cosf(run->yaw - yaw);
    for (int j = 0; j < 3; j++) o[26 + j] = run->desired_velocity[j] / 2.0f;
    const float g[3] = {w->goal[0] - st->position[0], w->goal[1] - st->position[1], w->goal[2] - st->position[2]};
    const float* v = st->linear_velocity;
    const float distance = sqrtf(g[0] * g[0] + g[1] * g[1] + g[2] * g[2]);
    o[29] = (g[0] * v[0] + g[1] * v[1] + g[2] * v[2]) / fmaxf(distance, 1e-6f) / 4.0f;
    o[30] = distance / 10.0f;
    o[31] = sqrtf(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]) / 4.0f;
}

/* The critic observation (sim_critic_obs, sim.metal:159-180) of `count`
 * environments from their state, `dim` = 32 or 64 (control-state critic)
 * floats per row; the room is the simulator's. */
void o_critic_obs_rows(const o_sim* s, const mdn_physics_state* states, const mdn_world* worlds,
                       const mdn_sim_run* runs, uint32_t count, uint32_t dim, float* out) {
    for (uint32_t n = 0; n < count; n++) {
        float* o = out + (size_t)n * dim;
        critic_obs(s, &states[n], &worlds[n], &runs[n], o);
        if (dim == 64) critic_control_state(&states[n], &worlds[n], &runs[n], o + COBS);
    }
}

/* sim.metal:182-228 (cpu_reference.hpp:303-377) */
static void observe_env(o_sim* s, uint32_t t, uint32_t n) {
    const mdn_sim_config* c = &s->cfg;
    const mdn_sim_run* run = &s->runs[n];
    if (c->eval && run->episodes) return;
    const mdn_physics_state* st = &s->states[n];
    const mdn_world* w = &s->worlds[n];
    float r[9];
    rotation(st->orientation_wxyz, r);
    const uint32_t delay = clean_env(s, s->env_base + n) ? 0 : c->sensor_delay;
    const uint32_t available = run->steps / c->sensor_period;
    const uint32_t frame = available > delay ? available - delay : 0;
    const uint32_t prev = frame > 0 ? frame - 1 : 0;
    float* o = s->obs + ((size_t)t * c->n + n) * AOBS;
    const float* ring = s->sensors + (size_t)n * NFRAMES * NPIX;
    for (uint32_t k = 0; k < 80; k++) {
        float cur = 12.0f, pre = 12.0f;
        const uint32_t y = (k / 10) * 2, x = (k % 10) * 2;
        for (uint32_t dy = 0; dy < 2; dy++)
            for (uint32_t dx = 0; dx < 2; dx++) {
                const uint32_t pixel = (y + dy) * 20 + x + dx;
                cur = smin(cur, ring[(frame % NFRAMES) * NPIX + pixel]);
                pre = smin(pre, ring[(prev % NFRAMES) * NPIX + pixel]);
            }
        o[k] = available >= delay ? cur / 12.0f : 1.0f;
        o[80 + k] = available >= delay ? pre / 12.0f : 1.0f;
    }
    if (c->mode == 18)
        for (uint32_t k = 0; k < 80; k++) o[80 + k] = o[k];
    const float delta[3] = {w->goal[0] - st->position[0], w->goal[1] - st->position[1], w->goal[2] - st->position[2]};
    const float distance = smax(len3(delta[0], delta[1], delta[2]), 1.0e-6f);
    float* ctx = o + 160;
    for (int j = 0; j < 3; j++) {
        ctx[j] = (r[j] * delta[0] + r[3 + j] * delta[1] + r[6 + j] * delta[2]) / distance;
        ctx[4 + j] = (r[j] * st->linear_velocity[0] + r[3 + j] * st->linear_velocity[1] + r[6 + j] * st->linear_velocity[2]) / 4.0f;
        ctx[7 + j] = st->angular_velocity_body[j] / 4.0f;
        ctx[10 + j] = r[6 + j];
    }
    ctx[3] = smin(distance / 10.0f, 1.5f);
    for (int j = 0; j < 4; j++) ctx[13 + j] = run->previous_nav[j];
    ctx[17] = (float)(run->steps - frame * c->sensor_period) * s->physics.dt * (float)c->substeps;
    const float ref[3] = {run->reference_position[0] - st->position[0], run->reference_position[1] - st->position[1],
                          run->reference_position[2] - st->position[2]};
    for (int j = 0; j < 3; j++) ctx[18 + j] = clampf_((r[j] * ref[0] + r[3 + j] * ref[1] + r[6 + j] * ref[2]) * 2.0f, -1.0f, 1.0f);
    float cur[80], pre[80], goal[3], vel[3], hint[3], pose[12];
    for (int j = 0; j < 80; j++) {
        cur[j] = o[j] * 12.0f;
        pre[j] = o[80 + j] * 12.0f;
    }
    for (int j = 0; j < 3; j++) {
        goal[j] = ctx[j];
        vel[j] = ctx[4 + j] * 4.0f;
        pose[j] = st->position[j];
    }
    for (int j = 0; j < 9; j++) pose[j + 3] = r[j];
    const float sensor_dt = (float)c->sensor_period * s->physics.dt * (float)c->substeps;
    if (c->geometry_memory) {
        const uint32_t valid = available >= delay ? (frame + 1 < NFRAMES - delay ? frame + 1 : NFRAMES - delay) : 0;
        o_nav_guidance_memory(cur, pre, goal, distance, vel, sensor_dt, 0.75f, ring, s->poses + (size_t)n * NFRAMES * 12,
                              pose, frame, valid, hint, ctx[17]);
    } else {
        o_nav_guidance(cur, pre, goal, distance, vel, sensor_dt, 0.75f, hint);
    }
    for (int j = 0; j < 3; j++) o[181 + j] = hint[j];
    critic_obs(s, st, w, run, s->co + ((size_t)t * c->n + n) * COBS);
}

/* Batched MLPs as cpu_reference.hpp:437-458 evaluates them: in-order dot
 * product from zero, then the bias. */
static void actor_forward_row(const float* actor, const float* obs, float* hidden, float* mean) {
    for (uint32_t h = 0; h < HID; h++) {
        float acc = 0.0f;
        for (uint32_t i = 0; i < AOBS; i++) acc += obs[i] * actor[h * AOBS + i];
        hidden[h] = tanhf(acc + actor[A_B1 + h]);
    }
    for (uint32_t a = 0; a < ACT; a++) {
        float acc = 0.0f;
        for (uint32_t h = 0; h < HID; h++) acc += hidden[h] * actor[A_W2 + a * HID + h];
        mean[a] = acc + actor[A_B2 + a];
        if (a < 3) mean[a] += obs[AOBS - 3 + a];
    }
}
static float critic_forward_row(const float* critic, const float* co, float* hidden) {
    for (uint32_t h = 0; h < HID; h++) {
        float acc = 0.0f;
        for (uint32_t i = 0; i < COBS; i++) acc += co[i] * critic[h * COBS + i];
        hidden[h] = tanhf(acc + critic[C_B1 + h]);
    }
    float acc = 0.0f;
    for (uint32_t h = 0; h < HID; h++) acc += hidden[h] * critic[C_W2 + h];
    return acc + critic[C_B2];
}

/* sim_act (sim.metal:229-271): value, mode-dependent mean (geometry-prior
 * blending for modes 9-21), sampling (cpu_reference.hpp:404-429 for mode 0),
 * deployed action map (mode 22), scripted goal velocity (modes 2, 3, 20),
 * command delay, velocity contract, fixed-speed ablation (mode 19). */
static void act_env(o_sim* s, uint32_t t, uint32_t n) {
    const mdn_sim_config* c = &s->cfg;
    mdn_sim_run* run = &s->runs[n];
    if (c->eval && run->episodes) return;
    const size_t row = (size_t)t * c->n + n;
    const float* ob = s->obs + row * AOBS;
    float hidden[HID], mean[ACT], a[ACT];
    actor_forward_row(s->actor, ob, hidden, mean);
    s->values[row] = critic_forward_row(s->critic, s->co + row * COBS, hidden);
    const uint32_t mode = c->mode;
    if (mode >= 9 && mode <= 21) {
        float scale = (mode == 9 || mode == 13) ? 0.0f
                    : ((mode == 10 || mode == 14 || mode == 16) ? 0.25f : (mode == 15 ? 1.0f : 0.5f));
        if (mode >= 17) {
            float overhead = 0;
            for (int k = 0; k < 20; k++) overhead += ob[k] * 12 > 2.5f;
            scale = .25f + .75f * (overhead / 20.0f);
        }
        if (mode == 12) {
            float near_ = 12;
            for (int k = 0; k < 80; k++) near_ = fminf(near_, ob[k] * 12);
            scale = fminf(fmaxf((near_ - .3f) / 2, 0.2f), 1.0f);
        }
        for (int j = 0; j < 3; j++) {
            const float prior = ob[AOBS - 3 + j];
            mean[j] = prior + scale * (mean[j] - prior);
        }
        mean[3] *= scale;
        if (mode == 16) {
            const float yaw = atan2f(ob[161], ob[160]);
            mean[3] += nav_atanh(fminf(fmaxf(yaw * 1.5f, -.85f), .85f));
        }
    }
    float deployed_scale = 1.0f;
    if (mode == 22) {
        float overhead = 0;
        for (int k = 0; k < 20; k++) overhead += ob[k] * 12 > 2.5f;
        deployed_scale = .25f + .75f * (overhead / 20.0f);
    }
    const float* log_std = s->actor + A_LS;
    uint32_t rng = run->rng;
    float* cmd = s->commands + (size_t)n * NFRAMES * ACT;
    for (uint32_t j = 0; j < ACT; j++) {
        a[j] = mean[j] + ((mode == 0 || mode == 22) ? expf(log_std[j]) * sim_normal(&rng) : 0);
        if (mode == 1) a[j] = sim_normal(&rng);
        s->actions[row * ACT + j] = a[j];
        float executed = a[j];
        if (mode == 22) executed = j < 3 ? ob[AOBS - 3 + j] + deployed_scale * (a[j] - ob[AOBS - 3 + j]) : deployed_scale * a[j];
        cmd[(run->steps % NFRAMES) * ACT + j] = tanhf(executed);
    }
    s->logp[row] = gaussian_log_prob(s->actions + row * ACT, mean, log_std);
    run->rng = rng;
    const mdn_physics_state* st = &s->states[n];
    if (mode == 2 || mode == 3 || mode == 20) {
        const mdn_world* w = &s->worlds[n];
        float d[3] = {w->goal[0] - st->position[0], w->goal[1] - st->position[1], w->goal[2] - st->position[2]};
        const float len = len3(d[0], d[1], d[2]);
        const float inv = 1.0f / len, keep = smin(len, c->speed);
        for (int j = 0; j < 3; j++) d[j] = d[j] * inv * keep;
        float r[9];
        rotation(st->orientation_wxyz, r);
        const float sc[4] = {(r[0] * d[0] + r[3] * d[1] + r[6] * d[2]) / c->speed,
                             (r[1] * d[0] + r[4] * d[1] + r[7] * d[2]) / c->speed,
                             (r[2] * d[0] + r[5] * d[1] + r[8] * d[2]) / c->speed, 0.0f};
        for (int j = 0; j < 4; j++) cmd[(run->steps % NFRAMES) * ACT + j] = sc[j];
    }
    const uint32_t delay = clean_env(s, s->env_base + n) ? 0 : c->command_delay;
    const uint32_t applied = run->steps > delay ? run->steps - delay : 0;
    for (uint32_t j = 0; j < ACT; j++) run->previous_nav[j] = run->steps < delay ? 0.0f : cmd[(applied % NFRAMES) * ACT + j];
    float r[9];
    rotation(st->orientation_wxyz, r);
    float v[3] = {run->previous_nav[0] * c->speed, run->previous_nav[1] * c->speed,
                  run->previous_nav[2] * c->speed * (c->velocity_contract == 0 ? 0.5f : 1.0f)};
    if (c->velocity_contract == 1) {
        const float scale = smin(1.0f, c->speed / smax(len3(v[0], v[1], v[2]), 1e-8f));
        for (int j = 0; j < 3; j++) v[j] *= scale;
    }
    if (mode == 19) {
        const float magnitude = len3(v[0], v[1], v[2]);
        if (magnitude > 1e-8f) {
            const float scale = c->speed / magnitude;
            for (int j = 0; j < 3; j++) v[j] *= scale;
        }
    }
    for (int j = 0; j < 3; j++) run->desired_velocity[j] = r[j * 3] * v[0] + r[j * 3 + 1] * v[1] + r[j * 3 + 2] * v[2];
    run->yaw += run->previous_nav[3] * s->physics.dt * (float)c->substeps * 0.5f;
}

static int finite3(const float* v) { return isfinite(v[0]) && isfinite(v[1]) && isfinite(v[2]); }

/* sim_advance (sim.metal:272-332) / advance_env (cpu_reference.hpp:460-513),
 * plus the nearest-obstacle id at the step's closest approach. */
static void advance_env(o_sim* s, uint32_t t, uint32_t n) {
    const mdn_sim_config* c = &s->cfg;
    mdn_sim_run* run = &s->runs[n];
    if (c->eval && run->episodes) return;
    const size_t row = (size_t)t * c->n + n;
    const mdn_physics_params* p = &s->physics;
    mdn_world* w = &s->worlds[n];
    mdn_physics_state st = s->states[n];
    float h[16], motors[4];
    memcpy(h, run->hidden, sizeof(h));
    memcpy(motors, run->motors, sizeof(motors));
    const float before = len3(w->goal[0] - st.position[0], w->goal[1] - st.position[1], w->goal[2] - st.position[2]);
    const float yaw = run->yaw, cy = cosf(yaw), sy = sinf(yaw);
    int collision = 0;
    float step_clearance = 12.0f;
    int32_t contact = -1;
    /* sim.metal:287: the episode plant integrates while the runtime config is on */
    const mdn_physics_params* plant = s->runtime.enabled ? &s->env_physics[n] : p;
    const float wind[3] = {w->wind[0] * plant->mass, w->wind[1] * plant->mass, w->wind[2] * plant->mass};
    for (uint32_t step = 0; step < c->substeps; step++) {
        float mo[22];
        const float v[3] = {run->desired_velocity[0], run->desired_velocity[1], run->desired_velocity[2]};
        for (int j = 0; j < 3; j++) run->reference_position[j] += v[j] * p->dt;
        const float dp[3] = {st.position[0] - run->reference_position[0], st.position[1] - run->reference_position[1],
                             st.position[2] - run->reference_position[2]};
        const float dv[3] = {st.linear_velocity[0] - v[0], st.linear_velocity[1] - v[1], st.linear_velocity[2] - v[2]};
        mo[0] = clampf_(cy * dp[0] + sy * dp[1], -.5f, .5f);
        mo[1] = clampf_(-sy * dp[0] + cy * dp[1], -.5f, .5f);
        mo[2] = clampf_(dp[2], -.5f, .5f);
        const float ch = cosf(yaw * .5f), sh = sinf(yaw * .5f);
        const float* qs = st.orientation_wxyz;
        const float q[4] = {ch * qs[0] + sh * qs[3], ch * qs[1] + sh * qs[2], ch * qs[2] - sh * qs[1], ch * qs[3] - sh * qs[0]};
        float r[9];
        rotation(q, r);
        for (int j = 0; j < 9; j++) mo[3 + j] = r[j];
        mo[12] = clampf_(cy * dv[0] + sy * dv[1], -1.0f, 1.0f);
        mo[13] = clampf_(-sy * dv[0] + cy * dv[1], -1.0f, 1.0f);
        mo[14] = clampf_(dv[2], -1.0f, 1.0f);
        for (int j = 0; j < 3; j++) mo[15 + j] = st.angular_velocity_body[j];
        for (int j = 0; j < 4; j++) mo[18 + j] = motors[j];
        o_raptor_forward(&s->raptor, mo, h, motors);
        for (int j = 0; j < 4; j++) motors[j] = smax(-1.0f, smin(1.0f, motors[j])); /* raptor.hpp:95-97 */
        mdn_physics_state next;
        o_physics_step(&st, motors, wind, plant, &next);
        const int valid = finite3(next.position) && finite3(next.linear_velocity) && finite3(next.angular_velocity_body) &&
                          isfinite(next.orientation_wxyz[0]) && isfinite(next.orientation_wxyz[1]) &&
                          isfinite(next.orientation_wxyz[2]) && isfinite(next.orientation_wxyz[3]) &&
                          isfinite(next.rpm[0]) && isfinite(next.rpm[1]) && isfinite(next.rpm[2]) && isfinite(next.rpm[3]);
        if (!valid) {
            collision = 1;
            break;
        }
        run->path += len3(st.position[0] - next.position[0], st.position[1] - next.position[1], st.position[2] - next.position[2]);
        st = next;
        run->elapsed += p->dt;
        int32_t id;
        const float clearance = o_wclearance(w, s->room, st.position, run->elapsed, &id);
        if (clearance < step_clearance) contact = id;
        step_clearance = smin(step_clearance, clearance);
        run->min_clearance = smin(run->min_clearance, clearance);
        run->peak_speed = smax(run->peak_speed, len3(st.linear_velocity[0], st.linear_velocity[1], st.linear_velocity[2]));
        if (clearance <= 0 || !finite3(st.position)) {
            collision = 1;
            break;
        }
    }
    run->steps++;
    s->states[n] = st;
    memcpy(run->hidden, h, sizeof(h));
    memcpy(run->motors, motors, sizeof(motors));
    const float after = len3(w->goal[0] - st.position[0], w->goal[1] - st.position[1], w->goal[2] - st.position[2]);
    int success = after < (c->mode == 20 ? .10f : .35f) && !collision, timeout = run->steps >= c->max_steps;
    s->rewards[row] = (before - after) * 2.0f - .01f - c->risk_coef * clampf_((0.6f - step_clearance) / 0.6f, 0.0f, 1.0f) +
                      (success ? 10.0f : 0.0f) - (collision ? 10.0f : 0.0f);
    s->term[row] = (uint8_t)(collision || success);
    s->trunc[row] = (uint8_t)(timeout && !s->term[row]);
    s->contact[row] = contact;
    if (s->task_ctl.enabled) {
        const float executed[4] = {run->desired_velocity[0], run->desired_velocity[1], run->desired_velocity[2],
                                   run->previous_nav[3] * 0.5f};
        uint32_t outcome[8];
        o_task_step(&s->tasks[n], &s->task_ctl.config, st.position, st.linear_velocity, executed, (uint32_t)collision,
                    (uint32_t)timeout, outcome);
        success = outcome[4] != 0 && !collision;
        timeout = outcome[6] != 0;
        memcpy(&s->rewards[row], &outcome[0], 4);
        s->term[row] = (uint8_t)(collision || success);
        s->trunc[row] = (uint8_t)(timeout && !s->term[row]);
    }
    float co[COBS], hidden[HID];
    critic_obs(s, &st, w, run, co);
    s->next_values[row] = critic_forward_row(s->critic, co, hidden);
    s->bank_transition[row] = s->bank.enabled ? s->bank_active[n] : 0xffffffffu; /* sim.metal:326 */
    if (success || collision || timeout) {
        run->successes += success;
        run->collisions += collision;
        run->timeouts += timeout && !s->term[row];
        run->episodes++;
        run->success_time += success ? run->elapsed : 0;
        run->total_path += run->path;
        run->total_elapsed += run->elapsed;
        run->final_progress += 1.0f - after / smax(run->initial_distance, 1.0e-4f);
        if (!c->eval) reset_one(s, n, 0, t + 1);
    }
}

void o_sim_observe(o_sim* s, uint32_t t) {
#pragma omp parallel for schedule(dynamic, 8)
    for (long n = 0; n < (long)s->cfg.n; n++) {
        depth_env(s, (uint32_t)n);
        observe_env(s, t, (uint32_t)n);
    }
}
void o_sim_act(o_sim* s, uint32_t t) {
#pragma omp parallel for schedule(static)
    for (long n = 0; n < (long)s->cfg.n; n++) act_env(s, t, (uint32_t)n);
}
void o_sim_advance(o_sim* s, uint32_t t) {
#pragma omp parallel for schedule(dynamic, 8)
    for (long n = 0; n < (long)s->cfg.n; n++) advance_env(s, t, (uint32_t)n);
}
void o_sim_step(o_sim* s, uint32_t t) {
    o_sim_observe(s, t);
    o_sim_act(s, t);
    o_sim_advance(s, t);
}
void o_sim_gae_normalize(o_sim* s, int normalize) {
    o_compute_gae(s->horizon, s->cfg.n, s->rewards, s->values, s->next_values, s->term, s->trunc, 0.99f, 0.95f, s->adv,
                  s->ret);
    if (normalize) o_normalize_advantages(s->adv, (size_t)s->cfg.n * s->horizon);
}

/* train_rollout (cpu_reference.hpp:569-608) with the chunk order supplied by
 * the caller, gradients as actor_gradients/critic_gradients (:515-551) and
 * clip_and_adam (:553-567). */
static void clip_and_adam(float* grad, float* params, float* m, float* v, size_t count, float b1c, float b2c, float lr,
                          float* norm_out) {
    float sum = 0.0f;
    for (size_t i = 0; i < count; i++) sum += grad[i] * grad[i];
    const float norm = sqrtf(sum + 1.0e-20f);
    if (norm_out) *norm_out = norm;
    const float scale = smin(1.0f, 0.5f / norm);
    for (size_t i = 0; i < count; i++) grad[i] *= scale;
    o_adam_update(params, grad, m, v, count, b1c, b2c, lr);
}
void o_sim_train_rollout(o_sim* s, uint32_t mb, uint32_t epochs, const uint32_t* order, uint32_t chunks,
                         const float* b1corr, const float* b2corr, float* out, float* grad_norms) {
    const uint32_t rows = s->cfg.n * s->horizon;
    float* ah = malloc((size_t)mb * HID * 4);
    float* am = malloc((size_t)mb * ACT * 4);
    float* ch = malloc((size_t)mb * HID * 4);
    float* cv = malloc((size_t)mb * 4);
    float* dm = malloc((size_t)mb * ACT * 4);
    float* dls = malloc((size_t)mb * ACT * 4);
    float* dv = malloc((size_t)mb * 4);
    float* adelta = malloc((size_t)mb * HID * 4);
    float* cdelta = malloc((size_t)mb * HID * 4);
    float* ag = malloc(A_P * 4);
    float* cg = malloc(C_P * 4);
    float policy_sum = 0, value_sum = 0, entropy_sum = 0, ratio_sum = 0;
    const float ecoef = s->cfg.entropy_coef, lr = s->cfg.learning_rate;
    uint32_t u = 0;
    for (uint32_t e = 0; e < epochs; e++)
        for (uint32_t ci = 0; ci < chunks; ci++, u++) {
            const uint32_t begin = order[(size_t)e * chunks + ci];
            const uint32_t b = mb < rows - begin ? mb : rows - begin;
            const float* ob = s->obs + (size_t)begin * AOBS;
            const float* co = s->co + (size_t)begin * COBS;
            for (uint32_t n = 0; n < b; n++) {
                actor_forward_row(s->actor, ob + (size_t)n * AOBS, ah + (size_t)n * HID, am + (size_t)n * ACT);
                cv[n] = critic_forward_row(s->critic, co + (size_t)n * COBS, ch + (size_t)n * HID);
            }
            for (uint32_t n = 0; n < b; n++) {
                float l[4];
                o_sample_loss_and_grad(s->actions + (size_t)(begin + n) * ACT, am + (size_t)n * ACT, s->actor + A_LS,
                                       s->logp[begin + n], cv[n], s->adv[begin + n], s->ret[begin + n], (float)b, 0.2f,
                                       0.5f, ecoef, dm + (size_t)n * ACT, dls + (size_t)n * ACT, &dv[n], l);
                policy_sum += l[0];
                value_sum += l[1];
                entropy_sum += l[2];
                ratio_sum += l[3] / (float)b;
            }
            /* actor_gradients, cpu_reference.hpp:515-533 */
            for (uint32_t n = 0; n < b; n++)
                for (uint32_t h = 0; h < HID; h++) {
                    float acc = 0.0f;
                    for (uint32_t a = 0; a < ACT; a++) acc += dm[n * ACT + a] * s->actor[A_W2 + a * HID + h];
                    adelta[n * HID + h] = acc;
                }
            for (uint32_t n = 0; n < b; n++)
                for (uint32_t h = 0; h < HID; h++) adelta[n * HID + h] *= 1.0f - ah[n * HID + h] * ah[n * HID + h];
            memset(ag, 0, A_P * 4);
            for (uint32_t h = 0; h < HID; h++)
                for (uint32_t i = 0; i < AOBS; i++) {
                    float acc = 0.0f;
                    for (uint32_t n = 0; n < b; n++) acc += adelta[n * HID + h] * ob[(size_t)n * AOBS + i];
                    ag[h * AOBS + i] = acc;
                }
            for (uint32_t a = 0; a < ACT; a++)
                for (uint32_t h = 0; h < HID; h++) {
                    float acc = 0.0f;
                    for (uint32_t n = 0; n < b; n++) acc += dm[n * ACT + a] * ah[n * HID + h];
                    ag[A_W2 + a * HID + h] = acc;
                }
            for (uint32_t n = 0; n < b; n++)
                for (uint32_t h = 0; h < HID; h++) ag[A_B1 + h] += adelta[n * HID + h];
            for (uint32_t n = 0; n < b; n++)
                for (uint32_t a = 0; a < ACT; a++) {
                    ag[A_B2 + a] += dm[n * ACT + a];
                    ag[A_LS + a] += dls[n * ACT + a];
                }
            /* critic_gradients, cpu_reference.hpp:535-551 */
            for (uint32_t n = 0; n < b; n++)
                for (uint32_t h = 0; h < HID; h++) cdelta[n * HID + h] = dv[n] * s->critic[C_W2 + h];
            for (uint32_t n = 0; n < b; n++)
                for (uint32_t h = 0; h < HID; h++) cdelta[n * HID + h] *= 1.0f - ch[n * HID + h] * ch[n * HID + h];
            memset(cg, 0, C_P * 4);
            for (uint32_t h = 0; h < HID; h++)
                for (uint32_t i = 0; i < COBS; i++) {
                    float acc = 0.0f;
                    for (uint32_t n = 0; n < b; n++) acc += cdelta[n * HID + h] * co[(size_t)n * COBS + i];
                    cg[h * COBS + i] = acc;
                }
            for (uint32_t h = 0; h < HID; h++) {
                float acc = 0.0f;
                for (uint32_t n = 0; n < b; n++) acc += dv[n] * ch[n * HID + h];
                cg[C_W2 + h] = acc;
            }
            for (uint32_t n = 0; n < b; n++) {
                cg[C_B2] += dv[n];
                for (uint32_t h = 0; h < HID; h++) cg[C_B1 + h] += cdelta[n * HID + h];
            }
            clip_and_adam(ag, s->actor, s->actor_m, s->actor_v, A_P, b1corr[u], b2corr[u], lr,
                          grad_norms ? grad_norms + 2 * u : NULL);
            clip_and_adam(cg, s->critic, s->critic_m, s->critic_v, C_P, b1corr[u], b2corr[u], lr,
                          grad_norms ? grad_norms + 2 * u + 1 : NULL);
            for (uint32_t a = 0; a < ACT; a++) s->actor[A_LS + a] = clampf_(s->actor[A_LS + a], -2.0f, .5f);
        }
    const float scale = 1.0f / (float)(epochs * chunks);
    out[0] = policy_sum * scale;
    out[1] = value_sum * scale;
    out[2] = entropy_sum * scale;
    out[3] = ratio_sum * scale;
    free(ah); free(am); free(ch); free(cv); free(dm); free(dls); free(dv); free(adelta); free(cdelta); free(ag); free(cg);
}

/* Raw gradient [actor | critic] of the clipped-PPO objective over the listed
 * rollout rows, each row's loss scaled by 1/batch (ppo.hpp:144-181 with
 * cpu_reference.hpp:515-551 as the per-row sums). Used to check the sharded
 * update: a global minibatch is the union of the ranks' chunks. */
void o_sim_rows_grad(o_sim* s, const uint32_t* rows, uint32_t count, float batch, float* grad) {
    memset(grad, 0, (A_P + C_P) * 4);
    float* ag = grad;
    float* cg = grad + A_P;
    float h[HID], ch[HID], mean[ACT];
    for (uint32_t k = 0; k < count; k++) {
        const uint32_t r = rows[k];
        const float* ob = s->obs + (size_t)r * AOBS;
        const float* co = s->co + (size_t)r * COBS;
        actor_forward_row(s->actor, ob, h, mean);
        const float v = critic_forward_row(s->critic, co, ch);
        float dm[ACT], dls[ACT], dv, l[4];
        o_sample_loss_and_grad(s->actions + (size_t)r * ACT, mean, s->actor + A_LS, s->logp[r], v, s->adv[r], s->ret[r],
                               batch, 0.2f, 0.5f, s->cfg.entropy_coef, dm, dls, &dv, l);
        for (uint32_t j = 0; j < HID; j++) {
            float acc = 0.0f;
            for (uint32_t a = 0; a < ACT; a++) acc += dm[a] * s->actor[A_W2 + a * HID + j];
            const float d = acc * (1.0f - h[j] * h[j]);
            for (uint32_t i = 0; i < AOBS; i++) ag[j * AOBS + i] += d * ob[i];
            ag[A_B1 + j] += d;
            const float cd = dv * s->critic[C_W2 + j] * (1.0f - ch[j] * ch[j]);
            for (uint32_t i = 0; i < COBS; i++) cg[j * COBS + i] += cd * co[i];
            cg[C_B1 + j] += cd;
            cg[C_W2 + j] += dv * ch[j];
        }
        for (uint32_t a = 0; a < ACT; a++) {
            for (uint32_t j = 0; j < HID; j++) ag[A_W2 + a * HID + j] += dm[a] * h[j];
            ag[A_B2 + a] += dm[a];
            ag[A_LS + a] += dls[a];
        }
        cg[C_B2] += dv;
    }
}

/* ----------------------------------------------------------- wide actor */
/* The one-hidden-layer tanh actor of ppo.hpp:65-80 at hidden width `hidden`
 * (the reference builds it with FIXED_PPO_HIDDEN_DIM; 5120 gives its
 * 967,688-parameter actor, navigation_wide_deployment.hpp:54-66). Parameter
 * offsets as ppo.hpp:35-40 with that width. */
uint32_t o_wide_param_count(uint32_t hidden) { return hidden * AOBS + hidden + ACT * hidden + ACT + ACT; }

/* main.mm:548-555 for an actor of width `hidden` and the 64-unit critic: one
 * seed-1789 stream, actor W1, actor W2, critic W1, critic W2 in that order. */
void o_wide_init(uint32_t hidden, float* actor, float* critic) {
    const size_t b1 = (size_t)hidden * AOBS, w2 = b1 + hidden, b2 = w2 + (size_t)ACT * hidden, ls = b2 + ACT;
    memset(actor, 0, o_wide_param_count(hidden) * sizeof(float));
    memset(critic, 0, C_P * sizeof(float));
    uint32_t seed = 1789;
    for (size_t i = 0; i < b1; i++) {
        const float u = smax(o_wurand(&seed), 1.0e-7f);
        const float a = sqrtf(-2.0f * logf(u));
        actor[i] = a * cosf(6.2831853f * o_wurand(&seed)) * 0.04f;
    }
    for (size_t i = w2; i < b2; i++) {
        const float u = smax(o_wurand(&seed), 1.0e-7f);
        const float a = sqrtf(-2.0f * logf(u));
        actor[i] = a * cosf(6.2831853f * o_wurand(&seed)) * 0.01f;
    }
    for (size_t i = 0; i < ACT; i++) actor[ls + i] = -1.0f;
    for (size_t i = 0; i < C_B1; i++) {
        const float u = smax(o_wurand(&seed), 1.0e-7f);
        const float a = sqrtf(-2.0f * logf(u));
        critic[i] = a * cosf(6.2831853f * o_wurand(&seed)) * 0.15f;
    }
    for (size_t i = C_W2; i < C_B2; i++) {
        const float u = smax(o_wurand(&seed), 1.0e-7f);
        const float a = sqrtf(-2.0f * logf(u));
        critic[i] = a * cosf(6.2831853f * o_wurand(&seed)) * 0.1f;
    }
}

/* fixed_ppo::actor_forward, ppo.hpp:65-80: z starts at the bias, in-order dot
 * product, tanh; mean = b2 + W2 . hidden (+ the geometry prior for a < 3). */
void o_wide_actor_forward(uint32_t hidden, const float* obs, const float* actor, float* hid, float* mean) {
    const size_t b1 = (size_t)hidden * AOBS, w2 = b1 + hidden, b2 = w2 + (size_t)ACT * hidden;
    for (uint32_t h = 0; h < hidden; h++) {
        float z = actor[b1 + h];
        const float* row = actor + (size_t)h * AOBS;
        for (uint32_t i = 0; i < AOBS; i++) z += row[i] * obs[i];
        hid[h] = tanhf(z);
    }
    for (uint32_t a = 0; a < ACT; a++) {
        float z = actor[b2 + a];
        const float* row = actor + w2 + (size_t)a * hidden;
        for (uint32_t h = 0; h < hidden; h++) z += row[h] * hid[h];
        if (a < 3) z += obs[AOBS - 3 + a];
        mean[a] = z;
    }
}
