// Pose-aware mechanical contact audit (vehicle_geometry.hpp:64-376,
// navigation_contact.metal:3-25): the declared vehicle - a 60 x 60 x 14 mm
// chassis box, two 84 mm arm bars and four 45 mm rotor discs at the L2F rotor
// positions - against the room planes and the world's obstacles, by GJK
// distance between convex shapes. An audit only: it changes no observation,
// reward or termination. Restated with the reference's operations in the
// reference's order (the kernels are built without FMA contraction), so the
// device results equal the CPU reference's bit for bit: the GJK loop, the
// exhaustive sub-simplex reduction with its small pivoted linear solve, the
// bounding-sphere pair skip and the conservative "ambiguous" outcomes are
// the reference's algorithm.
#pragma once
#include "mdn_device.cuh"

namespace mdn {
namespace contact {

struct V3 {
    float x, y, z;
};
__device__ __forceinline__ V3 v3(float x, float y, float z) { return {x, y, z}; }
__device__ __forceinline__ V3 add(V3 a, V3 b) { return v3(a.x + b.x, a.y + b.y, a.z + b.z); }
__device__ __forceinline__ V3 sub(V3 a, V3 b) { return v3(a.x - b.x, a.y - b.y, a.z - b.z); }
__device__ __forceinline__ V3 scale(V3 a, float s) { return v3(a.x * s, a.y * s, a.z * s); }
__device__ __forceinline__ float dot(V3 a, V3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
__device__ __forceinline__ float norm2(V3 a) { return dot(a, a); }
__device__ __forceinline__ float norm(V3 a) { return sqrtf(norm2(a)); }
__device__ __forceinline__ float comp(V3 a, int axis) { return axis == 0 ? a.x : (axis == 1 ? a.y : a.z); }
__device__ __forceinline__ float sgn(float x) { return x < 0.0f ? -1.0f : (x > 0.0f ? 1.0f : 0.0f); }

// Body -> world rotation by a unit wxyz quaternion: v + 2w (q x v) + 2 q x (q x v).
__device__ __forceinline__ V3 rotate(const float* q, V3 v) {
    const V3 t = scale(v3(q[2] * v.z - q[3] * v.y, q[3] * v.x - q[1] * v.z, q[1] * v.y - q[2] * v.x), 2.0f);
    const V3 qt = v3(q[2] * t.z - q[3] * t.y, q[3] * t.x - q[1] * t.z, q[1] * t.y - q[2] * t.x);
    return add(v, add(scale(t, q[0]), qt));
}
__device__ __forceinline__ V3 rotate_back(const float* q, V3 v) {
    const float c[4] = {q[0], -q[1], -q[2], -q[3]};
    return rotate(c, v);
}

// Vehicle part: kind 0 body-frame box, kind 1 disc (finite cylinder, axis = body z).
struct Part {
    uint32_t kind;
    V3 center, half;
    float radius, half_height;
};
__device__ __forceinline__ Part vehicle_part(uint32_t index) {
    Part s{};
    s.center = v3(0, 0, 0);
    s.half = v3(0, 0, 0);
    if (index == 0) {
        s.kind = 0;
        s.half = v3(0.030f, 0.030f, 0.007f);  // chassis
    } else if (index == 1) {
        s.kind = 0;
        s.half = v3(0.042f, 0.004f, 0.004f);  // arm bar along x
    } else if (index == 2) {
        s.kind = 0;
        s.half = v3(0.004f, 0.042f, 0.004f);  // arm bar along y
    } else {                                    // rotor discs at (+-28, +-28) mm
        s.kind = 1;
        const float sx = (index == 3 || index == 6) ? 1.0f : -1.0f;
        const float sy = (index == 5 || index == 6) ? 1.0f : -1.0f;
        s.center = v3(sx * 0.028f, sy * 0.028f, 0.0f);
        s.radius = 0.0225f;
        s.half_height = 0.0005f;
    }
    return s;
}
__device__ __forceinline__ float part_radius(const Part& s) {
    return s.kind == 0 ? norm(s.half) : sqrtf(s.radius * s.radius + s.half_height * s.half_height);
}

__device__ __forceinline__ V3 part_support(const Part& s, const float* p, const float* q, V3 dir) {
    const V3 db = rotate_back(q, dir);
    V3 pt = s.center;
    if (s.kind == 0) {
        pt.x += sgn(db.x) * s.half.x;
        pt.y += sgn(db.y) * s.half.y;
        pt.z += sgn(db.z) * s.half.z;
    } else {
        const float radial = sqrtf(db.x * db.x + db.y * db.y);
        if (radial > 1e-12f) {
            pt.x += s.radius * db.x / radial;
            pt.y += s.radius * db.y / radial;
        }
        pt.z += sgn(db.z) * s.half_height;
    }
    return add(v3(p[0], p[1], p[2]), rotate(q, pt));
}

// Obstacle kinds 0 (box), 1 (sphere), 2 (vertical cylinder), moving linearly.
__device__ __forceinline__ V3 obstacle_at(const mdn_obstacle& o, float t) {
    return v3(o.center[0] + o.velocity[0] * t, o.center[1] + o.velocity[1] * t, o.center[2] + o.velocity[2] * t);
}
__device__ __forceinline__ V3 obstacle_support(const mdn_obstacle& o, float t, V3 dir) {
    const V3 c = obstacle_at(o, t);
    if (o.kind == 0) return v3(c.x + sgn(dir.x) * o.size[0], c.y + sgn(dir.y) * o.size[1], c.z + sgn(dir.z) * o.size[2]);
    if (o.kind == 1) {
        const float len = norm(dir);
        if (len <= 1e-12f) return c;
        return add(c, scale(dir, o.size[0] / len));
    }
    const float radial = sqrtf(dir.x * dir.x + dir.y * dir.y);
    V3 pt = c;
    if (radial > 1e-12f) {
        pt.x += o.size[0] * dir.x / radial;
        pt.y += o.size[0] * dir.y / radial;
    }
    pt.z += sgn(dir.z) * o.size[2];
    return pt;
}
__device__ __forceinline__ float obstacle_radius(const mdn_obstacle& o) {
    if (o.kind == 0) return sqrtf(o.size[0] * o.size[0] + o.size[1] * o.size[1] + o.size[2] * o.size[2]);
    if (o.kind == 1) return o.size[0];
    return sqrtf(o.size[0] * o.size[0] + o.size[2] * o.size[2]);
}
__device__ __forceinline__ V3 minkowski(const Part& s, const float* p, const float* q, const mdn_obstacle& o, float t,
                                        V3 dir) {
    return sub(part_support(s, p, q, dir), obstacle_support(o, t, scale(dir, -1.0f)));
}

// Barycentric weights of the point of the selected vertices' affine hull
// nearest the origin: the (count+1) x (count+1) system [G 1; 1^T 0] by
// Gauss-Jordan elimination with partial pivoting. Fails on a singular pivot or
// a clearly negative weight (the point lies outside this sub-simplex).
__device__ __forceinline__ bool affine_weights(const V3* pts, const uint32_t* sel, uint32_t count, float* w) {
    float m[5][6];
    const uint32_t size = count + 1;
    for (uint32_t r = 0; r < size; r++)
        for (uint32_t c = 0; c <= size; c++) m[r][c] = 0.0f;
    for (uint32_t r = 0; r < count; r++) {
        for (uint32_t c = 0; c < count; c++) m[r][c] = dot(pts[sel[r]], pts[sel[c]]);
        m[r][count] = 1.0f;
        m[r][size] = 0.0f;
        m[count][r] = 1.0f;
    }
    m[count][count] = 0.0f;
    m[count][size] = 1.0f;
    for (uint32_t c = 0; c < size; c++) {
        uint32_t piv = c;
        for (uint32_t r = c + 1; r < size; r++)
            if (fabsf(m[r][c]) > fabsf(m[piv][c])) piv = r;
        if (fabsf(m[piv][c]) < 1e-12f) return false;
        if (piv != c)
            for (uint32_t j = c; j <= size; j++) {
                const float tmp = m[c][j];
                m[c][j] = m[piv][j];
                m[piv][j] = tmp;
            }
        const float d = m[c][c];
        for (uint32_t j = c; j <= size; j++) m[c][j] /= d;
        for (uint32_t r = 0; r < size; r++)
            if (r != c) {
                const float f = m[r][c];
                for (uint32_t j = c; j <= size; j++) m[r][j] -= f * m[c][j];
            }
    }
    float total = 0.0f;
    for (uint32_t i = 0; i < count; i++) {
        w[i] = m[i][size];
        if (w[i] < -1e-5f) return false;
        if (w[i] < 0.0f) w[i] = 0.0f;
        total += w[i];
    }
    if (total < 1e-10f) return false;
    for (uint32_t i = 0; i < count; i++) w[i] /= total;
    return true;
}

// Nearest point of the simplex (all faces, edges and vertices tried; the
// smallest feasible one kept); the simplex shrinks to that feature's vertices.
__device__ __forceinline__ bool reduce_simplex(V3* pts, uint32_t& count, V3& closest) {
    float best = 1e30f;
    uint32_t best_sel[4] = {0, 0, 0, 0}, best_count = 0;
    float best_w[4] = {0, 0, 0, 0};
    const uint32_t masks = 1u << count;
    for (uint32_t mask = 1; mask < masks; mask++) {
        uint32_t sel[4] = {0, 0, 0, 0}, k = 0;
        for (uint32_t i = 0; i < count; i++)
            if (mask & (1u << i)) sel[k++] = i;
        float w[4] = {0, 0, 0, 0};
        if (!affine_weights(pts, sel, k, w)) continue;
        V3 cand = v3(0, 0, 0);
        for (uint32_t i = 0; i < k; i++) cand = add(cand, scale(pts[sel[i]], w[i]));
        const float d2 = norm2(cand);
        if (d2 < best) {
            best = d2;
            closest = cand;
            best_count = k;
            for (uint32_t i = 0; i < k; i++) {
                best_sel[i] = sel[i];
                best_w[i] = w[i];
            }
        }
    }
    if (best_count == 0) return false;
    V3 kept[4];
    uint32_t n = 0;
    for (uint32_t i = 0; i < best_count; i++)
        if (best_w[i] > 1e-6f) kept[n++] = pts[best_sel[i]];
    if (n == 0) return false;
    for (uint32_t i = 0; i < n; i++) pts[i] = kept[i];
    count = n;
    return true;
}

// GJK separation of one vehicle part and one obstacle (0 on overlap);
// non-convergence counts as contact and is flagged ambiguous.
__device__ __forceinline__ void gjk(const Part& s, const float* p, const float* q, const mdn_obstacle& o, float t,
                                    float& distance, uint32_t& touching, uint32_t& ambiguous) {
    const V3 vc = add(v3(p[0], p[1], p[2]), rotate(q, s.center));
    V3 dir = sub(obstacle_at(o, t), vc);
    if (norm2(dir) < 1e-12f) dir = v3(1, 0, 0);
    V3 pts[4];
    uint32_t count = 1;
    pts[0] = minkowski(s, p, q, o, t, dir);
    V3 closest = pts[0];
    for (uint32_t it = 0; it < 32; it++) {
        if (!reduce_simplex(pts, count, closest)) {
            distance = 0.0f;
            touching = 1;
            ambiguous = 1;
            return;
        }
        const float d2 = norm2(closest);
        if (d2 <= 1e-10f) {
            distance = 0.0f;
            touching = 1;
            return;
        }
        dir = scale(closest, -1.0f);
        const V3 sp = minkowski(s, p, q, o, t, dir);
        const float gain = d2 - dot(closest, sp);
        if (gain <= 1e-7f * fmaxf(1.0f, d2)) {
            distance = sqrtf(d2);
            touching = distance <= 1e-5f;
            return;
        }
        bool repeat = false;
        for (uint32_t i = 0; i < count; i++)
            if (norm2(sub(pts[i], sp)) <= 1e-12f) repeat = true;
        if (repeat) {
            distance = sqrtf(d2);
            touching = distance <= 1e-5f;
            return;
        }
        if (count >= 4) {
            distance = 0.0f;
            touching = 1;
            ambiguous = 1;
            return;
        }
        pts[count++] = sp;
    }
    distance = 0.0f;
    touching = 1;
    ambiguous = 1;
}

// Whole audit of one pose (vg_world_contact): room planes x[-2,14] y[-5,5]
// z[0,5] and every obstacle, parts in order, early exit on contact.
__device__ __noinline__ mdn_contact_audit world_contact(const float* pos, const float* orient, const mdn_world& w,
                                                        float t, float margin) {
    mdn_contact_audit r;
    r.physical_clearance_m = 1e30f;
    r.safety_clearance_m = 1e30f;
    r.contact = 0;
    r.ambiguous = 0;
    auto fail = [&](uint32_t contact_flag) {
        r.physical_clearance_m = 0.0f;
        r.safety_clearance_m = -fmaxf(0.0f, margin);
        r.contact = contact_flag;
    };
    if (w.count > 16 || !isfinite(t) || !isfinite(margin)) {
        fail(1);
        r.ambiguous = 1;
        return r;
    }
    const float qn = sqrtf(orient[0] * orient[0] + orient[1] * orient[1] + orient[2] * orient[2] + orient[3] * orient[3]);
    if (!isfinite(qn) || qn < 1e-6f || !isfinite(pos[0]) || !isfinite(pos[1]) || !isfinite(pos[2])) {
        fail(1);
        r.ambiguous = 1;
        return r;
    }
    for (uint32_t i = 0; i < w.count; i++) {
        const mdn_obstacle& o = w.obstacles[i];
        bool ok = o.kind <= 2;
        for (int a = 0; a < 3 && ok; a++)
            ok = isfinite(o.center[a]) && isfinite(o.size[a]) && isfinite(o.velocity[a]) && o.size[a] >= 0.0f;
        if (!ok) {
            fail(1);
            r.ambiguous = 1;
            return r;
        }
    }
    const float q[4] = {orient[0] / qn, orient[1] / qn, orient[2] / qn, orient[3] / qn};
    const float lower[3] = {-2.0f, -5.0f, 0.0f}, upper[3] = {14.0f, 5.0f, 5.0f};
    for (uint32_t part = 0; part < 7; part++) {
        const Part s = vehicle_part(part);
        for (int a = 0; a < 3; a++) {
            const V3 up = a == 0 ? v3(1, 0, 0) : (a == 1 ? v3(0, 1, 0) : v3(0, 0, 1));
            const V3 down = a == 0 ? v3(-1, 0, 0) : (a == 1 ? v3(0, -1, 0) : v3(0, 0, -1));
            const float hi = comp(part_support(s, pos, q, up), a);
            const float lo = comp(part_support(s, pos, q, down), a);
            const float gap = fminf(lo - lower[a], upper[a] - hi);
            r.physical_clearance_m = fminf(r.physical_clearance_m, gap);
            if (gap <= 1e-5f) {
                fail(1);
                return r;
            }
        }
        for (uint32_t i = 0; i < w.count; i++) {
            const mdn_obstacle& o = w.obstacles[i];
            const V3 vc = add(v3(pos[0], pos[1], pos[2]), rotate(q, s.center));
            const float bound = norm(sub(vc, obstacle_at(o, t))) - part_radius(s) - obstacle_radius(o);
            if (bound >= r.physical_clearance_m) continue;  // cannot come nearer than the current gap
            float gap = 0.0f;
            uint32_t touching = 0, amb = 0;
            gjk(s, pos, q, o, t, gap, touching, amb);
            if (touching) {
                fail(1);
                r.ambiguous |= amb;
                return r;
            }
            r.physical_clearance_m = fminf(r.physical_clearance_m, gap);
            r.ambiguous |= amb;
        }
    }
    if (r.physical_clearance_m < 0.0f) {
        r.physical_clearance_m = 0.0f;
        r.contact = 1;
    }
    r.safety_clearance_m = r.physical_clearance_m - fmaxf(0.0f, margin);
    return r;
}

}  // namespace contact
}  // namespace mdn
