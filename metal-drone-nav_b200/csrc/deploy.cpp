// Deployment export of a trained actor in the reference's on-disk formats:
//   NAVPOL1 - the 12,104-parameter guided actor (deployment.hpp:41-88,
//             NavigationPolicy::write_file :166-201)
//   NAVWID4 - the width-aware actor (navigation_wide_deployment.hpp:10-40,
//             WideNavigationPolicy::load), e.g. the 967,688-parameter one.
// Both carry the 56-byte metadata block (deployment.hpp:70-88), the actor's
// flat parameters in ppo.hpp order and a provenance trailer with the FNV-1a
// 64-bit hash of the source checkpoint file (deployment.hpp:117-132).
// Files are written to a temporary name and renamed into place, as the
// reference writer does.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "host_common.h"

namespace mdn {
namespace {
constexpr uint32_t kBodyFrameFlu = 0x00554c46u;  // "FLU\0" little-endian

void put_u32(std::string& out, uint32_t v) {
    const char b[4] = {char(v & 0xff), char((v >> 8) & 0xff), char((v >> 16) & 0xff), char((v >> 24) & 0xff)};
    out.append(b, 4);
}
void put_f32(std::string& out, float v) {
    uint32_t bits;
    std::memcpy(&bits, &v, 4);
    put_u32(out, bits);
}
void put_u64(std::string& out, uint64_t v) {
    put_u32(out, uint32_t(v));
    put_u32(out, uint32_t(v >> 32));
}

// FNV-1a 64 over the file's bytes (offset basis 14695981039346656037,
// prime 1099511628211: the published FNV parameters).
bool fnv1a64_file(const char* path, uint64_t& hash) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    hash = 14695981039346656037ull;
    char buffer[16384];
    while (f) {
        f.read(buffer, sizeof(buffer));
        const std::streamsize count = f.gcount();
        for (std::streamsize i = 0; i < count; i++) {
            hash ^= static_cast<uint8_t>(buffer[i]);
            hash *= 1099511628211ull;
        }
    }
    return f.eof();
}
}  // namespace

void write_policy_file(const char* path, const float* actor, uint32_t hidden, const char* source_checkpoint,
                       float max_speed_mps) {
    require(path && actor && source_checkpoint, MDN_ERR_INVALID, "policy export: null argument");
    require(hidden == uint32_t(kHidden) || (hidden >= 64 && hidden <= 8192), MDN_ERR_INVALID,
            "policy export: hidden width must be 64..8192");
    require(std::isfinite(max_speed_mps) && max_speed_mps > 0.0f && max_speed_mps <= 10.0f, MDN_ERR_INVALID,
            "policy export: max speed must be in (0, 10] m/s");
    const uint32_t count = actor_param_count(hidden);
    for (uint32_t i = 0; i < count; i++)
        require(std::isfinite(actor[i]), MDN_ERR_INVALID, "policy export: actor has a non-finite parameter");
    uint64_t source_hash = 0;
    require(fnv1a64_file(source_checkpoint, source_hash), MDN_ERR_IO,
            std::string("policy export: cannot hash source checkpoint ") + source_checkpoint);
    const bool wide = hidden != uint32_t(kHidden);
    std::string out;
    out.reserve(size_t(count) * 4 + 128);
    out.append(wide ? "NAVWID4" : "NAVPOL1", 7);
    out.push_back('\0');
    // Metadata (deployment.hpp:70-88): version, observation count, hidden,
    // actions, policy mode 17, weight count, max speed, 16 x 20 sensor, 12 m
    // range, 0.05 s navigation and 0.01 s native periods, 8 memory frames, FLU.
    put_u32(out, wide ? 4u : 1u);
    put_u32(out, uint32_t(kActorObs));
    put_u32(out, hidden);
    put_u32(out, uint32_t(kActions));
    put_u32(out, 17u);
    put_u32(out, count);
    put_f32(out, max_speed_mps);
    put_u32(out, 16u);
    put_u32(out, 20u);
    put_f32(out, 12.0f);
    put_f32(out, 0.05f);
    put_f32(out, 0.01f);
    put_u32(out, 8u);
    put_u32(out, kBodyFrameFlu);
    if (wide) {
        // Camera contract (deployment.hpp:55-66): the legacy profile this
        // simulator renders (id 1, tan_h 1, tan_v 0.75, camera at the body
        // origin, 0.03-12 m, no noise).
        put_u32(out, 1u);
        put_f32(out, 1.0f);
        put_f32(out, 0.75f);
        put_f32(out, 0.0f);
        put_f32(out, 0.03f);
        put_f32(out, 12.0f);
        put_f32(out, 0.0f);
        put_u32(out, 0u);
    }
    for (uint32_t i = 0; i < count; i++) put_f32(out, actor[i]);
    out.append(wide ? "NAVSRC4" : "NAVSRC1", 7);
    out.push_back('\0');
    put_u64(out, source_hash);
    const std::string temp = std::string(path) + ".tmp";
    {
        std::ofstream f(temp, std::ios::binary | std::ios::trunc);
        require(bool(f), MDN_ERR_IO, "policy export: cannot create " + temp);
        f.write(out.data(), std::streamsize(out.size()));
        f.flush();
        if (!f) {
            f.close();
            std::remove(temp.c_str());
            throw Error(MDN_ERR_IO, "policy export: write failed");
        }
    }
    if (std::rename(temp.c_str(), path) != 0) {
        std::remove(temp.c_str());
        throw Error(MDN_ERR_IO, std::string("policy export: cannot replace ") + path);
    }
}

}  // namespace mdn

using namespace mdn;

extern "C" int mdn_policy_write(const char* path, const float* actor, uint32_t hidden, const char* source_checkpoint,
                                float max_speed_mps) {
    return guarded([&] { write_policy_file(path, actor, hidden, source_checkpoint, max_speed_mps); });
}

extern "C" int mdn_sim_export_policy(mdn_sim* sim, const char* path, const char* source_checkpoint,
                                     float max_speed_mps) {
    return guarded([&] {
        require(sim != nullptr, MDN_ERR_INVALID, "policy export: null simulator");
        require(!sim->layered, MDN_ERR_INVALID,
                "policy export: NAVPOL1/NAVWID4 hold one-hidden-layer tanh actors, not layered networks");
        cuda_check(cudaSetDevice(sim->dev->gpu), "cudaSetDevice");
        std::vector<float> actor(sim->actor_params);
        cuda_check(cudaMemcpyAsync(actor.data(), sim->buf[MDN_BUF_ACTOR], actor.size() * sizeof(float),
                                   cudaMemcpyDeviceToHost, sim->stream),
                   "download actor");
        cuda_check(cudaStreamSynchronize(sim->stream), "download actor");
        write_policy_file(path, actor.data(), sim->actor_hidden, source_checkpoint, max_speed_mps);
    });
}
