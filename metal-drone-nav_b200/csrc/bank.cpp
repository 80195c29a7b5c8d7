// Frozen challenge banks on the host:
//   - a strict JSON reader for the bank's JSONL rows,
//   - SHA-256 (FIPS 180-4) for the bank and checkpoint hashes,
//   - the split loader with every record check of challenge_evaluation::
//     parse_level / load_split (challenge_evaluation.hpp:163-313),
//   - the train-split level sampler challenge_training::ChallengeTraining
//     (challenge_training.hpp:53-427) with its CHTRN1 sidecar.
// The device side (sim_apply_challenge_world) is apply_challenge_world in
// world_gen.cuh; mdn_sim_set_challenge_bank in host.cpp wires the two.
#include <algorithm>
#include <array>
#include <cfloat>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <iomanip>
#include <locale>
#include <map>
#include <memory>
#include <set>
#include <sstream>
#include <string>
#include <vector>

#include "host_common.h"

namespace mdn {
namespace {

// ------------------------------------------------------------------ JSON
// A JSON value of one JSONL row (RFC 8259). Booleans count as numbers 1 / 0
// where a number is required: the reference reads rows with
// NSJSONSerialization, whose booleans are NSNumber objects.
struct Json {
    enum Kind { kNull, kBool, kNumber, kString, kArray, kObject } kind = kNull;
    double number = 0.0;
    std::string text;
    std::vector<Json> items;
    std::vector<std::pair<std::string, Json>> fields;
    const Json* get(const char* key) const {
        const Json* found = nullptr;
        for (const auto& f : fields)
            if (f.first == key) found = &f.second;  // the last duplicate wins
        return found;
    }
};

class JsonReader {
public:
    JsonReader(const char* begin, const char* end) : p_(begin), end_(end) {}
    bool parse(Json& out, std::string& error) {
        try {
            skip();
            value(out, 0);
            skip();
            if (p_ != end_) fail("unexpected data after the JSON value");
            return true;
        } catch (const std::runtime_error& e) {
            error = e.what();
            return false;
        }
    }

private:
    const char* p_;
    const char* end_;
    [[noreturn]] void fail(const char* what) { throw std::runtime_error(what); }
    void skip() {
        while (p_ != end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool literal(const char* word) {
        const size_t n = std::strlen(word);
        if (size_t(end_ - p_) < n || std::memcmp(p_, word, n) != 0) return false;
        p_ += n;
        return true;
    }
    void value(Json& out, int depth) {
        if (depth > 64) fail("JSON nesting too deep");
        if (p_ == end_) fail("unexpected end of JSON");
        const char c = *p_;
        if (c == '{') {
            object(out, depth);
        } else if (c == '[') {
            array(out, depth);
        } else if (c == '"') {
            out.kind = Json::kString;
            string(out.text);
        } else if (c == '-' || (c >= '0' && c <= '9')) {
            out.kind = Json::kNumber;
            out.number = number();
        } else if (literal("true")) {
            out.kind = Json::kBool;
            out.number = 1.0;
        } else if (literal("false")) {
            out.kind = Json::kBool;
            out.number = 0.0;
        } else if (literal("null")) {
            out.kind = Json::kNull;
        } else {
            fail("invalid JSON value");
        }
    }
    void object(Json& out, int depth) {
        out.kind = Json::kObject;
        ++p_;
        skip();
        if (p_ != end_ && *p_ == '}') {
            ++p_;
            return;
        }
        while (true) {
            skip();
            if (p_ == end_ || *p_ != '"') fail("expected an object key");
            std::string key;
            string(key);
            skip();
            if (p_ == end_ || *p_ != ':') fail("expected ':'");
            ++p_;
            skip();
            out.fields.emplace_back(std::move(key), Json{});
            value(out.fields.back().second, depth + 1);
            skip();
            if (p_ != end_ && *p_ == ',') {
                ++p_;
                continue;
            }
            if (p_ != end_ && *p_ == '}') {
                ++p_;
                return;
            }
            fail("expected ',' or '}'");
        }
    }
    void array(Json& out, int depth) {
        out.kind = Json::kArray;
        ++p_;
        skip();
        if (p_ != end_ && *p_ == ']') {
            ++p_;
            return;
        }
        while (true) {
            skip();
            out.items.emplace_back();
            value(out.items.back(), depth + 1);
            skip();
            if (p_ != end_ && *p_ == ',') {
                ++p_;
                continue;
            }
            if (p_ != end_ && *p_ == ']') {
                ++p_;
                return;
            }
            fail("expected ',' or ']'");
        }
    }
    static void utf8(std::string& s, uint32_t cp) {
        if (cp < 0x80) {
            s.push_back(char(cp));
        } else if (cp < 0x800) {
            s.push_back(char(0xc0 | (cp >> 6)));
            s.push_back(char(0x80 | (cp & 0x3f)));
        } else if (cp < 0x10000) {
            s.push_back(char(0xe0 | (cp >> 12)));
            s.push_back(char(0x80 | ((cp >> 6) & 0x3f)));
            s.push_back(char(0x80 | (cp & 0x3f)));
        } else {
            s.push_back(char(0xf0 | (cp >> 18)));
            s.push_back(char(0x80 | ((cp >> 12) & 0x3f)));
            s.push_back(char(0x80 | ((cp >> 6) & 0x3f)));
            s.push_back(char(0x80 | (cp & 0x3f)));
        }
    }
    uint32_t hex4() {
        if (end_ - p_ < 4) fail("short \\u escape");
        uint32_t v = 0;
        for (int k = 0; k < 4; k++) {
            const char h = *p_++;
            v <<= 4;
            if (h >= '0' && h <= '9') v |= uint32_t(h - '0');
            else if (h >= 'a' && h <= 'f') v |= uint32_t(h - 'a' + 10);
            else if (h >= 'A' && h <= 'F') v |= uint32_t(h - 'A' + 10);
            else fail("bad \\u escape");
        }
        return v;
    }
    void string(std::string& out) {
        ++p_;  // opening quote
        while (true) {
            if (p_ == end_) fail("unterminated string");
            const unsigned char c = static_cast<unsigned char>(*p_++);
            if (c == '"') return;
            if (c < 0x20) fail("control character in string");
            if (c != '\\') {
                out.push_back(char(c));
                continue;
            }
            if (p_ == end_) fail("unterminated escape");
            const char e = *p_++;
            switch (e) {
                case '"': out.push_back('"'); break;
                case '\\': out.push_back('\\'); break;
                case '/': out.push_back('/'); break;
                case 'b': out.push_back('\b'); break;
                case 'f': out.push_back('\f'); break;
                case 'n': out.push_back('\n'); break;
                case 'r': out.push_back('\r'); break;
                case 't': out.push_back('\t'); break;
                case 'u': {
                    uint32_t cp = hex4();
                    if (cp >= 0xd800 && cp <= 0xdbff) {
                        if (end_ - p_ < 6 || p_[0] != '\\' || p_[1] != 'u') fail("unpaired surrogate");
                        p_ += 2;
                        const uint32_t lo = hex4();
                        if (lo < 0xdc00 || lo > 0xdfff) fail("unpaired surrogate");
                        cp = 0x10000 + ((cp - 0xd800) << 10) + (lo - 0xdc00);
                    } else if (cp >= 0xdc00 && cp <= 0xdfff) {
                        fail("unpaired surrogate");
                    }
                    utf8(out, cp);
                    break;
                }
                default: fail("bad escape");
            }
        }
    }
    double number() {
        const char* start = p_;
        if (*p_ == '-') ++p_;
        if (p_ == end_) fail("bad number");
        if (*p_ == '0') {
            ++p_;
        } else if (*p_ >= '1' && *p_ <= '9') {
            while (p_ != end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        } else {
            fail("bad number");
        }
        if (p_ != end_ && *p_ == '.') {
            ++p_;
            if (p_ == end_ || *p_ < '0' || *p_ > '9') fail("bad number");
            while (p_ != end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        if (p_ != end_ && (*p_ == 'e' || *p_ == 'E')) {
            ++p_;
            if (p_ != end_ && (*p_ == '+' || *p_ == '-')) ++p_;
            if (p_ == end_ || *p_ < '0' || *p_ > '9') fail("bad number");
            while (p_ != end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        // strtod rounds correctly; the span is copied so it stops at the token.
        const std::string token(start, p_);
        return std::strtod(token.c_str(), nullptr);
    }
};

// ------------------------------------------------------------------ SHA-256
// FIPS 180-4 SHA-256.
class Sha256 {
public:
    Sha256() {
        static const uint32_t init[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                                         0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
        std::memcpy(h_, init, sizeof(h_));
    }
    void update(const unsigned char* data, size_t size) {
        total_ += size;
        while (size > 0) {
            const size_t take = std::min(size, size_t(64) - fill_);
            std::memcpy(block_ + fill_, data, take);
            fill_ += take;
            data += take;
            size -= take;
            if (fill_ == 64) {
                compress(block_);
                fill_ = 0;
            }
        }
    }
    std::string hex() {
        const uint64_t bits = total_ * 8;
        const unsigned char one = 0x80, zero = 0;
        update(&one, 1);
        while (fill_ != 56) update(&zero, 1);
        unsigned char length[8];
        for (int k = 0; k < 8; k++) length[k] = static_cast<unsigned char>(bits >> (56 - 8 * k));
        update(length, 8);
        static const char digits[] = "0123456789abcdef";
        std::string out;
        for (uint32_t word : h_)
            for (int k = 28; k >= 0; k -= 4) out.push_back(digits[(word >> k) & 0xf]);
        return out;
    }

private:
    uint32_t h_[8];
    unsigned char block_[64];
    size_t fill_ = 0;
    uint64_t total_ = 0;
    static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
    void compress(const unsigned char* b) {
        static const uint32_t k[64] = {
            0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
            0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
            0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
            0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
            0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
            0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
            0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
            0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};
        uint32_t w[64];
        for (int t = 0; t < 16; t++)
            w[t] = uint32_t(b[4 * t]) << 24 | uint32_t(b[4 * t + 1]) << 16 | uint32_t(b[4 * t + 2]) << 8 |
                   uint32_t(b[4 * t + 3]);
        for (int t = 16; t < 64; t++) {
            const uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
            const uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
            w[t] = w[t - 16] + s0 + w[t - 7] + s1;
        }
        uint32_t a = h_[0], bb = h_[1], c = h_[2], d = h_[3], e = h_[4], f = h_[5], g = h_[6], h = h_[7];
        for (int t = 0; t < 64; t++) {
            const uint32_t t1 = h + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + k[t] + w[t];
            const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & bb) ^ (a & c) ^ (bb & c));
            h = g;
            g = f;
            f = e;
            e = d + t1;
            d = c;
            c = bb;
            bb = a;
            a = t1 + t2;
        }
        h_[0] += a;
        h_[1] += bb;
        h_[2] += c;
        h_[3] += d;
        h_[4] += e;
        h_[5] += f;
        h_[6] += g;
        h_[7] += h;
    }
};

[[noreturn]] void bank_fail(const std::string& message) { throw Error(MDN_ERR_INVALID, "challenge bank: " + message); }

std::string sha256_file(const std::string& path) {
    std::ifstream file(path, std::ios::binary);
    if (!file) throw Error(MDN_ERR_IO, "challenge bank: cannot read for SHA-256: " + path);
    Sha256 hash;
    std::vector<char> buffer(64 * 1024);
    while (file) {
        file.read(buffer.data(), std::streamsize(buffer.size()));
        const std::streamsize count = file.gcount();
        if (count > 0) hash.update(reinterpret_cast<const unsigned char*>(buffer.data()), size_t(count));
    }
    if (!file.eof()) throw Error(MDN_ERR_IO, "challenge bank: read failed while hashing: " + path);
    return hash.hex();
}

bool is_sha256(const std::string& value) {
    return value.size() == 64 && std::all_of(value.begin(), value.end(), [](unsigned char c) {
               return (c >= '0' && c <= '9') || (c >= 'a' && c <= 'f');
           });
}

// ------------------------------------------------------------------ records
constexpr uint32_t kEnvStride = 747796405u;  // simulator env seed derivation (sim.metal:56)
constexpr uint32_t kEnvOffset = 2891336453u;
constexpr uint32_t kInvalidLevel = 0xffffffffu;

// Field readers with the reference's messages (challenge_evaluation.hpp:91-146).
const Json& field(const Json& object, const char* name, const std::string& where) {
    const Json* v = object.get(name);
    if (!v) bank_fail(where + " missing field " + name);
    return *v;
}
const Json& as_object(const Json& v, const std::string& where) {
    if (v.kind != Json::kObject) bank_fail(where + " must be an object");
    return v;
}
const Json& as_array(const Json& v, const std::string& where) {
    if (v.kind != Json::kArray) bank_fail(where + " must be an array");
    return v;
}
std::string as_string(const Json& v, const std::string& where) {
    if (v.kind != Json::kString) bank_fail(where + " must be a string");
    return v.text;
}
double as_number(const Json& v, const std::string& where) {
    if (v.kind != Json::kNumber && v.kind != Json::kBool) bank_fail(where + " must be a number");
    if (!std::isfinite(v.number)) bank_fail(where + " must be finite");
    return v.number;
}
uint32_t as_uint(const Json& v, const std::string& where) {
    const double number = as_number(v, where);
    if (number < 0 || number > double(UINT32_MAX) || std::floor(number) != number)
        bank_fail(where + " must be an unsigned 32-bit integer");
    return uint32_t(number);
}
float as_float(const Json& v, const std::string& where) {
    const double number = as_number(v, where);
    if (std::fabs(number) > double(FLT_MAX)) bank_fail(where + " is outside float32 range");
    return float(number);
}
void as_vec3(const Json& v, const std::string& where, float out[3]) {
    const Json& a = as_array(v, where);
    if (a.items.size() != 3) bank_fail(where + " must contain exactly 3 values");
    for (int k = 0; k < 3; k++) out[k] = as_float(a.items[size_t(k)], where + "[" + std::to_string(k) + "]");
}

// wclearance at t = 0 for the static kinds a record may hold (world.hpp:84-99).
float host_clearance(const mdn_world& w, const float p[3]) {
    float best = std::fmin(std::fmin(p[0] + 2, 14 - p[0]), std::fmin(std::fmin(p[1] + 5, 5 - p[1]), std::fmin(p[2], 5 - p[2]))) -
                 0.18f;
    for (uint32_t i = 0; i < w.count; i++) {
        const mdn_obstacle& o = w.obstacles[i];
        const float q[3] = {p[0] - (o.center[0] + 0.0f * o.velocity[0]), p[1] - (o.center[1] + 0.0f * o.velocity[1]),
                            p[2] - (o.center[2] + 0.0f * o.velocity[2])};
        float distance;
        if (o.kind == 1) {
            distance = std::sqrt(q[0] * q[0] + q[1] * q[1] + q[2] * q[2]) - o.size[0];
        } else if (o.kind == 2) {
            const float a = std::sqrt(q[0] * q[0] + q[1] * q[1]) - o.size[0], b = std::fabs(q[2]) - o.size[2];
            distance = std::sqrt(std::fmax(a, 0.0f) * std::fmax(a, 0.0f) + std::fmax(b, 0.0f) * std::fmax(b, 0.0f)) +
                       std::fmin(std::fmax(a, b), 0.0f);
        } else {
            const float k0 = std::fabs(q[0]) - o.size[0], k1 = std::fabs(q[1]) - o.size[1], k2 = std::fabs(q[2]) - o.size[2];
            const float m0 = std::fmax(k0, 0.0f), m1 = std::fmax(k1, 0.0f), m2 = std::fmax(k2, 0.0f);
            distance = std::sqrt(m0 * m0 + m1 * m1 + m2 * m2) + std::fmin(std::fmax(k0, std::fmax(k1, k2)), 0.0f);
        }
        best = std::fmin(best, distance - 0.18f);
    }
    return best;
}

struct Level {
    std::string failure_id, split, family_name, geometry_contract, difficulty_band, scene_sha256, world_source_sha256;
    mdn_bank_level info{};
    std::vector<float> witness_route;  // [points][3]
    mdn_world world{};
};

void require_room_bounds(const Json& record, const std::string& where) {
    const Json& bounds = as_object(field(record, "room_bounds", where), where + ".room_bounds");
    const float expected[3][2] = {{-2, 14}, {-5, 5}, {0, 5}};
    const char* names[3] = {"x", "y", "z"};
    for (int axis = 0; axis < 3; ++axis) {
        const Json& pair = as_array(field(bounds, names[axis], where + ".room_bounds"), where + ".room_bounds");
        if (pair.items.size() != 2) bank_fail(where + ".room_bounds axis must have two values");
        const float lo = as_float(pair.items[0], where + ".room_bounds lower");
        const float hi = as_float(pair.items[1], where + ".room_bounds upper");
        if (std::fabs(lo - expected[axis][0]) > 1e-5f || std::fabs(hi - expected[axis][1]) > 1e-5f)
            bank_fail(where + " uses room bounds incompatible with world.hpp");
    }
}

// parse_level, challenge_evaluation.hpp:163-280, check for check in its order.
Level parse_level(const Json& record, uint32_t line_number) {
    const std::string where = "JSONL line " + std::to_string(line_number);
    Level level;
    mdn_bank_level& info = level.info;
    info.line_number = line_number;
    if (as_string(field(record, "record_type", where), where + ".record_type") != "challenge")
        bank_fail(where + " has an unsupported record_type");
    if (as_uint(field(record, "schema_version", where), where + ".schema_version") != 1)
        bank_fail(where + " has an unsupported schema_version");
    level.failure_id = as_string(field(record, "failure_id", where), where + ".failure_id");
    level.split = as_string(field(record, "split", where), where + ".split");
    if (level.split != "train" && level.split != "dev" && level.split != "final") bank_fail(where + " has invalid split");
    info.family = as_uint(field(record, "family", where), where + ".family");
    if (info.family < 14 || info.family > 16) bank_fail(where + " family must be 14, 15, or 16");
    level.family_name = as_string(field(record, "family_name", where), where + ".family_name");
    level.geometry_contract = as_string(field(record, "geometry_contract", where), where + ".geometry_contract");
    const char* expected_name = info.family == 14   ? "bent_hallway_corner"
                                : info.family == 15 ? "connected_rooms_offset_doors_furniture"
                                                    : "vertical_over_under_choice";
    const Json* transform_field = record.get("coordinate_transform");
    const std::string transform =
        transform_field ? as_string(*transform_field, where + ".coordinate_transform") : "identity";
    const bool mirrored = transform == "mirror_y";
    if (transform != "identity" && !mirrored) bank_fail(where + " unsupported coordinate transform");
    info.mirrored = mirrored ? 1u : 0u;
    const char* corner_contract = mirrored ? "connected partitions force south turn, east hall, then north turn"
                                           : "connected partitions force north turn, east hall, then south turn";
    const char* expected_contract =
        info.family == 14   ? corner_contract
        : info.family == 15 ? "offset doors with intermediate table detour"
                            : "cross low barrier above, overhang below, then choose over or under slab";
    if (level.family_name != expected_name || level.geometry_contract != expected_contract)
        bank_fail(where + " family label/geometry contract does not match its family id");
    info.seed = as_uint(field(record, "seed", where), where + ".seed");
    info.environment_index = as_uint(field(record, "environment_index", where), where + ".environment_index");
    info.difficulty = as_float(field(record, "difficulty", where), where + ".difficulty");
    if (info.difficulty < 0 || info.difficulty >= 1) bank_fail(where + " difficulty must be in [0,1)");
    level.difficulty_band = as_string(field(record, "difficulty_band", where), where + ".difficulty_band");
    if (level.difficulty_band != "easy" && level.difficulty_band != "medium" && level.difficulty_band != "hard")
        bank_fail(where + " has invalid difficulty_band");
    const char* expected_band = info.difficulty < (1.0f / 3.0f) ? "easy" : info.difficulty < (2.0f / 3.0f) ? "medium" : "hard";
    if (level.difficulty_band != expected_band) bank_fail(where + " difficulty band does not match its difficulty value");
    level.scene_sha256 = as_string(field(record, "scene_sha256", where), where + ".scene_sha256");
    level.world_source_sha256 = as_string(field(record, "world_source_sha256", where), where + ".world_source_sha256");
    if (!is_sha256(level.scene_sha256) || !is_sha256(level.world_source_sha256))
        bank_fail(where + " has malformed source hashes");

    const Json& config = as_object(field(record, "sim_config", where), where + ".sim_config");
    if (as_uint(field(config, "family", where), where + ".sim_config.family") != info.family ||
        as_uint(field(config, "environment_index", where), where + ".sim_config.environment_index") !=
            info.environment_index)
        bank_fail(where + " sim_config does not match record family/index");
    info.base_seed = as_uint(field(config, "seed", where), where + ".sim_config.seed");
    info.distance = as_float(field(config, "distance", where), where + ".sim_config.distance");
    if (info.distance < 3.0f || info.distance > 10.0f) bank_fail(where + " distance must be in [3,10]");
    uint32_t seed_state = info.base_seed + info.environment_index * kEnvStride + kEnvOffset;
    seed_state ^= seed_state << 13;
    seed_state ^= seed_state >> 17;
    seed_state ^= seed_state << 5;
    if (seed_state != info.seed) bank_fail(where + " seed does not match simulator environment seed derivation");

    require_room_bounds(record, where);
    float goal[3], wind[3];
    as_vec3(field(record, "goal", where), where + ".goal", goal);
    as_vec3(field(record, "wind", where), where + ".wind", wind);
    const double body_radius = as_number(field(record, "body_radius_m", where), where + ".body_radius_m");
    if (std::fabs(body_radius - 0.18) > 1e-5) bank_fail(where + " body radius differs from simulator collision model");

    mdn_world& w = level.world;
    w = mdn_world{};
    w.family = info.family;
    w.seed = info.seed;
    for (int axis = 0; axis < 3; ++axis) {
        w.goal[axis] = goal[axis];
        w.wind[axis] = wind[axis];
    }
    const Json& obstacles = as_array(field(record, "obstacles", where), where + ".obstacles");
    if (obstacles.items.size() > 16) bank_fail(where + " contains more than 16 obstacles");
    w.count = uint32_t(obstacles.items.size());
    for (uint32_t i = 0; i < w.count; ++i) {
        const Json& object = as_object(obstacles.items[i], where + ".obstacles[]");
        mdn_obstacle& o = w.obstacles[i];
        o.kind = as_uint(field(object, "kind", where), where + ".obstacle.kind");
        if (o.kind > 2) bank_fail(where + " obstacle kind must be AABB(0), sphere(1), or cylinder(2)");
        float center[3], size[3], velocity[3];
        as_vec3(field(object, "center", where), where + ".obstacle.center", center);
        as_vec3(field(object, "half_extent", where), where + ".obstacle.half_extent", size);
        as_vec3(field(object, "velocity", where), where + ".obstacle.velocity", velocity);
        for (int axis = 0; axis < 3; ++axis) {
            if (size[axis] < 0) bank_fail(where + " obstacle size cannot be negative");
            o.center[axis] = center[axis];
            o.size[axis] = size[axis];
            o.velocity[axis] = velocity[axis];
        }
        if ((o.kind == 0 && (size[0] <= 0 || size[1] <= 0 || size[2] <= 0)) || (o.kind == 1 && size[0] <= 0) ||
            (o.kind == 2 && (size[0] <= 0 || size[2] <= 0)))
            bank_fail(where + " obstacle has a non-positive collision dimension");
        for (int axis = 0; axis < 3; ++axis) {
            const float lo = axis == 0 ? -2.0f : axis == 1 ? -5.0f : 0.0f;
            const float hi = axis == 0 ? 14.0f : 5.0f;
            const float extent = o.kind == 0 ? size[axis] : o.kind == 1 ? size[0] : axis == 2 ? size[2] : size[0];
            if (center[axis] - extent < lo - 1e-4f || center[axis] + extent > hi + 1e-4f)
                bank_fail(where + " obstacle extends outside the fixed room bounds");
        }
    }
    const float start[3] = {0, 0, 1.5f};
    if (host_clearance(w, start) <= 0.04f || host_clearance(w, goal) <= 0.04f)
        bank_fail(where + " has an unsafe start or goal for the 0.18 m vehicle");
    info.direct_route_clearance_m =
        as_float(field(record, "direct_route_clearance_m", where), where + ".direct_route_clearance_m");
    info.witness_min_clearance_m =
        as_float(field(record, "witness_min_clearance_m", where), where + ".witness_min_clearance_m");
    info.witness_sample_count = as_uint(field(record, "witness_sample_count", where), where + ".witness_sample_count");
    if (info.direct_route_clearance_m >= -0.02f || info.witness_min_clearance_m <= 0.04f || info.witness_sample_count == 0)
        bank_fail(where + " does not satisfy the stored obstructed-route/witness-clearance contract");
    const Json& route = as_array(field(record, "witness_route", where), where + ".witness_route");
    if (route.items.size() < 2) bank_fail(where + " witness_route needs at least two points");
    for (const Json& point : route.items) {
        float xyz[3];
        as_vec3(point, where + ".witness_route[]", xyz);
        level.witness_route.insert(level.witness_route.end(), xyz, xyz + 3);
    }
    const size_t last = level.witness_route.size() - 3;
    for (int axis = 0; axis < 3; ++axis) {
        if (std::fabs(level.witness_route[size_t(axis)] - start[axis]) > 1e-5f ||
            std::fabs(level.witness_route[last + size_t(axis)] - goal[axis]) > 1e-5f)
            bank_fail(where + " witness route endpoints do not match the simulator start and stored goal");
    }
    info.witness_point_count = uint32_t(route.items.size());
    return level;
}

}  // namespace

// load_split, challenge_evaluation.hpp:282-313.
struct BankData {
    std::vector<Level> levels;
    std::string bank_hash;
};

static void load_split(const std::string& path, const std::string& split, const std::string& expected_world_hash,
                       BankData& out) {
    if (split != "train" && split != "dev" && split != "final") bank_fail("split must be train, dev, or final");
    out.bank_hash = sha256_file(path);
    std::ifstream input(path);
    if (!input) throw Error(MDN_ERR_IO, "challenge bank: cannot open bank JSONL: " + path);
    std::set<std::string> failure_ids;
    std::string line;
    uint32_t line_number = 0;
    while (std::getline(input, line)) {
        ++line_number;
        if (line.empty()) bank_fail("blank JSONL row at line " + std::to_string(line_number));
        Json json;
        std::string error;
        const bool parsed = JsonReader(line.data(), line.data() + line.size()).parse(json, error);
        if (!parsed || json.kind != Json::kObject)
            bank_fail("invalid JSON object at line " + std::to_string(line_number) + (parsed ? "" : ": " + error));
        Level level = parse_level(json, line_number);
        if (level.world_source_sha256 != expected_world_hash)
            bank_fail("bank world.hpp hash does not match the running binary source");
        if (!failure_ids.insert(level.failure_id).second) bank_fail("duplicate failure_id: " + level.failure_id);
        if (level.split == split) out.levels.push_back(std::move(level));
        if (line_number > 1000000) bank_fail("bank exceeds one million records");
    }
    if (!input.eof()) throw Error(MDN_ERR_IO, "challenge bank: failed while reading bank JSONL");
    if (out.levels.empty()) bank_fail("bank contains no records for requested split " + split);
}

// ------------------------------------------------------------------ sampler
// Train-split level sampler of frozen-bank training. It reproduces the
// schedules, failure scores and CHTRN1 sidecar of challenge_training.hpp:53-427
// from this specification:
//
//  * Pools. The train levels fall into three family pools, 14, 15 and 16, each
//    listing its levels in bank order. All three must be non-empty.
//  * Quotas. Environments below `rehearsal_environments` never hold a bank
//    level: their slots are kInvalidLevel. Every other environment draws from
//    one fixed pool: the focus family when one is set, else pool
//    (env - rehearsal) mod 3 in the order 14, 15, 16.
//  * Schedules are env-major rows of horizon + 1 slots. A new run draws every
//    slot. Each later rollout keeps the caller's live level in slot 0 (checked
//    against the quota) and draws slots 1..horizon. Draws run environment by
//    environment, slot by slot, from one xorshift32 stream (shifts 13, 17, 5;
//    a zero state becomes 1; seed 0 means 1).
//  * One draw. Uniform selection: index = (u32 * pool size) >> 32. Failure-
//    weighted selection: u = u32 / 2^32 first; below the uniform floor, a
//    uniform index from the next draw; otherwise the next draw times the
//    pool's weight total is a remainder from which the weights are subtracted
//    in pool order, and the first level that takes it to zero or below wins.
//  * Weights, refreshed before each schedule: mix / (score rank + 1) +
//    (1 - mix) / (staleness rank + 1) in double. Score rank orders the pool by
//    failure score, highest first; staleness rank by the rollout of the last
//    visit, oldest first; equal keys go by level index.
//  * Scores. Each bank transition adds |raw GAE| to its environment's open
//    episode and stamps the level with the rollout index. When the episode
//    ends, the level's score becomes the episode's mean |GAE| and its
//    completion count grows.
//  * Sidecar CHTRN1 v3: a 256-byte header, the per-level ledger (scores f32,
//    last visit u64, last score u64, completions u64), the open episodes
//    (|GAE| sums f64, sample counts u32, levels u32) and the active ids u32.
//    Versions 1 and 2 load when no focus family is set.
namespace {

struct SamplerRng {
    uint32_t state = 1;
    uint32_t next() {
        uint32_t x = state ? state : 1u;
        x ^= x << 13;
        x ^= x >> 17;
        x ^= x << 5;
        state = x ? x : 1u;
        return state;
    }
    // in [0, 1): multiplying by 2^-32 is exact, as dividing by 2^32 is
    double unit() { return double(next()) * 0x1p-32; }
    size_t below(size_t count) { return size_t((uint64_t(next()) * count) >> 32); }
};

struct FamilyPool {
    uint32_t family = 0;
    std::vector<uint32_t> levels;  // bank indices, ascending
    std::vector<double> weight;    // failure-weighted replay weight of each entry
    double weight_total = 0.0;     // their sum in pool order
};

// Zero-based position of each pool entry once the entries are put in the
// strict total order `before`.
template <class Before>
std::vector<uint32_t> pool_ranks(const std::vector<uint32_t>& levels, Before before) {
    std::vector<uint32_t> order(levels.size());
    for (uint32_t i = 0; i < order.size(); i++) order[i] = i;
    std::sort(order.begin(), order.end(), [&](uint32_t x, uint32_t y) { return before(levels[x], levels[y]); });
    std::vector<uint32_t> rank(levels.size());
    for (uint32_t r = 0; r < order.size(); r++) rank[order[r]] = r;
    return rank;
}

// What the sampler knows about each train level.
struct LevelLedger {
    std::vector<float> score;         // mean |GAE| of the level's last completed episode
    std::vector<uint64_t> visited;    // rollout of the last transition on the level
    std::vector<uint64_t> scored;     // rollout of the last score
    std::vector<uint64_t> completed;  // completed episodes
    void reset(size_t levels) {
        score.assign(levels, 0.0f);
        visited.assign(levels, 0);
        scored.assign(levels, 0);
        completed.assign(levels, 0);
    }
};

// The episode each environment is in the middle of.
struct OpenEpisodes {
    std::vector<double> abs_gae;   // sum of |GAE| so far
    std::vector<uint32_t> samples; // transitions so far
    std::vector<uint32_t> level;   // its level, kInvalidLevel when none is open
    void reset(size_t envs) {
        abs_gae.assign(envs, 0.0);
        samples.assign(envs, 0);
        level.assign(envs, kInvalidLevel);
    }
};

// The CHTRN1 sidecar header (challenge_training.hpp:281-287): a file format.
struct SidecarHeader {
    char magic[8];
    uint32_t version, selection, environment_count, horizon, level_count, rng_state, focus_family, rehearsal;
    uint64_t last_rollout, completed_rollouts;
    float uniform_floor, score_staleness_mix;
    char bank_hash[64], world_hash[64], checkpoint_hash[64];
};
static_assert(sizeof(SidecarHeader) == 256, "challenge sidecar header layout");
constexpr char kSidecarMagic[8] = {'C', 'H', 'T', 'R', 'N', '1', 0, 0};
constexpr uint32_t kSidecarVersion = 3;

struct ByteSpan {
    void* data;
    size_t bytes;
};
template <class T>
ByteSpan span_of(std::vector<T>& v) {
    return {v.data(), v.size() * sizeof(T)};
}

// The sidecar body after the header, in file order.
std::vector<ByteSpan> sidecar_body(LevelLedger& l, OpenEpisodes& e, std::vector<uint32_t>& active) {
    return {span_of(l.score), span_of(l.visited), span_of(l.scored), span_of(l.completed),
            span_of(e.abs_gae), span_of(e.samples), span_of(e.level), span_of(active)};
}

}  // namespace

class ChallengeSampler {
public:
    ChallengeSampler(const std::string& bank_jsonl, const std::string& world_hash, const mdn_challenge_settings& s)
        : settings_(s), world_hash_(world_hash) {
        check_settings(s);
        load_split(bank_jsonl, "train", world_hash, bank_);
        build_pools();
        ledger_.reset(bank_.levels.size());
        open_.reset(s.environment_count);
        rng_.state = s.sampler_seed ? s.sampler_seed : 1u;
    }

    const BankData& bank() const { return bank_; }
    mdn_bank_control control() const {
        return {1u, uint32_t(bank_.levels.size()), settings_.horizon + 1, settings_.horizon};
    }
    const std::vector<uint32_t>& active_ids() const { return active_; }

    // A new run: every slot of every row is drawn; slot 0 becomes the active ids.
    void initial_schedule(uint32_t* schedule) {
        refresh_weights();
        const size_t stride = size_t(settings_.horizon) + 1;
        active_.resize(settings_.environment_count);
        for (uint32_t env = 0; env < settings_.environment_count; ++env) {
            uint32_t* row = schedule + env * stride;
            fill_row(env, row, 0);
            active_[env] = row[0];
        }
    }

    // A later rollout: slot 0 keeps each environment's live level; slots
    // 1..horizon serve the resets inside the rollout.
    void next_schedule(const uint32_t* active, uint64_t rollout_index, uint32_t* schedule) {
        last_rollout_ = rollout_index;
        refresh_weights();
        const uint32_t envs = settings_.environment_count;
        const size_t stride = size_t(settings_.horizon) + 1;
        for (uint32_t env = 0; env < envs; ++env) {
            check_active(env, active[env]);
            schedule[env * stride] = active[env];
        }
        active_.assign(active, active + envs);
        for (uint32_t env = 0; env < envs; ++env) fill_row(env, schedule + env * stride, 1);
    }

    // Rollout evidence in [tick][env] order: raw (unnormalised) GAE, episode
    // ends and the level of every transition.
    void observe_raw_gae(const float* raw_gae, const uint8_t* terminated, const uint8_t* truncated,
                         const uint32_t* transition_ids, uint64_t rollout_index) {
        if (!raw_gae || !terminated || !truncated || !transition_ids)
            throw Error(MDN_ERR_INVALID, "challenge rollout evidence buffer is null");
        const uint32_t envs = settings_.environment_count;
        for (uint32_t tick = 0; tick < settings_.horizon; ++tick)
            for (uint32_t env = 0; env < envs; ++env) {
                const size_t row = size_t(tick) * envs + env;
                const uint32_t level = transition_ids[row];
                if (is_rehearsal(env)) {
                    if (level != kInvalidLevel) throw Error(MDN_ERR_INVALID, "rehearsal transition contains a bank level");
                    continue;
                }
                if (level >= bank_.levels.size())
                    throw Error(MDN_ERR_INVALID, "transition level id is outside the frozen train bank");
                uint32_t& open_level = open_.level[env];
                if (open_level == kInvalidLevel)
                    open_level = level;
                else if (open_level != level)
                    throw Error(MDN_ERR_INVALID, "active challenge level changed before episode completion");
                if (!std::isfinite(raw_gae[row])) throw Error(MDN_ERR_INVALID, "raw GAE is non-finite");
                open_.abs_gae[env] += std::fabs(double(raw_gae[row]));
                open_.samples[env] += 1;
                ledger_.visited[level] = rollout_index;
                if (terminated[row] || truncated[row]) close_episode(env, level, rollout_index);
            }
        last_rollout_ = rollout_index;
    }

    void level_stats(uint32_t level, float* score, uint64_t* completed, uint64_t* last_visit) const {
        require(level < bank_.levels.size(), MDN_ERR_INVALID, "challenge level index out of range");
        if (score) *score = ledger_.score[level];
        if (completed) *completed = ledger_.completed[level];
        if (last_visit) *last_visit = ledger_.visited[level];
    }

    // Written to `path`.tmp, then renamed over `path`.
    void save_state(const std::string& path, const std::string& checkpoint_sha256, uint64_t completed_rollouts,
                    const uint32_t* active) {
        for (uint32_t env = 0; env < settings_.environment_count; env++) check_active(env, active[env]);
        active_.assign(active, active + settings_.environment_count);
        const SidecarHeader header = sidecar_header(checkpoint_sha256, completed_rollouts);
        const std::filesystem::path target(path);
        if (target.has_parent_path()) std::filesystem::create_directories(target.parent_path());
        const std::string temporary = path + ".tmp";
        std::ofstream file(temporary, std::ios::binary | std::ios::trunc);
        if (!file) throw Error(MDN_ERR_IO, "cannot write challenge sampler state: " + temporary);
        std::vector<ByteSpan> parts{{const_cast<SidecarHeader*>(&header), sizeof(header)}};
        for (const ByteSpan& b : sidecar_body(ledger_, open_, active_)) parts.push_back(b);
        for (const ByteSpan& b : parts) file.write(static_cast<const char*>(b.data), std::streamsize(b.bytes));
        file.flush();
        if (!file) throw Error(MDN_ERR_IO, "challenge sampler state write failed: " + temporary);
        file.close();
        if (std::rename(temporary.c_str(), path.c_str()) != 0)
            throw Error(MDN_ERR_IO, "cannot replace challenge sampler state: " + path);
    }

    // The state is read into copies and checked before it replaces the live
    // one, so a rejected sidecar leaves the sampler unchanged.
    void load_state(const std::string& path, const std::string& checkpoint_sha256, uint64_t completed_rollouts,
                    uint32_t* active_out) {
        std::ifstream file(path, std::ios::binary);
        if (!file) throw Error(MDN_ERR_IO, "cannot open challenge sampler state: " + path);
        SidecarHeader header{};
        read_span(file, {&header, sizeof(header)});
        if (!header_matches(header, checkpoint_sha256, completed_rollouts))
            throw Error(MDN_ERR_MISMATCH,
                        "challenge sampler sidecar does not match bank, world, PPO checkpoint, or rollout");
        LevelLedger ledger;
        ledger.reset(bank_.levels.size());
        OpenEpisodes open;
        open.reset(settings_.environment_count);
        std::vector<uint32_t> active(settings_.environment_count);
        for (const ByteSpan& b : sidecar_body(ledger, open, active)) read_span(file, b);
        char extra;
        if (file.read(&extra, 1)) throw Error(MDN_ERR_MISMATCH, "challenge sampler state has trailing bytes");
        for (size_t i = 0; i < ledger.score.size(); ++i) {
            const bool sane = std::isfinite(ledger.score[i]) && ledger.score[i] >= 0.0f &&
                              ledger.visited[i] <= header.last_rollout && ledger.scored[i] <= header.last_rollout;
            if (!sane) throw Error(MDN_ERR_MISMATCH, "challenge sampler sidecar has invalid priority data");
        }
        for (uint32_t env = 0; env < settings_.environment_count; env++) check_active(env, active[env]);
        for (uint32_t env = 0; env < settings_.environment_count; ++env) {
            const bool has_open = open.level[env] != kInvalidLevel;
            if (!std::isfinite(open.abs_gae[env]) || open.abs_gae[env] < 0.0 || has_open != (open.samples[env] != 0))
                throw Error(MDN_ERR_MISMATCH, "challenge sampler sidecar has invalid partial-episode state");
            if (has_open && open.level[env] != active[env])
                throw Error(MDN_ERR_MISMATCH, "challenge active id does not match partial episode score state");
        }
        std::swap(ledger_, ledger);
        std::swap(open_, open);
        active_.swap(active);
        rng_.state = header.rng_state;
        last_rollout_ = header.last_rollout;
        std::copy(active_.begin(), active_.end(), active_out);
    }

private:
    mdn_challenge_settings settings_;
    std::string world_hash_;
    BankData bank_;
    std::array<FamilyPool, 3> pools_;  // families 14, 15, 16
    LevelLedger ledger_;
    OpenEpisodes open_;
    std::vector<uint32_t> active_;
    SamplerRng rng_;
    uint64_t last_rollout_ = 0;

    static void check_settings(const mdn_challenge_settings& s) {
        auto fail = [](const char* m) { throw Error(MDN_ERR_INVALID, m); };
        if (s.environment_count == 0 || s.horizon == 0) fail("challenge training needs nonzero environments and horizon");
        if (s.environment_count < 3 || s.rehearsal_environments > s.environment_count - 3)
            fail("rehearsal must leave at least three bank environments");
        if (s.focus_family != 0u && (s.focus_family < 14u || s.focus_family > 16u))
            fail("focused challenge family must be 14, 15, 16, or 0 for balanced");
        if (s.selection > 1u) fail("unsupported challenge level selection mode");
        if (!(s.uniform_floor >= 0.5f && s.uniform_floor <= 1.0f))
            fail("failure-weighted replay uniform floor must be in [0.5,1]");
        if (!(s.score_staleness_mix >= 0.0f && s.score_staleness_mix <= 1.0f))
            fail("score/staleness mix must be in [0,1]");
        // a schedule holds environment_count x (horizon + 1) ids; keep it addressable
        if (uint64_t(s.environment_count) * (uint64_t(s.horizon) + 1) > (uint64_t(1) << 31))
            fail("challenge schedule larger than 2^31 slots");
    }

    void build_pools() {
        std::set<uint32_t> families;
        for (size_t i = 0; i < 3; i++) pools_[i].family = 14u + uint32_t(i);
        for (uint32_t i = 0; i < bank_.levels.size(); ++i) {
            const Level& level = bank_.levels[i];
            if (level.split != "train") throw Error(MDN_ERR_INVALID, "train loader returned a non-train challenge level");
            families.insert(level.info.family);
            if (level.info.family >= 14u && level.info.family <= 16u) pools_[level.info.family - 14u].levels.push_back(i);
        }
        if (families.size() < 3) throw Error(MDN_ERR_INVALID, "train bank must contain each family 14, 15, and 16");
        for (const FamilyPool& pool : pools_)
            if (pool.levels.empty())
                throw Error(MDN_ERR_INVALID, "train bank is missing family " + std::to_string(pool.family));
    }

    bool is_rehearsal(uint32_t env) const { return env < settings_.rehearsal_environments; }
    const FamilyPool& pool_of(uint32_t env) const {
        if (settings_.focus_family != 0u) return pools_[settings_.focus_family - 14u];
        return pools_[(env - settings_.rehearsal_environments) % 3u];
    }

    void check_active(uint32_t env, uint32_t id) const {
        if (is_rehearsal(env)) {
            if (id != kInvalidLevel) throw Error(MDN_ERR_INVALID, "rehearsal environment contains a bank level");
            return;
        }
        if (id >= bank_.levels.size()) throw Error(MDN_ERR_INVALID, "active challenge id is outside the train bank");
        if (bank_.levels[id].info.family != pool_of(env).family)
            throw Error(MDN_ERR_INVALID, "active challenge id violates its fixed per-environment family quota");
    }

    void fill_row(uint32_t env, uint32_t* row, uint32_t first_slot) {
        uint32_t* end = row + settings_.horizon + 1;
        if (is_rehearsal(env)) {
            std::fill(row + first_slot, end, kInvalidLevel);
            return;
        }
        const FamilyPool& pool = pool_of(env);
        for (uint32_t* slot = row + first_slot; slot != end; ++slot) *slot = draw(pool);
    }

    uint32_t draw(const FamilyPool& pool) {
        // the floor's draw is taken only under failure-weighted selection
        const bool weighted = settings_.selection == 1u && !(rng_.unit() < settings_.uniform_floor);
        if (!weighted) return pool.levels[rng_.below(pool.levels.size())];
        double remainder = rng_.unit() * pool.weight_total;
        const size_t last = pool.levels.size() - 1;
        for (size_t i = 0; i < last; ++i) {
            remainder -= pool.weight[i];
            if (remainder <= 0.0) return pool.levels[i];
        }
        return pool.levels[last];
    }

    void refresh_weights() {
        const double mix = settings_.score_staleness_mix;
        for (FamilyPool& pool : pools_) {
            pool.weight.clear();
            pool.weight_total = 0.0;
            if (settings_.selection != 1u) continue;
            const std::vector<float>& score = ledger_.score;
            const std::vector<uint64_t>& visited = ledger_.visited;
            const auto by_score = pool_ranks(pool.levels, [&](uint32_t a, uint32_t b) {
                return score[a] != score[b] ? score[a] > score[b] : a < b;
            });
            const auto by_age = pool_ranks(pool.levels, [&](uint32_t a, uint32_t b) {
                return visited[a] != visited[b] ? visited[a] < visited[b] : a < b;
            });
            pool.weight.resize(pool.levels.size());
            for (size_t i = 0; i < pool.levels.size(); ++i) {
                pool.weight[i] = mix / double(by_score[i] + 1) + (1.0 - mix) / double(by_age[i] + 1);
                pool.weight_total += pool.weight[i];
            }
        }
    }

    void close_episode(uint32_t env, uint32_t level, uint64_t rollout_index) {
        const uint32_t samples = open_.samples[env];
        if (samples == 0) throw Error(MDN_ERR_INVALID, "completed challenge episode has no GAE samples");
        ledger_.score[level] = float(open_.abs_gae[env] / samples);
        ledger_.scored[level] = rollout_index;
        ledger_.completed[level] += 1;
        open_.abs_gae[env] = 0.0;
        open_.samples[env] = 0;
        open_.level[env] = kInvalidLevel;
    }

    SidecarHeader sidecar_header(const std::string& checkpoint_hash, uint64_t completed_rollouts) const {
        if (checkpoint_hash.size() != 64)
            throw Error(MDN_ERR_INVALID, "challenge state requires a SHA-256 checkpoint hash");
        SidecarHeader h{};
        std::memcpy(h.magic, kSidecarMagic, 8);
        h.version = kSidecarVersion;
        h.selection = settings_.selection;
        h.environment_count = settings_.environment_count;
        h.horizon = settings_.horizon;
        h.level_count = uint32_t(bank_.levels.size());
        h.rng_state = rng_.state;
        h.focus_family = settings_.focus_family;
        h.rehearsal = settings_.rehearsal_environments;
        h.last_rollout = last_rollout_;
        h.completed_rollouts = completed_rollouts;
        h.uniform_floor = settings_.uniform_floor;
        h.score_staleness_mix = settings_.score_staleness_mix;
        std::memcpy(h.bank_hash, bank_.bank_hash.data(), 64);
        std::memcpy(h.world_hash, world_hash_.data(), 64);
        std::memcpy(h.checkpoint_hash, checkpoint_hash.data(), 64);
        return h;
    }

    // The header must describe this sampler, this bank and world, the given
    // checkpoint, and the rollout boundary the checkpoint was taken at.
    bool header_matches(const SidecarHeader& h, const std::string& checkpoint_hash, uint64_t completed_rollouts) const {
        const auto& s = settings_;
        const bool current = h.version == kSidecarVersion;
        if (std::memcmp(h.magic, kSidecarMagic, 8) != 0 || h.version < 1u || h.version > kSidecarVersion) return false;
        // before version 3 the field was zero and no focus family existed
        if (current ? h.focus_family != s.focus_family : (h.focus_family != 0u || s.focus_family != 0u)) return false;
        if (h.version == 1u && h.rehearsal != 0u) return false;
        if (h.selection != s.selection || h.environment_count != s.environment_count || h.horizon != s.horizon ||
            h.level_count != bank_.levels.size() || h.rehearsal != s.rehearsal_environments || h.rng_state == 0u)
            return false;
        const uint64_t expected_last = completed_rollouts == 0 ? 0 : completed_rollouts - 1;
        if (h.completed_rollouts != completed_rollouts || h.last_rollout != expected_last) return false;
        if (std::fabs(h.uniform_floor - s.uniform_floor) > 1e-7f ||
            std::fabs(h.score_staleness_mix - s.score_staleness_mix) > 1e-7f)
            return false;
        return std::memcmp(h.bank_hash, bank_.bank_hash.data(), 64) == 0 &&
               std::memcmp(h.world_hash, world_hash_.data(), 64) == 0 && is_sha256(checkpoint_hash) &&
               std::memcmp(h.checkpoint_hash, checkpoint_hash.data(), 64) == 0;
    }

    static void read_span(std::ifstream& file, const ByteSpan& b) {
        file.read(static_cast<char*>(b.data), std::streamsize(b.bytes));
        if (!file) throw Error(MDN_ERR_MISMATCH, "challenge sampler state is truncated");
    }
};

}  // namespace mdn

using namespace mdn;

struct mdn_bank {
    BankData data;
};
struct mdn_challenge {
    std::unique_ptr<ChallengeSampler> sampler;
    mdn_bank view;  // the train split, as a bank handle
};

static const Level& bank_level(const mdn_bank* bank, uint32_t index) {
    require(bank != nullptr, MDN_ERR_INVALID, "null challenge bank");
    require(index < bank->data.levels.size(), MDN_ERR_INVALID, "challenge level index out of range");
    return bank->data.levels[index];
}

static std::string hash_arg(const char* hash, const char* what) {
    require(hash != nullptr, MDN_ERR_INVALID, std::string(what) + ": null hash");
    return std::string(hash);
}

extern "C" int mdn_sha256_file(const char* path, char out[65]) {
    return guarded([&] {
        require(path && out, MDN_ERR_INVALID, "sha256: null argument");
        const std::string h = sha256_file(path);
        std::memcpy(out, h.c_str(), 65);
    });
}

extern "C" int mdn_bank_load(const char* jsonl_path, const char* split, const char* expected_world_sha256,
                             mdn_bank** out) {
    return guarded([&] {
        require(jsonl_path && split && out, MDN_ERR_INVALID, "challenge bank: null argument");
        *out = nullptr;
        auto bank = std::make_unique<mdn_bank>();
        load_split(jsonl_path, split, hash_arg(expected_world_sha256, "challenge bank"), bank->data);
        *out = bank.release();
    });
}

extern "C" int mdn_bank_free(mdn_bank* bank) {
    delete bank;
    return MDN_OK;
}

extern "C" int mdn_bank_info(const mdn_bank* bank, uint32_t* level_count, char bank_sha256[65]) {
    return guarded([&] {
        require(bank != nullptr, MDN_ERR_INVALID, "null challenge bank");
        if (level_count) *level_count = uint32_t(bank->data.levels.size());
        if (bank_sha256) std::memcpy(bank_sha256, bank->data.bank_hash.c_str(), 65);
    });
}

extern "C" int mdn_bank_level_get(const mdn_bank* bank, uint32_t index, mdn_bank_level* level, mdn_world* world) {
    return guarded([&] {
        const Level& l = bank_level(bank, index);
        if (level) *level = l.info;
        if (world) *world = l.world;
    });
}

extern "C" int mdn_bank_worlds(const mdn_bank* bank, mdn_world* out, uint32_t capacity) {
    return guarded([&] {
        require(bank && out, MDN_ERR_INVALID, "challenge bank: null argument");
        require(capacity >= bank->data.levels.size(), MDN_ERR_INVALID, "challenge bank: world capacity too small");
        for (size_t i = 0; i < bank->data.levels.size(); i++) out[i] = bank->data.levels[i].world;
    });
}

extern "C" const char* mdn_bank_level_text(const mdn_bank* bank, uint32_t index, int field) {
    if (!bank || index >= bank->data.levels.size()) return nullptr;
    const Level& l = bank->data.levels[index];
    switch (field) {
        case MDN_BANK_FAILURE_ID: return l.failure_id.c_str();
        case MDN_BANK_SPLIT: return l.split.c_str();
        case MDN_BANK_FAMILY_NAME: return l.family_name.c_str();
        case MDN_BANK_GEOMETRY_CONTRACT: return l.geometry_contract.c_str();
        case MDN_BANK_DIFFICULTY_BAND: return l.difficulty_band.c_str();
        case MDN_BANK_SCENE_SHA256: return l.scene_sha256.c_str();
        case MDN_BANK_WORLD_SOURCE_SHA256: return l.world_source_sha256.c_str();
        default: return nullptr;
    }
}

extern "C" int mdn_bank_witness_route(const mdn_bank* bank, uint32_t index, float* xyz, uint32_t capacity,
                                      uint32_t* count) {
    return guarded([&] {
        const Level& l = bank_level(bank, index);
        const uint32_t points = uint32_t(l.witness_route.size() / 3);
        if (count) *count = points;
        if (xyz) {
            require(capacity >= points, MDN_ERR_INVALID, "challenge bank: witness route capacity too small");
            std::copy(l.witness_route.begin(), l.witness_route.end(), xyz);
        }
    });
}

extern "C" void mdn_challenge_settings_default(mdn_challenge_settings* out) {
    if (!out) return;
    *out = mdn_challenge_settings{};
    out->environment_count = 128;  // challenge_training.hpp:40-49
    out->horizon = 32;
    out->sampler_seed = 1;
    out->rehearsal_environments = 0;
    out->selection = 0;
    out->uniform_floor = 0.50f;
    out->score_staleness_mix = 0.50f;
    out->focus_family = 0;
}

static ChallengeSampler& sampler_of(const mdn_challenge* c) {
    require(c != nullptr && c->sampler != nullptr, MDN_ERR_INVALID, "null challenge sampler");
    return *c->sampler;
}

extern "C" int mdn_challenge_create(const char* bank_jsonl, const char* expected_world_sha256,
                                    const mdn_challenge_settings* settings, mdn_challenge** out) {
    return guarded([&] {
        require(bank_jsonl && settings && out, MDN_ERR_INVALID, "challenge sampler: null argument");
        *out = nullptr;
        auto c = std::make_unique<mdn_challenge>();
        c->sampler = std::make_unique<ChallengeSampler>(bank_jsonl, hash_arg(expected_world_sha256, "challenge sampler"),
                                                        *settings);
        c->view.data = c->sampler->bank();
        *out = c.release();
    });
}

extern "C" int mdn_challenge_destroy(mdn_challenge* sampler) {
    delete sampler;
    return MDN_OK;
}

extern "C" int mdn_challenge_bank(mdn_challenge* sampler, const mdn_bank** out) {
    return guarded([&] {
        sampler_of(sampler);
        require(out != nullptr, MDN_ERR_INVALID, "challenge sampler: null out");
        *out = &sampler->view;
    });
}

extern "C" int mdn_challenge_control(const mdn_challenge* sampler, mdn_bank_control* out) {
    return guarded([&] {
        require(out != nullptr, MDN_ERR_INVALID, "challenge sampler: null out");
        *out = sampler_of(sampler).control();
    });
}

extern "C" int mdn_challenge_initial_schedule(mdn_challenge* sampler, uint32_t* schedule) {
    return guarded([&] {
        require(schedule != nullptr, MDN_ERR_INVALID, "challenge sampler: null schedule");
        sampler_of(sampler).initial_schedule(schedule);
    });
}

extern "C" int mdn_challenge_next_schedule(mdn_challenge* sampler, const uint32_t* active_ids, uint64_t rollout_index,
                                           uint32_t* schedule) {
    return guarded([&] {
        require(active_ids && schedule, MDN_ERR_INVALID, "challenge sampler: null argument");
        sampler_of(sampler).next_schedule(active_ids, rollout_index, schedule);
    });
}

extern "C" int mdn_challenge_active_ids(const mdn_challenge* sampler, uint32_t* out) {
    return guarded([&] {
        require(out != nullptr, MDN_ERR_INVALID, "challenge sampler: null out");
        const auto& a = sampler_of(sampler).active_ids();
        require(!a.empty(), MDN_ERR_STATE, "challenge sampler: no schedule issued yet");
        std::copy(a.begin(), a.end(), out);
    });
}

extern "C" int mdn_challenge_observe_raw_gae(mdn_challenge* sampler, const float* raw_gae, const uint8_t* terminated,
                                             const uint8_t* truncated, const uint32_t* transition_ids,
                                             uint64_t rollout_index) {
    return guarded([&] {
        sampler_of(sampler).observe_raw_gae(raw_gae, terminated, truncated, transition_ids, rollout_index);
    });
}

extern "C" int mdn_challenge_level_stats(const mdn_challenge* sampler, uint32_t level, float* score,
                                         uint64_t* completed_episodes, uint64_t* last_visit_rollout) {
    return guarded([&] { sampler_of(sampler).level_stats(level, score, completed_episodes, last_visit_rollout); });
}

extern "C" int mdn_challenge_save_state(mdn_challenge* sampler, const char* path, const char* checkpoint_sha256,
                                        uint64_t completed_rollouts, const uint32_t* active_ids) {
    return guarded([&] {
        require(path && active_ids, MDN_ERR_INVALID, "challenge sampler: null argument");
        sampler_of(sampler).save_state(path, hash_arg(checkpoint_sha256, "challenge sampler"), completed_rollouts,
                                       active_ids);
    });
}

extern "C" int mdn_challenge_load_state(mdn_challenge* sampler, const char* path, const char* checkpoint_sha256,
                                        uint64_t completed_rollouts, uint32_t* active_ids) {
    return guarded([&] {
        require(path && active_ids, MDN_ERR_INVALID, "challenge sampler: null argument");
        sampler_of(sampler).load_state(path, hash_arg(checkpoint_sha256, "challenge sampler"), completed_rollouts,
                                       active_ids);
    });
}

// ------------------------------------------------------------------ evaluation
// challenge_evaluation::run (challenge_evaluation.hpp:352-497).
namespace mdn {
namespace {

std::string csv_cell(const std::string& value) {  // :316-321
    if (value.find_first_of(",\"\r\n") == std::string::npos) return value;
    std::string escaped = "\"";
    for (char c : value) {
        if (c == '"') escaped += '"';
        escaped += c;
    }
    return escaped + '"';
}
std::string number_cell(double value) {  // :323-328
    std::ostringstream out;
    out.imbue(std::locale::classic());
    out << std::setprecision(9) << value;
    return out.str();
}
std::string uint_cell(uint64_t value) { return std::to_string(value); }
std::string witness_route_cell(const Level& level) {  // :332-342
    std::ostringstream out;
    out.imbue(std::locale::classic());
    out << std::setprecision(9) << '[';
    for (size_t i = 0; i < level.witness_route.size() / 3; ++i) {
        if (i) out << ',';
        out << '[' << level.witness_route[3 * i] << ',' << level.witness_route[3 * i + 1] << ','
            << level.witness_route[3 * i + 2] << ']';
    }
    out << ']';
    return out.str();
}
void write_csv_row(std::ofstream& file, const std::vector<std::string>& cells) {
    for (size_t i = 0; i < cells.size(); ++i) {
        if (i) file << ',';
        file << csv_cell(cells[i]);
    }
    file << '\n';
}

// Status -> exception, for calls into this library's own C-ABI.
void ok(int status) {
    if (status != MDN_OK) throw Error(status, mdn_last_error());
}

struct SimGuard {
    mdn_sim* sim = nullptr;
    ~SimGuard() {
        if (sim) mdn_sim_destroy(sim);
    }
};

mdn_bank_score evaluate(mdn_device* dev, const mdn_raptor_weights* raptor, const std::string& checkpoint_path,
                        const std::string& bank_path, const std::string& split, const std::string& world_hash,
                        const std::string& output_path, uint32_t mode, float speed, uint32_t max_steps) {
    auto fail = [](const std::string& m) { bank_fail(m); };
    if (mode != 2 && mode != 13 && mode != 17) fail("mode must be 2, 13, or 17");
    if (!std::isfinite(speed) || speed <= 0 || speed > 3.0f) fail("speed must be finite and in (0,3]");
    if (max_steps == 0 || max_steps > 400) fail("max_steps must be in 1..400 (maximum 20 seconds)");
    require(dev != nullptr && raptor != nullptr, MDN_ERR_INVALID, "challenge bank: null device or controller");

    const std::string checkpoint_hash = sha256_file(checkpoint_path);
    std::ifstream checkpoint(checkpoint_path, std::ios::binary);
    if (!checkpoint) throw Error(MDN_ERR_IO, "challenge bank: cannot open checkpoint: " + checkpoint_path);
    mdn_checkpoint_header header;
    read_checkpoint_header(checkpoint, header);
    // The actor may be the 64-unit one or a wide one (hidden*189 + 8 floats).
    const uint32_t hidden = header.actor_count >= 8 ? (header.actor_count - 8) / 189 : 0;
    const bool actor_ok = header.actor_count == actor_param_count(hidden) &&
                          (hidden == uint32_t(kHidden) || (hidden % 256 == 0 && hidden >= 256 && hidden <= 8192));
    if (!actor_ok || header.critic_count != uint32_t(kCriticParams) || header.version < 3 || header.version > 9)
        fail("checkpoint header/dimensions are unsupported");
    std::vector<float> actor(header.actor_count), critic(header.critic_count);
    checkpoint.read(reinterpret_cast<char*>(actor.data()), std::streamsize(actor.size() * sizeof(float)));
    checkpoint.read(reinterpret_cast<char*>(critic.data()), std::streamsize(critic.size() * sizeof(float)));
    if (!checkpoint) fail("checkpoint is missing actor or critic weights");
    auto finite = [](float v) { return std::isfinite(v); };
    if (!std::all_of(actor.begin(), actor.end(), finite) || !std::all_of(critic.begin(), critic.end(), finite))
        fail("checkpoint contains non-finite weights");

    BankData bank;
    load_split(bank_path, split, world_hash, bank);
    const std::vector<Level>& levels = bank.levels;
    const std::filesystem::path output_file(output_path);
    if (output_file.has_parent_path()) std::filesystem::create_directories(output_file.parent_path());
    const std::filesystem::path temporary_output = output_file.string() + ".tmp";
    std::ofstream csv(temporary_output, std::ios::out | std::ios::trunc);
    if (!csv) throw Error(MDN_ERR_IO, "challenge bank: cannot write output CSV: " + temporary_output.string());
    csv.imbue(std::locale::classic());
    write_csv_row(csv, {"failure_id", "scene_sha256", "split", "family", "family_name", "seed", "base_seed",
                        "environment_index", "distance_m", "geometry_contract", "difficulty", "difficulty_band", "mode",
                        "speed_mps", "max_steps", "wind_x", "wind_y", "wind_z", "obstacle_count", "witness_route_json",
                        "episodes", "success", "collision", "timeout", "progress", "path_m", "elapsed_s",
                        "goal_time_s", "mean_speed_mps", "peak_speed_mps", "min_clearance_m", "physics_invalid",
                        "direct_route_clearance_m", "witness_min_clearance_m", "witness_sample_count",
                        "checkpoint_sha256", "bank_sha256", "world_source_sha256"});

    mdn_bank_score score{};
    constexpr uint32_t kBatch = 128;  // challenge_evaluation.hpp:30
    for (size_t begin = 0; begin < levels.size(); begin += kBatch) {
        const uint32_t count = uint32_t(std::min<size_t>(kBatch, levels.size() - begin));
        mdn_sim_config config;
        mdn_sim_config_default(&config);
        config.n = count;
        config.family = 0;  // the bank's geometry replaces the reset's worlds before any observation
        config.mode = mode;
        config.seed = levels[begin].info.seed;
        config.eval = 1;
        config.speed = speed;
        config.distance = levels[begin].info.distance;
        config.max_steps = max_steps;
        config.sensor_delay = 0;
        config.command_delay = 0;
        config.wind = 0;
        config.depth_noise = 0;
        config.dropout = 0;
        config.velocity_contract = header.config.velocity_contract;
        config.geometry_memory = header.config.geometry_memory;
        mdn_rollout_shape shape;
        mdn_rollout_shape_default(&shape);
        shape.actor_hidden = hidden;
        SimGuard guard;
        ok(mdn_sim_create(dev, &config, &shape, 32, raptor, nullptr, &guard.sim));
        mdn_sim* sim = guard.sim;
        ok(mdn_sim_upload(sim, MDN_BUF_ACTOR, actor.data(), 0, actor.size() * sizeof(float)));
        ok(mdn_sim_upload(sim, MDN_BUF_CRITIC, critic.data(), 0, critic.size() * sizeof(float)));
        std::vector<mdn_world> worlds(count);
        std::vector<mdn_sim_run> runs(count);
        ok(mdn_sim_download(sim, MDN_BUF_RUNS, runs.data(), 0, runs.size() * sizeof(mdn_sim_run)));
        for (uint32_t n = 0; n < count; ++n) {
            const Level& level = levels[begin + n];
            worlds[n] = level.world;
            // The reset's policy-sampling seed of this bank environment, independent of its batch slot.
            runs[n].rng = level.info.base_seed + level.info.environment_index * kEnvStride + kEnvOffset;
            runs[n].steps = 0;
            const float* g = level.world.goal;
            runs[n].initial_distance = std::sqrt(g[0] * g[0] + g[1] * g[1] + (g[2] - 1.5f) * (g[2] - 1.5f));
            runs[n].reference_position[0] = 0;
            runs[n].reference_position[1] = 0;
            runs[n].reference_position[2] = 1.5f;
        }
        ok(mdn_sim_upload(sim, MDN_BUF_WORLDS, worlds.data(), 0, worlds.size() * sizeof(mdn_world)));
        ok(mdn_sim_upload(sim, MDN_BUF_RUNS, runs.data(), 0, runs.size() * sizeof(mdn_sim_run)));
        ok(mdn_sim_collect(sim, max_steps));
        ok(mdn_sync(dev, nullptr));
        std::vector<mdn_physics_state> states(count);
        ok(mdn_sim_download(sim, MDN_BUF_RUNS, runs.data(), 0, runs.size() * sizeof(mdn_sim_run)));
        ok(mdn_sim_download(sim, MDN_BUF_STATES, states.data(), 0, states.size() * sizeof(mdn_physics_state)));
        for (uint32_t n = 0; n < count; ++n) {
            const Level& level = levels[begin + n];
            const mdn_sim_run& run = runs[n];
            if (run.episodes != 1 || run.successes + run.collisions + run.timeouts != 1)
                fail("level did not produce exactly one terminal outcome: " + level.failure_id);
            const float progress = run.final_progress;
            const float mean_speed = run.elapsed > 0 ? run.path / run.elapsed : 0;
            const float values[] = {progress, run.path, run.elapsed, run.success_time, mean_speed, run.peak_speed,
                                    run.min_clearance};
            if (!std::all_of(std::begin(values), std::end(values), finite))
                fail("non-finite episode metric for " + level.failure_id);
            for (int j = 0; j < 3; ++j)
                if (!std::isfinite(states[n].position[j]) || !std::isfinite(states[n].linear_velocity[j]))
                    fail("non-finite terminal simulator state for " + level.failure_id);
            score.episodes += run.episodes;
            score.successes += run.successes;
            score.collisions += run.collisions;
            score.timeouts += run.timeouts;
            score.successful_time_s += run.success_time;
            const size_t slot = level.info.family - 14;
            score.family_episodes[slot] += run.episodes;
            score.family_successes[slot] += run.successes;
            const mdn_bank_level& i = level.info;
            write_csv_row(csv, {level.failure_id, level.scene_sha256, level.split, uint_cell(i.family), level.family_name,
                                uint_cell(i.seed), uint_cell(i.base_seed), uint_cell(i.environment_index),
                                number_cell(i.distance), level.geometry_contract, number_cell(i.difficulty),
                                level.difficulty_band, uint_cell(mode), number_cell(speed), uint_cell(max_steps),
                                number_cell(level.world.wind[0]), number_cell(level.world.wind[1]),
                                number_cell(level.world.wind[2]), uint_cell(level.world.count),
                                witness_route_cell(level), uint_cell(run.episodes), uint_cell(run.successes),
                                uint_cell(run.collisions), uint_cell(run.timeouts), number_cell(progress),
                                number_cell(run.path), number_cell(run.elapsed),
                                run.successes ? number_cell(run.success_time) : "", number_cell(mean_speed),
                                number_cell(run.peak_speed), number_cell(run.min_clearance), "not_instrumented",
                                number_cell(i.direct_route_clearance_m), number_cell(i.witness_min_clearance_m),
                                uint_cell(i.witness_sample_count), checkpoint_hash, bank.bank_hash,
                                level.world_source_sha256});
        }
        csv.flush();
        if (!csv) throw Error(MDN_ERR_IO, "challenge bank: write failed for output CSV: " + temporary_output.string());
    }
    csv.close();
    if (!csv) throw Error(MDN_ERR_IO, "challenge bank: close failed for output CSV: " + temporary_output.string());
    std::error_code rename_error;
    std::filesystem::rename(temporary_output, output_file, rename_error);
    if (rename_error)
        throw Error(MDN_ERR_IO, "challenge bank: cannot atomically publish output CSV: " + rename_error.message());
    return score;
}

}  // namespace
}  // namespace mdn

extern "C" int mdn_bank_evaluate(mdn_device* dev, const mdn_raptor_weights* raptor, const char* checkpoint_path,
                                 const char* bank_jsonl, const char* split, const char* world_sha256,
                                 const char* output_csv, uint32_t mode, float speed, uint32_t max_steps,
                                 mdn_bank_score* score) {
    return guarded([&] {
        require(checkpoint_path && bank_jsonl && split && world_sha256 && output_csv, MDN_ERR_INVALID,
                "challenge bank: null argument");
        const mdn_bank_score s = mdn::evaluate(dev, raptor, checkpoint_path, bank_jsonl, split, world_sha256,
                                               output_csv, mode, speed, max_steps);
        if (score) *score = s;
    });
}
