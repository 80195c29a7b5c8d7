/*
 * TEST INFRASTRUCTURE ONLY - a stand-in for the reference's
 * challenge_evaluation.hpp when compiling its challenge_training.hpp on Linux.
 *
 * The reference header parses JSONL with Foundation (NSJSONSerialization) and
 * hashes with CommonCrypto, neither of which exists here. The sampler in
 * challenge_training.hpp only needs, from it, Level::{split, family, world},
 * load_split() and is_sha256(). This stand-in provides those, with load_split
 * reading levels that the tests have already parsed, from a flat file:
 *   char magic[8] = "MDNLVL1\0"; uint32 count; char bank_hash[64];
 *   count x { uint32 split (0 train, 1 dev, 2 final); uint32 family; WWorld world; }
 * oracle/Makefile puts this directory first on the quoted-include path with
 * -I- so that the unmodified challenge_training.hpp includes this file.
 */
#pragma once
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "world.hpp"

namespace challenge_evaluation {

struct Level {
    std::string split;
    uint32_t family = 0;
    WWorld world{};
};

inline bool is_sha256(const std::string& value) {
    return value.size() == 64 && std::all_of(value.begin(), value.end(), [](unsigned char c) {
        return (c >= '0' && c <= '9') || (c >= 'a' && c <= 'f');
    });
}

inline std::vector<Level> load_split(const std::string& path, const std::string& split,
                                     const std::string& /*expected_world_hash*/, std::string& bank_hash) {
    std::ifstream f(path, std::ios::binary);
    char magic[8];
    uint32_t count = 0;
    char hash[64];
    if (!f.read(magic, 8) || std::memcmp(magic, "MDNLVL1", 8) != 0 || !f.read(reinterpret_cast<char*>(&count), 4) ||
        !f.read(hash, 64))
        throw std::runtime_error("level file: bad header");
    bank_hash.assign(hash, 64);
    static const char* names[3] = {"train", "dev", "final"};
    std::vector<Level> selected;
    for (uint32_t i = 0; i < count; i++) {
        uint32_t s = 0;
        Level level;
        if (!f.read(reinterpret_cast<char*>(&s), 4) || s > 2 ||
            !f.read(reinterpret_cast<char*>(&level.family), 4) ||
            !f.read(reinterpret_cast<char*>(&level.world), sizeof(WWorld)))
            throw std::runtime_error("level file: truncated");
        level.split = names[s];
        if (level.split == split) selected.push_back(level);
    }
    if (selected.empty()) throw std::runtime_error("level file: no records for the split");
    return selected;
}

}  // namespace challenge_evaluation
