/*
 * TEST INFRASTRUCTURE ONLY - never linked into, or called by, the product.
 *
 * C entry points over the reference's own challenge-bank sampler,
 * challenge_training::ChallengeTraining (challenge_training.hpp), compiled
 * unmodified from the reference checkout by oracle/Makefile into
 * oracle/_ref/libref_bank.so. Its JSONL reader (challenge_evaluation.hpp) needs
 * Foundation and cannot be built here; ref/bank_shim/challenge_evaluation.hpp
 * stands in for it and reads levels that the tests parsed beforehand. The tests
 * use this library to pin libmdn's sampler: schedules, failure scores and the
 * CHTRN1 sidecar bytes.
 */
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "challenge_training.hpp"

namespace {
thread_local std::string g_error;
template <class F>
int guard(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return 1;
    }
}
}  // namespace

extern "C" {

const char* refb_error(void) { return g_error.c_str(); }

/* settings: environment_count, horizon, sampler_seed, rehearsal, selection,
 * focus_family as u32[6]; uniform_floor and score_staleness_mix as floats. */
int refb_create(const char* levels, const char* world_hash, const uint32_t* u, float uniform_floor,
                float score_staleness_mix, void** out) {
    return guard([&] {
        challenge_training::Settings s;
        s.environment_count = u[0];
        s.horizon = u[1];
        s.sampler_seed = u[2];
        s.rehearsal_environments = u[3];
        s.selection = challenge_training::SelectionMode(u[4]);
        s.focus_family = u[5];
        s.uniform_floor = uniform_floor;
        s.score_staleness_mix = score_staleness_mix;
        *out = new challenge_training::ChallengeTraining(levels, world_hash, s);
    });
}
void refb_destroy(void* h) { delete static_cast<challenge_training::ChallengeTraining*>(h); }
int refb_control(void* h, uint32_t out[4]) {
    return guard([&] {
        const auto c = static_cast<challenge_training::ChallengeTraining*>(h)->control();
        std::memcpy(out, &c, 16);
    });
}
int refb_initial_schedule(void* h, uint32_t* out) {
    return guard([&] {
        const auto v = static_cast<challenge_training::ChallengeTraining*>(h)->initial_schedule();
        std::memcpy(out, v.data(), v.size() * 4);
    });
}
int refb_next_schedule(void* h, const uint32_t* active, uint32_t envs, uint64_t rollout, uint32_t* out) {
    return guard([&] {
        const auto v = static_cast<challenge_training::ChallengeTraining*>(h)->next_schedule(
            std::vector<uint32_t>(active, active + envs), rollout);
        std::memcpy(out, v.data(), v.size() * 4);
    });
}
int refb_observe(void* h, const float* gae, const uint8_t* term, const uint8_t* trunc, const uint32_t* ids,
                 uint64_t rollout) {
    return guard([&] { static_cast<challenge_training::ChallengeTraining*>(h)->observe_raw_gae(gae, term, trunc, ids, rollout); });
}
int refb_level(void* h, uint32_t level, float* score, uint64_t* completed) {
    return guard([&] {
        auto* t = static_cast<challenge_training::ChallengeTraining*>(h);
        *score = t->level_score(level);
        *completed = t->level_completed_episodes(level);
    });
}
int refb_save(void* h, const char* path, const char* checkpoint_hash, uint64_t completed, const uint32_t* active,
              uint32_t envs) {
    return guard([&] {
        static_cast<challenge_training::ChallengeTraining*>(h)->save_state(path, checkpoint_hash, completed,
                                                                          std::vector<uint32_t>(active, active + envs));
    });
}
int refb_load(void* h, const char* path, const char* checkpoint_hash, uint64_t completed, uint32_t* active) {
    return guard([&] {
        const auto v = static_cast<challenge_training::ChallengeTraining*>(h)->load_state(path, checkpoint_hash, completed);
        std::memcpy(active, v.data(), v.size() * 4);
    });
}
}
