// Drives the C++ host veneer (include/mdn.hpp) end to end on one GPU:
// evaluation of a fresh actor twice (deterministic), a two-rollout task
// training run from a warm-start checkpoint, and its resume for a third
// rollout. Prints the scores and the trainer state for the Python test.
//   argv: workdir
#include <cstdio>
#include <string>
#include <vector>

#include "mdn.hpp"

using namespace mdn::host;

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    const std::string dir = argv[1];
    try {
        Device device(0);
        mdn_sim_config cfg;
        mdn_sim_config_default(&cfg);
        cfg.n = 128;
        cfg.mode = 22;
        cfg.family = 1;
        cfg.seed = 11;
        cfg.speed = 1.5f;
        cfg.distance = 8;
        cfg.max_steps = 400;
        cfg.geometry_memory = 1;
        Sim warm(device, cfg, 32);
        PPOTrainer warm_trainer(warm);
        warm_trainer.save_checkpoint(dir + "/warm.bin", 1, 11, 0);
        const auto actor = warm.download<float>(MDN_BUF_ACTOR);
        // deployment inference of the fresh actor on a constant observation row
        std::vector<float> row(184, 0.5f);
        const auto means = warm.actor_means(row);
        std::printf("means %.9g %.9g %.9g %.9g\n", means[0], means[1], means[2], means[3]);
        const auto a = navigation_training::evaluate(device, actor.data(), 2, 1, 0.0f, 800001, dir + "/eval.csv");
        const auto b = navigation_training::evaluate(device, actor.data(), 2, 1, 0.0f, 800001);
        std::printf("eval %.9g %.9g %.9g %.9g\n", a.success, a.collision, a.timeout, a.successful_time_s);
        std::printf("eval_again %.9g %.9g %.9g %.9g\n", b.success, b.collision, b.timeout, b.successful_time_s);
        navigation_training::train(device, 2, dir + "/task.bin", dir + "/warm.bin", 2, 1, 0.0f, 11, 1);
        navigation_training::train(device, 1, dir + "/task.bin", dir + "/warm.bin", 2, 1, 0.0f, 11, 1);
        std::printf("done\n");
    } catch (const Error& e) {
        std::printf("error %d %s\n", e.code, e.what());
        return 1;
    }
    return 0;
}
