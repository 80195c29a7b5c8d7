/*
 * Stand-in for libdispatch (GCD), test infrastructure only: the reference CPU
 * path runs its per-environment loops through dispatch_apply_f
 * (cpu_reference.hpp:106-110). This maps it to an OpenMP parallel loop over the
 * host's cores; each iteration touches only its own environment.
 */
#pragma once
#include <cstddef>
typedef void* dispatch_queue_t;
#define QOS_CLASS_USER_INITIATED 0x19
inline dispatch_queue_t dispatch_get_global_queue(long, unsigned long) { return nullptr; }
inline void dispatch_apply_f(size_t iterations, dispatch_queue_t, void* context, void (*work)(void*, size_t)) {
#pragma omp parallel for schedule(dynamic, 4)
    for (long i = 0; i < long(iterations); ++i) work(context, size_t(i));
}
