// profile.h — launch counting and optional CUDA-event timing per kernel category.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace arcqml {

enum ProfCategory {
    PROF_GATE = 0,       // per-gate kernels (gate, diagonal, dense, derivative)
    PROF_FUSED_FWD = 1,  // fused forward passes
    PROF_FUSED_ADJ = 2,  // fused adjoint passes
    PROF_ADJ_STEP = 3,   // per-gate adjoint steps
    PROF_PAULI = 4,      // observable passes
    PROF_OTHER = 5,      // reductions, scaling, norms, basis states
    PROF_SHARD = 6,      // shard slice packing for global-qubit swaps
};
constexpr int kProfCategories = 7;

struct ProfToken {
    int cat = -1;
    cudaEvent_t a = nullptr, b = nullptr;
};

// Counts one launch; when timing is on, records a start event on s.
ProfToken prof_begin(int cat, cudaStream_t s);
// Records the stop event; `bytes` is the launch's algorithmic HBM traffic.
void prof_end(const ProfToken &t, cudaStream_t s, double bytes);
void prof_count_launch();
void prof_enable(bool on);
void prof_read(int cat, uint64_t *launches, double *ms, double *bytes);
uint64_t prof_launch_count();

}  // namespace arcqml
