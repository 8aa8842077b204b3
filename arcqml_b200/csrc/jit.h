// jit.h — per-pass fused kernels compiled at run time (jit.cpp).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "planner.h"

namespace arcqml {

// False when ARCQML_JIT=0.
bool jit_enabled();
// The `struct PassOps` source the run-time compiler generates for a pass (empty when the pass
// has no compiled form); a test builds it as host code (ARCQML_HOST_RUN) and runs it.
std::string jit_pass_code(const Step &st, bool adjoint);
// Per step of the schedule: its compiled kernel, or nullptr where the step has no compiled form
// (a dense barrier, an op without a fast path, or a failed compile) and the precompiled pass
// kernel runs instead. Kernels are compiled once per circuit structure and device.
std::vector<void *> jit_kernels(const Schedule &sch, bool adjoint);
// True when the compiled kernel of an (adjoint, rb) pass keeps one accumulator column per warp.
// Threads per gradient accumulator column of compiled adjoint kernels (1, 4 or 32).
uint32_t jit_acc_lanes(bool adjoint, uint32_t rb);
// Whether compiled forward kernels are single-buffered at two CTAs per SM (on unless
// ARCQML_FWD_SINGLE=0).
bool jit_forward_single();
// Whether compiled kernels take their pass's matrix table as a by-value kernel parameter
// (constant-bank operands; forward and adjoint kernels unless ARCQML_JIT_MATS_SMEM=1, which
// stages it in shared memory: 30-qubit adjoint passes 6.3 % slower that way).
bool jit_mats_in_params(bool adjoint);
// Compiles the schedule's passes; true if every pass has a compiled kernel.
bool jit_schedule_compiles(const Schedule &sch, bool adjoint);
// ARCQML_ADJ_WIDE=1 (with the run-time compiler on): adjoint sweeps use 12-qubit tiles with 4
// register bits when every pass compiles.
bool adjoint_wide_tiles();
// Persistent grid of a compiled kernel: resident CTAs per SM x SMs for this launch shape.
uint32_t jit_grid_blocks(void *fn, uint32_t threads, size_t smem);
// Launches a compiled pass kernel with the precompiled kernel's argument list.
void jit_launch(void *fn, unsigned grid, unsigned threads, size_t smem, cudaStream_t s,
                void **args);
// Compiles the schedule's passes with NVRTC only (no device needed); returns how many compiled,
// with the number that have a compiled form in *eligible and the first error in *err.
size_t jit_compile_check(const Schedule &sch, bool adjoint, size_t *eligible, std::string *err);
void jit_info(uint64_t *compiled, uint64_t *launches, uint64_t *fallbacks, std::string *last);

}  // namespace arcqml
