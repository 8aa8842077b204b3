// planner.h — fused-pass schedules built from a plan (host side).
#pragma once

#include <utility>
#include <vector>

#include "fused.h"
#include "rt_internal.h"

namespace arcqml {

struct Step {
    bool is_pass = true;
    const OpRecord *dense_op = nullptr;  // !is_pass: a custom gate on > 2 targets
    PassHeader header{};
    std::vector<SubBlock> subs;
    std::vector<FOp> ops;
    std::vector<double2> mats;
    std::vector<size_t> parents;         // per accumulator of the pass (adjoint)
    // (accumulator, parent): further parents that receive an accumulator's gradient (rotations
    // merged into the rotation that owns the accumulator)
    std::vector<std::pair<uint32_t, size_t>> alias;
    // Scaled pass (compiled kernels only): the state in the tile carries a common factor sigma,
    // true = sigma * stored, multiplied in once at the end from mats[sfin].
    bool scaled = false;
    uint32_t sfin = 0;
};

struct Schedule {
    uint32_t k = 0, rb = 0;
    std::vector<Step> steps;
    uint32_t total_acc = 0;
};

// Forward (adjoint = false) or reverse-daggered (adjoint = true) schedule of the plan's gates
// for an n-qubit state, with tiles of k qubits and rb register bits per thread. With grads,
// every bound slot whose parent has req[parent] != 0 gets an accumulator.
Schedule build_schedule(const Plan &plan, uint32_t n, bool adjoint, const uint8_t *req,
                        bool grads, uint32_t k, uint32_t rb);

// Whether X and single-control CNOT gates on register bits use their register-exchange fast
// paths (on unless ARCQML_FAST_CNOT=0) instead of a dense 2x2 / the generic path.
bool fast_cnot();

// Whether passes merge a Pauli rotation into the previous rotation about the same axis on its
// qubit anywhere in the pass (on unless ARCQML_ROT_MERGE=0; forward passes still merge
// one-qubit gates within a register sub-block without it).
bool rotation_merge();

// Whether each pass also tries tile qubits picked by lookahead (each qubit the one whose tile
// holds the most remaining gates) and keeps whichever choice takes more gates (on unless
// ARCQML_LOOKAHEAD=0: tile qubits in the order the gates need them).
bool lookahead_tiles();

// Whether the run-time compiled kernels run diagonal gates with controls, two-qubit diagonals,
// controlled one-target gates and generic slot gradients (on unless ARCQML_FAST_DIAG=0).
bool fast_diag();

// Whether consecutive sub-blocks that can keep every element in the same warp do so and
// exchange with __syncwarp instead of a CTA barrier (on unless ARCQML_WARP_LOCAL=0).
bool warp_local_exchanges();

// Whether passes pack commuting gates into fewer register sub-blocks than circuit order gives
// (on unless ARCQML_SUBBLOCK_REORDER=0).
bool subblock_reorder();

// Register bits of forward passes on tiles of k qubits (ARCQML_FORWARD_RB may force 3 or 4).
uint32_t forward_rb(uint32_t k);

// Runs the engine's schedule of the plan on a host state (emulate.cpp; diagnostic, no CUDA):
// psi forward, or the adjoint sweep over psi and lam (lam already scaled by the upstream
// factor) adding 2 Re<lam| dU |psi> per required slot into grads[parent].
void emulate_schedule(const Plan &plan, uint32_t n, bool adjoint, double2 *psi, double2 *lam,
                      const uint8_t *req, size_t req_len, double *grads, size_t grads_len);

// Whether compiled passes run Pauli rotations and unitary one-qubit diagonals in their scaled
// unit-diagonal forms (ARCQML_SCALED=0 turns it off).
bool scaled_passes();

// Runs a schedule on device states (fused.cu). psi/lam are [batch, 2^n]; lam is null in
// forward mode. Accumulator partials go to partials[acc * partial_stride + block].
void run_schedule(const Schedule &sch, double2 *psi, double2 *lam, size_t batch, uint32_t n,
                  double *partials, uint32_t partial_stride, ThreadContext &ctx, cudaStream_t s);
// Persistent grid size of the fused kernel for tiles of k qubits with rb register bits
// (resident CTAs on the current device), and its block size 2^(k - rb).
uint32_t fused_grid_blocks(bool adjoint, uint32_t k, uint32_t rb);
uint32_t fused_threads(uint32_t k, uint32_t rb);

// Tile shape the engine uses for an n-qubit state: forward k = min(n, 12) with 4 register bits
// at k = 12 (3 below), adjoint k = min(n, 11) with 3. Fused passes need n >= 8 (a full warp).
// ARCQML_ADJ_TILE=10 caps adjoint tiles at 10 qubits (128 threads, four CTAs per SM);
// ARCQML_FWD_TILE=11 caps forward tiles at 11 (with ARCQML_FORWARD_RB=4: 128 threads, four CTAs).
constexpr uint32_t kFusedMinQubits = 8;
uint32_t adjoint_tile_cap();
uint32_t forward_tile_cap();
inline uint32_t fused_k(uint32_t n, bool adjoint) {
    const uint32_t cap = adjoint ? adjoint_tile_cap() : forward_tile_cap();
    return n < cap ? n : cap;
}
inline uint32_t fused_rb(uint32_t k, bool adjoint) { return (!adjoint && k >= 12) ? 4u : 3u; }

}  // namespace arcqml
