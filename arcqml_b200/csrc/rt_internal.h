// rt_internal.h — internal types of the ArcQML B200 statevector runtime (host + device).
//
// Layout in HBM: a state of n qubits is 2^n complex128 amplitudes stored as double2
// {re, im}, basis index bit q <-> qubit q (q0 = LSB). A batch is [batch, 2^n] row-major.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/arcqml_runtime.h"

namespace arcqml {

// ------------------------------------------------------------------ errors

// Sets the calling thread's last error message (read back by arcqml_rt_last_error).
void set_last_error(const std::string &msg);

struct Error {
    std::string msg;
};

[[noreturn]] void fail(const std::string &msg);
void check_cuda(cudaError_t e, const char *what);

// ------------------------------------------------------------------ gate lowering

// Maximum number of qubits a state may have (2^n amplitudes must be addressable).
constexpr uint32_t kMaxQubits = 40;
// Custom unitaries of arity above this go through the generic dense kernel; the
// matrix of a k-qubit gate holds 4^k complex entries.
constexpr uint32_t kMaxDenseArity = 10;

enum GateKind : int32_t {
    KIND_NONE = 0,   // identity (I), nothing to do
    KIND_1Q = 1,     // dense 2x2 on one target, optional controls
    KIND_2Q = 2,     // dense 4x4 on two targets, optional controls
    KIND_DIAG1 = 3,  // diagonal 2x2 on one target, optional controls
    KIND_DIAG2 = 4,  // diagonal 4x4 on two targets, optional controls
    KIND_DENSE = 5,  // dense 2^k x 2^k, no controls, matrix in device memory
};

// One gate lowered to the form the kernels consume. `positions` lists every qubit position
// the kernel must hold fixed while enumerating groups (targets and controls), sorted
// ascending. Amplitudes whose control bits are not all 1 are untouched (or zeroed when
// `zero_uncontrolled` is set, which is how derivative matrices of controlled gates act).
struct DevGate {
    int32_t kind;
    int32_t nt;                // number of targets (1, 2, or k for KIND_DENSE)
    int32_t npos;              // number of entries in positions
    int32_t zero_uncontrolled; // derivative form: control-0 block is zero
    int32_t t[2];              // targets: local bit j of the gate matrix <-> t[j]
    uint64_t cmask;            // control mask
    uint8_t positions[kMaxQubits];
    double2 m[16];             // 2x2 (KIND_1Q/DIAG1 uses m[0..3] or diag m[0], m[1]),
                               // 4x4 (KIND_2Q), diag m[0..3] (KIND_DIAG2)
    const double2 *dense;      // KIND_DENSE: device matrix, row-major 2^k x 2^k
    uint8_t dense_targets[kMaxDenseArity];
};

// Host copy of one plan operation (deep copy of an OperationDescriptor).
struct OpRecord {
    uint32_t opcode = 0;
    std::vector<uint32_t> qubits;
    double params[3] = {0, 0, 0};
    std::vector<double2> custom;  // CUSTOM_UNITARY matrix, 4^arity entries
    std::string name;
    uint32_t num_bindings = 0;
    size_t slots[3] = {0, 0, 0};
    size_t parents[3] = {0, 0, 0};
};

enum LowerMode { LOWER_FORWARD = 0, LOWER_ADJOINT = 1, LOWER_DERIVATIVE = 2 };

// Validates a GateDescriptor + qubit list against a state of num_qubits qubits and fills
// an OpRecord (no bindings). Throws Error with the reference's wording on invalid input.
OpRecord record_from_descriptor(const GateDescriptor *gate, const size_t *qubits,
                                size_t qubits_len, int64_t num_qubits /* -1: unchecked */);
void check_qubits_for_state(const OpRecord &op, uint32_t num_qubits);
// Number of differentiable slots of an opcode.
uint32_t slot_count(uint32_t opcode);
// Small matrix form (controls, targets, 2x2/4x4) of an op. `dense` receives the full
// 2^k x 2^k matrix only for custom unitaries of arity > 2.
DevGate lower(const OpRecord &op, LowerMode mode, uint32_t slot, bool allow_diag = true);
// Dense 2^arity x 2^arity matrix of the op (forward) or of its slot derivative.
std::vector<double2> dense_matrix(const OpRecord &op, bool derivative, uint32_t slot);

// ------------------------------------------------------------------ plans

// The tile qubits each pass of a schedule took (planner.cpp), kept with the plan so that a
// schedule of the same gate structure skips the lookahead search.
struct TileChoices {
    uint64_t key = 0;                                // n, k, rb, direction
    std::vector<uint64_t> signature;                 // per gate, what the choice depended on
    std::vector<std::pair<uint64_t, uint32_t>> take; // per pass: start tile, free qubits
};

struct Plan {
    std::vector<OpRecord> ops;
    mutable std::mutex tiles_mu;
    mutable std::vector<TileChoices> tiles;  // a few entries (one per schedule kind)
};

// ------------------------------------------------------------------ observables

struct PauliGroup {
    uint64_t flip;      // common flip mask
    uint32_t first;     // first term index in the sorted term arrays
    uint32_t count;     // number of terms with this flip mask
};

struct Observable {
    uint32_t num_qubits = 0;
    // Terms sorted by flip mask (stable, diagonal group first when present).
    std::vector<double> coef;         // coefficient * real/imag part of i^y handled below
    std::vector<uint64_t> zmask;      // phase masks
    std::vector<uint32_t> ymod4;      // y count mod 4
    std::vector<PauliGroup> groups;
    // Host tables derived from the terms on first use, per state size (pauli_tile.cu: the tile
    // passes that cover the flip masks). The terms never change after creation.
    mutable std::mutex cache_mu;
    mutable std::vector<std::pair<uint32_t, std::shared_ptr<const void>>> tile_cache;
};

// ------------------------------------------------------------------ execution context

// Per-thread execution resources on the current device: a stream and growable device
// buffers for the host-pointer (v1) entry points and for reduction partials.
struct ThreadContext {
    int device = -1;
    cudaStream_t stream = nullptr;
    void *buf[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};  // 0-2: states, 3: tables,
    size_t cap[5] = {0, 0, 0, 0, 0};                               // 4: fused-pass tables
    double *partials = nullptr;  // block partial sums
    size_t partials_cap = 0;     // in doubles
    double *dgrads = nullptr;    // gradient accumulators
    size_t dgrads_cap = 0;
    double *hvals = nullptr;     // pinned host mirror for small results
    size_t hvals_cap = 0;
    cudaStream_t table_stream = nullptr;  // stream of the last table upload
};

ThreadContext &thread_context();
void *ctx_buffer(ThreadContext &c, int which, size_t bytes);
double *ctx_partials(ThreadContext &c, size_t count);
double *ctx_dgrads(ThreadContext &c, size_t count);
double *ctx_hvals(ThreadContext &c, size_t count);

// ------------------------------------------------------------------ engine (device work)

// All of these run on `stream` over device buffers and do not synchronize.
void launch_gate(double2 *amps, size_t batch, uint32_t n, const DevGate &g, cudaStream_t s);
void launch_gate_out(const double2 *in, double2 *out, size_t batch, uint32_t n,
                     const DevGate &g, cudaStream_t s);
// Adjoint step for one op: psi <- U^dag psi, partial[slot][block] = Re<lam|dU_slot psi>,
// lam <- U^dag lam. Returns the number of blocks written per slot (0 if no slot).
struct AdjointSlots {
    int32_t count;           // number of slots needing gradients (0..3)
    DevGate d[3];            // derivative gates
    int32_t grad_index[3];   // index into the device gradient array
};
void launch_adjoint_step(double2 *psi, double2 *lam, size_t batch, uint32_t n,
                         const DevGate &uadj, const AdjointSlots &slots, double *dgrads,
                         const double *row_scale, ThreadContext &ctx, cudaStream_t s);
void launch_scale(double2 *amps, size_t batch, uint32_t n, const double *row_scale_dev,
                  cudaStream_t s);

void plan_apply_device(Plan &plan, double2 *amps, size_t batch, uint32_t n, ThreadContext &ctx,
                       cudaStream_t s);
void adjoint_backward_device(Plan &plan, double2 *psi, double2 *lam, size_t batch, uint32_t n,
                             const double *upstream_host, const uint8_t *req, size_t req_len,
                             double *grads_host, size_t grads_len, ThreadContext &ctx,
                             cudaStream_t s);
// values_host[b] = <psi_b|H|psi_b>; when out != null also writes out = H psi, or adds H psi
// to out when `accumulate` is set.
void observable_device(Observable &obs, const double2 *psi, double2 *out, size_t batch,
                       uint32_t n, double *values_host, ThreadContext &ctx, cudaStream_t s,
                       bool accumulate = false);

// Large states (pauli_tile.cu, n >= 20): <psi|H|psi> into *value_host and, when out != null,
// H psi into out (added to it with `accumulate`), as passes over 12-qubit tiles that cover the
// observable's flip masks. Returns false, having launched nothing, when the state is smaller or
// a flip mask fits no tile. observable_tile_passes: the pass count (0: not applicable).
bool observable_tiled(const Observable &obs, const double2 *psi, double2 *out, uint32_t n,
                      double *value_host, bool accumulate, ThreadContext &ctx, cudaStream_t s);
uint32_t observable_tile_passes(const Observable &obs, uint32_t n);
// Whether large states use observable_tiled (ARCQML_PAULI_TILE=0 keeps k_pauli).
bool pauli_tiles_enabled();

// One-kernel run + backward of a small single state (small.cu): value <- <H> after the plan
// applied to init (null: |0...0>), grads[parent] += 2 Re<lambda| dU/dp |psi> with lambda = H psi,
// lam0 (may be null) <- lambda_0.
void small_step_device(Plan &plan, Observable &obs, const double2 *init, uint32_t n,
                       const uint8_t *req, size_t req_len, double *grads_host, size_t grads_len,
                       double *value_host, double2 *lam0, ThreadContext &ctx, cudaStream_t s);

// Device optimizer loop (small.cu): `steps` Adam steps of <H> over the parameters (parent
// indexed, params[0..req_len) in and out; req[p] != 0 marks a trained parameter, p >= 1), each
// step forward + <H> + adjoint + Adam in one CTA; energies[i] = <H> before update i. adam_m /
// adam_v (may be null: zero) continue an optimizer that has taken t0 steps.
struct SmallAdam;
// Argument checks of small_adam_device (host only, no CUDA call); returns the plan's ops with
// their bound slots set from params.
std::vector<OpRecord> validate_small_adam(const Plan &plan, const Observable &obs, uint32_t n,
                                          const uint8_t *req, size_t req_len,
                                          const double *params, size_t steps, const SmallAdam &h,
                                          const double *energies);
void small_adam_device(const Plan &plan, Observable &obs, const double2 *init, uint32_t n,
                       const uint8_t *req, size_t req_len, double *params, double *adam_m,
                       double *adam_v, uint64_t t0, size_t steps, const SmallAdam &h,
                       double *energies, ThreadContext &ctx, cudaStream_t s);

// Copies host tables (dense matrices of custom gates) into the context's table buffer;
// returns device pointers in the same order. Valid until the next call on this thread.
std::vector<const double2 *> upload_tables(const std::vector<const std::vector<double2> *> &ms,
                                           ThreadContext &ctx, cudaStream_t s);

}  // namespace arcqml
