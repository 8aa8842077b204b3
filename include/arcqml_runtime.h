/*
 * arcqml_runtime.h — C ABI of the ArcQML statevector runtime, B200 (sm_100a) build.
 *
 * This header declares the 14 `arcqml_rt_*` symbols that ArcQML's Rust crate
 * `arcqml-runtime-sys` links against (static library name `arcqml_runtime_private`),
 * with the exact `repr(C)` layouts of `arcqml-runtime-abi`. Linking this library
 * in place of the closed CPU runtime leaves every Rust and Python caller unchanged.
 *
 * Reference interface replaced (paths inside the ArcQML project):
 *   crates/arcqml-runtime-sys/src/lib.rs:28-103   raw extern "C" declarations
 *   crates/arcqml-runtime-abi/src/lib.rs:8-153    ABI_VERSION, descriptors, opcodes
 *
 * Conventions (crates/arcqml-circuit/src/gate.rs:4-10, docs/ArcQML技术手册.md:223-247):
 *   - amplitudes are complex128 stored as `double[2]` = {re, im} (num_complex::Complex64);
 *   - basis index bit q <-> qubit q (q0 is the least significant bit);
 *   - the local basis index of a k-qubit gate has bit j <-> qubits[j]; controlled gates
 *     list controls first and targets last;
 *   - custom matrices are row-major, matrix[row * dim + col] = <row|U|col>.
 *
 * Status: every function returning int32_t returns 0 on success and a non-zero code on
 * failure; the message of the calling thread's last failure is read back with
 * arcqml_rt_last_error. No function aborts or throws across this boundary.
 *
 * Amplitude buffers passed to the v1 entry points are HOST memory owned by the caller
 * (borrowed for the call). The runtime copies them to the current CUDA device, runs the
 * sm_100a kernels there and copies the result back before returning. Device-resident
 * entry points that avoid those copies are declared in arcqml_runtime_v2.h.
 */
#ifndef ARCQML_RUNTIME_H
#define ARCQML_RUNTIME_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* crates/arcqml-runtime-abi/src/lib.rs:8 */
#define ARCQML_RT_ABI_VERSION 1u

/* num_complex::Complex64 is repr(C) and layout-compatible with [f64; 2]
 * (crates/arcqml-runtime-abi/src/lib.rs:10-12). */
typedef struct arcqml_c128 {
    double re;
    double im;
} arcqml_c128;

/* crates/arcqml-runtime-abi/src/lib.rs:13-24 */
typedef struct GateDescriptor {
    uint32_t abi_version;
    uint32_t opcode;
    size_t arity;
    double parameters[3];
    const arcqml_c128 *matrix;
    size_t matrix_len;
    const uint8_t *name;
    size_t name_len;
} GateDescriptor;

/* crates/arcqml-runtime-abi/src/lib.rs:29-35 — runtime-owned derivative matrix. */
typedef struct DerivativeMatrixHandle {
    arcqml_c128 *data;
    size_t len;
    size_t capacity;
} DerivativeMatrixHandle;

/* crates/arcqml-runtime-abi/src/lib.rs:81-86 */
typedef struct ParameterBindingDescriptor {
    size_t parameter_slot;
    size_t parent_index;
} ParameterBindingDescriptor;

/* crates/arcqml-runtime-abi/src/lib.rs:88-96 */
typedef struct OperationDescriptor {
    GateDescriptor gate;
    const size_t *qubits;
    size_t qubits_len;
    const ParameterBindingDescriptor *parameters;
    size_t parameters_len;
} OperationDescriptor;

/* crates/arcqml-runtime-abi/src/lib.rs:98-102 */
typedef struct CircuitPlanHandle {
    void *opaque;
} CircuitPlanHandle;

/* Stable gate opcodes, crates/arcqml-runtime-abi/src/lib.rs:113-153. */
enum {
    ARCQML_OP_I = 0,
    ARCQML_OP_X = 1,
    ARCQML_OP_Y = 2,
    ARCQML_OP_Z = 3,
    ARCQML_OP_H = 4,
    ARCQML_OP_S = 5,
    ARCQML_OP_SDG = 6,
    ARCQML_OP_T = 7,
    ARCQML_OP_TDG = 8,
    ARCQML_OP_SX = 9,
    ARCQML_OP_SXDG = 10,
    ARCQML_OP_RX = 11,
    ARCQML_OP_RY = 12,
    ARCQML_OP_RZ = 13,
    ARCQML_OP_PHASE = 14,
    ARCQML_OP_U3 = 15,
    ARCQML_OP_CNOT = 16,
    ARCQML_OP_CY = 17,
    ARCQML_OP_CZ = 18,
    ARCQML_OP_CH = 19,
    ARCQML_OP_CS = 20,
    ARCQML_OP_CT = 21,
    ARCQML_OP_CPHASE = 22,
    ARCQML_OP_CRX = 23,
    ARCQML_OP_CRY = 24,
    ARCQML_OP_CRZ = 25,
    ARCQML_OP_SWAP = 26,
    ARCQML_OP_ISWAP = 27,
    ARCQML_OP_DCX = 28,
    ARCQML_OP_ECR = 29,
    ARCQML_OP_RXX = 30,
    ARCQML_OP_RYY = 31,
    ARCQML_OP_RZZ = 32,
    ARCQML_OP_RZX = 33,
    ARCQML_OP_FSIM = 34,
    ARCQML_OP_TOFFOLI = 35,
    ARCQML_OP_CSWAP = 36,
    ARCQML_OP_MCX = 37,
    ARCQML_OP_CUSTOM_UNITARY = 38
};

/* crates/arcqml-runtime-sys/src/lib.rs:29 — returns ARCQML_RT_ABI_VERSION. */
uint32_t arcqml_rt_abi_version(void);

/* crates/arcqml-runtime-sys/src/lib.rs:30-37 — amplitudes <- U amplitudes, in place. */
int32_t arcqml_rt_v1_apply_gate(arcqml_c128 *amplitudes, size_t amplitudes_len, size_t num_qubits,
                                const GateDescriptor *gate, const size_t *qubits,
                                size_t qubits_len);

/* crates/arcqml-runtime-sys/src/lib.rs:38-45 — amplitudes <- U^dagger amplitudes, in place. */
int32_t arcqml_rt_v1_apply_adjoint_gate(arcqml_c128 *amplitudes, size_t amplitudes_len,
                                        size_t num_qubits, const GateDescriptor *gate,
                                        const size_t *qubits, size_t qubits_len);

/* crates/arcqml-runtime-sys/src/lib.rs:46-55 — output <- (dU/dp_slot) input. For controlled
 * rotations the control-0 block of dU is zero. */
int32_t arcqml_rt_v1_parameter_derivative_into(const arcqml_c128 *input, size_t input_len,
                                               arcqml_c128 *output, size_t output_len,
                                               const GateDescriptor *gate, const size_t *qubits,
                                               size_t qubits_len, size_t parameter_slot);

/* crates/arcqml-runtime-sys/src/lib.rs:56-60 — builds the dense 2^k x 2^k row-major matrix
 * dU/dp_slot; the handle owns it until arcqml_rt_v1_derivative_matrix_destroy. */
int32_t arcqml_rt_v1_derivative_matrix_create(const GateDescriptor *gate, size_t parameter_slot,
                                              DerivativeMatrixHandle *output);

/* crates/arcqml-runtime-sys/src/lib.rs:61-67 — amplitudes <- M amplitudes (M need not be
 * unitary), local index bit j <-> qubits[j]. The state dimension is amplitudes_len. */
int32_t arcqml_rt_v1_derivative_matrix_apply(arcqml_c128 *amplitudes, size_t amplitudes_len,
                                             const DerivativeMatrixHandle *matrix,
                                             const size_t *qubits, size_t qubits_len);

/* crates/arcqml-runtime-sys/src/lib.rs:68 — idempotent; null handle or null data is a no-op. */
void arcqml_rt_v1_derivative_matrix_destroy(DerivativeMatrixHandle *matrix);

/* crates/arcqml-runtime-sys/src/lib.rs:69-73 — plan from a descriptor array (deep copied). */
int32_t arcqml_rt_v1_circuit_plan_create(const OperationDescriptor *operations,
                                         size_t operations_len, CircuitPlanHandle *output);

/* crates/arcqml-runtime-sys/src/lib.rs:74-77 */
int32_t arcqml_rt_v1_circuit_plan_create_empty(size_t operation_capacity,
                                               CircuitPlanHandle *output);

/* crates/arcqml-runtime-sys/src/lib.rs:78-81 — appends one bound operation. Qubits, parameter
 * bindings, custom matrix and name are deep-copied (callers pass pointers to temporaries). */
int32_t arcqml_rt_v1_circuit_plan_push(CircuitPlanHandle *plan,
                                       const OperationDescriptor *operation);

/* crates/arcqml-runtime-sys/src/lib.rs:82-87 — applies every operation in order. */
int32_t arcqml_rt_v1_circuit_plan_apply(const CircuitPlanHandle *plan, arcqml_c128 *amplitudes,
                                        size_t amplitudes_len, size_t num_qubits);

/* crates/arcqml-runtime-sys/src/lib.rs:88-100 — adjoint reverse sweep.
 * In:  forward_state = psi_m, adjoint_state = H psi_m (unscaled), upstream = g,
 *      gradients zero-filled by the caller, parameter_requires_grad[parent] in {0,1}.
 * Out: forward_state = psi_0, adjoint_state = g * lambda_0,
 *      gradients[parent] += 2 g Re<lambda_k| dU_k/dp |psi_{k-1}> for every bound slot whose
 *      parent requires a gradient (docs/ArcQML技术手册.md:426-454).
 * derivative_state must have state_len elements; this build needs no scratch state and only
 * checks its length. */
int32_t arcqml_rt_v1_adjoint_backward(const CircuitPlanHandle *plan, arcqml_c128 *forward_state,
                                      arcqml_c128 *adjoint_state, size_t state_len,
                                      arcqml_c128 *derivative_state, size_t num_qubits,
                                      double upstream, const uint8_t *parameter_requires_grad,
                                      size_t parameter_requires_grad_len, double *gradients,
                                      size_t gradients_len);

/* crates/arcqml-runtime-sys/src/lib.rs:101 — idempotent; null is a no-op. */
void arcqml_rt_v1_circuit_plan_destroy(CircuitPlanHandle *plan);

/* crates/arcqml-runtime-sys/src/lib.rs:102, :330-336 — returns the length in bytes of the
 * calling thread's last error message and copies min(len, capacity) bytes into buffer. */
size_t arcqml_rt_last_error(uint8_t *buffer, size_t capacity);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* ARCQML_RUNTIME_H */
