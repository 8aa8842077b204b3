/*
 * oracle.h — CPU f64 restatement of ArcQML's statevector path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the sm_100a runtime: only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may load
 * it. The product library never links or calls it.
 *
 * Parity pin: the restatement is checked against the reference's own known-answer tests
 * (kernel_tests.rs, compiled_hamiltonian_tests.rs, run_tests.rs, row_major_batch_tests.rs,
 * dense_tests.rs, python/tests/test_single.py) and against the end-to-end H2 VQE trajectory
 * printed in docs/tutorial/h2_vqe.md:499-501 (energy after Adam steps 1 and 100, 12 digits).
 * The reference runtime itself is a closed Windows/MSVC static library and cannot run here.
 *
 * Conventions (crates/arcqml-circuit/src/gate.rs:4-10, docs/ArcQML技术手册.md:223-247):
 * basis index bit q <-> qubit q; gate local index bit j <-> qubits[j]; controls first;
 * matrices row-major m[row * dim + col].
 */
#ifndef ARCQML_ORACLE_H
#define ARCQML_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct oc128 {
    double re;
    double im;
} oc128;

/* One bound plan operation, the oracle's copy of OperationDescriptor
 * (crates/arcqml-runtime-abi/src/lib.rs:88-96). */
typedef struct oracle_op {
    uint32_t opcode;
    uint32_t arity;
    double params[3];
    const oc128 *matrix; /* custom unitary, 4^arity entries, or NULL */
    const size_t *qubits;
    uint32_t num_bindings;
    size_t slots[3];
    size_t parents[3];
} oracle_op;

/* One compiled Pauli term (crates/arcqml-observable/src/compiled_hamiltonian.rs:20-26). */
typedef struct oracle_term {
    double coefficient;
    uint64_t flip_mask;
    uint64_t phase_mask;
    uint32_t y_count_mod_four;
} oracle_term;

/* Number of qubits the oracle accepts in a dense gate matrix. */
#define ORACLE_MAX_DENSE_ARITY 10

int oracle_gate_matrix(uint32_t opcode, uint32_t arity, const double *params,
                       const oc128 *custom, oc128 *out);
int oracle_derivative_matrix(uint32_t opcode, uint32_t arity, const double *params,
                             size_t slot, oc128 *out);
void oracle_apply_dense(oc128 *amps, uint32_t num_qubits, const oc128 *m, uint32_t k,
                        const size_t *qubits);
int oracle_apply_gate(oc128 *amps, uint32_t num_qubits, const oracle_op *op, int adjoint);
int oracle_parameter_derivative(const oc128 *in, oc128 *out, uint32_t num_qubits,
                                const oracle_op *op, size_t slot);
int oracle_plan_apply(const oracle_op *ops, size_t num_ops, oc128 *amps, uint32_t num_qubits);
int oracle_adjoint_backward(const oracle_op *ops, size_t num_ops, oc128 *psi, oc128 *lambda,
                            uint32_t num_qubits, double upstream, const uint8_t *req,
                            size_t req_len, double *grads, size_t grads_len);

void oracle_hamiltonian_diagonal(const oracle_term *terms, size_t num_terms,
                                 uint32_t num_qubits, double *diagonal);
double oracle_expectation(const oracle_term *terms, size_t num_terms, const oc128 *amps,
                          uint32_t num_qubits);
void oracle_apply_hamiltonian(const oracle_term *terms, size_t num_terms, const oc128 *amps,
                              oc128 *out, uint32_t num_qubits);
double oracle_expectation_and_apply(const oracle_term *terms, size_t num_terms,
                                    const oc128 *amps, oc128 *out, uint32_t num_qubits);

/* Batch forms: rows of [batch, 2^n], one independent state per row (OpenMP over rows). */
int oracle_batch_plan_apply(const oracle_op *ops, size_t num_ops, oc128 *amps, size_t batch,
                            uint32_t num_qubits);
int oracle_batch_adjoint_backward(const oracle_op *ops, size_t num_ops, oc128 *psi,
                                  oc128 *lambda, size_t batch, uint32_t num_qubits,
                                  const double *upstream, const uint8_t *req, size_t req_len,
                                  double *grads, size_t grads_len);

/* Threads used by the OpenMP loops (1 when built without OpenMP). */
/* Sampling (crates/arcqml-sim/src/statevector/api/measurement.rs:18-60): shot s's basis index
 * in out[s]. The ChaCha block and the StdRng key/stream helpers are exported for tests. */
int oracle_sample_indices(const oc128 *amps, uint32_t num_qubits, uint64_t shots, uint64_t seed,
                          uint64_t *out);
void oracle_chacha_block(const uint32_t key[8], uint64_t counter, uint64_t stream, int rounds,
                         uint32_t out[16]);
void oracle_stdrng_key(uint64_t seed, uint32_t key[8]);
uint64_t oracle_stdrng_u64(uint64_t seed, uint64_t k);
int oracle_num_threads(void);
void oracle_set_num_threads(int n);

/* Analysis of a state (crates/arcqml-analysis/src/statevector): probabilities (2^n), marginal
 * probabilities of a qubit selection (2^k, selected qubits in descending order from the most
 * significant output bit; non-zero return for an empty, out-of-range or duplicate selection),
 * the Bloch vector of one qubit, and <lhs|rhs> with the fidelity |<lhs|rhs>|^2. */
void oracle_probabilities(const oc128 *amps, uint32_t num_qubits, double *out);
int oracle_marginal_probabilities(const oc128 *amps, uint32_t num_qubits, const uint32_t *qubits,
                                  size_t num_selected, double *out);
int oracle_bloch_vector(const oc128 *amps, uint32_t num_qubits, uint32_t qubit, double xyz[3]);
void oracle_overlap_fidelity(const oc128 *lhs, const oc128 *rhs, uint32_t num_qubits,
                             double out[3]);

#ifdef __cplusplus
}
#endif

#endif
