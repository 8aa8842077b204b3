// launch.h — host entry points of the kernels in kernels.cu.
#pragma once

#include "rt_internal.h"

namespace arcqml {

// Adjoint step over psi and lambda for one reversed gate with `ns` required slots.
// uadj must be a dense small form (KIND_1Q / KIND_2Q); d[s] holds dU/dp_s on the same targets.
// Writes partials[s * blocks + b]; returns the block count (<= adjoint_max_blocks()).
unsigned launch_adjoint_raw(double2 *psi, double2 *lam, size_t batch, uint32_t n,
                            const DevGate &uadj, const double2 (*d)[16], int ns,
                            double *partials, cudaStream_t s);
unsigned adjoint_max_blocks();
// sums[r] = sum_b partials[r * nblocks + b] in a fixed order.
void launch_reduce_rows(const double *partials, uint32_t rows, uint32_t nblocks, double *sums,
                        cudaStream_t s);
void launch_basis_state(double2 *amps, size_t batch, uint32_t n, uint64_t index, cudaStream_t s);
unsigned launch_norms(const double2 *amps, size_t batch, uint32_t n, double *partials,
                      cudaStream_t s);
// Coset traversal of the observable pass (see k_pauli); tables == nullptr: index order.
struct PauliTraversal {
    const uint64_t *tables = nullptr;  // device, ntables x 256 entries
    uint32_t coset_bits = 0, nb = 0, ntables = 0;
};
// Host-side choice of the coset qubits for an n-qubit state and the given group flip masks;
// fills `tables` (host, ntables x 256) and the counts, or leaves it empty for index order.
void pauli_traversal_tables(uint32_t n, const std::vector<uint64_t> &flips,
                            std::vector<uint64_t> &tables, PauliTraversal &tr);
// Device tables of an observable in one block at `base` (`bytes` long, 16-byte aligned), byte
// offsets of each array: single-term groups (s_*: weight, flip, phase mask per group) and the
// other groups (m_*: weight and phase mask per term, flip per group, first term per group plus
// an end index). Weights are coefficient * i^(y mod 4) * (-1)^popc(flip & phase).
struct PauliTables {
    const unsigned char *base = nullptr;
    uint32_t s_w = 0, s_f = 0, s_z = 0, m_w = 0, m_z = 0, m_f = 0, m_e = 0;
    uint32_t ns = 0, nm = 0;
    size_t bytes = 0;
};
unsigned launch_pauli(const double2 *psi, double2 *out, size_t batch, uint32_t n,
                      const PauliTables &tab, const PauliTraversal &tr, double *partials,
                      bool accumulate, cudaStream_t s);

// Moves the slices of a shard with slice value y != skip (bit i of y at positions[i]) between
// the shard and staging blocks [block][chunk_len], for other-index o in [chunk_begin, +chunk_len).
void launch_slices(double2 *amps, uint32_t n_local, const uint32_t *positions, uint32_t k,
                   uint64_t chunk_begin, uint64_t chunk_len, uint64_t skip, double2 *staging,
                   bool unpack, cudaStream_t s);
constexpr uint32_t kMaxSliceBits = 8;
// Swaps the global qubits at rank bits global_bits[i] with the shard's local positions
// local_positions[i] over an NCCL communicator (shard_nccl.cpp): pack, grouped send/receive with
// each peer, unpack, in chunks that fit staging (2 x (2^k - 1) x chunk amplitudes).
void shard_swap_nccl(double2 *shard, uint32_t n_local, const uint32_t *global_bits,
                     const uint32_t *local_positions, uint32_t k, void *comm, double2 *staging,
                     size_t staging_len, cudaStream_t s);
// amps[index(y, o)] <- sources[y][o - chunk_begin] for every slice value y whose source is
// non-null (sources may be peer mappings of other GPUs' buffers).
void launch_slices_from(double2 *amps, const uint32_t *positions, uint32_t k,
                        uint64_t chunk_begin, uint64_t chunk_len, const double2 *const *sources,
                        cudaStream_t s);

// cum[i] = sequential f64 sum of |amps[j]|^2 for j <= i (no FMA); out[s] = basis index of
// shot s of StdRng::seed_from_u64(seed). cum holds 2^n doubles, out `shots` entries.
void launch_sample(const double2 *amps, uint32_t n, uint64_t shots, uint64_t seed, double *cum,
                   uint64_t *out, cudaStream_t s);

// One op of the one-kernel small-state step: U for the forward sweep, U^dagger (a dense small
// form when slots need gradients) with dU/dp per such slot for the reverse sweep.
struct SmallOp {
    DevGate u;
    DevGate ua;
    int32_t ns;
    int32_t pad;
    double2 d[3][16];
};
constexpr uint32_t kSmallMaxQubits = 10;
// One CTA: psi <- plan |init>, lam <- H psi, out[0] = <H>, then the reverse sweep with
// out[1 + j] = sum Re<lam| dU/dp |psi> for the j-th (op, slot); lam0 (may be null) <- lambda_0.
void launch_small_step(const double2 *init, uint32_t n, const SmallOp *ops, uint32_t nops,
                       const PauliTables &tab, double *out, double2 *lam0, cudaStream_t s);

// A trained op of the device optimizer loop: its one bound slot's parameter is `parent` and its
// dense small form (D = dim) is U(t) = a0 + cos(alpha t) a1 + sin(alpha t) a2 (rotations:
// alpha = 1/2, a0 = 0; phase gates: alpha = 1); dU/dt goes to d[slot_row] of the op.
struct SmallParamOp {
    uint32_t op, parent;
    int32_t slot_row, dim;
    double alpha, pad;
    double2 a0[16], a1[16], a2[16];
};
struct SmallAdam {
    double lr, beta1, beta2, eps, weight_decay;
};
// Dynamic shared memory of the loop: psi, lambda, the op table, theta / m / v / grad per parent.
size_t small_adam_smem(uint32_t n, uint32_t nops, uint32_t nparents);
// `steps` steps of: U, U^dagger and dU/dp of the trained ops from the parameters; forward, <H>,
// reverse sweep (as launch_small_step); grad[parent] = sum 2 x rows (row_parent[j] per row);
// energies[step] = <H>; Adam on the parents in `trained` with bias corrections
// bc[2 step] = 1 - beta1^t, bc[2 step + 1] = 1 - beta2^t. state = theta, m, v per parent
// (nparents each), read at the start and written at the end.
void launch_small_adam(const double2 *init, uint32_t n, const SmallOp *ops, uint32_t nops,
                       const SmallParamOp *pops, uint32_t npops, const uint32_t *row_parent,
                       const uint32_t *trained, uint32_t ntrained, uint32_t nparents,
                       const PauliTables &tab, const SmallAdam &h, const double *bc,
                       uint32_t steps, double *state, double *energies, cudaStream_t s);

Observable *make_observable(size_t num_qubits, const double *coef, const uint64_t *flip,
                            const uint64_t *phase, size_t num_terms);
const std::string &last_error();
void check_bindings(const Plan &plan, size_t req_len, size_t grads_len);
void validate_plan_for_state(const Plan &plan, uint32_t n);

}  // namespace arcqml
