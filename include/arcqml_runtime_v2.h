/*
 * arcqml_runtime_v2.h — device-resident extension of the ArcQML runtime C ABI (B200 build).
 *
 * The v1 entry points (arcqml_runtime.h) take host buffers and copy them to the GPU on every
 * call, as the reference's callers hand over host `Vec<Complex64>` states. These additive
 * `arcqml_rt_v2_*` entry points keep states in HBM across calls: amplitude pointers are
 * DEVICE pointers on the calling thread's current CUDA device, laid out [batch, 2^n]
 * row-major complex128, and `stream` is a cudaStream_t (NULL selects CUDA's legacy default
 * stream). Small results (values, gradients, norms) are written to HOST arrays; calls that
 * return them synchronize the stream before returning.
 *
 * Each entry point restates a step of the reference's `run` / backward path on device:
 *   plan apply           crates/arcqml-runtime-sys/src/lib.rs:82-87 (circuit_plan_apply)
 *   observable           crates/arcqml-observable/src/compiled_hamiltonian.rs:30-182
 *   adjoint backward     crates/arcqml-runtime-sys/src/lib.rs:88-100 (adjoint_backward),
 *                        batch rows as crates/arcqml-sim/src/statevector/execution/adjoint/
 *                        row_major.rs:108-162 (per-row upstream, gradients summed over rows)
 * Status and errors follow the v1 convention (0 = success, message via arcqml_rt_last_error).
 */
#ifndef ARCQML_RUNTIME_V2_H
#define ARCQML_RUNTIME_V2_H

#include "arcqml_runtime.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Compiled sparse Pauli observable (CompiledHamiltonian, compiled_hamiltonian.rs:13-26). */
typedef struct ArcqmlObservableHandle {
    void *opaque;
} ArcqmlObservableHandle;

/* Term k is coefficients[k] * i^{popcount(flip & phase) mod 4} * X^{flip} Z^{phase} applied as
 * P|i> = i^y (-1)^{popcount(i & phase_masks[k])} |i ^ flip_masks[k]> (flip = X|Y bits,
 * phase = Y|Z bits, compiled_hamiltonian.rs:37-62, :198-210). */
int32_t arcqml_rt_v2_observable_create(size_t num_qubits, const double *coefficients,
                                       const uint64_t *flip_masks, const uint64_t *phase_masks,
                                       size_t num_terms, ArcqmlObservableHandle *output);
void arcqml_rt_v2_observable_destroy(ArcqmlObservableHandle *observable);

/* amplitudes[b] <- U_m ... U_1 amplitudes[b] for every row b. */
int32_t arcqml_rt_v2_plan_apply(const CircuitPlanHandle *plan, arcqml_c128 *amplitudes,
                                size_t batch, size_t num_qubits, void *stream);

/* One gate (adjoint != 0 applies U^dagger) on every row. */
int32_t arcqml_rt_v2_apply_gate(arcqml_c128 *amplitudes, size_t batch, size_t num_qubits,
                                const GateDescriptor *gate, const size_t *qubits,
                                size_t qubits_len, int32_t adjoint, void *stream);

/* output[b] <- (dU/dp_slot) input[b] (control-0 block of controlled gates is zero). */
int32_t arcqml_rt_v2_parameter_derivative(const arcqml_c128 *input, arcqml_c128 *output,
                                          size_t batch, size_t num_qubits,
                                          const GateDescriptor *gate, const size_t *qubits,
                                          size_t qubits_len, size_t parameter_slot,
                                          void *stream);

/* *passes <- how many passes over 12-qubit tiles the observable takes on a state of num_qubits
 * qubits (states of 20 qubits and more, when every flip mask fits a tile); 0 when the gather
 * kernel evaluates it instead. Host only. No counterpart in the reference (its CompiledHamiltonian
 * is one CPU loop, crates/arcqml-observable/src/compiled_hamiltonian.rs:81-132). */
int32_t arcqml_rt_v2_observable_tile_passes(const ArcqmlObservableHandle *observable,
                                            size_t num_qubits, uint32_t *passes);

/* values[b] <- Re<psi_b|H|psi_b> (host array of batch doubles). */
int32_t arcqml_rt_v2_expectation(const ArcqmlObservableHandle *observable,
                                 const arcqml_c128 *amplitudes, size_t batch, size_t num_qubits,
                                 double *values, void *stream);

/* output[b] <- H psi_b and values[b] <- Re<psi_b|H psi_b> in one pass. */
int32_t arcqml_rt_v2_expectation_and_apply(const ArcqmlObservableHandle *observable,
                                           const arcqml_c128 *amplitudes, arcqml_c128 *output,
                                           size_t batch, size_t num_qubits, double *values,
                                           void *stream);

/* Reverse sweep over device states. In: psi = psi_m, lambda = H psi_m (unscaled) per row,
 * upstream[b] = g_b (host array). Out: psi = psi_0, lambda = g_b lambda_0, and
 * gradients[parent] += sum_b 2 g_b Re<lambda_k| dU_k/dp |psi_{k-1}> over every bound slot whose
 * parent has parameter_requires_grad[parent] != 0. No scratch state is needed. */
int32_t arcqml_rt_v2_adjoint_backward(const CircuitPlanHandle *plan, arcqml_c128 *forward_state,
                                      arcqml_c128 *adjoint_state, size_t batch,
                                      size_t num_qubits, const double *upstream,
                                      const uint8_t *parameter_requires_grad,
                                      size_t parameter_requires_grad_len, double *gradients,
                                      size_t gradients_len, void *stream);

/* Same as arcqml_rt_v2_expectation_and_apply but ADDS H psi to `output` (output += H psi) and
 * returns this call's <psi|H|psi> in values. Lets a caller sum H psi over several observables
 * that share one output buffer; a sharded state evaluates its terms in groups, one group per
 * qubit layout (no reference counterpart: the reference's observables run in one piece,
 * compiled_hamiltonian.rs:104-182). */
int32_t arcqml_rt_v2_expectation_and_accumulate(const ArcqmlObservableHandle *observable,
                                                const arcqml_c128 *amplitudes, arcqml_c128 *output,
                                                size_t batch, size_t num_qubits, double *values,
                                                void *stream);

/* Global-qubit swap support for one state sharded over ranks on its highest qubits (no
 * reference counterpart: the reference runs one process). The local index of a shard of
 * num_local_qubits qubits splits into the slice bits at positions[0..num_positions) (bit i of a
 * slice value y sits at positions[i]) and the other bits o, in ascending order. For every slice
 * value y != skip_value and o in [chunk_begin, chunk_begin + chunk_len):
 *   unpack == 0: staging[block(y) * chunk_len + o - chunk_begin] <- amplitudes[index(y, o)]
 *   unpack != 0: amplitudes[index(y, o)] <- staging[block(y) * chunk_len + o - chunk_begin]
 * where block(y) numbers the slice values in increasing order without skip_value (pass 2^k or
 * more to keep every value). At most 8 positions; o must stay below 2^(num_local_qubits - k). */
int32_t arcqml_rt_v2_shard_slices(arcqml_c128 *amplitudes, size_t num_local_qubits,
                                  const uint32_t *positions, size_t num_positions,
                                  uint64_t chunk_begin, uint64_t chunk_len, uint64_t skip_value,
                                  arcqml_c128 *staging, int32_t unpack, void *stream);

/* Shot sampling from one device state, bit-exact with the reference's sample_counts
 * (crates/arcqml-sim/src/statevector/api/measurement.rs:18-60): p_i = re^2 + im^2 (no fused
 * multiply-add), a sequential f64 running sum, and per shot target = u * total with u the next
 * f64 of StdRng::seed_from_u64(seed) (ChaCha12); indices[s] (host array of `shots` entries)
 * receives the first basis index whose running sum exceeds target (the last index if none).
 * norm_sqr (optional) receives the total. Fails, as the reference does, for shots == 0 and
 * when |total - 1| > 1e-10 (state.rs:108-114). Uses 8 * 2^n bytes of device scratch; the running
 * sum is one dependency chain (about 2-4 ns per amplitude). */
int32_t arcqml_rt_v2_sample(const arcqml_c128 *amplitudes, size_t num_qubits, uint64_t shots,
                            uint64_t seed, uint64_t *indices, double *norm_sqr, void *stream);

/* Global-qubit swap of a sharded state over the caller's NCCL communicator (nccl_comm is an
 * ncclComm_t whose ranks each hold one shard: rank r the 2^num_local_qubits amplitudes whose top
 * log2(size) index bits equal r). Exchanges, for every i < num_pairs, the qubit at rank bit
 * global_bits[i] with the qubit at the shard's position local_positions[i]: each rank sends the
 * slices whose local bits differ from its own rank bits to the rank holding them and receives
 * the matching slices in their place (the all-to-all among the 2^num_pairs ranks that differ in
 * those rank bits). staging (device) must hold 2 x (2^num_pairs - 1) x chunk amplitudes for some
 * chunk >= 1; larger buffers move larger chunks. Every rank of the communicator calls it with
 * the same pairs. Runs on `stream`; the NCCL library is the one loaded in the process. No
 * counterpart in the reference: this is the data movement under the sharded 32- and 35-qubit
 * configurations, for callers (an arcqml-sim with device-resident shards) that own the
 * communicator and the layout. */
int32_t arcqml_rt_v2_shard_swap_nccl(arcqml_c128 *shard, size_t num_local_qubits,
                                     const uint32_t *global_bits, const uint32_t *local_positions,
                                     size_t num_pairs, void *nccl_comm, arcqml_c128 *staging,
                                     size_t staging_len, void *stream);

/* Same slice layout as arcqml_rt_v2_shard_slices, gathering into the shard: for every slice
 * value y with sources[y] != NULL (sources has 2^num_positions entries) and o in
 * [chunk_begin, chunk_begin + chunk_len): amplitudes[index(y, o)] <- sources[y][o - chunk_begin].
 * A source may be another GPU's buffer mapped with arcqml_rt_v2_peer_buffer_open: the swap of a
 * sharded state then reads each peer's packed slices over NVLink with plain loads. */
int32_t arcqml_rt_v2_shard_slices_from(arcqml_c128 *amplitudes, size_t num_local_qubits,
                                       const uint32_t *positions, size_t num_positions,
                                       uint64_t chunk_begin, uint64_t chunk_len,
                                       const arcqml_c128 *const *sources, void *stream);

/* Device buffers shared between the processes of one node (CUDA IPC; no reference counterpart).
 * create: cudaMalloc of `bytes` on the current device, its 64-byte IPC handle in handle[64];
 * open: maps another process's buffer from its handle (peer access enabled on demand); close
 * unmaps an opened buffer; destroy frees a created one. */
int32_t arcqml_rt_v2_peer_buffer_create(size_t bytes, void **device_ptr, uint8_t *handle);
int32_t arcqml_rt_v2_peer_buffer_open(const uint8_t *handle, void **device_ptr);
int32_t arcqml_rt_v2_peer_buffer_close(void *device_ptr);
int32_t arcqml_rt_v2_peer_buffer_destroy(void *device_ptr);

/* One-kernel run + backward for a small single state (num_qubits <= 10; no reference
 * counterpart: it fuses plan apply, expectation_and_apply and adjoint_backward with upstream 1
 * into one launch and one read-back). psi = plan |initial_state> (device, or NULL for |0...0>),
 * *value = <psi|H|psi>, gradients[parent] += 2 Re<lambda| dU/dp |psi> over the reverse sweep with
 * lambda = H psi (as arcqml_rt_v2_adjoint_backward with upstream 1; scale by an upstream factor
 * afterwards, the sweep is linear in it), and lambda0 (device, may be NULL) <- lambda at the
 * start of the circuit (the initial state's gradient is 2 * upstream * lambda0). Custom gates
 * must act on at most 4 qubits. */
int32_t arcqml_rt_v2_small_run(const CircuitPlanHandle *plan,
                               const ArcqmlObservableHandle *observable,
                               const arcqml_c128 *initial_state, size_t num_qubits,
                               const uint8_t *parameter_requires_grad,
                               size_t parameter_requires_grad_len, double *gradients,
                               size_t gradients_len, double *value, arcqml_c128 *lambda0,
                               void *stream);

/* Device optimizer loop for a small single state (num_qubits <= 10; no reference counterpart:
 * it runs `steps` iterations of the loop a caller writes around arcqml_rt_v2_small_run — run,
 * backward with upstream 1, then the f64 Adam step of crates/arcqml-optim/src/adam.rs:190-240 —
 * in one launch). parameters[num_parameters] is indexed by parent (as the requires-grad list;
 * entry 0 is the initial-state slot and is never updated): read as the starting values, written
 * with the values after the last step. Parameters with parameter_requires_grad[p] != 0 (p >= 1)
 * are trained; every op with such a parameter must be a one-parameter rotation (RX, RY, RZ,
 * CRX, CRY, CRZ, RXX, RYY, RZZ, RZX) or phase gate (PHASE, CPHASE). energies[i] = <H> before
 * update i (host, `steps` entries). adam_m / adam_v (host, num_parameters each, may be NULL for
 * zero moments and then not written) carry the moments of an optimizer that has taken
 * steps_taken steps (bias corrections use t = steps_taken + i + 1). initial_state: device, or
 * NULL for |0...0>. The op table, state and parameters must fit in one CTA's shared memory
 * (an error names the sizes). */
int32_t arcqml_rt_v2_small_adam(const CircuitPlanHandle *plan,
                                const ArcqmlObservableHandle *observable,
                                const arcqml_c128 *initial_state, size_t num_qubits,
                                const uint8_t *parameter_requires_grad, double *parameters,
                                size_t num_parameters, double *adam_m, double *adam_v,
                                uint64_t steps_taken, size_t steps, double learning_rate,
                                double beta1, double beta2, double epsilon, double weight_decay,
                                double *energies, void *stream);

/* State analysis (crates/arcqml-analysis/src/statevector), on every row of a device state.
 * probabilities: probabilities[row][i] = |psi_row[i]|^2 (device, [batch, 2^n];
 *   probabilities.rs:22-25).
 * marginal_probabilities: marginals[row][m] = summed probabilities over the basis indices whose
 *   selected qubits read m, the selected qubits taken in descending order with the highest as
 *   the most significant bit of m (device, [batch, 2^num_selected]; marginal.rs:17-67). An empty
 *   selection, a qubit >= num_qubits or a repeated qubit fails with the reference's message.
 * bloch_vector: xyz[3 row + 0..2] = <X_q>, <Y_q>, <Z_q> (host, 3 per row; bloch.rs:23-56).
 * overlap: overlaps[2 row], [2 row + 1] = real and imaginary part of <lhs_row|rhs_row> (host,
 *   2 per row); the fidelity of fidelity.rs:14-30 is its squared modulus.
 * Reductions are deterministic (fixed summation order on the device). */
int32_t arcqml_rt_v2_probabilities(const arcqml_c128 *amplitudes, size_t batch,
                                   size_t num_qubits, double *probabilities, void *stream);
int32_t arcqml_rt_v2_marginal_probabilities(const arcqml_c128 *amplitudes, size_t batch,
                                            size_t num_qubits, const size_t *qubits,
                                            size_t num_selected, double *marginals,
                                            void *stream);
int32_t arcqml_rt_v2_bloch_vector(const arcqml_c128 *amplitudes, size_t batch, size_t num_qubits,
                                  size_t qubit, double *xyz, void *stream);
int32_t arcqml_rt_v2_overlap(const arcqml_c128 *lhs, const arcqml_c128 *rhs, size_t batch,
                             size_t num_qubits, double *overlaps, void *stream);

/* Cotangents for arcqml_rt_v2_adjoint_backward (its lambda; gradients += 2 Re<lambda|dU|psi>)
 * of the analysis outputs, so that losses built on them train through the reverse sweep as the
 * reference's autograd does (statevector_analysis.rs:109-181).
 * probability_cotangent: cotangent[row][i] = upstream[row][bin(i)] psi_row[i] for upstream
 *   gradients of marginal probabilities (device, [batch, 2^num_selected]); qubits = NULL with
 *   num_selected = 0 means the full probability vector (bin(i) = i).
 * scaled_copy: output[row] = factor[row] input[row] with a complex factor (host, re and im per
 *   row): lambda = <a|psi> a for the fidelity |<a|psi>|^2, lambda = upstream / 2 for a complex
 *   upstream gradient of the amplitudes. */
int32_t arcqml_rt_v2_probability_cotangent(const arcqml_c128 *amplitudes, size_t batch,
                                           size_t num_qubits, const size_t *qubits,
                                           size_t num_selected, const double *upstream,
                                           arcqml_c128 *cotangent, void *stream);
int32_t arcqml_rt_v2_scaled_copy(const arcqml_c128 *input, size_t batch, size_t num_qubits,
                                 const double *factors, arcqml_c128 *output, void *stream);

/* norms[b] <- sum_i |psi_b[i]|^2 (host array). */
int32_t arcqml_rt_v2_norms(const arcqml_c128 *amplitudes, size_t batch, size_t num_qubits,
                           double *norms, void *stream);

/* Same result as arcqml_rt_v2_norms, for callers that cannot allocate device memory while they
 * run (their memory is all handed to their own pool, or an allocation would synchronise the
 * device at a point they cannot afford). No counterpart in the reference. It allocates nothing:
 * its scratch is a static 192 KiB device array that every GPU loading the library keeps until
 * exit. At most 8192 rows per call (larger batches are rejected with an error). The first call
 * on a device looks up the array's device address (cudaGetSymbolAddress) with that device
 * current; make that first call before any stream capture. That first call may also load the
 * library's kernels onto the device (lazy module loading), which can allocate: a caller that
 * needs every later call to allocate nothing makes one call ahead of time. Every call waits for
 * its stream (the norms are copied to the host array before it returns). The address is kept
 * for the life of the process: cudaDeviceReset is not supported between calls. All calls share
 * the array: calls that overlap on the GPU race. */
int32_t arcqml_rt_v2_norms_noalloc(const arcqml_c128 *amplitudes, size_t batch,
                                   size_t num_qubits, double *norms, void *stream);

/* Every row <- |index>. */
int32_t arcqml_rt_v2_set_basis_state(arcqml_c128 *amplitudes, size_t batch, size_t num_qubits,
                                     uint64_t index, void *stream);

/* Replaces the bound value of every (slot, parent) binding of the plan with
 * parent_values[parent]; the plan's structure is unchanged. Lets a training loop update
 * parameters without rebuilding the plan. */
int32_t arcqml_rt_v2_plan_set_parameters(CircuitPlanHandle *plan, const double *parent_values,
                                         size_t parent_values_len);

/* Number of operations in the plan. */
size_t arcqml_rt_v2_plan_len(const CircuitPlanHandle *plan);

/* Fused-pass schedule of the plan for an n-qubit state (host only; no reference counterpart).
 * adjoint != 0 plans the reverse sweep with every bound slot required. Writes the number of
 * HBM passes, register sub-blocks and fused gates; states below the fused-path size report
 * one pass per gate. */
int32_t arcqml_rt_v2_plan_schedule_stats(const CircuitPlanHandle *plan, size_t num_qubits,
                                         int32_t adjoint, uint64_t *passes, uint64_t *sub_blocks,
                                         uint64_t *gates);

/* Generates the run-time kernels of the plan's fused passes for an n-qubit state (forward, or
 * the adjoint sweep when adjoint != 0) and compiles them with NVRTC without loading them: needs
 * no GPU. compiled / eligible receive the passes that compiled and the passes that have a
 * compiled form; message the first compile error. Diagnostic and test support. */
int32_t arcqml_rt_v2_plan_jit_check(const CircuitPlanHandle *plan, size_t num_qubits,
                                    int32_t adjoint, uint64_t *compiled, uint64_t *eligible,
                                    char *message, size_t capacity);
/* The fused-pass schedule the engine builds for the plan (diagnostic and test support; no
 * reference counterpart, no CUDA call), serialised into buffer when capacity allows; *size
 * receives the byte count (call with buffer NULL to size it). Little-endian: u32 steps; per step
 * u32 is_pass, then for a custom gate u32 op index, else the PassHeader, u32 count + SubBlocks,
 * u32 count + FOps, u32 count + matrix entries (two doubles each), u32 count + u64 gradient
 * parents (one per accumulator), u32 count + (u64 accumulator, u64 parent) pairs (further
 * parents that receive an accumulator's gradient: rotations merged in the adjoint sweep),
 * u32 length + the `struct PassOps` source of the pass's run-time compiled kernel (empty
 * without one). The layouts are those of arcqml_b200/csrc/fused.h. */
int32_t arcqml_rt_v2_plan_schedule_export(const CircuitPlanHandle *plan, size_t num_qubits,
                                          int32_t adjoint, const uint8_t *parameter_requires_grad,
                                          size_t parameter_requires_grad_len, uint8_t *buffer,
                                          size_t capacity, size_t *size);

/* Runs the fused-pass schedule the engine builds for the plan on a host state, on the CPU
 * (diagnostic and test support; no reference counterpart, no CUDA call): the same passes, tile
 * mapping, encoded ops, scaled forms and gradient factors as the device kernels, so the
 * planner can be checked against a CPU reference without a GPU. adjoint == 0: state <- plan
 * state. adjoint != 0: the reverse sweep over state (psi) and lambda (already scaled by the
 * upstream factor), gradients[parent] += 2 Re<lambda| dU |psi> per required slot. 8 to 22
 * qubits. */
int32_t arcqml_rt_v2_plan_emulate(const CircuitPlanHandle *plan, arcqml_c128 *state,
                                  size_t num_qubits, int32_t adjoint, arcqml_c128 *lambda,
                                  const uint8_t *parameter_requires_grad,
                                  size_t parameter_requires_grad_len, double *gradients,
                                  size_t gradients_len);

/* Run-time compiled pass kernels (no reference counterpart). Fused passes whose gates all have
 * fast paths run as kernels compiled for the circuit's structure (NVRTC, sm_100a) and cached per
 * device; ARCQML_JIT=0 in the environment keeps every pass on the precompiled kernel. Reports the
 * kernels compiled, the launches of compiled kernels and the passes that fell back to the
 * precompiled kernel since the library was loaded, and copies the last compile or load error
 * (NUL-terminated, at most capacity - 1 bytes); returns that message's length. */
size_t arcqml_rt_v2_jit_info(uint64_t *kernels_compiled, uint64_t *launches, uint64_t *fallbacks,
                             char *last_error, size_t capacity);

/* Kernel timing (no reference counterpart; measurement support). While enabled, every kernel
 * launch of the runtime in these categories is bracketed by CUDA events on its own stream:
 * 0 per-gate kernels, 1 fused forward passes, 2 fused adjoint passes, 3 per-gate adjoint steps,
 * 4 observable passes, 5 other (scaling, norms, basis states), 6 shard slice packing for
 * global-qubit swaps. Enabling (or disabling) resets
 * the totals. */
void arcqml_rt_v2_profile_enable(int32_t on);
/* Totals of one category since the last enable: launches, summed device time (ms) and summed
 * algorithmic HBM bytes (each touched amplitude read and written once). Waits for pending
 * events. Returns non-zero for an unknown category. */
int32_t arcqml_rt_v2_profile_read(uint32_t category, uint64_t *launches, double *total_ms,
                                  double *algorithmic_bytes);
/* Kernel launches issued by the runtime since the library was loaded (all categories). */
uint64_t arcqml_rt_v2_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* ARCQML_RUNTIME_V2_H */
