// abi.cpp — the exported C ABI: the 14 v1 symbols of arcqml-runtime-sys
// (crates/arcqml-runtime-sys/src/lib.rs:28-103) and the device-resident v2 extension.
//
// Every entry point converts C++ failures into a non-zero status plus a thread-local
// message; nothing throws or aborts across the boundary.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <sstream>

#include "../../include/arcqml_runtime.h"
#include "../../include/arcqml_runtime_v2.h"
#include "analysis.h"
#include "jit.h"
#include "launch.h"
#include "planner.h"
#include "profile.h"
#include "rt_internal.h"

using namespace arcqml;

namespace {

template <class F>
int32_t guarded(F &&f) {
    try {
        f();
        return 0;
    } catch (const Error &e) {
        set_last_error(e.msg);
        return 1;
    } catch (const std::bad_alloc &) {
        set_last_error("out of host memory");
        return 2;
    } catch (const std::exception &e) {
        set_last_error(std::string("runtime failure: ") + e.what());
        return 3;
    } catch (...) {
        set_last_error("runtime failure");
        return 3;
    }
}

// 2^num_qubits with the reference's overflow and length errors
// (crates/arcqml-kernel/src/statevector/single.rs:137-148).
size_t state_dimension(size_t num_qubits) {
    if (num_qubits >= kMaxQubits) {
        std::ostringstream s;
        s << "state dimension overflow for " << num_qubits << " qubits";
        fail(s.str());
    }
    return size_t(1) << num_qubits;
}

void check_state_length(size_t len, size_t num_qubits) {
    const size_t expected = state_dimension(num_qubits);
    if (len != expected) {
        std::ostringstream s;
        s << "state length mismatch for " << num_qubits << " qubits: expected " << expected
          << ", got " << len;
        fail(s.str());
    }
}

uint32_t qubits_of_length(size_t len) {
    if (len == 0 || (len & (len - 1)) != 0) {
        std::ostringstream s;
        s << "state length " << len << " is not a power of two";
        fail(s.str());
    }
    uint32_t n = 0;
    while ((size_t(1) << n) < len) ++n;
    if (n >= kMaxQubits) fail("state dimension overflow");
    return n;
}

Plan *plan_of(const CircuitPlanHandle *h) {
    if (!h || !h->opaque) fail("circuit plan handle is null");
    return static_cast<Plan *>(h->opaque);
}

Observable *obs_of(const ArcqmlObservableHandle *h) {
    if (!h || !h->opaque) fail("observable handle is null");
    return static_cast<Observable *>(h->opaque);
}

// v2 calls run on the caller's stream; NULL is CUDA's legacy default stream, so work queued
// by other libraries on it (e.g. torch's default stream) stays ordered with ours.
cudaStream_t pick_stream(ThreadContext &, void *stream) { return static_cast<cudaStream_t>(stream); }

// Host state -> device buffer `which` of this thread's context.
double2 *upload_state(ThreadContext &ctx, int which, const arcqml_c128 *host, size_t len) {
    if (!host) fail("amplitude buffer is null");
    auto *d = static_cast<double2 *>(ctx_buffer(ctx, which, len * sizeof(double2)));
    check_cuda(cudaMemcpyAsync(d, host, len * sizeof(double2), cudaMemcpyHostToDevice, ctx.stream),
               "cudaMemcpyAsync (host to device)");
    return d;
}

void download_state(ThreadContext &ctx, const double2 *dev, arcqml_c128 *host, size_t len) {
    check_cuda(cudaMemcpyAsync(host, dev, len * sizeof(double2), cudaMemcpyDeviceToHost, ctx.stream),
               "cudaMemcpyAsync (device to host)");
}

void sync(cudaStream_t s) { check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize"); }

OpRecord push_record(const OperationDescriptor *op) {
    if (!op) fail("operation descriptor is null");
    OpRecord r = record_from_descriptor(&op->gate, op->qubits, op->qubits_len, -1);
    if (op->parameters_len > 3)
        fail("a gate has more parameter slots than the runtime ABI supports");
    if (op->parameters_len && !op->parameters) fail("parameter binding list is null");
    r.num_bindings = uint32_t(op->parameters_len);
    for (size_t b = 0; b < op->parameters_len; ++b) {
        const size_t slot = op->parameters[b].parameter_slot;
        if (slot >= slot_count(r.opcode)) {
            std::ostringstream s;
            s << "gate " << r.name << " does not have parameter slot " << slot;
            fail(s.str());
        }
        r.slots[b] = slot;
        r.parents[b] = op->parameters[b].parent_index;
    }
    return r;
}

// Applies one host-described gate to device amplitudes.
void apply_gate_device(double2 *d, size_t batch, uint32_t n, const OpRecord &rec, bool adjoint,
                       ThreadContext &ctx, cudaStream_t s) {
    DevGate g = lower(rec, adjoint ? LOWER_ADJOINT : LOWER_FORWARD, 0);
    if (g.kind == KIND_DENSE) {
        std::vector<double2> m = rec.custom;
        if (adjoint) {
            const size_t dim = size_t(1) << rec.qubits.size();
            for (size_t i = 0; i < dim; ++i)
                for (size_t j = 0; j < dim; ++j)
                    m[j * dim + i] = make_double2(rec.custom[i * dim + j].x, -rec.custom[i * dim + j].y);
        }
        std::vector<const std::vector<double2> *> refs{&m};
        g.dense = upload_tables(refs, ctx, s)[0];
        launch_gate(d, batch, n, g, s);
        sync(s);  // the table lives in host memory owned by this frame
        return;
    }
    launch_gate(d, batch, n, g, s);
}

void check_slot(const OpRecord &rec, size_t slot) {
    if (slot >= slot_count(rec.opcode)) {
        std::ostringstream s;
        s << "gate " << rec.name << " does not have parameter slot " << slot;
        fail(s.str());
    }
}

}  // namespace

// The library is built with -fvisibility=hidden; only the C ABI below is exported.
#pragma GCC visibility push(default)
extern "C" {

// ============================================================================ v1

uint32_t arcqml_rt_abi_version(void) { return ARCQML_RT_ABI_VERSION; }

static int32_t apply_gate_v1(arcqml_c128 *amplitudes, size_t len, size_t num_qubits,
                             const GateDescriptor *gate, const size_t *qubits, size_t qlen,
                             bool adjoint) {
    return guarded([&] {
        check_state_length(len, num_qubits);
        OpRecord rec = record_from_descriptor(gate, qubits, qlen, int64_t(num_qubits));
        ThreadContext &ctx = thread_context();
        double2 *d = upload_state(ctx, 0, amplitudes, len);
        apply_gate_device(d, 1, uint32_t(num_qubits), rec, adjoint, ctx, ctx.stream);
        download_state(ctx, d, amplitudes, len);
        sync(ctx.stream);
    });
}

int32_t arcqml_rt_v1_apply_gate(arcqml_c128 *amplitudes, size_t amplitudes_len, size_t num_qubits,
                                const GateDescriptor *gate, const size_t *qubits,
                                size_t qubits_len) {
    return apply_gate_v1(amplitudes, amplitudes_len, num_qubits, gate, qubits, qubits_len, false);
}

int32_t arcqml_rt_v1_apply_adjoint_gate(arcqml_c128 *amplitudes, size_t amplitudes_len,
                                        size_t num_qubits, const GateDescriptor *gate,
                                        const size_t *qubits, size_t qubits_len) {
    return apply_gate_v1(amplitudes, amplitudes_len, num_qubits, gate, qubits, qubits_len, true);
}

int32_t arcqml_rt_v1_parameter_derivative_into(const arcqml_c128 *input, size_t input_len,
                                               arcqml_c128 *output, size_t output_len,
                                               const GateDescriptor *gate, const size_t *qubits,
                                               size_t qubits_len, size_t parameter_slot) {
    return guarded([&] {
        const uint32_t n = qubits_of_length(input_len);
        if (output_len != input_len) {
            std::ostringstream s;
            s << "state length mismatch for " << n << " qubits: expected " << input_len
              << ", got " << output_len;
            fail(s.str());
        }
        if (!output) fail("output buffer is null");
        OpRecord rec = record_from_descriptor(gate, qubits, qubits_len, int64_t(n));
        check_slot(rec, parameter_slot);
        ThreadContext &ctx = thread_context();
        double2 *din = upload_state(ctx, 0, input, input_len);
        auto *dout = static_cast<double2 *>(ctx_buffer(ctx, 1, input_len * sizeof(double2)));
        DevGate g = lower(rec, LOWER_DERIVATIVE, uint32_t(parameter_slot));
        launch_gate_out(din, dout, 1, n, g, ctx.stream);
        download_state(ctx, dout, output, output_len);
        sync(ctx.stream);
    });
}

int32_t arcqml_rt_v1_derivative_matrix_create(const GateDescriptor *gate, size_t parameter_slot,
                                              DerivativeMatrixHandle *output) {
    return guarded([&] {
        if (!output) fail("derivative matrix handle is null");
        if (!gate) fail("gate descriptor is null");
        // Validate against a canonical qubit list 0..arity-1 (the matrix is position-free).
        std::vector<size_t> q(gate->arity);
        for (size_t i = 0; i < q.size(); ++i) q[i] = i;
        OpRecord rec = record_from_descriptor(gate, q.data(), q.size(), -1);
        check_slot(rec, parameter_slot);
        std::vector<double2> m = dense_matrix(rec, true, uint32_t(parameter_slot));
        auto *data = new arcqml_c128[m.size()];
        for (size_t i = 0; i < m.size(); ++i) data[i] = arcqml_c128{m[i].x, m[i].y};
        output->data = data;
        output->len = m.size();
        output->capacity = m.size();
    });
}

int32_t arcqml_rt_v1_derivative_matrix_apply(arcqml_c128 *amplitudes, size_t amplitudes_len,
                                             const DerivativeMatrixHandle *matrix,
                                             const size_t *qubits, size_t qubits_len) {
    return guarded([&] {
        if (!matrix || !matrix->data) fail("derivative matrix handle is null");
        const uint32_t n = qubits_of_length(amplitudes_len);
        const size_t k = qubits_len;
        if (k == 0 || k > kMaxDenseArity || matrix->len != (size_t(1) << (2 * k))) {
            std::ostringstream s;
            s << "derivative matrix of " << matrix->len << " entries does not act on " << k
              << " qubits";
            fail(s.str());
        }
        if (!qubits) fail("qubit list is null");
        OpRecord rec;
        rec.opcode = ARCQML_OP_CUSTOM_UNITARY;
        rec.name = "derivative";
        for (size_t i = 0; i < k; ++i) {
            if (qubits[i] >= n) {
                std::ostringstream s;
                s << "qubit index " << qubits[i] << " is out of range for " << n << " qubits";
                fail(s.str());
            }
            for (size_t j = 0; j < i; ++j)
                if (qubits[j] == qubits[i]) fail("duplicate qubit index " + std::to_string(qubits[i]));
            rec.qubits.push_back(uint32_t(qubits[i]));
        }
        rec.custom.resize(matrix->len);
        for (size_t i = 0; i < matrix->len; ++i)
            rec.custom[i] = make_double2(matrix->data[i].re, matrix->data[i].im);
        ThreadContext &ctx = thread_context();
        double2 *d = upload_state(ctx, 0, amplitudes, amplitudes_len);
        DevGate g = lower(rec, LOWER_FORWARD, 0, false);
        if (g.kind == KIND_DENSE) {
            std::vector<const std::vector<double2> *> refs{&rec.custom};
            g.dense = upload_tables(refs, ctx, ctx.stream)[0];
        }
        launch_gate(d, 1, n, g, ctx.stream);
        download_state(ctx, d, amplitudes, amplitudes_len);
        sync(ctx.stream);
    });
}

void arcqml_rt_v1_derivative_matrix_destroy(DerivativeMatrixHandle *matrix) {
    if (!matrix || !matrix->data) return;
    delete[] matrix->data;
    matrix->data = nullptr;
    matrix->len = 0;
    matrix->capacity = 0;
}

int32_t arcqml_rt_v1_circuit_plan_create(const OperationDescriptor *operations,
                                         size_t operations_len, CircuitPlanHandle *output) {
    return guarded([&] {
        if (!output) fail("circuit plan handle is null");
        if (operations_len && !operations) fail("operation list is null");
        std::unique_ptr<Plan> p(new Plan());
        p->ops.reserve(operations_len);
        for (size_t i = 0; i < operations_len; ++i) p->ops.push_back(push_record(&operations[i]));
        output->opaque = p.release();
    });
}

int32_t arcqml_rt_v1_circuit_plan_create_empty(size_t operation_capacity,
                                               CircuitPlanHandle *output) {
    return guarded([&] {
        if (!output) fail("circuit plan handle is null");
        std::unique_ptr<Plan> p(new Plan());
        p->ops.reserve(operation_capacity < (size_t(1) << 24) ? operation_capacity : 0);
        output->opaque = p.release();
    });
}

int32_t arcqml_rt_v1_circuit_plan_push(CircuitPlanHandle *plan,
                                       const OperationDescriptor *operation) {
    return guarded([&] { plan_of(plan)->ops.push_back(push_record(operation)); });
}

int32_t arcqml_rt_v1_circuit_plan_apply(const CircuitPlanHandle *plan, arcqml_c128 *amplitudes,
                                        size_t amplitudes_len, size_t num_qubits) {
    return guarded([&] {
        Plan *p = plan_of(plan);
        check_state_length(amplitudes_len, num_qubits);
        validate_plan_for_state(*p, uint32_t(num_qubits));
        ThreadContext &ctx = thread_context();
        double2 *d = upload_state(ctx, 0, amplitudes, amplitudes_len);
        plan_apply_device(*p, d, 1, uint32_t(num_qubits), ctx, ctx.stream);
        download_state(ctx, d, amplitudes, amplitudes_len);
        sync(ctx.stream);
    });
}

int32_t arcqml_rt_v1_adjoint_backward(const CircuitPlanHandle *plan, arcqml_c128 *forward_state,
                                      arcqml_c128 *adjoint_state, size_t state_len,
                                      arcqml_c128 *derivative_state, size_t num_qubits,
                                      double upstream, const uint8_t *parameter_requires_grad,
                                      size_t parameter_requires_grad_len, double *gradients,
                                      size_t gradients_len) {
    return guarded([&] {
        Plan *p = plan_of(plan);
        check_state_length(state_len, num_qubits);
        if (!derivative_state) fail("derivative state buffer is null");
        if (parameter_requires_grad_len && !parameter_requires_grad)
            fail("requires-grad list is null");
        if (gradients_len && !gradients) fail("gradient buffer is null");
        validate_plan_for_state(*p, uint32_t(num_qubits));
        check_bindings(*p, parameter_requires_grad_len, gradients_len);
        ThreadContext &ctx = thread_context();
        double2 *dpsi = upload_state(ctx, 0, forward_state, state_len);
        double2 *dlam = upload_state(ctx, 1, adjoint_state, state_len);
        adjoint_backward_device(*p, dpsi, dlam, 1, uint32_t(num_qubits), &upstream,
                                parameter_requires_grad, parameter_requires_grad_len, gradients,
                                gradients_len, ctx, ctx.stream);
        download_state(ctx, dpsi, forward_state, state_len);
        download_state(ctx, dlam, adjoint_state, state_len);
        sync(ctx.stream);
    });
}

void arcqml_rt_v1_circuit_plan_destroy(CircuitPlanHandle *plan) {
    if (!plan || !plan->opaque) return;
    delete static_cast<Plan *>(plan->opaque);
    plan->opaque = nullptr;
}

size_t arcqml_rt_last_error(uint8_t *buffer, size_t capacity) {
    const std::string &m = last_error();
    if (buffer && capacity) {
        const size_t n = m.size() < capacity ? m.size() : capacity;
        std::memcpy(buffer, m.data(), n);
        if (n < capacity) buffer[n] = 0;
    }
    return m.size();
}

// ============================================================================ v2

int32_t arcqml_rt_v2_observable_create(size_t num_qubits, const double *coefficients,
                                       const uint64_t *flip_masks, const uint64_t *phase_masks,
                                       size_t num_terms, ArcqmlObservableHandle *output) {
    return guarded([&] {
        if (!output) fail("observable handle is null");
        output->opaque = make_observable(num_qubits, coefficients, flip_masks, phase_masks, num_terms);
    });
}

void arcqml_rt_v2_observable_destroy(ArcqmlObservableHandle *observable) {
    if (!observable || !observable->opaque) return;
    delete static_cast<Observable *>(observable->opaque);
    observable->opaque = nullptr;
}

static void check_device_state(const void *amps, size_t batch, size_t num_qubits) {
    if (!amps) fail("amplitude buffer is null");
    if (batch == 0) fail("batch size must be non-zero");
    state_dimension(num_qubits);
}

int32_t arcqml_rt_v2_plan_apply(const CircuitPlanHandle *plan, arcqml_c128 *amplitudes,
                                size_t batch, size_t num_qubits, void *stream) {
    return guarded([&] {
        Plan *p = plan_of(plan);
        check_device_state(amplitudes, batch, num_qubits);
        ThreadContext &ctx = thread_context();
        cudaStream_t s = pick_stream(ctx, stream);
        plan_apply_device(*p, reinterpret_cast<double2 *>(amplitudes), batch, uint32_t(num_qubits),
                          ctx, s);
        // Tables uploaded for dense gates live in a per-thread buffer; the next call on this
        // thread may overwrite them only after this stream's work (stream order).
    });
}

int32_t arcqml_rt_v2_apply_gate(arcqml_c128 *amplitudes, size_t batch, size_t num_qubits,
                                const GateDescriptor *gate, const size_t *qubits,
                                size_t qubits_len, int32_t adjoint, void *stream) {
    return guarded([&] {
        check_device_state(amplitudes, batch, num_qubits);
        OpRecord rec = record_from_descriptor(gate, qubits, qubits_len, int64_t(num_qubits));
        ThreadContext &ctx = thread_context();
        apply_gate_device(reinterpret_cast<double2 *>(amplitudes), batch, uint32_t(num_qubits), rec,
                          adjoint != 0, ctx, pick_stream(ctx, stream));
    });
}

int32_t arcqml_rt_v2_parameter_derivative(const arcqml_c128 *input, arcqml_c128 *output,
                                          size_t batch, size_t num_qubits,
                                          const GateDescriptor *gate, const size_t *qubits,
                                          size_t qubits_len, size_t parameter_slot,
                                          void *stream) {
    return guarded([&] {
        check_device_state(input, batch, num_qubits);
        if (!output) fail("output buffer is null");
        OpRecord rec = record_from_descriptor(gate, qubits, qubits_len, int64_t(num_qubits));
        check_slot(rec, parameter_slot);
        ThreadContext &ctx = thread_context();
        DevGate g = lower(rec, LOWER_DERIVATIVE, uint32_t(parameter_slot));
        launch_gate_out(reinterpret_cast<const double2 *>(input), reinterpret_cast<double2 *>(output),
                        batch, uint32_t(num_qubits), g, pick_stream(ctx, stream));
    });
}

int32_t arcqml_rt_v2_expectation(const ArcqmlObservableHandle *observable,
                                 const arcqml_c128 *amplitudes, size_t batch, size_t num_qubits,
                                 double *values, void *stream) {
    return guarded([&] {
        check_device_state(amplitudes, batch, num_qubits);
        if (!values) fail("value buffer is null");
        ThreadContext &ctx = thread_context();
        observable_device(*obs_of(observable), reinterpret_cast<const double2 *>(amplitudes), nullptr,
                          batch, uint32_t(num_qubits), values, ctx, pick_stream(ctx, stream));
    });
}

int32_t arcqml_rt_v2_observable_tile_passes(const ArcqmlObservableHandle *observable,
                                            size_t num_qubits, uint32_t *passes) {
    return guarded([&] {
        if (!passes) fail("output pointer is null");
        if (num_qubits >= kMaxQubits) fail("state dimension overflow");
        const Observable &o = *obs_of(observable);
        *passes = (o.num_qubits == num_qubits && pauli_tiles_enabled())
                      ? observable_tile_passes(o, uint32_t(num_qubits))
                      : 0u;
    });
}

int32_t arcqml_rt_v2_expectation_and_apply(const ArcqmlObservableHandle *observable,
                                           const arcqml_c128 *amplitudes, arcqml_c128 *output,
                                           size_t batch, size_t num_qubits, double *values,
                                           void *stream) {
    return guarded([&] {
        check_device_state(amplitudes, batch, num_qubits);
        if (!values || !output) fail("output buffer is null");
        ThreadContext &ctx = thread_context();
        observable_device(*obs_of(observable), reinterpret_cast<const double2 *>(amplitudes),
                          reinterpret_cast<double2 *>(output), batch, uint32_t(num_qubits), values,
                          ctx, pick_stream(ctx, stream));
    });
}

// Shared validation of the slice entry points.
static void check_slices(const void *amplitudes, size_t num_local_qubits, const uint32_t *positions,
                         size_t num_positions, uint64_t chunk_begin, uint64_t chunk_len) {
    if (!amplitudes) fail("amplitude buffer is null");
    if (num_local_qubits >= 63) fail("shard qubit count must be below 63");
    if (num_positions == 0 || num_positions > kMaxSliceBits)
        fail("slice must have between 1 and 8 positions");
    if (num_positions > num_local_qubits) fail("slice has more positions than the shard has qubits");
    if (!positions) fail("slice position list is null");
    uint64_t seen = 0;
    for (size_t i = 0; i < num_positions; ++i) {
        if (positions[i] >= num_local_qubits) {
            std::ostringstream m;
            m << "slice position " << positions[i] << " is outside the " << num_local_qubits
              << "-qubit shard";
            fail(m.str());
        }
        if ((seen >> positions[i]) & 1) fail("slice positions repeat");
        seen |= uint64_t(1) << positions[i];
    }
    const uint64_t others = uint64_t(1) << (num_local_qubits - num_positions);
    if (chunk_begin > others || chunk_len > others - chunk_begin)
        fail("slice chunk exceeds the shard");
}

int32_t arcqml_rt_v2_expectation_and_accumulate(const ArcqmlObservableHandle *observable,
                                                const arcqml_c128 *amplitudes, arcqml_c128 *output,
                                                size_t batch, size_t num_qubits, double *values,
                                                void *stream) {
    return guarded([&] {
        check_device_state(amplitudes, batch, num_qubits);
        if (!values || !output) fail("output buffer is null");
        ThreadContext &ctx = thread_context();
        observable_device(*obs_of(observable), reinterpret_cast<const double2 *>(amplitudes),
                          reinterpret_cast<double2 *>(output), batch, uint32_t(num_qubits), values,
                          ctx, pick_stream(ctx, stream), true);
    });
}

int32_t arcqml_rt_v2_shard_slices(arcqml_c128 *amplitudes, size_t num_local_qubits,
                                  const uint32_t *positions, size_t num_positions,
                                  uint64_t chunk_begin, uint64_t chunk_len, uint64_t skip_value,
                                  arcqml_c128 *staging, int32_t unpack, void *stream) {
    return guarded([&] {
        if (!amplitudes || !staging) fail("amplitude or staging buffer is null");
        check_slices(amplitudes, num_local_qubits, positions, num_positions, chunk_begin,
                     chunk_len);
        ThreadContext &ctx = thread_context();
        launch_slices(reinterpret_cast<double2 *>(amplitudes), uint32_t(num_local_qubits),
                      positions, uint32_t(num_positions), chunk_begin, chunk_len, skip_value,
                      reinterpret_cast<double2 *>(staging), unpack != 0, pick_stream(ctx, stream));
    });
}

int32_t arcqml_rt_v2_sample(const arcqml_c128 *amplitudes, size_t num_qubits, uint64_t shots,
                            uint64_t seed, uint64_t *indices, double *norm_sqr, void *stream) {
    return guarded([&] {
        if (shots == 0) fail("invalid shot count: shots must be greater than zero");
        check_device_state(amplitudes, 1, num_qubits);
        if (!indices) fail("index buffer is null");
        const size_t dim = state_dimension(num_qubits);
        ThreadContext &ctx = thread_context();
        cudaStream_t s = pick_stream(ctx, stream);
        // the v2 entry points never use the state slots 1 and 2 of the thread's buffers
        auto *cum = static_cast<double *>(ctx_buffer(ctx, 1, dim * sizeof(double)));
        auto *out = static_cast<uint64_t *>(ctx_buffer(ctx, 2, shots * sizeof(uint64_t)));
        launch_sample(reinterpret_cast<const double2 *>(amplitudes), uint32_t(num_qubits), shots,
                      seed, cum, out, s);
        double total = 0.0;
        check_cuda(cudaMemcpyAsync(&total, cum + dim - 1, sizeof(double), cudaMemcpyDeviceToHost, s),
                   "cudaMemcpyAsync (norm)");
        check_cuda(cudaMemcpyAsync(indices, out, shots * sizeof(uint64_t), cudaMemcpyDeviceToHost, s),
                   "cudaMemcpyAsync (indices)");
        check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
        if (norm_sqr) *norm_sqr = total;
        if (!(std::fabs(total - 1.0) <= 1e-10)) {
            std::ostringstream m;
            m << "tensor state is not normalized: expected norm squared close to 1, got " << total;
            fail(m.str());
        }
    });
}

int32_t arcqml_rt_v2_plan_jit_check(const CircuitPlanHandle *plan, size_t num_qubits,
                                    int32_t adjoint, uint64_t *compiled, uint64_t *eligible,
                                    char *message, size_t capacity) {
    return guarded([&] {
        Plan *p = plan_of(plan);
        state_dimension(num_qubits);
        const uint32_t n = uint32_t(num_qubits);
        if (n < kFusedMinQubits) fail("plans below 8 qubits run no fused passes");
        validate_plan_for_state(*p, n);
        size_t parents = 1;
        for (const auto &op : p->ops)
            for (uint32_t b = 0; b < op.num_bindings; ++b)
                parents = std::max(parents, op.parents[b] + 1);
        std::vector<uint8_t> req(parents, 1);
        const bool wide = adjoint && adjoint_wide_tiles() && n >= 12;
        const uint32_t k = wide ? 12u : fused_k(n, adjoint != 0);
        Schedule sch = build_schedule(*p, n, adjoint != 0, req.data(), adjoint != 0, k,
                                      wide ? 4u : (adjoint ? fused_rb(k, true) : forward_rb(k)));
        size_t el = 0;
        std::string err;
        const size_t ok = jit_compile_check(sch, adjoint != 0, &el, &err);
        if (compiled) *compiled = ok;
        if (eligible) *eligible = el;
        if (message && capacity) {
            const size_t m = std::min(capacity - 1, err.size());
            std::memcpy(message, err.data(), m);
            message[m] = '\0';
        }
    });
}

size_t arcqml_rt_v2_jit_info(uint64_t *kernels_compiled, uint64_t *launches, uint64_t *fallbacks,
                             char *last_error, size_t capacity) {
    std::string last;
    jit_info(kernels_compiled, launches, fallbacks, &last);
    if (last_error && capacity) {
        const size_t n = std::min(capacity - 1, last.size());
        std::memcpy(last_error, last.data(), n);
        last_error[n] = '\0';
    }
    return last.size();
}

int32_t arcqml_rt_v2_shard_swap_nccl(arcqml_c128 *shard, size_t num_local_qubits,
                                     const uint32_t *global_bits, const uint32_t *local_positions,
                                     size_t num_pairs, void *nccl_comm, arcqml_c128 *staging,
                                     size_t staging_len, void *stream) {
    return guarded([&] {
        if (!nccl_comm) fail("NCCL communicator is null");
        if (!global_bits) fail("global bit list is null");
        if (!staging) fail("staging buffer is null");
        check_slices(shard, num_local_qubits, local_positions, num_pairs, 0, 0);
        ThreadContext &ctx = thread_context();
        shard_swap_nccl(reinterpret_cast<double2 *>(shard), uint32_t(num_local_qubits),
                        global_bits, local_positions, uint32_t(num_pairs), nccl_comm,
                        reinterpret_cast<double2 *>(staging), staging_len,
                        pick_stream(ctx, stream));
    });
}

int32_t arcqml_rt_v2_shard_slices_from(arcqml_c128 *amplitudes, size_t num_local_qubits,
                                       const uint32_t *positions, size_t num_positions,
                                       uint64_t chunk_begin, uint64_t chunk_len,
                                       const arcqml_c128 *const *sources, void *stream) {
    return guarded([&] {
        check_slices(amplitudes, num_local_qubits, positions, num_positions, chunk_begin,
                     chunk_len);
        if (!sources) fail("slice source list is null");
        ThreadContext &ctx = thread_context();
        launch_slices_from(reinterpret_cast<double2 *>(amplitudes), positions,
                           uint32_t(num_positions), chunk_begin, chunk_len,
                           reinterpret_cast<const double2 *const *>(sources),
                           pick_stream(ctx, stream));
    });
}

int32_t arcqml_rt_v2_peer_buffer_create(size_t bytes, void **device_ptr, uint8_t *handle) {
    return guarded([&] {
        if (!device_ptr || !handle) fail("output pointer is null");
        if (bytes == 0) fail("peer buffer size must be non-zero");
        void *p = nullptr;
        check_cuda(cudaMalloc(&p, bytes), "cudaMalloc (peer buffer)");
        cudaIpcMemHandle_t h;
        const cudaError_t e = cudaIpcGetMemHandle(&h, p);
        if (e != cudaSuccess) {
            cudaFree(p);
            check_cuda(e, "cudaIpcGetMemHandle");
        }
        static_assert(sizeof(h) == 64, "IPC handle size");
        std::memcpy(handle, &h, sizeof(h));
        *device_ptr = p;
    });
}

int32_t arcqml_rt_v2_peer_buffer_open(const uint8_t *handle, void **device_ptr) {
    return guarded([&] {
        if (!device_ptr || !handle) fail("handle or output pointer is null");
        cudaIpcMemHandle_t h;
        std::memcpy(&h, handle, sizeof(h));
        void *p = nullptr;
        check_cuda(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess),
                   "cudaIpcOpenMemHandle");
        *device_ptr = p;
    });
}

int32_t arcqml_rt_v2_peer_buffer_close(void *device_ptr) {
    return guarded([&] {
        if (device_ptr) check_cuda(cudaIpcCloseMemHandle(device_ptr), "cudaIpcCloseMemHandle");
    });
}

int32_t arcqml_rt_v2_peer_buffer_destroy(void *device_ptr) {
    return guarded([&] {
        if (device_ptr) check_cuda(cudaFree(device_ptr), "cudaFree (peer buffer)");
    });
}

int32_t arcqml_rt_v2_small_run(const CircuitPlanHandle *plan,
                               const ArcqmlObservableHandle *observable,
                               const arcqml_c128 *initial_state, size_t num_qubits,
                               const uint8_t *parameter_requires_grad,
                               size_t parameter_requires_grad_len, double *gradients,
                               size_t gradients_len, double *value, arcqml_c128 *lambda0,
                               void *stream) {
    return guarded([&] {
        Plan *p = plan_of(plan);
        state_dimension(num_qubits);
        if (!value) fail("value pointer is null");
        if (parameter_requires_grad_len && !parameter_requires_grad)
            fail("requires-grad list is null");
        if (gradients_len && !gradients) fail("gradient buffer is null");
        ThreadContext &ctx = thread_context();
        small_step_device(*p, *obs_of(observable),
                          reinterpret_cast<const double2 *>(initial_state), uint32_t(num_qubits),
                          parameter_requires_grad, parameter_requires_grad_len, gradients,
                          gradients_len, value, reinterpret_cast<double2 *>(lambda0), ctx,
                          pick_stream(ctx, stream));
    });
}

int32_t arcqml_rt_v2_small_adam(const CircuitPlanHandle *plan,
                                const ArcqmlObservableHandle *observable,
                                const arcqml_c128 *initial_state, size_t num_qubits,
                                const uint8_t *parameter_requires_grad, double *parameters,
                                size_t num_parameters, double *adam_m, double *adam_v,
                                uint64_t steps_taken, size_t steps, double learning_rate,
                                double beta1, double beta2, double epsilon, double weight_decay,
                                double *energies, void *stream) {
    return guarded([&] {
        Plan *p = plan_of(plan);
        state_dimension(num_qubits);
        SmallAdam h{learning_rate, beta1, beta2, epsilon, weight_decay};
        Observable &obs = *obs_of(observable);
        validate_small_adam(*p, obs, uint32_t(num_qubits), parameter_requires_grad,
                            num_parameters, parameters, steps, h, energies);
        ThreadContext &ctx = thread_context();
        small_adam_device(*p, obs, reinterpret_cast<const double2 *>(initial_state),
                          uint32_t(num_qubits), parameter_requires_grad, num_parameters,
                          parameters, adam_m, adam_v, steps_taken, steps, h, energies, ctx,
                          pick_stream(ctx, stream));
    });
}

int32_t arcqml_rt_v2_adjoint_backward(const CircuitPlanHandle *plan, arcqml_c128 *forward_state,
                                      arcqml_c128 *adjoint_state, size_t batch,
                                      size_t num_qubits, const double *upstream,
                                      const uint8_t *parameter_requires_grad,
                                      size_t parameter_requires_grad_len, double *gradients,
                                      size_t gradients_len, void *stream) {
    return guarded([&] {
        Plan *p = plan_of(plan);
        check_device_state(forward_state, batch, num_qubits);
        if (!adjoint_state) fail("adjoint state buffer is null");
        if (!upstream) fail("upstream buffer is null");
        if (parameter_requires_grad_len && !parameter_requires_grad)
            fail("requires-grad list is null");
        if (gradients_len && !gradients) fail("gradient buffer is null");
        ThreadContext &ctx = thread_context();
        adjoint_backward_device(*p, reinterpret_cast<double2 *>(forward_state),
                                reinterpret_cast<double2 *>(adjoint_state), batch,
                                uint32_t(num_qubits), upstream, parameter_requires_grad,
                                parameter_requires_grad_len, gradients, gradients_len, ctx,
                                pick_stream(ctx, stream));
    });
}

int32_t arcqml_rt_v2_plan_schedule_export(const CircuitPlanHandle *plan, size_t num_qubits,
                                          int32_t adjoint, const uint8_t *parameter_requires_grad,
                                          size_t parameter_requires_grad_len, uint8_t *buffer,
                                          size_t capacity, size_t *size) {
    return guarded([&] {
        Plan *p = plan_of(plan);
        state_dimension(num_qubits);
        if (!size) fail("size pointer is null");
        const uint32_t n = uint32_t(num_qubits);
        if (n < kFusedMinQubits) fail("plans below 8 qubits run no fused passes");
        validate_plan_for_state(*p, n);
        std::vector<uint8_t> req(parameter_requires_grad,
                                 parameter_requires_grad + parameter_requires_grad_len);
        if (adjoint) check_bindings(*p, req.size(), req.size());
        const uint32_t k = fused_k(n, adjoint != 0);
        const uint32_t rb = adjoint ? fused_rb(k, true) : forward_rb(k);
        const Schedule sch = build_schedule(*p, n, adjoint != 0, req.empty() ? nullptr : req.data(),
                                            adjoint != 0, k, rb);
        std::vector<uint8_t> out;
        auto put = [&](const void *src, size_t bytes) {
            const uint8_t *b = static_cast<const uint8_t *>(src);
            out.insert(out.end(), b, b + bytes);
        };
        auto put32 = [&](uint64_t v) {
            const uint32_t x = uint32_t(v);
            put(&x, 4);
        };
        put32(sch.steps.size());
        for (const Step &st : sch.steps) {
            put32(st.is_pass ? 1 : 0);
            if (!st.is_pass) {
                put32(uint64_t(st.dense_op - p->ops.data()));
                continue;
            }
            put(&st.header, sizeof(PassHeader));
            put32(st.subs.size());
            put(st.subs.data(), st.subs.size() * sizeof(SubBlock));
            put32(st.ops.size());
            put(st.ops.data(), st.ops.size() * sizeof(FOp));
            put32(st.mats.size());
            put(st.mats.data(), st.mats.size() * sizeof(double2));
            put32(st.parents.size());
            for (size_t pa : st.parents) {
                const uint64_t x = pa;
                put(&x, 8);
            }
            put32(st.alias.size());
            for (const auto &al : st.alias) {
                const uint64_t x[2] = {al.first, al.second};
                put(x, 16);
            }
            const std::string code = jit_pass_code(st, adjoint != 0);
            put32(code.size());
            put(code.data(), code.size());
        }
        *size = out.size();
        if (buffer && capacity >= out.size()) std::memcpy(buffer, out.data(), out.size());
    });
}

int32_t arcqml_rt_v2_plan_emulate(const CircuitPlanHandle *plan, arcqml_c128 *state,
                                  size_t num_qubits, int32_t adjoint, arcqml_c128 *lambda,
                                  const uint8_t *parameter_requires_grad,
                                  size_t parameter_requires_grad_len, double *gradients,
                                  size_t gradients_len) {
    return guarded([&] {
        Plan *p = plan_of(plan);
        state_dimension(num_qubits);
        if (!state) fail("state buffer is null");
        if (adjoint) {
            if (!lambda) fail("adjoint state buffer is null");
            if (parameter_requires_grad_len && !parameter_requires_grad)
                fail("requires-grad list is null");
            if (gradients_len && !gradients) fail("gradient buffer is null");
        }
        emulate_schedule(*p, uint32_t(num_qubits), adjoint != 0,
                         reinterpret_cast<double2 *>(state), reinterpret_cast<double2 *>(lambda),
                         parameter_requires_grad, parameter_requires_grad_len, gradients,
                         gradients_len);
    });
}

// ---------------------------------------------------------------- state analysis

// The qubit selection of crates/arcqml-analysis/src/statevector/marginal.rs:38-59 (same errors
// and messages as AnalysisError); qubits == NULL with num_selected == 0 selects every qubit when
// allow_all is set.
static Selection analysis_selection(size_t num_qubits, const size_t *qubits, size_t num_selected,
                                    bool allow_all) {
    std::vector<uint32_t> q;
    if (!qubits && num_selected == 0 && allow_all) {
        for (size_t i = num_qubits; i-- > 0;) q.push_back(uint32_t(i));
        return make_selection(uint32_t(num_qubits), q);
    }
    if (num_selected == 0) fail("at least one qubit must be selected");
    if (!qubits) fail("qubit list is null");
    for (size_t j = 0; j < num_selected; ++j) {
        if (qubits[j] >= num_qubits) {
            std::ostringstream m;
            m << "qubit index out of range: simulator has " << num_qubits << " qubits, got "
              << qubits[j];
            fail(m.str());
        }
        for (size_t i = 0; i < j; ++i)
            if (qubits[i] == qubits[j]) {
                std::ostringstream m;
                m << "duplicate qubit in selection: " << qubits[j];
                fail(m.str());
            }
        q.push_back(uint32_t(qubits[j]));
    }
    return make_selection(uint32_t(num_qubits), q);
}

int32_t arcqml_rt_v2_probabilities(const arcqml_c128 *amplitudes, size_t batch,
                                   size_t num_qubits, double *probabilities, void *stream) {
    return guarded([&] {
        check_device_state(amplitudes, batch, num_qubits);
        if (!probabilities) fail("probability buffer is null");
        ThreadContext &ctx = thread_context();
        probabilities_device(reinterpret_cast<const double2 *>(amplitudes), batch,
                             uint32_t(num_qubits), probabilities, pick_stream(ctx, stream));
    });
}

int32_t arcqml_rt_v2_marginal_probabilities(const arcqml_c128 *amplitudes, size_t batch,
                                            size_t num_qubits, const size_t *qubits,
                                            size_t num_selected, double *marginals,
                                            void *stream) {
    return guarded([&] {
        check_device_state(amplitudes, batch, num_qubits);
        const Selection S = analysis_selection(num_qubits, qubits, num_selected, false);
        if (!marginals) fail("marginal buffer is null");
        ThreadContext &ctx = thread_context();
        marginal_device(reinterpret_cast<const double2 *>(amplitudes), batch,
                        uint32_t(num_qubits), S, marginals, ctx, pick_stream(ctx, stream));
    });
}

int32_t arcqml_rt_v2_bloch_vector(const arcqml_c128 *amplitudes, size_t batch, size_t num_qubits,
                                  size_t qubit, double *xyz, void *stream) {
    return guarded([&] {
        check_device_state(amplitudes, batch, num_qubits);
        if (qubit >= num_qubits) {
            std::ostringstream m;
            m << "qubit index out of range: simulator has " << num_qubits << " qubits, got "
              << qubit;
            fail(m.str());
        }
        if (!xyz) fail("Bloch vector buffer is null");
        ThreadContext &ctx = thread_context();
        bloch_device(reinterpret_cast<const double2 *>(amplitudes), batch, uint32_t(num_qubits),
                     uint32_t(qubit), xyz, ctx, pick_stream(ctx, stream));
    });
}

int32_t arcqml_rt_v2_overlap(const arcqml_c128 *lhs, const arcqml_c128 *rhs, size_t batch,
                             size_t num_qubits, double *overlaps, void *stream) {
    return guarded([&] {
        check_device_state(lhs, batch, num_qubits);
        check_device_state(rhs, batch, num_qubits);
        if (!overlaps) fail("overlap buffer is null");
        ThreadContext &ctx = thread_context();
        overlap_device(reinterpret_cast<const double2 *>(lhs),
                       reinterpret_cast<const double2 *>(rhs), batch, uint32_t(num_qubits),
                       overlaps, ctx, pick_stream(ctx, stream));
    });
}

int32_t arcqml_rt_v2_probability_cotangent(const arcqml_c128 *amplitudes, size_t batch,
                                           size_t num_qubits, const size_t *qubits,
                                           size_t num_selected, const double *upstream,
                                           arcqml_c128 *cotangent, void *stream) {
    return guarded([&] {
        check_device_state(amplitudes, batch, num_qubits);
        const Selection S = analysis_selection(num_qubits, qubits, num_selected, true);
        if (!upstream) fail("upstream buffer is null");
        if (!cotangent) fail("cotangent buffer is null");
        ThreadContext &ctx = thread_context();
        probability_cotangent_device(reinterpret_cast<const double2 *>(amplitudes), batch,
                                     uint32_t(num_qubits), S, upstream,
                                     reinterpret_cast<double2 *>(cotangent),
                                     pick_stream(ctx, stream));
    });
}

int32_t arcqml_rt_v2_scaled_copy(const arcqml_c128 *input, size_t batch, size_t num_qubits,
                                 const double *factors, arcqml_c128 *output, void *stream) {
    return guarded([&] {
        check_device_state(input, batch, num_qubits);
        if (!factors) fail("factor list is null");
        if (!output) fail("output buffer is null");
        for (size_t r = 0; r < 2 * batch; ++r)
            if (!std::isfinite(factors[r])) fail("factors must be finite");
        ThreadContext &ctx = thread_context();
        scaled_copy_device(reinterpret_cast<const double2 *>(input), batch, uint32_t(num_qubits),
                           factors, reinterpret_cast<double2 *>(output), ctx,
                           pick_stream(ctx, stream));
    });
}

int32_t arcqml_rt_v2_norms(const arcqml_c128 *amplitudes, size_t batch, size_t num_qubits,
                           double *norms, void *stream) {
    return guarded([&] {
        check_device_state(amplitudes, batch, num_qubits);
        if (!norms) fail("norm buffer is null");
        ThreadContext &ctx = thread_context();
        cudaStream_t s = pick_stream(ctx, stream);
        const size_t chunk = 65535;
        const size_t dim = size_t(1) << num_qubits;
        for (size_t b0 = 0; b0 < batch; b0 += chunk) {
            const size_t rows = std::min(chunk, batch - b0);
            double *partials = ctx_partials(ctx, rows * size_t(adjoint_max_blocks()));
            const unsigned bx = launch_norms(reinterpret_cast<const double2 *>(amplitudes) + b0 * dim,
                                             rows, uint32_t(num_qubits), partials, s);
            double *sums = ctx_dgrads(ctx, rows);
            launch_reduce_rows(partials, uint32_t(rows), bx, sums, s);
            double *h = ctx_hvals(ctx, rows);
            check_cuda(cudaMemcpyAsync(h, sums, rows * sizeof(double), cudaMemcpyDeviceToHost, s),
                       "cudaMemcpyAsync (norms)");
            sync(s);
            std::memcpy(norms + b0, h, rows * sizeof(double));
        }
    });
}

int32_t arcqml_rt_v2_set_basis_state(arcqml_c128 *amplitudes, size_t batch, size_t num_qubits,
                                     uint64_t index, void *stream) {
    return guarded([&] {
        check_device_state(amplitudes, batch, num_qubits);
        if (index >= (uint64_t(1) << num_qubits)) fail("basis index out of range");
        ThreadContext &ctx = thread_context();
        launch_basis_state(reinterpret_cast<double2 *>(amplitudes), batch, uint32_t(num_qubits),
                           index, pick_stream(ctx, stream));
    });
}

int32_t arcqml_rt_v2_plan_set_parameters(CircuitPlanHandle *plan, const double *parent_values,
                                         size_t parent_values_len) {
    return guarded([&] {
        Plan *p = plan_of(plan);
        if (parent_values_len && !parent_values) fail("parameter value list is null");
        for (auto &op : p->ops)
            for (uint32_t b = 0; b < op.num_bindings; ++b)
                if (op.parents[b] >= parent_values_len)
                    fail("parameter parent index " + std::to_string(op.parents[b]) + " is out of range");
        for (auto &op : p->ops)
            for (uint32_t b = 0; b < op.num_bindings; ++b) {
                const double v = parent_values[op.parents[b]];
                if (!std::isfinite(v)) fail("parameter value is not finite");
                op.params[op.slots[b]] = v;
            }
    });
}

size_t arcqml_rt_v2_plan_len(const CircuitPlanHandle *plan) {
    if (!plan || !plan->opaque) return 0;
    return static_cast<const Plan *>(plan->opaque)->ops.size();
}

int32_t arcqml_rt_v2_plan_schedule_stats(const CircuitPlanHandle *plan, size_t num_qubits,
                                         int32_t adjoint, uint64_t *passes, uint64_t *sub_blocks,
                                         uint64_t *gates) {
    return guarded([&] {
        Plan *p = plan_of(plan);
        state_dimension(num_qubits);
        if (!passes || !sub_blocks || !gates) fail("output pointer is null");
        validate_plan_for_state(*p, uint32_t(num_qubits));
        if (num_qubits < kFusedMinQubits) {
            *passes = p->ops.size();
            *sub_blocks = p->ops.size();
            *gates = p->ops.size();
            return;
        }
        size_t parents = 1;
        for (const auto &op : p->ops)
            for (uint32_t b = 0; b < op.num_bindings; ++b)
                parents = std::max(parents, op.parents[b] + 1);
        std::vector<uint8_t> req(parents, 1);
        const uint32_t k = fused_k(uint32_t(num_qubits), adjoint != 0);
        Schedule sch = build_schedule(*p, uint32_t(num_qubits), adjoint != 0, req.data(),
                                      adjoint != 0, k, adjoint ? fused_rb(k, true) : forward_rb(k));
        *passes = sch.steps.size();
        uint64_t sb = 0, g = 0;
        for (const auto &st : sch.steps) {
            sb += st.is_pass ? st.subs.size() : 1;
            g += st.is_pass ? st.ops.size() : 1;
        }
        *sub_blocks = sb;
        *gates = g;
    });
}

void arcqml_rt_v2_profile_enable(int32_t on) { prof_enable(on != 0); }

int32_t arcqml_rt_v2_profile_read(uint32_t category, uint64_t *launches, double *total_ms,
                                  double *algorithmic_bytes) {
    return guarded([&] {
        if (category >= uint32_t(kProfCategories)) fail("unknown profile category");
        if (!launches || !total_ms || !algorithmic_bytes) fail("output pointer is null");
        prof_read(int(category), launches, total_ms, algorithmic_bytes);
    });
}

uint64_t arcqml_rt_v2_launch_count(void) { return prof_launch_count(); }

}  // extern "C"
#pragma GCC visibility pop
