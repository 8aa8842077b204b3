// engine.cpp — device orchestration: per-thread contexts, plan execution, the adjoint
// reverse sweep and Pauli observables on device-resident states.
//
// Reverse sweep (docs/ArcQML技术手册.md:426-454, loop order of
// crates/arcqml-unitary/src/fit/adjoint.rs:19-66): lambda <- g lambda; for k = m..1:
// psi <- U_k^dag psi; grads[parent] += 2 Re<lambda|dU_k/dp psi>; lambda <- U_k^dag lambda.
// Each reversed gate with a required slot is ONE kernel pass over psi and lambda
// (k_adjoint): 64 bytes of HBM traffic per touched amplitude, no derivative scratch state.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <sstream>
#include <unordered_map>

#include "jit.h"
#include "launch.h"
#include "planner.h"
#include "rt_internal.h"

namespace arcqml {

// ------------------------------------------------------------------ errors

namespace {
thread_local std::string t_last_error;
}

void set_last_error(const std::string &msg) { t_last_error = msg; }
const std::string &last_error() { return t_last_error; }

void fail(const std::string &msg) { throw Error{msg}; }

void check_cuda(cudaError_t e, const char *what) {
    if (e != cudaSuccess) {
        std::ostringstream s;
        s << what << " failed: " << cudaGetErrorString(e);
        throw Error{s.str()};
    }
}

// ------------------------------------------------------------------ thread contexts

namespace {

struct ContextSlot {
    ThreadContext ctx;
    ~ContextSlot() {
        // Thread exit: release device buffers (the CUDA context may already be gone at
        // process exit; errors are ignored).
        int prev = -1;
        if (cudaGetDevice(&prev) != cudaSuccess) return;
        if (ctx.device >= 0 && cudaSetDevice(ctx.device) == cudaSuccess) {
            for (int i = 0; i < 5; ++i)
                if (ctx.buf[i]) cudaFree(ctx.buf[i]);
            if (ctx.partials) cudaFree(ctx.partials);
            if (ctx.dgrads) cudaFree(ctx.dgrads);
            if (ctx.hvals) cudaFreeHost(ctx.hvals);
            if (ctx.stream) cudaStreamDestroy(ctx.stream);
        }
        cudaSetDevice(prev);
    }
};

thread_local std::unordered_map<int, std::unique_ptr<ContextSlot>> t_contexts;

}  // namespace

ThreadContext &thread_context() {
    int dev = 0;
    check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    auto &slot = t_contexts[dev];
    if (!slot) {
        slot.reset(new ContextSlot());
        slot->ctx.device = dev;
        check_cuda(cudaStreamCreateWithFlags(&slot->ctx.stream, cudaStreamNonBlocking),
                   "cudaStreamCreateWithFlags");
    }
    return slot->ctx;
}

void *ctx_buffer(ThreadContext &c, int which, size_t bytes) {
    if (bytes > c.cap[which]) {
        if (c.buf[which]) {
            check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
            check_cuda(cudaFree(c.buf[which]), "cudaFree");
            c.buf[which] = nullptr;
            c.cap[which] = 0;
        }
        check_cuda(cudaMalloc(&c.buf[which], bytes), "cudaMalloc");
        c.cap[which] = bytes;
    }
    return c.buf[which];
}

double *ctx_partials(ThreadContext &c, size_t count) {
    if (count > c.partials_cap) {
        if (c.partials) {
            check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
            check_cuda(cudaFree(c.partials), "cudaFree");
            c.partials = nullptr;
            c.partials_cap = 0;
        }
        check_cuda(cudaMalloc(&c.partials, count * sizeof(double)), "cudaMalloc");
        c.partials_cap = count;
    }
    return c.partials;
}

double *ctx_dgrads(ThreadContext &c, size_t count) {
    if (count > c.dgrads_cap) {
        if (c.dgrads) {
            check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
            check_cuda(cudaFree(c.dgrads), "cudaFree");
            c.dgrads = nullptr;
            c.dgrads_cap = 0;
        }
        check_cuda(cudaMalloc(&c.dgrads, count * sizeof(double)), "cudaMalloc");
        c.dgrads_cap = count;
    }
    return c.dgrads;
}

double *ctx_hvals(ThreadContext &c, size_t count) {
    if (count > c.hvals_cap) {
        if (c.hvals) {
            check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
            check_cuda(cudaFreeHost(c.hvals), "cudaFreeHost");
            c.hvals = nullptr;
            c.hvals_cap = 0;
        }
        check_cuda(cudaMallocHost(&c.hvals, count * sizeof(double)), "cudaMallocHost");
        c.hvals_cap = count;
    }
    return c.hvals;
}

std::vector<const double2 *> upload_tables(const std::vector<const std::vector<double2> *> &ms,
                                           ThreadContext &ctx, cudaStream_t s) {
    size_t total = 0;
    for (auto *m : ms) total += m->size();
    std::vector<const double2 *> out;
    if (total == 0) return out;
    // The table buffer may still be read by kernels queued on another stream by an earlier
    // call of this thread; wait for them before overwriting it.
    if (ctx.table_stream && ctx.table_stream != s)
        check_cuda(cudaStreamSynchronize(ctx.table_stream), "cudaStreamSynchronize");
    ctx.table_stream = s;
    auto *dev = static_cast<double2 *>(ctx_buffer(ctx, 3, total * sizeof(double2)));
    size_t off = 0;
    for (auto *m : ms) {
        check_cuda(cudaMemcpyAsync(dev + off, m->data(), m->size() * sizeof(double2),
                                   cudaMemcpyHostToDevice, s),
                   "cudaMemcpyAsync (tables)");
        out.push_back(dev + off);
        off += m->size();
    }
    return out;
}

// ------------------------------------------------------------------ plan execution

void validate_plan_for_state(const Plan &plan, uint32_t n) {
    for (const auto &op : plan.ops) check_qubits_for_state(op, n);
}

// ARCQML_FUSE=0 selects the per-gate kernels everywhere (for A/B measurements);
// ARCQML_FORWARD_RB=3 runs 12-qubit forward tiles with 8 instead of 16 amplitudes per thread.
bool fusion_enabled() {
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_FUSE");
        return !(e && e[0] == '0');
    }();
    return on;
}

uint32_t forward_rb(uint32_t k) {
    static const int forced = [] {
        const char *e = std::getenv("ARCQML_FORWARD_RB");
        return e ? std::atoi(e) : 0;
    }();
    if (k >= 11 && (forced == 3 || forced == 4)) return uint32_t(forced);
    return fused_rb(k, false);
}

void plan_apply_device(Plan &plan, double2 *amps, size_t batch, uint32_t n, ThreadContext &ctx,
                       cudaStream_t s) {
    validate_plan_for_state(plan, n);
    if (fusion_enabled() && n >= kFusedMinQubits) {
        const uint32_t k = fused_k(n, false);
        Schedule sch = build_schedule(plan, n, false, nullptr, false, k, forward_rb(k));
        run_schedule(sch, amps, nullptr, batch, n, nullptr, 0, ctx, s);
        return;
    }
    std::vector<std::vector<double2>> dense;
    std::vector<DevGate> gates;
    gates.reserve(plan.ops.size());
    for (const auto &op : plan.ops) {
        DevGate g = lower(op, LOWER_FORWARD, 0);
        if (g.kind == KIND_DENSE) dense.push_back(op.custom);
        gates.push_back(g);
    }
    std::vector<const std::vector<double2> *> refs;
    for (auto &d : dense) refs.push_back(&d);
    auto ptrs = upload_tables(refs, ctx, s);
    size_t di = 0;
    for (auto &g : gates) {
        if (g.kind == KIND_DENSE) g.dense = ptrs[di++];
        launch_gate(amps, batch, n, g, s);
    }
}

namespace {

// Dense (conjugate-transposed) custom matrix for the adjoint of a KIND_DENSE gate.
std::vector<double2> dagger(const std::vector<double2> &m, size_t dim) {
    std::vector<double2> t(dim * dim);
    for (size_t i = 0; i < dim; ++i)
        for (size_t j = 0; j < dim; ++j) t[j * dim + i] = make_double2(m[i * dim + j].x, -m[i * dim + j].y);
    return t;
}

}  // namespace

void check_bindings(const Plan &plan, size_t req_len, size_t grads_len) {
    for (const auto &op : plan.ops)
        for (uint32_t b = 0; b < op.num_bindings; ++b) {
            if (op.parents[b] >= req_len || op.parents[b] >= grads_len) {
                std::ostringstream s;
                s << "parameter parent index " << op.parents[b]
                  << " is out of range (requires_grad length " << req_len
                  << ", gradients length " << grads_len << ")";
                fail(s.str());
            }
        }
}

void adjoint_backward_device(Plan &plan, double2 *psi, double2 *lam, size_t batch, uint32_t n,
                             const double *upstream_host, const uint8_t *req, size_t req_len,
                             double *grads_host, size_t grads_len, ThreadContext &ctx,
                             cudaStream_t s) {
    validate_plan_for_state(plan, n);
    check_bindings(plan, req_len, grads_len);

    // lambda <- g lambda (per row); factors of exactly 1 leave lambda unchanged
    bool unit = true;
    for (size_t b = 0; b < batch; ++b) unit = unit && upstream_host[b] == 1.0;
    if (!unit) {
        // pack the per-row factors as doubles inside the table buffer
        std::vector<double2> packed((batch + 1) / 2);
        std::memcpy(packed.data(), upstream_host, batch * sizeof(double));
        std::vector<const std::vector<double2> *> refs{&packed};
        auto p = upload_tables(refs, ctx, s);
        launch_scale(lam, batch, n, reinterpret_cast<const double *>(p[0]), s);
        // The table buffer is reused below for dense matrices; keep the scale ordered first.
    }

    if (fusion_enabled() && n >= kFusedMinQubits) {
        uint32_t k = fused_k(n, true);
        uint32_t rb = fused_rb(k, true);
        Schedule sch;
        bool wide = false;
        if (adjoint_wide_tiles() && n >= 12) {
            sch = build_schedule(plan, n, true, req, true, 12, 4);
            wide = jit_schedule_compiles(sch, true);
            if (wide) {
                k = 12;
                rb = 4;
            }
        }
        if (!wide) sch = build_schedule(plan, n, true, req, true, k, rb);
        // room for two resident CTAs per SM (run-time compiled adjoint kernels may have them)
        const uint32_t stride = 2 * fused_grid_blocks(true, k, rb);
        double *partials = nullptr;
        if (sch.total_acc) {
            partials = ctx_partials(ctx, size_t(sch.total_acc) * stride);
            check_cuda(cudaMemsetAsync(partials, 0, size_t(sch.total_acc) * stride * sizeof(double), s),
                       "cudaMemsetAsync");
        }
        run_schedule(sch, psi, lam, batch, n, partials, stride, ctx, s);
        if (sch.total_acc) {
            double *sums = ctx_dgrads(ctx, sch.total_acc);
            launch_reduce_rows(partials, sch.total_acc, stride, sums, s);
            double *h = ctx_hvals(ctx, sch.total_acc);
            check_cuda(cudaMemcpyAsync(h, sums, sch.total_acc * sizeof(double),
                                       cudaMemcpyDeviceToHost, s),
                       "cudaMemcpyAsync (gradients)");
            check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
            size_t a = 0;
            for (const auto &st : sch.steps) {
                for (const auto &al : st.alias) grads_host[al.second] += 2.0 * h[a + al.first];
                for (size_t p : st.parents) grads_host[p] += 2.0 * h[a++];
            }
        }
        return;
    }

    // Rows of partial sums, one per (op, binding) that needs a gradient, in sweep order.
    struct Row {
        size_t parent;
    };
    std::vector<Row> rows;
    for (size_t k = plan.ops.size(); k-- > 0;) {
        const auto &op = plan.ops[k];
        for (uint32_t b = 0; b < op.num_bindings; ++b)
            if (req[op.parents[b]]) rows.push_back({op.parents[b]});
    }
    const unsigned cap = adjoint_max_blocks();
    double *partials = nullptr;
    if (!rows.empty()) {
        partials = ctx_partials(ctx, rows.size() * size_t(cap));
        check_cuda(cudaMemsetAsync(partials, 0, rows.size() * size_t(cap) * sizeof(double), s),
                   "cudaMemsetAsync");
    }

    // Dense custom gates (arity > 2) need their adjoint matrices on the device.
    std::vector<std::vector<double2>> dense;
    for (size_t k = plan.ops.size(); k-- > 0;) {
        const auto &op = plan.ops[k];
        if (op.opcode == ARCQML_OP_CUSTOM_UNITARY && op.qubits.size() > 2)
            dense.push_back(dagger(op.custom, size_t(1) << op.qubits.size()));
    }
    std::vector<const std::vector<double2> *> refs;
    for (auto &d : dense) refs.push_back(&d);
    auto dptr = upload_tables(refs, ctx, s);
    size_t di = 0;

    size_t row = 0;
    for (size_t k = plan.ops.size(); k-- > 0;) {
        const auto &op = plan.ops[k];
        double2 d[3][16];
        int ns = 0;
        for (uint32_t b = 0; b < op.num_bindings; ++b) {
            if (!req[op.parents[b]]) continue;
            DevGate dg = lower(op, LOWER_DERIVATIVE, uint32_t(op.slots[b]), false);
            for (int i = 0; i < 16; ++i) d[ns][i] = dg.m[i];
            ++ns;
        }
        if (ns == 0) {
            DevGate u = lower(op, LOWER_ADJOINT, 0);
            if (u.kind == KIND_DENSE) u.dense = dptr[di++];
            launch_gate(psi, batch, n, u, s);
            launch_gate(lam, batch, n, u, s);
            continue;
        }
        DevGate u = lower(op, LOWER_ADJOINT, 0, false);
        launch_adjoint_raw(psi, lam, batch, n, u, d, ns, partials + row * size_t(cap), s);
        row += size_t(ns);
    }

    if (!rows.empty()) {
        double *sums = ctx_dgrads(ctx, rows.size());
        launch_reduce_rows(partials, uint32_t(rows.size()), cap, sums, s);
        double *h = ctx_hvals(ctx, rows.size());
        check_cuda(cudaMemcpyAsync(h, sums, rows.size() * sizeof(double), cudaMemcpyDeviceToHost, s),
                   "cudaMemcpyAsync (gradients)");
        check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
        for (size_t j = 0; j < rows.size(); ++j) grads_host[rows[j].parent] += 2.0 * h[j];
    }
}

// ------------------------------------------------------------------ observables

void pauli_traversal_tables(uint32_t n, const std::vector<uint64_t> &flips,
                            std::vector<uint64_t> &tables, PauliTraversal &tr) {
    constexpr uint32_t kCoset = 21;  // 2^21 amplitudes = 32 MB of psi per coset
    tables.clear();
    tr = PauliTraversal{};
    if (n <= kCoset) return;
    // qubits 0-5 always (coalesced 1 KB runs); then the qubits the most flip groups act on
    std::vector<std::pair<uint32_t, uint32_t>> cnt;  // (-count, qubit) sorts by count desc
    for (uint32_t q = 6; q < n; ++q) {
        uint32_t c = 0;
        for (uint64_t f : flips) c += uint32_t((f >> q) & 1u);
        cnt.push_back({~c, q});
    }
    std::sort(cnt.begin(), cnt.end());
    std::vector<uint32_t> in, out;
    for (size_t i = 0; i < cnt.size(); ++i)
        (i < kCoset - 6 ? in : out).push_back(cnt[i].second);
    std::sort(in.begin(), in.end());
    std::sort(out.begin(), out.end());
    auto add = [&](const std::vector<uint32_t> &pos) {
        uint32_t made = 0;
        for (size_t j = 0; j < pos.size(); j += 8, ++made)
            for (uint32_t v = 0; v < 256; ++v) {
                uint64_t e = 0;
                for (uint32_t i = 0; i < 8; ++i)
                    if (j + i < pos.size() && ((v >> i) & 1u)) e |= uint64_t(1) << pos[j + i];
                tables.push_back(e);
            }
        return made;
    };
    tr.nb = add(in);
    tr.ntables = tr.nb + add(out);
    tr.coset_bits = kCoset;
}

// Observable tables for k_pauli / the one-kernel step in one host block (layout in PauliTables;
// tab.base left null), followed at `*perm_off` by the traversal tables of an n-qubit state.
std::vector<double2> pack_pauli(const Observable &obs, uint32_t n, PauliTables &tab,
                                PauliTraversal &tr, size_t *perm_off) {
    const size_t ng = obs.groups.size();
    std::vector<uint64_t> gflips(ng), ptab;
    for (size_t g = 0; g < ng; ++g) gflips[g] = obs.groups[g].flip;
    tr = PauliTraversal{};
    pauli_traversal_tables(n, gflips, ptab, tr);
    auto weight = [&](const PauliGroup &grp, uint32_t k) {
        // (-1)^popc((t ^ f) & z) = (-1)^popc(f & z) (-1)^popc(t & z): fold the first factor
        const double c = (__builtin_popcountll(grp.flip & obs.zmask[k]) & 1) ? -obs.coef[k]
                                                                             : obs.coef[k];
        switch (obs.ymod4[k] & 3u) {
        case 0: return make_double2(c, 0.0);
        case 1: return make_double2(0.0, c);
        case 2: return make_double2(-c, 0.0);
        default: return make_double2(0.0, -c);
        }
    };
    std::vector<double2> sw, mw;
    std::vector<uint64_t> sf, sz, mz, mf;
    std::vector<uint32_t> me;
    for (size_t g = 0; g < ng; ++g) {
        const auto &grp = obs.groups[g];
        if (grp.count == 1) {
            sw.push_back(weight(grp, grp.first));
            sf.push_back(grp.flip);
            sz.push_back(obs.zmask[grp.first]);
        } else {
            mf.push_back(grp.flip);
            me.push_back(uint32_t(mw.size()));
            for (uint32_t k = grp.first; k < grp.first + grp.count; ++k) {
                mw.push_back(weight(grp, k));
                mz.push_back(obs.zmask[k]);
            }
        }
    }
    me.push_back(uint32_t(mw.size()));
    tab = PauliTables{};
    size_t off = 0;
    auto place = [&](size_t bytes) {
        const size_t at = off;
        off = (off + bytes + 15) & ~size_t(15);
        return uint32_t(at);
    };
    tab.s_w = place(sw.size() * 16);
    tab.s_f = place(sf.size() * 8);
    tab.s_z = place(sz.size() * 8);
    tab.m_w = place(mw.size() * 16);
    tab.m_z = place(mz.size() * 8);
    tab.m_f = place(mf.size() * 8);
    tab.m_e = place(me.size() * 4);
    tab.bytes = off;
    tab.ns = uint32_t(sw.size());
    tab.nm = uint32_t(mf.size());
    std::vector<double2> pack((off + ptab.size() * 8 + 15) / 16 + 1);
    char *base = reinterpret_cast<char *>(pack.data());
    auto put = [&](uint32_t at, const void *src, size_t bytes) {
        if (bytes) std::memcpy(base + at, src, bytes);
    };
    put(tab.s_w, sw.data(), sw.size() * 16);
    put(tab.s_f, sf.data(), sf.size() * 8);
    put(tab.s_z, sz.data(), sz.size() * 8);
    put(tab.m_w, mw.data(), mw.size() * 16);
    put(tab.m_z, mz.data(), mz.size() * 8);
    put(tab.m_f, mf.data(), mf.size() * 8);
    put(tab.m_e, me.data(), me.size() * 4);
    if (!ptab.empty()) std::memcpy(base + off, ptab.data(), ptab.size() * 8);
    *perm_off = off;
    return pack;
}

bool pauli_tiles_enabled() {
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_PAULI_TILE");
        return !(e && e[0] == '0');
    }();
    return on;
}

void observable_device(Observable &obs, const double2 *psi, double2 *out, size_t batch,
                       uint32_t n, double *values_host, ThreadContext &ctx, cudaStream_t s,
                       bool accumulate) {
    if (obs.num_qubits != n) {
        std::ostringstream m;
        m << "observable acts on " << obs.num_qubits << " qubits, state has " << n;
        fail(m.str());
    }
    if (pauli_tiles_enabled() &&
        observable_tiled(obs, psi, out, n, values_host, accumulate, ctx, s)) {
        const size_t dim = size_t(1) << n;
        for (size_t b = 1; b < batch; ++b)
            observable_tiled(obs, psi + b * dim, out ? out + b * dim : nullptr, n,
                             values_host + b, accumulate, ctx, s);
        return;
    }
    PauliTables tab;
    PauliTraversal tr;
    size_t off = 0;
    std::vector<double2> pack = pack_pauli(obs, n, tab, tr, &off);
    std::vector<const std::vector<double2> *> refs{&pack};
    auto p = upload_tables(refs, ctx, s);
    const char *dbase = reinterpret_cast<const char *>(p[0]);
    if (tr.ntables) tr.tables = reinterpret_cast<const uint64_t *>(dbase + off);
    tab.base = reinterpret_cast<const unsigned char *>(dbase);

    const size_t dim = size_t(1) << n;
    const size_t chunk = 65535;  // grid.y limit
    for (size_t b0 = 0; b0 < batch; b0 += chunk) {
        const size_t rows = std::min(chunk, batch - b0);
        const unsigned bx_cap = adjoint_max_blocks();
        double *partials = ctx_partials(ctx, rows * size_t(bx_cap));
        const unsigned bx = launch_pauli(psi + b0 * dim, out ? out + b0 * dim : nullptr, rows, n,
                                         tab, tr, partials, accumulate, s);
        double *sums = ctx_dgrads(ctx, rows);
        launch_reduce_rows(partials, uint32_t(rows), bx, sums, s);
        double *h = ctx_hvals(ctx, rows);
        check_cuda(cudaMemcpyAsync(h, sums, rows * sizeof(double), cudaMemcpyDeviceToHost, s),
                   "cudaMemcpyAsync (values)");
        check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
        std::memcpy(values_host + b0, h, rows * sizeof(double));
    }
}

void small_step_device(Plan &plan, Observable &obs, const double2 *init, uint32_t n,
                       const uint8_t *req, size_t req_len, double *grads_host, size_t grads_len,
                       double *value_host, double2 *lam0, ThreadContext &ctx, cudaStream_t s) {
    validate_plan_for_state(plan, n);
    check_bindings(plan, req_len, grads_len);
    if (n > kSmallMaxQubits) {
        std::ostringstream m;
        m << "the one-kernel step takes states of at most " << kSmallMaxQubits << " qubits";
        fail(m.str());
    }
    if (obs.num_qubits != n) {
        std::ostringstream m;
        m << "observable acts on " << obs.num_qubits << " qubits, state has " << n;
        fail(m.str());
    }
    // per op: U, U^dagger (dense small form when a slot needs its gradient) and dU/dp per slot
    std::vector<SmallOp> ops(plan.ops.size());
    std::vector<std::vector<double2>> dense;  // matrices of custom gates, forward then dagger
    std::vector<std::pair<size_t, int>> dense_use;  // (op, 0 = u / 1 = ua)
    std::vector<size_t> parents;  // per output row, in reverse-sweep order
    for (size_t k = 0; k < plan.ops.size(); ++k) {
        const OpRecord &op = plan.ops[k];
        SmallOp &so = ops[k];
        std::memset(&so, 0, sizeof(so));
        so.u = lower(op, LOWER_FORWARD, 0);
        if (so.u.kind == KIND_DENSE) {
            if (op.qubits.size() > 4) fail("the one-kernel step takes custom gates on at most 4 qubits");
            dense.push_back(op.custom);
            dense_use.push_back({k, 0});
        }
        int ns = 0;
        for (uint32_t b = 0; b < op.num_bindings; ++b) {
            if (!req[op.parents[b]]) continue;
            DevGate dg = lower(op, LOWER_DERIVATIVE, uint32_t(op.slots[b]), false);
            for (int i = 0; i < 16; ++i) so.d[ns][i] = dg.m[i];
            ++ns;
        }
        so.ns = ns;
        so.ua = lower(op, LOWER_ADJOINT, 0, ns == 0);
        if (so.ua.kind == KIND_DENSE) {
            dense.push_back(dagger(op.custom, size_t(1) << op.qubits.size()));
            dense_use.push_back({k, 1});
        }
        if (ns > 0 && so.ua.kind != KIND_1Q && so.ua.kind != KIND_2Q)
            fail("internal: adjoint step needs a dense small form");
    }
    for (size_t k = plan.ops.size(); k-- > 0;) {
        const OpRecord &op = plan.ops[k];
        for (uint32_t b = 0; b < op.num_bindings; ++b)
            if (req[op.parents[b]]) parents.push_back(op.parents[b]);
    }
    PauliTables tab;
    PauliTraversal tr;
    size_t off = 0;
    std::vector<double2> pauli = pack_pauli(obs, n, tab, tr, &off);
    // one upload: the op table, the custom matrices, the observable tables
    std::vector<double2> optab((ops.size() * sizeof(SmallOp) + 15) / 16 + 1);
    if (!ops.empty()) std::memcpy(optab.data(), ops.data(), ops.size() * sizeof(SmallOp));
    std::vector<const std::vector<double2> *> refs{&optab, &pauli};
    for (auto &d : dense) refs.push_back(&d);
    auto ptrs = upload_tables(refs, ctx, s);
    if (!dense.empty()) {
        // patch the device matrix pointers into the op table on the device copy
        for (size_t j = 0; j < dense.size(); ++j) {
            SmallOp &so = ops[dense_use[j].first];
            (dense_use[j].second == 0 ? so.u : so.ua).dense = ptrs[2 + j];
        }
        check_cuda(cudaMemcpyAsync(const_cast<double2 *>(ptrs[0]), ops.data(),
                                   ops.size() * sizeof(SmallOp), cudaMemcpyHostToDevice, s),
                   "cudaMemcpyAsync (step table)");
    }
    tab.base = reinterpret_cast<const unsigned char *>(ptrs[1]);
    double *out = ctx_dgrads(ctx, 1 + parents.size());
    launch_small_step(init, n, reinterpret_cast<const SmallOp *>(ptrs[0]),
                      uint32_t(ops.size()), tab, out, lam0, s);
    double *h = ctx_hvals(ctx, 1 + parents.size());
    check_cuda(cudaMemcpyAsync(h, out, (1 + parents.size()) * sizeof(double),
                               cudaMemcpyDeviceToHost, s),
               "cudaMemcpyAsync (step results)");
    check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    if (value_host) *value_host = h[0];
    for (size_t j = 0; j < parents.size(); ++j) grads_host[parents[j]] += 2.0 * h[1 + j];
}

namespace {

// Opcodes whose one parameter the device optimizer loop rebuilds on the device: the Pauli
// rotations U = cos(t/2) a1 + sin(t/2) a2 and the phase gates U = a0 + cos(t) a1 + sin(t) a2.
bool loop_rotation(uint32_t opcode) {
    return (opcode >= 11 && opcode <= 13) || (opcode >= 23 && opcode <= 25) ||
           (opcode >= 30 && opcode <= 33);
}
bool loop_phase(uint32_t opcode) { return opcode == 14 || opcode == 22; }

}  // namespace

std::vector<OpRecord> validate_small_adam(const Plan &plan, const Observable &obs, uint32_t n,
                                          const uint8_t *req, size_t req_len,
                                          const double *params, size_t steps, const SmallAdam &h,
                                          const double *energies) {
    validate_plan_for_state(plan, n);
    check_bindings(plan, req_len, req_len);
    if (n > kSmallMaxQubits) {
        std::ostringstream m;
        m << "the optimizer loop takes states of at most " << kSmallMaxQubits << " qubits";
        fail(m.str());
    }
    if (obs.num_qubits != n) {
        std::ostringstream m;
        m << "observable acts on " << obs.num_qubits << " qubits, state has " << n;
        fail(m.str());
    }
    if (req_len == 0 || !req || !params) fail("parameter arrays are empty or null");
    if (req_len > (size_t(1) << 20)) fail("too many parameters for the optimizer loop");
    if (steps == 0 || steps > (size_t(1) << 24)) fail("step count must be in 1..2^24");
    if (!energies) fail("energy buffer is null");
    if (!std::isfinite(h.lr) || !(h.beta1 >= 0.0 && h.beta1 < 1.0) ||
        !(h.beta2 >= 0.0 && h.beta2 < 1.0) || !std::isfinite(h.eps) || h.eps < 0.0 ||
        !std::isfinite(h.weight_decay))
        fail("invalid Adam hyperparameters (finite lr and weight decay, 0 <= beta < 1, eps >= 0)");
    for (size_t p = 0; p < req_len; ++p)
        if (!std::isfinite(params[p])) fail("parameter values must be finite");
    // the plan's ops with every bound slot set from params (the plan itself stays as it is)
    std::vector<OpRecord> rec(plan.ops);
    for (auto &op : rec)
        for (uint32_t b = 0; b < op.num_bindings; ++b) op.params[op.slots[b]] = params[op.parents[b]];
    for (const auto &op : rec) {
        bool trained = false;
        for (uint32_t b = 0; b < op.num_bindings; ++b) trained = trained || req[op.parents[b]];
        if (!trained) continue;
        if (!(loop_rotation(op.opcode) || loop_phase(op.opcode)) || op.num_bindings != 1) {
            std::ostringstream m;
            m << "the optimizer loop rebuilds only one-parameter rotation and phase gates on the "
                 "device; op with opcode "
              << op.opcode << " has a trained parameter";
            fail(m.str());
        }
    }
    return rec;
}

void small_adam_device(const Plan &plan, Observable &obs, const double2 *init, uint32_t n,
                       const uint8_t *req, size_t req_len, double *params, double *adam_m,
                       double *adam_v, uint64_t t0, size_t steps, const SmallAdam &h,
                       double *energies, ThreadContext &ctx, cudaStream_t s) {
    const std::vector<OpRecord> rec =
        validate_small_adam(plan, obs, n, req, req_len, params, steps, h, energies);

    // --- tables: ops (trained ones as dense small forms), their parameter forms, rows
    std::vector<SmallOp> ops(rec.size());
    std::vector<SmallParamOp> pops;
    std::vector<std::vector<double2>> dense;
    std::vector<std::pair<size_t, int>> dense_use;
    for (size_t k = 0; k < rec.size(); ++k) {
        const OpRecord &op = rec[k];
        SmallOp &so = ops[k];
        std::memset(&so, 0, sizeof(so));
        const bool trained = op.num_bindings == 1 && req[op.parents[0]];
        so.u = lower(op, LOWER_FORWARD, 0, !trained);
        if (so.u.kind == KIND_DENSE) {
            if (op.qubits.size() > 4) fail("the optimizer loop takes custom gates on at most 4 qubits");
            dense.push_back(op.custom);
            dense_use.push_back({k, 0});
        }
        so.ns = trained ? 1 : 0;
        so.ua = lower(op, LOWER_ADJOINT, 0, !trained);
        if (so.ua.kind == KIND_DENSE) {
            dense.push_back(dagger(op.custom, size_t(1) << op.qubits.size()));
            dense_use.push_back({k, 1});
        }
        if (!trained) continue;
        if (so.u.kind != KIND_1Q && so.u.kind != KIND_2Q) fail("internal: loop op without a dense form");
        const DevGate dg = lower(op, LOWER_DERIVATIVE, uint32_t(op.slots[0]), false);
        for (int i = 0; i < 16; ++i) so.d[0][i] = dg.m[i];
        SmallParamOp P;
        std::memset(&P, 0, sizeof(P));
        P.op = uint32_t(k);
        P.parent = uint32_t(op.parents[0]);
        P.slot_row = 0;
        P.dim = so.u.kind == KIND_2Q ? 4 : 2;
        OpRecord zero = op;
        zero.params[op.slots[0]] = 0.0;
        const DevGate u0 = lower(zero, LOWER_FORWARD, 0, false);
        const DevGate d0 = lower(zero, LOWER_DERIVATIVE, uint32_t(op.slots[0]), false);
        const int dd = P.dim * P.dim;
        if (loop_rotation(op.opcode)) {  // U(0) = a1, dU/dt(0) = a2 / 2
            P.alpha = 0.5;
            for (int i = 0; i < dd; ++i) {
                P.a1[i] = u0.m[i];
                P.a2[i] = make_double2(2.0 * d0.m[i].x, 2.0 * d0.m[i].y);
            }
        } else {  // diag(1, e^{it}): a2 = dU/dt(0), a1 = U(0) where a2 is non-zero, a0 the rest
            P.alpha = 1.0;
            for (int i = 0; i < dd; ++i) {
                P.a2[i] = d0.m[i];
                const bool on = d0.m[i].x != 0.0 || d0.m[i].y != 0.0;
                P.a1[i] = on ? u0.m[i] : make_double2(0.0, 0.0);
                P.a0[i] = on ? make_double2(0.0, 0.0) : u0.m[i];
            }
        }
        // the forms must reproduce the host's own matrices at the current value
        const double t = op.params[op.slots[0]];
        const double c = std::cos(P.alpha * t), sn = std::sin(P.alpha * t);
        for (int i = 0; i < dd; ++i) {
            const double rx = P.a0[i].x + c * P.a1[i].x + sn * P.a2[i].x;
            const double ry = P.a0[i].y + c * P.a1[i].y + sn * P.a2[i].y;
            if (std::fabs(rx - so.u.m[i].x) > 1e-14 || std::fabs(ry - so.u.m[i].y) > 1e-14)
                fail("internal: optimizer-loop matrix form does not reproduce the gate");
        }
        pops.push_back(P);
    }
    std::vector<uint32_t> row_parent, trained;
    for (size_t k = rec.size(); k-- > 0;)
        if (ops[k].ns) row_parent.push_back(uint32_t(rec[k].parents[0]));
    for (size_t p = 1; p < req_len; ++p)
        if (req[p]) trained.push_back(uint32_t(p));
    const uint32_t np = uint32_t(req_len);
    const size_t smem = small_adam_smem(n, uint32_t(ops.size()), np);
    int dev = 0, optin = 0;
    check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    check_cuda(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev),
               "cudaDeviceGetAttribute");
    if (smem + 1024 > size_t(optin)) {
        std::ostringstream m;
        m << "the optimizer loop keeps the state, the op table and the parameters in shared "
             "memory: "
          << rec.size() << " ops and " << req_len << " parameters need " << smem
          << " bytes, the device allows " << optin;
        fail(m.str());
    }

    // --- one upload: op table, parameter forms, index lists, bias corrections, observable,
    // custom matrices, theta / m / v
    auto words = [](const void *src, size_t bytes) {
        std::vector<double2> v((bytes + 15) / 16 + 1);
        if (bytes) std::memcpy(v.data(), src, bytes);
        return v;
    };
    std::vector<double2> optab = words(ops.data(), ops.size() * sizeof(SmallOp));
    std::vector<double2> ptab = words(pops.data(), pops.size() * sizeof(SmallParamOp));
    std::vector<uint32_t> idx(row_parent);
    idx.insert(idx.end(), trained.begin(), trained.end());
    std::vector<double2> itab = words(idx.data(), idx.size() * sizeof(uint32_t));
    std::vector<double2> bc(steps);
    for (size_t i = 0; i < steps; ++i) {
        const double t = double(t0 + i + 1);
        bc[i] = make_double2(1.0 - std::pow(h.beta1, t), 1.0 - std::pow(h.beta2, t));
    }
    std::vector<double> st(3 * size_t(np), 0.0);
    std::memcpy(st.data(), params, np * sizeof(double));
    if (adam_m) std::memcpy(st.data() + np, adam_m, np * sizeof(double));
    if (adam_v) std::memcpy(st.data() + 2 * size_t(np), adam_v, np * sizeof(double));
    std::vector<double2> stab = words(st.data(), st.size() * sizeof(double));
    PauliTables tab;
    PauliTraversal tr;
    size_t off = 0;
    std::vector<double2> pauli = pack_pauli(obs, n, tab, tr, &off);
    std::vector<const std::vector<double2> *> refs{&optab, &ptab, &itab, &bc, &pauli, &stab};
    for (auto &d : dense) refs.push_back(&d);
    auto ptrs = upload_tables(refs, ctx, s);
    if (!dense.empty()) {
        for (size_t j = 0; j < dense.size(); ++j) {
            SmallOp &so = ops[dense_use[j].first];
            (dense_use[j].second == 0 ? so.u : so.ua).dense = ptrs[6 + j];
        }
        check_cuda(cudaMemcpyAsync(const_cast<double2 *>(ptrs[0]), ops.data(),
                                   ops.size() * sizeof(SmallOp), cudaMemcpyHostToDevice, s),
                   "cudaMemcpyAsync (loop table)");
    }
    tab.base = reinterpret_cast<const unsigned char *>(ptrs[4]);
    const uint32_t *ip = reinterpret_cast<const uint32_t *>(ptrs[2]);
    double *state = reinterpret_cast<double *>(const_cast<double2 *>(ptrs[5]));
    double *dev_e = ctx_dgrads(ctx, steps);
    launch_small_adam(init, n, reinterpret_cast<const SmallOp *>(ptrs[0]), uint32_t(ops.size()),
                      reinterpret_cast<const SmallParamOp *>(ptrs[1]), uint32_t(pops.size()), ip,
                      ip + row_parent.size(), uint32_t(trained.size()), np, tab, h,
                      reinterpret_cast<const double *>(ptrs[3]), uint32_t(steps), state, dev_e, s);
    double *hb = ctx_hvals(ctx, steps + 3 * size_t(np));
    check_cuda(cudaMemcpyAsync(hb, dev_e, steps * sizeof(double), cudaMemcpyDeviceToHost, s),
               "cudaMemcpyAsync (energies)");
    check_cuda(cudaMemcpyAsync(hb + steps, state, 3 * size_t(np) * sizeof(double),
                               cudaMemcpyDeviceToHost, s),
               "cudaMemcpyAsync (parameters)");
    check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    std::memcpy(energies, hb, steps * sizeof(double));
    std::memcpy(params, hb + steps, np * sizeof(double));
    if (adam_m) std::memcpy(adam_m, hb + steps + np, np * sizeof(double));
    if (adam_v) std::memcpy(adam_v, hb + steps + 2 * size_t(np), np * sizeof(double));
}

Observable *make_observable(size_t num_qubits, const double *coef, const uint64_t *flip,
                            const uint64_t *phase, size_t num_terms) {
    if (num_qubits >= 64) fail("observable qubit count must be below 64");
    if (num_terms && (!coef || !flip || !phase)) fail("observable term arrays are null");
    std::unique_ptr<Observable> o(new Observable());
    o->num_qubits = uint32_t(num_qubits);
    const uint64_t limit = num_qubits >= 64 ? ~uint64_t(0) : ((uint64_t(1) << num_qubits) - 1);
    // Group terms by flip mask in first-appearance order; the diagonal group (flip 0) is
    // evaluated with the same code path.
    std::vector<uint64_t> order;
    std::unordered_map<uint64_t, std::vector<size_t>> by_flip;
    for (size_t k = 0; k < num_terms; ++k) {
        if ((flip[k] | phase[k]) & ~limit) fail("Pauli term acts on a qubit outside the observable");
        if (!std::isfinite(coef[k])) fail("Pauli term coefficient is not finite");
        auto it = by_flip.find(flip[k]);
        if (it == by_flip.end()) {
            order.push_back(flip[k]);
            by_flip[flip[k]] = {k};
        } else {
            it->second.push_back(k);
        }
    }
    for (uint64_t f : order) {
        PauliGroup g;
        g.flip = f;
        g.first = uint32_t(o->coef.size());
        g.count = uint32_t(by_flip[f].size());
        for (size_t k : by_flip[f]) {
            o->coef.push_back(coef[k]);
            o->zmask.push_back(phase[k]);
            o->ymod4.push_back(uint32_t(__builtin_popcountll(flip[k] & phase[k]) & 3));
        }
        o->groups.push_back(g);
    }
    return o.release();
}

}  // namespace arcqml
