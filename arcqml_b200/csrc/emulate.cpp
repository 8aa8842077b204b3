// emulate.cpp — host execution of fused-pass schedules (diagnostic and test support; no CUDA).
//
// Runs the schedule the engine would run for a plan — the same build_schedule call, tile size
// and register bits — on a host state, interpreting every encoded op as the pass kernels do:
// a tile-local bit t is qubit header.S[t], register bit r of a sub-block is tile bit R[r], a
// diagonal qubit is a tile bit or a global position, controls are the tile bits of lcmask and
// the positions of gcmask. Passes the planner scaled (compiled kernels) run their ops in the
// scaled unit-diagonal forms with the pass factor multiplied in at the end and the gradient
// factors of the matrix table; the others run the plain forms. Adjoint passes take, per op,
// the Pauli-rotation gradient before U^dagger, U^dagger on psi, a generic slot gradient on
// (U^dagger psi, lambda), then U^dagger on lambda. A test compares the result with the oracle
// to check the planner's encoding without a GPU.
#include <complex>
#include <cstring>
#include <vector>

#include "launch.h"
#include "planner.h"
#include "rt_internal.h"

namespace arcqml {
namespace {

using cplx = std::complex<double>;

cplx cx(double2 a) { return cplx(a.x, a.y); }

struct Emu {
    std::vector<cplx> &psi;
    std::vector<cplx> *lam;  // adjoint only
    uint32_t n;
};

uint32_t reg_qubit(const Step &st, const SubBlock &sb, int r) {
    return st.header.S[sb.R[r]];
}
uint32_t diag_qubit(const Step &st, const FOp &o, int slot) {
    return o.dq_in_tile[slot] ? st.header.S[o.dq_pos[slot]] : o.dq_pos[slot];
}
uint64_t control_mask(const Step &st, const FOp &o) {
    uint64_t m = o.gcmask;
    for (uint32_t t = 0; t < st.header.k; ++t)
        if ((o.lcmask >> t) & 1u) m |= uint64_t(1) << st.header.S[t];
    return m;
}

// An op as (qubits, dense D x D matrix or diagonal, controls); matrix bit j <-> qubits[j].
struct Shape {
    std::vector<uint32_t> q;
    bool diag = false;
    uint64_t ctrl = 0;
};

// CZ-type sign flips (FC_SIGN_*): -1 where both of their qubits are 1; the classifier keeps
// them in rb0 / rb1 / the diagonal slots, and the sign code ignores the control masks.
bool sign_shape(const Step &st, const SubBlock &sb, const FOp &o, Shape &s) {
    if (o.code == FC_SIGN_RR) s.q = {reg_qubit(st, sb, o.rb0), reg_qubit(st, sb, o.rb1)};
    else if (o.code == FC_SIGN_RC) s.q = {reg_qubit(st, sb, o.rb0), diag_qubit(st, o, 0)};
    else if (o.code == FC_SIGN_CC) s.q = {diag_qubit(st, o, 0), diag_qubit(st, o, 1)};
    else return false;
    s.diag = true;
    s.ctrl = 0;
    return true;
}

// X and CNOT fast paths (FC_X / FC_CX_*): the target is register bit rb0; the control (if any)
// is register bit rb1 or the diagonal slot 0, and the control masks are not read.
bool x_shape(const Step &st, const SubBlock &sb, const FOp &o, Shape &s) {
    if (o.code != FC_X && o.code != FC_CX_RR && o.code != FC_CX_CR) return false;
    s.q = {reg_qubit(st, sb, o.rb0)};
    s.diag = false;
    s.ctrl = 0;
    if (o.code == FC_CX_RR) s.ctrl = uint64_t(1) << reg_qubit(st, sb, o.rb1);
    if (o.code == FC_CX_CR) s.ctrl = uint64_t(1) << diag_qubit(st, o, 0);
    return true;
}

Shape shape_of(const Step &st, const SubBlock &sb, const FOp &o) {
    Shape s;
    if (sign_shape(st, sb, o, s)) return s;
    if (x_shape(st, sb, o, s)) return s;
    s.ctrl = control_mask(st, o);
    switch (o.kind) {
    case FK_D1: s.q = {diag_qubit(st, o, 0)}; s.diag = true; break;
    case FK_D2: s.q = {diag_qubit(st, o, 0), diag_qubit(st, o, 1)}; s.diag = true; break;
    case FK_M4: s.q = {reg_qubit(st, sb, o.rb0), reg_qubit(st, sb, o.rb1)}; break;
    default: s.q = {reg_qubit(st, sb, o.rb0)}; break;
    }
    return s;
}

// The op's U (plain form) as D x D, or D diagonal entries.
std::vector<cplx> plain_matrix(const FOp &o, const double2 *m) {
    switch (o.kind) {
    case FK_RX: return {cplx(m[0].x, 0), cplx(0, -m[0].y), cplx(0, -m[0].y), cplx(m[0].x, 0)};
    case FK_RY: return {cplx(m[0].x, 0), cplx(-m[0].y, 0), cplx(m[0].y, 0), cplx(m[0].x, 0)};
    case FK_D1: return {cx(m[0]), cx(m[1])};
    case FK_D2: case FK_M2: return {cx(m[0]), cx(m[1]), cx(m[2]), cx(m[3])};
    default: {
        std::vector<cplx> u(16);
        for (int i = 0; i < 16; ++i) u[i] = cx(m[i]);
        return u;
    }
    }
}

// The scaled unit-diagonal form of an RX / RY / one-qubit diagonal op: tau = mats[soff].x.
std::vector<cplx> scaled_matrix(const FOp &o, double tau) {
    if (o.kind == FK_RX) return {1.0, cplx(0, -tau), cplx(0, -tau), 1.0};
    if (o.kind == FK_RY) return {1.0, -tau, tau, 1.0};
    return {cplx(1.0, -tau), cplx(1.0, tau)};
}

// Member amplitudes of every group of the shape (controls satisfied), visited as f(indices).
template <class F>
void for_groups(uint32_t n, const Shape &s, F f) {
    uint64_t qmask = 0;
    for (uint32_t q : s.q) qmask |= uint64_t(1) << q;
    const size_t D = size_t(1) << s.q.size();
    std::vector<uint64_t> idx(D);
    for (uint64_t base = 0; base < (uint64_t(1) << n); ++base) {
        if ((base & qmask) || (base & s.ctrl) != s.ctrl) continue;
        for (size_t j = 0; j < D; ++j) {
            uint64_t i = base;
            for (size_t b = 0; b < s.q.size(); ++b)
                if ((j >> b) & 1u) i |= uint64_t(1) << s.q[b];
            idx[j] = i;
        }
        f(idx);
    }
}

void apply(std::vector<cplx> &a, uint32_t n, const Shape &s, const std::vector<cplx> &u) {
    const size_t D = size_t(1) << s.q.size();
    std::vector<cplx> x(D);
    for_groups(n, s, [&](const std::vector<uint64_t> &idx) {
        for (size_t j = 0; j < D; ++j) x[j] = a[idx[j]];
        for (size_t r = 0; r < D; ++r) {
            if (s.diag) {
                a[idx[r]] = u[r] * x[r];
                continue;
            }
            cplx acc = 0.0;
            for (size_t c = 0; c < D; ++c) acc += u[r * D + c] * x[c];
            a[idx[r]] = acc;
        }
    });
}

// sum over the controlled groups of Re<lam| M |psi> (M dense D x D or diagonal)
double re_inner(const std::vector<cplx> &l, const std::vector<cplx> &p, uint32_t n,
                const Shape &s, const std::vector<cplx> &m) {
    const size_t D = size_t(1) << s.q.size();
    double z = 0.0;
    for_groups(n, s, [&](const std::vector<uint64_t> &idx) {
        for (size_t r = 0; r < D; ++r) {
            cplx y = 0.0;
            if (s.diag) y = m[r] * p[idx[r]];
            else
                for (size_t c = 0; c < D; ++c) y += m[r * D + c] * p[idx[c]];
            z += (std::conj(l[idx[r]]) * y).real();
        }
    });
    return z;
}

// Im<lam| P |psi> of the op's Pauli rotation over the controlled groups.
double pauli_grad(const std::vector<cplx> &l, const std::vector<cplx> &p, uint32_t n,
                  const Shape &s, uint8_t gkind) {
    std::vector<cplx> P;
    Shape t = s;
    if (gkind == GK_PX) P = {0.0, 1.0, 1.0, 0.0};
    else if (gkind == GK_PY) P = {0.0, cplx(0, -1), cplx(0, 1), 0.0};
    else {
        t.diag = true;
        P = {1.0, -1.0};
    }
    // Im<l|P p> = Re<l| (-i P) p>
    for (auto &x : P) x *= cplx(0, -1);
    return re_inner(l, p, n, t, P);
}

void run_step(const Step &st, bool adjoint, Emu &E, const uint8_t *req, double *grads) {
    const uint32_t n = E.n;
    if (!st.is_pass) {  // a custom gate on more than two targets
        const OpRecord &op = *st.dense_op;
        std::vector<double2> u = dense_matrix(op, false, 0);
        const size_t D = size_t(1) << op.qubits.size();
        Shape s;
        s.q = op.qubits;
        std::vector<cplx> m(D * D);
        for (size_t r = 0; r < D; ++r)
            for (size_t c = 0; c < D; ++c)
                m[r * D + c] = adjoint ? std::conj(cx(u[c * D + r])) : cx(u[r * D + c]);
        apply(E.psi, n, s, m);
        if (adjoint) apply(*E.lam, n, s, m);
        return;
    }
    (void)req;
    std::vector<double> acc(st.parents.size(), 0.0);
    for (const SubBlock &sb : st.subs) {
        for (uint32_t oi = sb.op_begin; oi < sb.op_end; ++oi) {
            const FOp &o = st.ops[oi];
            const double2 *m = st.mats.data() + o.moff;
            const Shape s = shape_of(st, sb, o);
            const bool sc = st.scaled && o.sform;
            const bool sign = o.code == FC_SIGN_RR || o.code == FC_SIGN_RC || o.code == FC_SIGN_CC;
            const bool xop = o.code == FC_X || o.code == FC_CX_RR || o.code == FC_CX_CR;
            const std::vector<cplx> u =
                sign ? std::vector<cplx>{1.0, 1.0, 1.0, -1.0}
                     : xop ? std::vector<cplx>{0.0, 1.0, 1.0, 0.0}
                           : (sc ? scaled_matrix(o, st.mats[o.soff].x) : plain_matrix(o, m));
            Shape su = s;
            if (sc && o.kind == FK_D1) su.diag = true;
            if (adjoint && (o.gkind == GK_PX || o.gkind == GK_PY || o.gkind == GK_PZ)) {
                const double f = (st.scaled && o.sgrad) ? st.mats[o.soff].y : 0.5;
                Shape ps = s;
                if (o.gkind == GK_PZ) ps.q = {diag_qubit(st, o, 0)};
                acc[o.acc[0]] += f * pauli_grad(*E.lam, E.psi, n, ps, o.gkind);
            }
            apply(E.psi, n, su, u);
            if (adjoint && o.gkind == GK_GENERIC) {
                // the op keeps its plain form, so psi and lambda both carry the pass factor
                // sigma from before it: the stored sum times |sigma|^2 = 2 * mats[soff].y
                const double f = (st.scaled && o.sgrad) ? 2.0 * st.mats[o.soff].y : 1.0;
                static const int ulen[6] = {4, 1, 1, 2, 4, 16};
                const int dl = o.kind == FK_D1 ? 2 : (o.kind == FK_D2 ? 4 : (o.kind == FK_M4 ? 16 : 4));
                for (uint32_t sl = 0; sl < o.nslots; ++sl) {
                    const double2 *d = m + ulen[o.kind] + sl * dl;
                    std::vector<cplx> dm(dl);
                    for (int i = 0; i < dl; ++i) dm[i] = cx(d[i]);
                    Shape ds = s;
                    ds.diag = (o.kind == FK_D1 || o.kind == FK_D2);
                    acc[o.acc[sl]] += f * re_inner(*E.lam, E.psi, n, ds, dm);
                }
            }
            if (adjoint) apply(*E.lam, n, su, u);
        }
    }
    if (st.scaled) {
        const cplx sigma = cx(st.mats[st.sfin]);
        for (auto &x : E.psi) x *= sigma;
        if (adjoint)
            for (auto &x : *E.lam) x *= sigma;
    }
    for (size_t a = 0; a < acc.size(); ++a) grads[st.parents[a]] += 2.0 * acc[a];
    for (const auto &al : st.alias) grads[al.second] += 2.0 * acc[al.first];
}

}  // namespace

void emulate_schedule(const Plan &plan, uint32_t n, bool adjoint, double2 *psi, double2 *lam,
                      const uint8_t *req, size_t req_len, double *grads, size_t grads_len) {
    validate_plan_for_state(plan, n);
    if (n < kFusedMinQubits) fail("plans below 8 qubits run no fused passes");
    if (n > 22) fail("the schedule emulator takes states of at most 22 qubits");
    if (adjoint) check_bindings(plan, req_len, grads_len);
    const uint32_t k = fused_k(n, adjoint);
    const uint32_t rb = adjoint ? fused_rb(k, true) : forward_rb(k);
    Schedule sch = build_schedule(plan, n, adjoint, req, adjoint, k, rb);
    const size_t dim = size_t(1) << n;
    std::vector<cplx> p(dim), l;
    for (size_t i = 0; i < dim; ++i) p[i] = cx(psi[i]);
    if (adjoint) {
        l.resize(dim);
        for (size_t i = 0; i < dim; ++i) l[i] = cx(lam[i]);
    }
    Emu E{p, adjoint ? &l : nullptr, n};
    for (const Step &st : sch.steps) run_step(st, adjoint, E, req, grads);
    for (size_t i = 0; i < dim; ++i) psi[i] = make_double2(p[i].real(), p[i].imag());
    if (adjoint)
        for (size_t i = 0; i < dim; ++i) lam[i] = make_double2(l[i].real(), l[i].imag());
}

}  // namespace arcqml
