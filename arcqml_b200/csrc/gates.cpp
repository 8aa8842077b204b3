// gates.cpp — opcode semantics and lowering of ArcQML gates to kernel form.
//
// Gate conventions follow crates/arcqml-circuit/src/gate.rs:4-109: rotations are
// R_P(t) = cos(t/2) I - i sin(t/2) P; U3(t, f, l) = [[c, -e^{il} s], [e^{if} s, e^{i(f+l)} c]];
// fSim(t, f) = [[1,0,0,0],[0,cos t,-i sin t,0],[0,-i sin t,cos t,0],[0,0,0,e^{-if}]];
// local basis index bit j <-> qubits[j]; controlled gates list the control first
// (gate.rs:6-10, circuit_gates_multi.rs:142-179). Descriptor validation mirrors
// crates/arcqml-kernel/src/statevector/single.rs:108-197.
#include <algorithm>
#include <cmath>
#include <sstream>

#include "rt_internal.h"

namespace arcqml {

namespace {

inline double2 C(double re, double im) { return make_double2(re, im); }
inline double2 cmul(double2 a, double2 b) {
    return C(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
inline double2 cscale(double2 a, double s) { return C(a.x * s, a.y * s); }
inline double2 cexpi(double t) { return C(std::cos(t), std::sin(t)); }
inline double2 cconj(double2 a) { return C(a.x, -a.y); }

const char *kNames[39] = {"I",    "X",    "Y",     "Z",   "H",    "S",     "Sdg",  "T",
                          "Tdg",  "SX",   "SXdg",  "Rx",  "Ry",   "Rz",    "Phase", "U3",
                          "CNot", "CY",   "CZ",    "CH",  "CS",   "CT",    "CP",   "CRx",
                          "CRy",  "CRz",  "Swap",  "iSwap", "DCX", "ECR",  "RXX",  "RYY",
                          "RZZ",  "RZX",  "fSim",  "Toffoli", "CSwap", "MCX", "CustomUnitary"};

// 2x2 matrix of a 1-qubit opcode (0..15), row-major.
void one_qubit(uint32_t op, const double *p, double2 u[4]) {
    const double r = 1.0 / std::sqrt(2.0);
    const double c = std::cos(0.5 * p[0]), s = std::sin(0.5 * p[0]);
    switch (op) {
    case 0: u[0] = C(1, 0); u[1] = C(0, 0); u[2] = C(0, 0); u[3] = C(1, 0); break;
    case 1: u[0] = C(0, 0); u[1] = C(1, 0); u[2] = C(1, 0); u[3] = C(0, 0); break;
    case 2: u[0] = C(0, 0); u[1] = C(0, -1); u[2] = C(0, 1); u[3] = C(0, 0); break;
    case 3: u[0] = C(1, 0); u[1] = C(0, 0); u[2] = C(0, 0); u[3] = C(-1, 0); break;
    case 4: u[0] = C(r, 0); u[1] = C(r, 0); u[2] = C(r, 0); u[3] = C(-r, 0); break;
    case 5: u[0] = C(1, 0); u[1] = C(0, 0); u[2] = C(0, 0); u[3] = C(0, 1); break;
    case 6: u[0] = C(1, 0); u[1] = C(0, 0); u[2] = C(0, 0); u[3] = C(0, -1); break;
    case 7: u[0] = C(1, 0); u[1] = C(0, 0); u[2] = C(0, 0); u[3] = C(r, r); break;
    case 8: u[0] = C(1, 0); u[1] = C(0, 0); u[2] = C(0, 0); u[3] = C(r, -r); break;
    case 9: u[0] = C(.5, .5); u[1] = C(.5, -.5); u[2] = C(.5, -.5); u[3] = C(.5, .5); break;
    case 10: u[0] = C(.5, -.5); u[1] = C(.5, .5); u[2] = C(.5, .5); u[3] = C(.5, -.5); break;
    case 11: u[0] = C(c, 0); u[1] = C(0, -s); u[2] = C(0, -s); u[3] = C(c, 0); break;
    case 12: u[0] = C(c, 0); u[1] = C(-s, 0); u[2] = C(s, 0); u[3] = C(c, 0); break;
    case 13: u[0] = C(c, -s); u[1] = C(0, 0); u[2] = C(0, 0); u[3] = C(c, s); break;
    case 14: u[0] = C(1, 0); u[1] = C(0, 0); u[2] = C(0, 0); u[3] = cexpi(p[0]); break;
    case 15:
        u[0] = C(c, 0);
        u[1] = cscale(cexpi(p[2]), -s);
        u[2] = cscale(cexpi(p[1]), s);
        u[3] = cscale(cexpi(p[1] + p[2]), c);
        break;
    default: fail("internal: not a 1-qubit opcode");
    }
}

// 1-qubit opcode applied to the target of a controlled opcode (16..25).
uint32_t controlled_base(uint32_t op) {
    static const uint32_t base[10] = {1, 2, 3, 4, 5, 7, 14, 11, 12, 13};
    return base[op - 16];
}

void two_qubit(uint32_t op, const double *p, double2 m[16]) {
    const double r = 1.0 / std::sqrt(2.0);
    const double c = std::cos(0.5 * p[0]), s = std::sin(0.5 * p[0]);
    for (int i = 0; i < 16; ++i) m[i] = C(0, 0);
    auto M = [&](int i, int j) -> double2 & { return m[i * 4 + j]; };
    switch (op) {
    case 26: M(0, 0) = C(1, 0); M(1, 2) = C(1, 0); M(2, 1) = C(1, 0); M(3, 3) = C(1, 0); break;
    case 27: M(0, 0) = C(1, 0); M(1, 2) = C(0, 1); M(2, 1) = C(0, 1); M(3, 3) = C(1, 0); break;
    case 28: M(0, 0) = C(1, 0); M(1, 3) = C(1, 0); M(2, 1) = C(1, 0); M(3, 2) = C(1, 0); break;
    case 29:
        M(0, 1) = C(r, 0); M(0, 3) = C(0, r); M(1, 0) = C(r, 0); M(1, 2) = C(0, -r);
        M(2, 1) = C(0, r); M(2, 3) = C(r, 0); M(3, 0) = C(0, -r); M(3, 2) = C(r, 0);
        break;
    case 30:
        for (int b = 0; b < 4; ++b) { M(b, b) = C(c, 0); M(b ^ 3, b) = C(0, -s); }
        break;
    case 31:
        for (int b = 0; b < 4; ++b) M(b, b) = C(c, 0);
        M(3, 0) = C(0, s); M(0, 3) = C(0, s); M(2, 1) = C(0, -s); M(1, 2) = C(0, -s);
        break;
    case 32: M(0, 0) = C(c, -s); M(1, 1) = C(c, s); M(2, 2) = C(c, s); M(3, 3) = C(c, -s); break;
    case 33:
        for (int b = 0; b < 4; ++b) { M(b, b) = C(c, 0); M(b ^ 2, b) = C(0, (b & 1) ? s : -s); }
        break;
    case 34:
        M(0, 0) = C(1, 0);
        M(1, 1) = C(std::cos(p[0]), 0); M(1, 2) = C(0, -std::sin(p[0]));
        M(2, 1) = C(0, -std::sin(p[0])); M(2, 2) = C(std::cos(p[0]), 0);
        M(3, 3) = cexpi(-p[1]);
        break;
    default: fail("internal: not a 2-qubit opcode");
    }
}

// -(i/2) P R for dim x dim matrices.
void rot_deriv(const double2 *P, const double2 *R, double2 *out, int dim) {
    for (int i = 0; i < dim; ++i)
        for (int j = 0; j < dim; ++j) {
            double2 acc = C(0, 0);
            for (int k = 0; k < dim; ++k) {
                double2 t = cmul(P[i * dim + k], R[k * dim + j]);
                acc.x += t.x;
                acc.y += t.y;
            }
            out[i * dim + j] = C(0.5 * acc.y, -0.5 * acc.x);
        }
}

void one_qubit_deriv(uint32_t op, const double *p, uint32_t slot, double2 d[4]) {
    double2 P[4], R[4];
    switch (op) {
    case 11: case 12: case 13:
        one_qubit(op - 10, p, P);
        one_qubit(op, p, R);
        rot_deriv(P, R, d, 2);
        return;
    case 14:
        d[0] = d[1] = d[2] = C(0, 0);
        d[3] = cmul(C(0, 1), cexpi(p[0]));
        return;
    case 15: {
        const double c = std::cos(0.5 * p[0]), s = std::sin(0.5 * p[0]);
        if (slot == 0) {
            d[0] = C(-0.5 * s, 0);
            d[1] = cscale(cexpi(p[2]), -0.5 * c);
            d[2] = cscale(cexpi(p[1]), 0.5 * c);
            d[3] = cscale(cexpi(p[1] + p[2]), -0.5 * s);
        } else if (slot == 1) {
            d[0] = d[1] = C(0, 0);
            d[2] = cmul(C(0, 1), cscale(cexpi(p[1]), s));
            d[3] = cmul(C(0, 1), cscale(cexpi(p[1] + p[2]), c));
        } else {
            d[0] = d[2] = C(0, 0);
            d[1] = cmul(C(0, 1), cscale(cexpi(p[2]), -s));
            d[3] = cmul(C(0, 1), cscale(cexpi(p[1] + p[2]), c));
        }
        return;
    }
    default: fail("internal: opcode has no 1-qubit derivative");
    }
}

void two_qubit_deriv(uint32_t op, const double *p, uint32_t slot, double2 d[16]) {
    if (op == 34) {
        for (int i = 0; i < 16; ++i) d[i] = C(0, 0);
        if (slot == 0) {
            d[1 * 4 + 1] = C(-std::sin(p[0]), 0);
            d[1 * 4 + 2] = C(0, -std::cos(p[0]));
            d[2 * 4 + 1] = C(0, -std::cos(p[0]));
            d[2 * 4 + 2] = C(-std::sin(p[0]), 0);
        } else {
            d[3 * 4 + 3] = cmul(C(0, -1), cexpi(-p[1]));
        }
        return;
    }
    static const uint32_t first[4] = {1, 2, 3, 3};   // XX, YY, ZZ, ZX: Pauli on qubits[0]
    static const uint32_t second[4] = {1, 2, 3, 1};  // Pauli on qubits[1]
    double2 a[4], b[4], P[16], R[16];
    const double zero[3] = {0, 0, 0};
    one_qubit(first[op - 30], zero, a);
    one_qubit(second[op - 30], zero, b);
    for (int i = 0; i < 4; ++i)
        for (int j = 0; j < 4; ++j)
            P[i * 4 + j] = cmul(a[(i & 1) * 2 + (j & 1)], b[(i >> 1) * 2 + (j >> 1)]);
    two_qubit(op, p, R);
    rot_deriv(P, R, d, 4);
}

// The gate as (controls, targets, small matrix over the targets).
struct SmallForm {
    std::vector<uint32_t> controls;
    std::vector<uint32_t> targets;
    std::vector<double2> m;  // (2^|targets|)^2, row-major
    bool zero_uncontrolled = false;
    bool identity = false;
};

SmallForm small_form(const OpRecord &op, LowerMode mode, uint32_t slot) {
    SmallForm f;
    const auto &q = op.qubits;
    const uint32_t o = op.opcode;
    const double *p = op.params;
    const bool deriv = mode == LOWER_DERIVATIVE;
    if (deriv && slot >= slot_count(o)) fail("internal: invalid derivative slot");
    if (o <= 15) {
        f.targets = {q[0]};
        f.m.resize(4);
        if (deriv) one_qubit_deriv(o, p, slot, f.m.data());
        else one_qubit(o, p, f.m.data());
        f.identity = (o == 0);
    } else if (o <= 25) {
        f.controls = {q[0]};
        f.targets = {q[1]};
        f.m.resize(4);
        if (deriv) {
            one_qubit_deriv(controlled_base(o), p, 0, f.m.data());
            f.zero_uncontrolled = true;
        } else {
            one_qubit(controlled_base(o), p, f.m.data());
        }
    } else if (o <= 34) {
        f.targets = {q[0], q[1]};
        f.m.resize(16);
        if (deriv) two_qubit_deriv(o, p, slot, f.m.data());
        else two_qubit(o, p, f.m.data());
    } else if (o == 35 || o == 37) {
        for (size_t i = 0; i + 1 < q.size(); ++i) f.controls.push_back(q[i]);
        f.targets = {q.back()};
        f.m = {C(0, 0), C(1, 0), C(1, 0), C(0, 0)};
    } else if (o == 36) {
        f.controls = {q[0]};
        f.targets = {q[1], q[2]};
        f.m.resize(16);
        two_qubit(26, p, f.m.data());
    } else if (o == 38) {
        f.targets = q;
        f.m = op.custom;
    } else {
        fail("internal: unknown opcode");
    }
    if (mode == LOWER_ADJOINT) {
        const size_t dim = size_t(1) << f.targets.size();
        std::vector<double2> t(dim * dim);
        for (size_t i = 0; i < dim; ++i)
            for (size_t j = 0; j < dim; ++j) t[j * dim + i] = cconj(f.m[i * dim + j]);
        f.m.swap(t);
    }
    return f;
}

bool is_diagonal(const std::vector<double2> &m, size_t dim) {
    for (size_t i = 0; i < dim; ++i)
        for (size_t j = 0; j < dim; ++j)
            if (i != j && (m[i * dim + j].x != 0.0 || m[i * dim + j].y != 0.0)) return false;
    return true;
}

void set_positions(DevGate &g, std::vector<uint32_t> pos) {
    std::sort(pos.begin(), pos.end());
    g.npos = int32_t(pos.size());
    for (size_t i = 0; i < pos.size(); ++i) g.positions[i] = uint8_t(pos[i]);
}

}  // namespace

uint32_t slot_count(uint32_t opcode) {
    switch (opcode) {
    case 11: case 12: case 13: case 14: case 22: case 23: case 24: case 25:
    case 30: case 31: case 32: case 33:
        return 1;
    case 15: return 3;
    case 34: return 2;
    default: return 0;
    }
}

static uint32_t builtin_arity(uint32_t op) {
    if (op <= 15) return 1;
    if (op <= 34) return 2;
    if (op <= 36) return 3;
    return 0;
}

OpRecord record_from_descriptor(const GateDescriptor *gate, const size_t *qubits,
                                size_t qubits_len, int64_t num_qubits) {
    if (!gate) fail("gate descriptor is null");
    if (gate->abi_version != ARCQML_RT_ABI_VERSION) {
        std::ostringstream s;
        s << "ArcQML runtime ABI mismatch: expected " << ARCQML_RT_ABI_VERSION << ", got "
          << gate->abi_version;
        fail(s.str());
    }
    if (gate->opcode > ARCQML_OP_CUSTOM_UNITARY) {
        fail("unknown gate opcode " + std::to_string(gate->opcode));
    }
    OpRecord r;
    r.opcode = gate->opcode;
    r.name = (gate->name && gate->name_len)
                 ? std::string(reinterpret_cast<const char *>(gate->name), gate->name_len)
                 : std::string(kNames[gate->opcode]);
    const size_t arity = gate->arity;
    if (r.opcode == ARCQML_OP_MCX) {
        if (arity < 1 || arity > kMaxQubits) fail("gate MCX has invalid arity " + std::to_string(arity));
    } else if (r.opcode == ARCQML_OP_CUSTOM_UNITARY) {
        if (arity < 1 || arity > kMaxDenseArity)
            fail("custom unitary " + r.name + " has unsupported arity " + std::to_string(arity));
        const size_t expected = size_t(1) << (2 * arity);
        if (!gate->matrix || gate->matrix_len != expected) {
            std::ostringstream s;
            s << "custom unitary " << r.name << " of arity " << arity << " expects " << expected
              << " matrix entries, got " << (gate->matrix ? gate->matrix_len : 0);
            fail(s.str());
        }
        r.custom.resize(expected);
        for (size_t i = 0; i < expected; ++i) {
            r.custom[i] = make_double2(gate->matrix[i].re, gate->matrix[i].im);
            if (!std::isfinite(r.custom[i].x) || !std::isfinite(r.custom[i].y))
                fail("custom unitary " + r.name + " has non-finite entries");
        }
    } else if (builtin_arity(r.opcode) != arity) {
        std::ostringstream s;
        s << "gate " << r.name << " has arity " << builtin_arity(r.opcode) << ", descriptor says "
          << arity;
        fail(s.str());
    }
    if (qubits_len != arity) {
        std::ostringstream s;
        s << "gate " << r.name << " expects " << arity << " qubits, got " << qubits_len;
        fail(s.str());
    }
    if (arity && !qubits) fail("qubit list is null");
    for (int i = 0; i < 3; ++i) {
        r.params[i] = gate->parameters[i];
        if (i < int(slot_count(r.opcode)) && !std::isfinite(r.params[i]))
            fail("gate " + r.name + " has a non-finite parameter");
    }
    r.qubits.resize(arity);
    for (size_t i = 0; i < arity; ++i) {
        if (qubits[i] >= kMaxQubits) {
            fail("qubit index " + std::to_string(qubits[i]) + " is out of range");
        }
        r.qubits[i] = uint32_t(qubits[i]);
        for (size_t j = 0; j < i; ++j)
            if (r.qubits[j] == r.qubits[i])
                fail("duplicate qubit index " + std::to_string(qubits[i]));
    }
    if (num_qubits >= 0) check_qubits_for_state(r, uint32_t(num_qubits));
    return r;
}

void check_qubits_for_state(const OpRecord &op, uint32_t num_qubits) {
    for (uint32_t q : op.qubits)
        if (q >= num_qubits) {
            std::ostringstream s;
            s << "qubit index " << q << " is out of range for " << num_qubits << " qubits";
            fail(s.str());
        }
}

DevGate lower(const OpRecord &op, LowerMode mode, uint32_t slot, bool allow_diag) {
    SmallForm f = small_form(op, mode, slot);
    DevGate g;
    std::memset(&g, 0, sizeof(g));
    g.zero_uncontrolled = f.zero_uncontrolled ? 1 : 0;
    for (uint32_t c : f.controls) g.cmask |= uint64_t(1) << c;
    const size_t nt = f.targets.size();
    const size_t dim = size_t(1) << nt;
    g.nt = int32_t(nt);
    if (f.identity && mode != LOWER_DERIVATIVE) {
        g.kind = KIND_NONE;
        return g;
    }
    if (nt > 2) {
        g.kind = KIND_DENSE;
        for (size_t j = 0; j < nt; ++j) g.dense_targets[j] = uint8_t(f.targets[j]);
        set_positions(g, f.targets);
        return g;  // matrix uploaded by the caller (dense_matrix)
    }
    for (size_t j = 0; j < nt; ++j) g.t[j] = int32_t(f.targets[j]);
    std::vector<uint32_t> pos = f.controls;
    for (uint32_t t : f.targets) pos.push_back(t);
    if (allow_diag && is_diagonal(f.m, dim)) {
        g.kind = nt == 1 ? KIND_DIAG1 : KIND_DIAG2;
        for (size_t i = 0; i < dim; ++i) g.m[i] = f.m[i * dim + i];
        // Only the target's |1> phase differs from 1 (Z, S, T, Phase, CZ, CP ...): act on the
        // target=1 half alone by treating the target as one more control.
        if (nt == 1 && !g.zero_uncontrolled && g.m[0].x == 1.0 && g.m[0].y == 0.0) {
            g.cmask |= uint64_t(1) << f.targets[0];
            set_positions(g, pos);
        } else {
            set_positions(g, f.controls);
        }
        return g;
    }
    g.kind = nt == 1 ? KIND_1Q : KIND_2Q;
    for (size_t i = 0; i < dim * dim; ++i) g.m[i] = f.m[i];
    set_positions(g, pos);
    return g;
}

std::vector<double2> dense_matrix(const OpRecord &op, bool derivative, uint32_t slot) {
    SmallForm f = small_form(op, derivative ? LOWER_DERIVATIVE : LOWER_FORWARD, slot);
    const size_t k = op.qubits.size();
    const size_t dim = size_t(1) << k;
    std::vector<double2> out(dim * dim, make_double2(0, 0));
    // Local index over op.qubits; the small form acts on targets when every control is 1.
    std::vector<int> tpos(f.targets.size()), cpos(f.controls.size());
    for (size_t j = 0; j < f.targets.size(); ++j)
        tpos[j] = int(std::find(op.qubits.begin(), op.qubits.end(), f.targets[j]) - op.qubits.begin());
    for (size_t j = 0; j < f.controls.size(); ++j)
        cpos[j] = int(std::find(op.qubits.begin(), op.qubits.end(), f.controls[j]) - op.qubits.begin());
    const size_t tdim = size_t(1) << f.targets.size();
    for (size_t col = 0; col < dim; ++col) {
        bool ctl = true;
        for (int c : cpos) ctl = ctl && ((col >> c) & 1);
        if (!ctl) {
            if (!f.zero_uncontrolled) out[col * dim + col] = make_double2(1, 0);
            continue;
        }
        size_t tin = 0, rest = col;
        for (size_t j = 0; j < tpos.size(); ++j) {
            tin |= ((col >> tpos[j]) & 1) << j;
            rest &= ~(size_t(1) << tpos[j]);
        }
        for (size_t tout = 0; tout < tdim; ++tout) {
            size_t row = rest;
            for (size_t j = 0; j < tpos.size(); ++j) row |= ((tout >> j) & 1) << tpos[j];
            out[row * dim + col] = f.m[tout * tdim + tin];
        }
    }
    return out;
}

}  // namespace arcqml
