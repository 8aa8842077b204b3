/*
 * oracle.c — CPU f64 restatement of ArcQML's statevector path (TEST INFRASTRUCTURE ONLY).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline may load this file's
 * library; the product runtime never does. See oracle.h for the parity pin.
 *
 * What each part restates:
 *   gate matrices        crates/arcqml-circuit/src/gate.rs:4-109 (doc formulas), opcode map
 *                        crates/arcqml-kernel/src/statevector/single.rs:199-256
 *   derivative slots     crates/arcqml-kernel/src/statevector/single.rs:169-197
 *   Pauli observable     crates/arcqml-observable/src/compiled_hamiltonian.rs:30-210,
 *                        same term compile, phase rule and summation order
 *   adjoint sweep        docs/ArcQML技术手册.md:426-462, loop order of
 *                        crates/arcqml-unitary/src/fit/adjoint.rs:19-66, buffer contract of
 *                        crates/arcqml-sim/src/statevector/execution/adjoint/single.rs:104-163
 *   batch rows           crates/arcqml-sim/src/statevector/execution/adjoint/row_major.rs:108-162
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- complex helpers */

static inline oc128 cmk(double re, double im) {
    oc128 z;
    z.re = re;
    z.im = im;
    return z;
}
static inline oc128 cmul(oc128 a, oc128 b) {
    return cmk(a.re * b.re - a.im * b.im, a.re * b.im + a.im * b.re);
}
static inline oc128 cadd(oc128 a, oc128 b) { return cmk(a.re + b.re, a.im + b.im); }
static inline oc128 cconj(oc128 a) { return cmk(a.re, -a.im); }
static inline oc128 cscale(oc128 a, double s) { return cmk(a.re * s, a.im * s); }
static inline oc128 cexpi(double t) { return cmk(cos(t), sin(t)); }

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oracle_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ---------------------------------------------------------------- gate matrices */

static void identity(oc128 *m, size_t dim) {
    memset(m, 0, dim * dim * sizeof(oc128));
    for (size_t i = 0; i < dim; ++i) m[i * dim + i] = cmk(1.0, 0.0);
}

/* 2x2 single-qubit matrix of a built-in opcode, or -1 if the opcode is not 1-qubit. */
static int one_qubit(uint32_t op, const double *p, oc128 u[4]) {
    const double r = 1.0 / sqrt(2.0);
    double c, s;
    switch (op) {
    case 0: u[0] = cmk(1, 0); u[1] = cmk(0, 0); u[2] = cmk(0, 0); u[3] = cmk(1, 0); return 0;
    case 1: u[0] = cmk(0, 0); u[1] = cmk(1, 0); u[2] = cmk(1, 0); u[3] = cmk(0, 0); return 0;
    case 2: u[0] = cmk(0, 0); u[1] = cmk(0, -1); u[2] = cmk(0, 1); u[3] = cmk(0, 0); return 0;
    case 3: u[0] = cmk(1, 0); u[1] = cmk(0, 0); u[2] = cmk(0, 0); u[3] = cmk(-1, 0); return 0;
    case 4: u[0] = cmk(r, 0); u[1] = cmk(r, 0); u[2] = cmk(r, 0); u[3] = cmk(-r, 0); return 0;
    case 5: u[0] = cmk(1, 0); u[1] = cmk(0, 0); u[2] = cmk(0, 0); u[3] = cmk(0, 1); return 0;
    case 6: u[0] = cmk(1, 0); u[1] = cmk(0, 0); u[2] = cmk(0, 0); u[3] = cmk(0, -1); return 0;
    case 7: u[0] = cmk(1, 0); u[1] = cmk(0, 0); u[2] = cmk(0, 0); u[3] = cmk(r, r); return 0;
    case 8: u[0] = cmk(1, 0); u[1] = cmk(0, 0); u[2] = cmk(0, 0); u[3] = cmk(r, -r); return 0;
    case 9:
        u[0] = cmk(0.5, 0.5); u[1] = cmk(0.5, -0.5); u[2] = cmk(0.5, -0.5); u[3] = cmk(0.5, 0.5);
        return 0;
    case 10:
        u[0] = cmk(0.5, -0.5); u[1] = cmk(0.5, 0.5); u[2] = cmk(0.5, 0.5); u[3] = cmk(0.5, -0.5);
        return 0;
    case 11: /* RX = cI - i s X */
        c = cos(0.5 * p[0]); s = sin(0.5 * p[0]);
        u[0] = cmk(c, 0); u[1] = cmk(0, -s); u[2] = cmk(0, -s); u[3] = cmk(c, 0);
        return 0;
    case 12: /* RY = cI - i s Y */
        c = cos(0.5 * p[0]); s = sin(0.5 * p[0]);
        u[0] = cmk(c, 0); u[1] = cmk(-s, 0); u[2] = cmk(s, 0); u[3] = cmk(c, 0);
        return 0;
    case 13: /* RZ = diag(e^{-i t/2}, e^{i t/2}) */
        c = cos(0.5 * p[0]); s = sin(0.5 * p[0]);
        u[0] = cmk(c, -s); u[1] = cmk(0, 0); u[2] = cmk(0, 0); u[3] = cmk(c, s);
        return 0;
    case 14:
        u[0] = cmk(1, 0); u[1] = cmk(0, 0); u[2] = cmk(0, 0); u[3] = cexpi(p[0]);
        return 0;
    case 15: /* U3(theta, phi, lambda), gate.rs:43-47 */
        c = cos(0.5 * p[0]); s = sin(0.5 * p[0]);
        u[0] = cmk(c, 0);
        u[1] = cscale(cexpi(p[2]), -s);
        u[2] = cscale(cexpi(p[1]), s);
        u[3] = cscale(cexpi(p[1] + p[2]), c);
        return 0;
    default:
        return -1;
    }
}

/* Target matrix of the controlled 2-qubit family (control = local bit 0, target = bit 1). */
static int controlled_target(uint32_t op, const double *p, oc128 u[4]) {
    switch (op) {
    case 16: return one_qubit(1, p, u);  /* CNOT */
    case 17: return one_qubit(2, p, u);  /* CY */
    case 18: return one_qubit(3, p, u);  /* CZ */
    case 19: return one_qubit(4, p, u);  /* CH */
    case 20: return one_qubit(5, p, u);  /* CS */
    case 21: return one_qubit(7, p, u);  /* CT */
    case 22: return one_qubit(14, p, u); /* CPHASE = controlled PHASE */
    case 23: return one_qubit(11, p, u); /* CRX */
    case 24: return one_qubit(12, p, u); /* CRY */
    case 25: return one_qubit(13, p, u); /* CRZ */
    default: return -1;
    }
}

/* Embed a 2x2 target matrix as the control-1 block of a 4x4 (index = c + 2 t). The control-0
 * block is `zero_block ? 0 : I`. */
static void embed_controlled(const oc128 u[4], oc128 *m, int zero_block) {
    memset(m, 0, 16 * sizeof(oc128));
    if (!zero_block) {
        m[0 * 4 + 0] = cmk(1, 0);
        m[2 * 4 + 2] = cmk(1, 0);
    }
    m[1 * 4 + 1] = u[0];
    m[1 * 4 + 3] = u[1];
    m[3 * 4 + 1] = u[2];
    m[3 * 4 + 3] = u[3];
}

/* 4x4 of the 2-target family on local index b = bit(q0) + 2 bit(q1). */
static int two_qubit(uint32_t op, const double *p, oc128 *m) {
    const double r = 1.0 / sqrt(2.0);
    double c, s;
    memset(m, 0, 16 * sizeof(oc128));
#define M(i, j) m[(i) * 4 + (j)]
    switch (op) {
    case 26: /* SWAP */
        M(0, 0) = cmk(1, 0); M(1, 2) = cmk(1, 0); M(2, 1) = cmk(1, 0); M(3, 3) = cmk(1, 0);
        return 0;
    case 27: /* ISWAP: |01> -> i|10>, |10> -> i|01> */
        M(0, 0) = cmk(1, 0); M(1, 2) = cmk(0, 1); M(2, 1) = cmk(0, 1); M(3, 3) = cmk(1, 0);
        return 0;
    case 28: /* DCX = CNOT(q0->q1) then CNOT(q1->q0) */
        M(0, 0) = cmk(1, 0); M(1, 3) = cmk(1, 0); M(2, 1) = cmk(1, 0); M(3, 2) = cmk(1, 0);
        return 0;
    case 29: /* ECR (echoed cross-resonance), little-endian local index */
        M(0, 1) = cmk(r, 0); M(0, 3) = cmk(0, r);
        M(1, 0) = cmk(r, 0); M(1, 2) = cmk(0, -r);
        M(2, 1) = cmk(0, r); M(2, 3) = cmk(r, 0);
        M(3, 0) = cmk(0, -r); M(3, 2) = cmk(r, 0);
        return 0;
    case 30: /* RXX = cI - i s XX */
        c = cos(0.5 * p[0]); s = sin(0.5 * p[0]);
        for (int b = 0; b < 4; ++b) { M(b, b) = cmk(c, 0); M(b ^ 3, b) = cmk(0, -s); }
        return 0;
    case 31: /* RYY = cI - i s YY; YY|00>=-|11>, YY|01>=|10> */
        c = cos(0.5 * p[0]); s = sin(0.5 * p[0]);
        for (int b = 0; b < 4; ++b) M(b, b) = cmk(c, 0);
        M(3, 0) = cmk(0, s); M(0, 3) = cmk(0, s); M(2, 1) = cmk(0, -s); M(1, 2) = cmk(0, -s);
        return 0;
    case 32: /* RZZ = cI - i s ZZ */
        c = cos(0.5 * p[0]); s = sin(0.5 * p[0]);
        M(0, 0) = cmk(c, -s); M(1, 1) = cmk(c, s); M(2, 2) = cmk(c, s); M(3, 3) = cmk(c, -s);
        return 0;
    case 33: /* RZX = cI - i s Z(q0) X(q1); ZX|b> = (-1)^{b0} |b ^ 2> */
        c = cos(0.5 * p[0]); s = sin(0.5 * p[0]);
        for (int b = 0; b < 4; ++b) {
            M(b, b) = cmk(c, 0);
            M(b ^ 2, b) = cmk(0, (b & 1) ? s : -s);
        }
        return 0;
    case 34: /* FSIM(theta, phi), gate.rs:86-90 */
        M(0, 0) = cmk(1, 0);
        M(1, 1) = cmk(cos(p[0]), 0); M(1, 2) = cmk(0, -sin(p[0]));
        M(2, 1) = cmk(0, -sin(p[0])); M(2, 2) = cmk(cos(p[0]), 0);
        M(3, 3) = cexpi(-p[1]);
        return 0;
    default:
        return -1;
    }
#undef M
}

static size_t builtin_arity(uint32_t op) {
    if (op <= 15) return 1;
    if (op <= 34) return 2;
    if (op <= 36) return 3;
    return 0; /* MCX and custom carry their own arity */
}

int oracle_gate_matrix(uint32_t op, uint32_t arity, const double *p, const oc128 *custom,
                       oc128 *out) {
    if (arity == 0 || arity > ORACLE_MAX_DENSE_ARITY) return -1;
    const size_t dim = (size_t)1 << arity;
    if (op == 38) {
        if (!custom) return -1;
        memcpy(out, custom, dim * dim * sizeof(oc128));
        return 0;
    }
    if (op > 38) return -1;
    if (op != 37 && builtin_arity(op) != arity) return -1;
    oc128 u[4];
    if (op <= 15) return one_qubit(op, p, out);
    if (controlled_target(op, p, u) == 0) {
        embed_controlled(u, out, 0);
        return 0;
    }
    if (two_qubit(op, p, out) == 0) return 0;
    identity(out, dim);
    if (op == 35 || op == 37) { /* TOFFOLI / MCX: X on the last qubit iff every control is 1 */
        const size_t ctl = dim / 2 - 1; /* all control bits set, target bit clear */
        const size_t a = ctl, b = ctl | (dim / 2);
        out[a * dim + a] = cmk(0, 0);
        out[b * dim + b] = cmk(0, 0);
        out[a * dim + b] = cmk(1, 0);
        out[b * dim + a] = cmk(1, 0);
        return 0;
    }
    if (op == 36) { /* CSWAP: control bit 0, swap bits 1 and 2 */
        const size_t a = 3, b = 5;
        out[a * dim + a] = cmk(0, 0);
        out[b * dim + b] = cmk(0, 0);
        out[a * dim + b] = cmk(1, 0);
        out[b * dim + a] = cmk(1, 0);
        return 0;
    }
    return -1;
}

/* Number of differentiable slots, crates/arcqml-kernel/src/statevector/single.rs:169-197. */
static size_t slot_count(uint32_t op) {
    switch (op) {
    case 11: case 12: case 13: case 14: case 22: case 23: case 24: case 25:
    case 30: case 31: case 32: case 33:
        return 1;
    case 15: return 3;
    case 34: return 2;
    default: return 0;
    }
}

/* -(i/2) P R for a Pauli-rotation matrix R of dimension dim with P given as a matrix. */
static void rotation_derivative(const oc128 *pauli, const oc128 *rot, oc128 *out, size_t dim) {
    for (size_t i = 0; i < dim; ++i)
        for (size_t j = 0; j < dim; ++j) {
            oc128 acc = cmk(0, 0);
            for (size_t k = 0; k < dim; ++k) acc = cadd(acc, cmul(pauli[i * dim + k], rot[k * dim + j]));
            out[i * dim + j] = cmk(0.5 * acc.im, -0.5 * acc.re); /* -(i/2) * acc */
        }
}

int oracle_derivative_matrix(uint32_t op, uint32_t arity, const double *p, size_t slot,
                             oc128 *out) {
    if (slot >= slot_count(op) || builtin_arity(op) != arity) return -1;
    const double zero[3] = {0, 0, 0};
    oc128 u[4], pm[16], rm[16], d[4];
    (void)zero;
    switch (op) {
    case 11: case 12: case 13: { /* 1-qubit rotations: -(i/2) P R */
        oc128 pu[4];
        one_qubit(op - 10, p, pu); /* X, Y, Z = 1, 2, 3 */
        one_qubit(op, p, u);
        rotation_derivative(pu, u, out, 2);
        return 0;
    }
    case 14: /* PHASE: diag(0, i e^{i t}) */
        out[0] = cmk(0, 0); out[1] = cmk(0, 0); out[2] = cmk(0, 0);
        out[3] = cmul(cmk(0, 1), cexpi(p[0]));
        return 0;
    case 15: { /* U3 elementwise */
        const double c = cos(0.5 * p[0]), s = sin(0.5 * p[0]);
        if (slot == 0) {
            out[0] = cmk(-0.5 * s, 0);
            out[1] = cscale(cexpi(p[2]), -0.5 * c);
            out[2] = cscale(cexpi(p[1]), 0.5 * c);
            out[3] = cscale(cexpi(p[1] + p[2]), -0.5 * s);
        } else if (slot == 1) {
            out[0] = cmk(0, 0);
            out[1] = cmk(0, 0);
            out[2] = cmul(cmk(0, 1), cscale(cexpi(p[1]), s));
            out[3] = cmul(cmk(0, 1), cscale(cexpi(p[1] + p[2]), c));
        } else {
            out[0] = cmk(0, 0);
            out[1] = cmul(cmk(0, 1), cscale(cexpi(p[2]), -s));
            out[2] = cmk(0, 0);
            out[3] = cmul(cmk(0, 1), cscale(cexpi(p[1] + p[2]), c));
        }
        return 0;
    }
    case 22: /* CPHASE: diag(0, 0, 0, i e^{i t}); the control-0 block is zero */
        one_qubit(14, p, u);
        oracle_derivative_matrix(14, 1, p, 0, d);
        embed_controlled(d, out, 1);
        return 0;
    case 23: case 24: case 25: /* controlled rotations: control-0 block zero */
        oracle_derivative_matrix(op - 12, 1, p, 0, d);
        embed_controlled(d, out, 1);
        return 0;
    case 30: case 31: case 32: case 33: { /* two-qubit Pauli rotations */
        oc128 a[4], b[4];
        static const uint32_t first[4] = {1, 2, 3, 3};  /* XX, YY, ZZ, ZX: op on q0 */
        static const uint32_t second[4] = {1, 2, 3, 1}; /* op on q1 */
        one_qubit(first[op - 30], p, a);
        one_qubit(second[op - 30], p, b);
        /* (P0 on bit 0) (x) (P1 on bit 1): M[(i0 + 2 i1)][(j0 + 2 j1)] = a[i0][j0] b[i1][j1] */
        for (int i = 0; i < 4; ++i)
            for (int j = 0; j < 4; ++j)
                pm[i * 4 + j] = cmul(a[(i & 1) * 2 + (j & 1)], b[(i >> 1) * 2 + (j >> 1)]);
        two_qubit(op, p, rm);
        rotation_derivative(pm, rm, out, 4);
        return 0;
    }
    case 34: /* FSIM */
        memset(out, 0, 16 * sizeof(oc128));
        if (slot == 0) {
            out[1 * 4 + 1] = cmk(-sin(p[0]), 0);
            out[1 * 4 + 2] = cmk(0, -cos(p[0]));
            out[2 * 4 + 1] = cmk(0, -cos(p[0]));
            out[2 * 4 + 2] = cmk(-sin(p[0]), 0);
        } else {
            out[3 * 4 + 3] = cmul(cmk(0, -1), cexpi(-p[1]));
        }
        return 0;
    default:
        return -1;
    }
}

/* ---------------------------------------------------------------- state kernels */

/* Deposit the bits of `j` (k bits) at the positions qubits[0..k) of a zero index. */
static inline size_t scatter(size_t j, uint32_t k, const size_t *qubits) {
    size_t idx = 0;
    for (uint32_t b = 0; b < k; ++b)
        if ((j >> b) & 1) idx |= (size_t)1 << qubits[b];
    return idx;
}

/* Insert zero bits at the sorted positions into `g`. */
static inline size_t insert_zeros(size_t g, uint32_t k, const size_t *sorted) {
    for (uint32_t b = 0; b < k; ++b) {
        const size_t low = g & (((size_t)1 << sorted[b]) - 1);
        g = ((g >> sorted[b]) << (sorted[b] + 1)) | low;
    }
    return g;
}

static void sort_positions(const size_t *q, uint32_t k, size_t *out) {
    for (uint32_t i = 0; i < k; ++i) out[i] = q[i];
    for (uint32_t i = 1; i < k; ++i)
        for (uint32_t j = i; j > 0 && out[j - 1] > out[j]; --j) {
            size_t t = out[j]; out[j] = out[j - 1]; out[j - 1] = t;
        }
}

void oracle_apply_dense(oc128 *amps, uint32_t n, const oc128 *m, uint32_t k,
                        const size_t *qubits) {
    const size_t dim = (size_t)1 << k;
    const size_t groups = (size_t)1 << (n - k);
    size_t sorted[64];
    sort_positions(qubits, k, sorted);
    size_t offs[1 << ORACLE_MAX_DENSE_ARITY];
    for (size_t j = 0; j < dim; ++j) offs[j] = scatter(j, k, qubits);
#pragma omp parallel for schedule(static) if (groups >= 4096)
    for (size_t g = 0; g < groups; ++g) {
        oc128 in[1 << ORACLE_MAX_DENSE_ARITY];
        const size_t base = insert_zeros(g, k, sorted);
        for (size_t j = 0; j < dim; ++j) in[j] = amps[base | offs[j]];
        for (size_t r = 0; r < dim; ++r) {
            oc128 acc = cmk(0, 0);
            for (size_t c = 0; c < dim; ++c) acc = cadd(acc, cmul(m[r * dim + c], in[c]));
            amps[base | offs[r]] = acc;
        }
    }
}

/* MCX with many controls: swap the target pair where every control bit is set. */
static void apply_mcx(oc128 *amps, uint32_t n, uint32_t arity, const size_t *qubits) {
    size_t cmask = 0;
    for (uint32_t i = 0; i + 1 < arity; ++i) cmask |= (size_t)1 << qubits[i];
    const size_t tbit = (size_t)1 << qubits[arity - 1];
    const size_t dim = (size_t)1 << n;
#pragma omp parallel for schedule(static) if (dim >= 65536)
    for (size_t i = 0; i < dim; ++i) {
        if ((i & cmask) == cmask && !(i & tbit)) {
            oc128 t = amps[i];
            amps[i] = amps[i | tbit];
            amps[i | tbit] = t;
        }
    }
}

static void conj_transpose(const oc128 *m, oc128 *out, size_t dim) {
    for (size_t i = 0; i < dim; ++i)
        for (size_t j = 0; j < dim; ++j) out[j * dim + i] = cconj(m[i * dim + j]);
}

static int op_arity_ok(const oracle_op *op, uint32_t n) {
    if (op->arity == 0 || op->arity > n) return 0;
    for (uint32_t i = 0; i < op->arity; ++i) {
        if (op->qubits[i] >= n) return 0;
        for (uint32_t j = 0; j < i; ++j)
            if (op->qubits[j] == op->qubits[i]) return 0;
    }
    return 1;
}

int oracle_apply_gate(oc128 *amps, uint32_t n, const oracle_op *op, int adjoint) {
    if (!op_arity_ok(op, n)) return -1;
    if (op->opcode == 37 && op->arity > ORACLE_MAX_DENSE_ARITY) {
        apply_mcx(amps, n, op->arity, op->qubits); /* self-inverse */
        return 0;
    }
    const size_t dim = (size_t)1 << op->arity;
    oc128 *m = (oc128 *)malloc(dim * dim * sizeof(oc128));
    oc128 *mt = (oc128 *)malloc(dim * dim * sizeof(oc128));
    int rc = oracle_gate_matrix(op->opcode, op->arity, op->params, op->matrix, m);
    if (rc == 0) {
        if (adjoint) conj_transpose(m, mt, dim);
        oracle_apply_dense(amps, n, adjoint ? mt : m, op->arity, op->qubits);
    }
    free(m);
    free(mt);
    return rc;
}

int oracle_parameter_derivative(const oc128 *in, oc128 *out, uint32_t n, const oracle_op *op,
                                size_t slot) {
    if (!op_arity_ok(op, n)) return -1;
    oc128 d[16];
    if (oracle_derivative_matrix(op->opcode, op->arity, op->params, slot, d) != 0) return -1;
    const size_t len = (size_t)1 << n;
    memcpy(out, in, len * sizeof(oc128));
    oracle_apply_dense(out, n, d, op->arity, op->qubits);
    return 0;
}

int oracle_plan_apply(const oracle_op *ops, size_t num_ops, oc128 *amps, uint32_t n) {
    for (size_t k = 0; k < num_ops; ++k)
        if (oracle_apply_gate(amps, n, &ops[k], 0) != 0) return -1;
    return 0;
}

/* Re sum_i conj(a_i) b_i */
static double re_inner(const oc128 *a, const oc128 *b, size_t len) {
    double acc = 0.0;
#pragma omp parallel for reduction(+ : acc) schedule(static) if (len >= 65536)
    for (size_t i = 0; i < len; ++i) acc += a[i].re * b[i].re + a[i].im * b[i].im;
    return acc;
}

int oracle_adjoint_backward(const oracle_op *ops, size_t num_ops, oc128 *psi, oc128 *lambda,
                            uint32_t n, double upstream, const uint8_t *req, size_t req_len,
                            double *grads, size_t grads_len) {
    const size_t len = (size_t)1 << n;
    for (size_t k = 0; k < num_ops; ++k)
        for (uint32_t b = 0; b < ops[k].num_bindings; ++b)
            if (ops[k].parents[b] >= req_len || ops[k].parents[b] >= grads_len) return -1;
    for (size_t i = 0; i < len; ++i) lambda[i] = cscale(lambda[i], upstream);
    oc128 *scratch = (oc128 *)malloc(len * sizeof(oc128));
    if (!scratch) return -1;
    for (size_t kk = num_ops; kk-- > 0;) {
        const oracle_op *op = &ops[kk];
        if (oracle_apply_gate(psi, n, op, 1) != 0) { free(scratch); return -1; }
        for (uint32_t b = 0; b < op->num_bindings; ++b) {
            if (!req[op->parents[b]]) continue;
            if (oracle_parameter_derivative(psi, scratch, n, op, op->slots[b]) != 0) {
                free(scratch);
                return -1;
            }
            grads[op->parents[b]] += 2.0 * re_inner(lambda, scratch, len);
        }
        if (oracle_apply_gate(lambda, n, op, 1) != 0) { free(scratch); return -1; }
    }
    free(scratch);
    return 0;
}

int oracle_batch_plan_apply(const oracle_op *ops, size_t num_ops, oc128 *amps, size_t batch,
                            uint32_t n) {
    const size_t len = (size_t)1 << n;
    int bad = 0;
#pragma omp parallel for schedule(dynamic) reduction(| : bad)
    for (size_t b = 0; b < batch; ++b) bad |= oracle_plan_apply(ops, num_ops, amps + b * len, n) != 0;
    return bad ? -1 : 0;
}

int oracle_batch_adjoint_backward(const oracle_op *ops, size_t num_ops, oc128 *psi,
                                  oc128 *lambda, size_t batch, uint32_t n,
                                  const double *upstream, const uint8_t *req, size_t req_len,
                                  double *grads, size_t grads_len) {
    const size_t len = (size_t)1 << n;
    double *rows = (double *)calloc(batch * grads_len, sizeof(double));
    if (!rows) return -1;
    int bad = 0;
#pragma omp parallel for schedule(dynamic) reduction(| : bad)
    for (size_t b = 0; b < batch; ++b)
        bad |= oracle_adjoint_backward(ops, num_ops, psi + b * len, lambda + b * len, n,
                                       upstream[b], req, req_len, rows + b * grads_len,
                                       grads_len) != 0;
    /* per-row gradient vectors summed in row order, row_major.rs:150-160 */
    for (size_t b = 0; b < batch; ++b)
        for (size_t j = 0; j < grads_len; ++j) grads[j] += rows[b * grads_len + j];
    free(rows);
    return bad ? -1 : 0;
}

/* ---------------------------------------------------------------- Pauli observable */

static inline int parity(uint64_t x) { return __builtin_popcountll(x) & 1; }

/* CompiledPauliTerm::phase, compiled_hamiltonian.rs:198-210 */
static inline oc128 term_phase(const oracle_term *t, uint64_t index) {
    oc128 base;
    switch (t->y_count_mod_four & 3u) {
    case 0: base = cmk(1, 0); break;
    case 1: base = cmk(0, 1); break;
    case 2: base = cmk(-1, 0); break;
    default: base = cmk(0, -1); break;
    }
    return parity(index & t->phase_mask) ? cmk(-base.re, -base.im) : base;
}

/* compiled_hamiltonian.rs:64-67: Z-only terms summed into a diagonal table. */
void oracle_hamiltonian_diagonal(const oracle_term *terms, size_t num_terms, uint32_t n,
                                 double *diagonal) {
    const size_t len = (size_t)1 << n;
    memset(diagonal, 0, len * sizeof(double));
    for (size_t t = 0; t < num_terms; ++t) {
        if (terms[t].flip_mask != 0) continue;
#pragma omp parallel for schedule(static) if (len >= 65536)
        for (size_t i = 0; i < len; ++i) diagonal[i] += terms[t].coefficient * term_phase(&terms[t], i).re;
    }
}

/* compiled_hamiltonian.rs:81-101 */
double oracle_expectation(const oracle_term *terms, size_t num_terms, const oc128 *amps,
                          uint32_t n) {
    const size_t len = (size_t)1 << n;
    double *diag = (double *)malloc(len * sizeof(double));
    oracle_hamiltonian_diagonal(terms, num_terms, n, diag);
    double value = 0.0;
#pragma omp parallel for reduction(+ : value) schedule(static) if (len >= 65536)
    for (size_t i = 0; i < len; ++i) value += diag[i] * (amps[i].re * amps[i].re + amps[i].im * amps[i].im);
    free(diag);
    for (size_t t = 0; t < num_terms; ++t) {
        const oracle_term *term = &terms[t];
        if (term->flip_mask == 0) continue;
        double part = 0.0;
#pragma omp parallel for reduction(+ : part) schedule(static) if (len >= 65536)
        for (size_t i = 0; i < len; ++i) {
            const size_t j = i ^ term->flip_mask;
            const oc128 v = cmul(cscale(cmul(cconj(amps[j]), term_phase(term, i)), term->coefficient), amps[i]);
            part += v.re;
        }
        value += part;
    }
    return value;
}

/* compiled_hamiltonian.rs:104-132 */
void oracle_apply_hamiltonian(const oracle_term *terms, size_t num_terms, const oc128 *amps,
                              oc128 *out, uint32_t n) {
    const size_t len = (size_t)1 << n;
    double *diag = (double *)malloc(len * sizeof(double));
    oracle_hamiltonian_diagonal(terms, num_terms, n, diag);
#pragma omp parallel for schedule(static) if (len >= 65536)
    for (size_t target = 0; target < len; ++target) {
        oc128 value = cscale(amps[target], diag[target]);
        for (size_t t = 0; t < num_terms; ++t) {
            const oracle_term *term = &terms[t];
            if (term->flip_mask == 0) continue;
            const size_t source = target ^ term->flip_mask;
            value = cadd(value, cmul(cscale(term_phase(term, source), term->coefficient), amps[source]));
        }
        out[target] = value;
    }
    free(diag);
}

/* compiled_hamiltonian.rs:157-168 */
double oracle_expectation_and_apply(const oracle_term *terms, size_t num_terms,
                                    const oc128 *amps, oc128 *out, uint32_t n) {
    oracle_apply_hamiltonian(terms, num_terms, amps, out, n);
    return re_inner(amps, out, (size_t)1 << n);
}

/* ---------------------------------------------------------------- sampling
 *
 * sample_counts, crates/arcqml-sim/src/statevector/api/measurement.rs:18-60: p_i = re^2 + im^2
 * (two products and a sum, no fused multiply-add), a sequential f64 running sum, and per shot
 * target = u * total with u the next f64 of StdRng::seed_from_u64(seed); the shot lands on the
 * first index whose running sum exceeds target (the last index if none does).
 *
 * The generator comes from crates the reference pins but does not ship (rand 0.10.2,
 * rand_core 0.10.1, chacha20 0.10.2, Cargo.lock:482-497, :201-204); this restates their
 * published algorithms:
 *   seed_from_u64  the 32-byte seed is eight outputs of PCG32 (XSH-RR) on a 64-bit state
 *                  advanced as s = s * 6364136223846793005 + 11634580027462260723 before each
 *                  output, each output stored little-endian;
 *   StdRng         ChaCha with 12 rounds (6 double rounds): words 0-3 the "expand 32-byte k"
 *                  constants, 4-11 the seed as little-endian words, 12-13 a 64-bit block
 *                  counter from 0, 14-15 a zero stream id; the keystream is the blocks' output
 *                  words in order;
 *   next_u64       two consecutive keystream words, the first as the low half;
 *   f64            (next_u64 >> 11) * 2^-53.
 */

static inline uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

#define QR(a, b, c, d)                 \
    do {                               \
        a += b; d ^= a; d = rotl32(d, 16); \
        c += d; b ^= c; b = rotl32(b, 12); \
        a += b; d ^= a; d = rotl32(d, 8);  \
        c += d; b ^= c; b = rotl32(b, 7);  \
    } while (0)

void oracle_chacha_block(const uint32_t key[8], uint64_t counter, uint64_t stream, int rounds,
                         uint32_t out[16]) {
    uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u};
    for (int i = 0; i < 8; ++i) s[4 + i] = key[i];
    s[12] = (uint32_t)counter;
    s[13] = (uint32_t)(counter >> 32);
    s[14] = (uint32_t)stream;
    s[15] = (uint32_t)(stream >> 32);
    uint32_t x[16];
    memcpy(x, s, sizeof x);
    for (int r = 0; r < rounds; r += 2) {
        QR(x[0], x[4], x[8], x[12]);
        QR(x[1], x[5], x[9], x[13]);
        QR(x[2], x[6], x[10], x[14]);
        QR(x[3], x[7], x[11], x[15]);
        QR(x[0], x[5], x[10], x[15]);
        QR(x[1], x[6], x[11], x[12]);
        QR(x[2], x[7], x[8], x[13]);
        QR(x[3], x[4], x[9], x[14]);
    }
    for (int i = 0; i < 16; ++i) out[i] = x[i] + s[i];
}

void oracle_stdrng_key(uint64_t seed, uint32_t key[8]) {
    uint64_t st = seed;
    for (int i = 0; i < 8; ++i) {
        st = st * 6364136223846793005ull + 11634580027462260723ull;
        const uint32_t xorshifted = (uint32_t)(((st >> 18) ^ st) >> 27);
        const uint32_t rot = (uint32_t)(st >> 59);
        key[i] = (xorshifted >> rot) | (xorshifted << ((32 - rot) & 31));
    }
}

/* The k-th u64 of StdRng::seed_from_u64(seed) (k = 0 first). */
uint64_t oracle_stdrng_u64(uint64_t seed, uint64_t k) {
    uint32_t key[8], blk[16];
    oracle_stdrng_key(seed, key);
    oracle_chacha_block(key, k / 8, 0, 12, blk);
    const int w = (int)(k % 8) * 2;
    return (uint64_t)blk[w] | ((uint64_t)blk[w + 1] << 32);
}

int oracle_sample_indices(const oc128 *amps, uint32_t num_qubits, uint64_t shots, uint64_t seed,
                          uint64_t *out) {
    if (num_qubits >= 63 || shots == 0) return 1;
    const size_t dim = (size_t)1 << num_qubits;
    double *cum = (double *)malloc(dim * sizeof(double));
    if (!cum) return 2;
    double run = 0.0;
    for (size_t i = 0; i < dim; ++i) {
        const double re2 = amps[i].re * amps[i].re;
        const double im2 = amps[i].im * amps[i].im;
        run += re2 + im2;
        cum[i] = run;
    }
    const double total = run;
    uint32_t key[8], blk[16];
    oracle_stdrng_key(seed, key);
    for (uint64_t s = 0; s < shots; ++s) {
        if (s % 8 == 0) oracle_chacha_block(key, s / 8, 0, 12, blk);
        const int w = (int)(s % 8) * 2;
        const uint64_t x = (uint64_t)blk[w] | ((uint64_t)blk[w + 1] << 32);
        const double target = (double)(x >> 11) * (1.0 / 9007199254740992.0) * total;
        /* first i with target < cum[i]: the running sum never decreases, so the linear scan
         * of the reference and this bisection land on the same index */
        size_t lo = 0, hi = dim;
        while (lo < hi) {
            const size_t mid = lo + (hi - lo) / 2;
            if (target < cum[mid]) hi = mid;
            else lo = mid + 1;
        }
        out[s] = lo < dim ? lo : dim - 1;
    }
    free(cum);
    return 0;
}

/* ---------------------------------------------------------------- analysis
 * crates/arcqml-analysis/src/statevector/{probabilities,marginal,bloch,fidelity}.rs. */

/* probabilities.rs:22-25: square(abs(amplitude)); abs of a Complex64 is re.hypot(im). */
void oracle_probabilities(const oc128 *amps, uint32_t num_qubits, double *out) {
    const size_t dim = (size_t)1 << num_qubits;
    for (size_t i = 0; i < dim; ++i) {
        const double h = hypot(amps[i].re, amps[i].im);
        out[i] = h * h;
    }
}

/* marginal.rs:17-32 and :62-67: display order = selected qubits descending; output index bit j
 * (counted from the most significant) is the basis index's bit display[j]; segment sums in
 * basis-index order. Returns non-zero for an empty, duplicate or out-of-range selection. */
int oracle_marginal_probabilities(const oc128 *amps, uint32_t num_qubits, const uint32_t *qubits,
                                  size_t num_selected, double *out) {
    if (num_selected == 0 || num_selected > num_qubits) return 1;
    uint32_t disp[64];
    for (size_t j = 0; j < num_selected; ++j) {
        if (qubits[j] >= num_qubits) return 2;
        for (size_t m = 0; m < j; ++m)
            if (qubits[m] == qubits[j]) return 3;
        disp[j] = qubits[j];
    }
    for (size_t a = 0; a < num_selected; ++a)  /* descending */
        for (size_t b = a + 1; b < num_selected; ++b)
            if (disp[b] > disp[a]) {
                const uint32_t t = disp[a];
                disp[a] = disp[b];
                disp[b] = t;
            }
    const size_t dim = (size_t)1 << num_qubits, bins = (size_t)1 << num_selected;
    for (size_t m = 0; m < bins; ++m) out[m] = 0.0;
    for (size_t i = 0; i < dim; ++i) {
        size_t m = 0;
        for (size_t j = 0; j < num_selected; ++j) m = (m << 1) | ((i >> disp[j]) & 1u);
        const double h = hypot(amps[i].re, amps[i].im);
        out[m] += h * h;
    }
    return 0;
}

/* bloch.rs:23-56: x += 2 Re(conj(a0) a1), y += 2 Im(conj(a0) a1), z += |a0|^2 - |a1|^2 over the
 * index pairs (a0, a1) of the qubit, in index order. */
int oracle_bloch_vector(const oc128 *amps, uint32_t num_qubits, uint32_t qubit, double xyz[3]) {
    if (qubit >= num_qubits) return 1;
    const size_t dim = (size_t)1 << num_qubits, mask = (size_t)1 << qubit;
    double x = 0.0, y = 0.0, z = 0.0;
    for (size_t i = 0; i < dim; ++i) {
        if (i & mask) continue;
        const oc128 a0 = amps[i], a1 = amps[i | mask];
        const double cre = a0.re * a1.re + a0.im * a1.im;
        const double cim = a0.re * a1.im - a0.im * a1.re;
        x += 2.0 * cre;
        y += 2.0 * cim;
        z += (a0.re * a0.re + a0.im * a0.im) - (a1.re * a1.re + a1.im * a1.im);
    }
    xyz[0] = x;
    xyz[1] = y;
    xyz[2] = z;
    return 0;
}

/* fidelity.rs:14-30: overlap = sum(conj(lhs) * rhs) in index order; fidelity = square(abs(.)),
 * returned in out[2] after the overlap's real and imaginary parts in out[0], out[1]. */
void oracle_overlap_fidelity(const oc128 *lhs, const oc128 *rhs, uint32_t num_qubits,
                             double out[3]) {
    const size_t dim = (size_t)1 << num_qubits;
    double re = 0.0, im = 0.0;
    for (size_t i = 0; i < dim; ++i) {
        re += lhs[i].re * rhs[i].re + lhs[i].im * rhs[i].im;
        im += lhs[i].re * rhs[i].im - lhs[i].im * rhs[i].re;
    }
    const double h = hypot(re, im);
    out[0] = re;
    out[1] = im;
    out[2] = h * h;
}
