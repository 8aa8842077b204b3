// planner.cpp — partitions a gate sequence into fused passes (see fused.h).
//
// Greedy, order-preserving: a pass picks its tile qubits S (qubits 0..L-1 plus either the first
// non-diagonal targets met in circuit order, or qubits picked by lookahead, each the one whose
// tile holds the most remaining gates: whichever takes more gates) and takes every gate it can,
// in order, whose non-diagonal targets lie in S and that does not need to move past a gate it
// left behind (a gate sharing a qubit with a skipped gate is skipped too, so the relative order
// of all gates on any qubit is kept). Inside a pass, consecutive gates are grouped into sub-blocks whose
// non-diagonal targets fit in RB register bits. Custom gates on more than two targets cannot be
// fused and run as separate per-gate kernels between passes.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "fused.h"
#include "planner.h"
#include "rt_internal.h"

namespace arcqml {

namespace {

bool is_diag(const std::vector<double2> &m, size_t dim) {
    for (size_t i = 0; i < dim; ++i)
        for (size_t j = 0; j < dim; ++j)
            if (i != j && (m[i * dim + j].x != 0.0 || m[i * dim + j].y != 0.0)) return false;
    return true;
}

bool eq(double2 a, double2 b) { return a.x == b.x && a.y == b.y; }

// One gate in kernel-ready small form, with its planning footprint.
struct PGate {
    const OpRecord *op = nullptr;
    bool noop = false;                 // identity gate
    bool dense_barrier = false;        // arity > 2 custom: per-gate kernel
    std::vector<uint32_t> controls;
    std::vector<uint32_t> targets;
    std::vector<double2> m;            // (2^nt)^2, U or U^dagger
    bool diag = false;
    uint64_t touched = 0;              // every qubit of the gate
    uint64_t needs = 0;                // non-diagonal targets (must be in the tile)
    uint8_t gkind = GK_NONE;           // adjoint
    std::vector<std::vector<double2>> dm;  // generic slots: dU in small form
    std::vector<size_t> parents;           // per required slot
};

PGate make_pgate(const OpRecord &op, bool adjoint, const uint8_t *req, bool grads) {
    PGate g;
    g.op = &op;
    for (uint32_t q : op.qubits) g.touched |= uint64_t(1) << q;
    if (op.opcode == ARCQML_OP_CUSTOM_UNITARY && op.qubits.size() > 2) {
        g.dense_barrier = true;
        return g;
    }
    // allow_diag = false keeps the dense small form: positions = controls + targets.
    DevGate u = lower(op, adjoint ? LOWER_ADJOINT : LOWER_FORWARD, 0, false);
    if (u.kind == KIND_NONE) {  // the identity gate: nothing to apply, nothing to differentiate
        g.noop = true;
        return g;
    }
    for (int i = 0; i < u.nt; ++i) g.targets.push_back(uint32_t(u.t[i]));
    for (uint32_t q = 0; q < 64; ++q)
        if ((u.cmask >> q) & 1) g.controls.push_back(q);
    const size_t dim = size_t(1) << u.nt;
    g.m.assign(u.m, u.m + dim * dim);
    g.diag = is_diag(g.m, dim);
    if (!g.diag)
        for (uint32_t t : g.targets) g.needs |= uint64_t(1) << t;
    if (adjoint && grads) {
        const uint32_t o = op.opcode;
        std::vector<uint32_t> slots;
        for (uint32_t b = 0; b < op.num_bindings; ++b)
            if (req[op.parents[b]]) {
                slots.push_back(uint32_t(op.slots[b]));
                g.parents.push_back(op.parents[b]);
            }
        if (!slots.empty()) {
            if (o == ARCQML_OP_RX || o == ARCQML_OP_CRX) g.gkind = GK_PX;
            else if (o == ARCQML_OP_RY || o == ARCQML_OP_CRY) g.gkind = GK_PY;
            else if (o == ARCQML_OP_RZ || o == ARCQML_OP_CRZ) g.gkind = GK_PZ;
            else g.gkind = GK_GENERIC;
            if (g.gkind == GK_GENERIC)
                for (uint32_t s : slots) {
                    DevGate d = lower(op, LOWER_DERIVATIVE, s, false);
                    g.dm.emplace_back(d.m, d.m + dim * dim);
                    // U can be diagonal at particular angles (U3(0, f, l), fSim(0, f), RXX(0))
                    // while its derivative is not: then the targets must sit in registers
                    if (g.diag && !is_diag(g.dm.back(), dim)) {
                        g.diag = false;
                        for (uint32_t t : g.targets) g.needs |= uint64_t(1) << t;
                    }
                }
            // X/Y gradients pair amplitudes across the target even when the angle makes the
            // matrix diagonal (e.g. RX(0)): keep the target in registers.
            if ((g.gkind == GK_PX || g.gkind == GK_PY) && g.diag) {
                g.diag = false;
                for (uint32_t t : g.targets) g.needs |= uint64_t(1) << t;
            }
        }
    }
    return g;
}

// Upper bound of the matrix-table entries a gate adds to its pass.
// (a forward single-qubit gate may be merged into a 2x2 of 4 entries: count it as 4)
size_t mat_entries(const PGate &g) {
    const size_t dim = size_t(1) << g.targets.size();
    const size_t per = (g.diag && dim > 2) ? dim : dim * dim;
    return per * (1 + g.dm.size());
}

// Full 2x2 of an emitted single-target op from its kind and matrix-table entries.
void op_matrix2(const FOp &o, const std::vector<double2> &mats, double2 u[4]) {
    const double2 *m = mats.data() + o.moff;
    switch (o.kind) {
    case FK_RX: u[0] = make_double2(m[0].x, 0); u[1] = make_double2(0, -m[0].y);
                u[2] = u[1]; u[3] = u[0]; break;
    case FK_RY: u[0] = make_double2(m[0].x, 0); u[1] = make_double2(-m[0].y, 0);
                u[2] = make_double2(m[0].y, 0); u[3] = u[0]; break;
    case FK_D1: u[0] = m[0]; u[1] = make_double2(0, 0); u[2] = u[1]; u[3] = m[1]; break;
    default: for (int i = 0; i < 4; ++i) u[i] = m[i]; break;
    }
}

void mul2(const double2 a[4], const double2 b[4], double2 out[4]) {  // out = a * b
    for (int i = 0; i < 2; ++i)
        for (int j = 0; j < 2; ++j) {
            double re = 0, im = 0;
            for (int k = 0; k < 2; ++k) {
                const double2 x = a[i * 2 + k], y = b[k * 2 + j];
                re += x.x * y.x - x.y * y.y;
                im += x.x * y.y + x.y * y.x;
            }
            out[i * 2 + j] = make_double2(re, im);
        }
}

// FK_RX or FK_RY when a 2x2 (row-major) is [[c, -is], [-is, c]] or [[c, -s], [s, c]] with real
// c and s (the patterns the op emitter stores as (c, s)), else 0.
int rotation_form(const double2 m[4]) {
    const bool same_diag = eq(m[0], m[3]) && m[0].y == 0.0;
    if (same_diag && m[1].x == 0.0 && eq(m[1], m[2])) return FK_RX;
    if (same_diag && m[1].y == 0.0 && m[2].y == 0.0 && m[1].x == -m[2].x) return FK_RY;
    return 0;
}

// Whether a 2x2 (row-major) has the form of `kind` (FK_RX or FK_RY). rotation_form tests the RX
// form first, so it calls the identity (either form with s = 0) an RX form.
bool has_rotation_form(const double2 m[4], int kind) {
    const bool same_diag = eq(m[0], m[3]) && m[0].y == 0.0;
    if (kind == FK_RX) return same_diag && m[1].x == 0.0 && eq(m[1], m[2]);
    if (kind == FK_RY) return same_diag && m[1].y == 0.0 && m[2].y == 0.0 && m[1].x == -m[2].x;
    return false;
}

// Whether a 2x2 (row-major) has a scaled unit-diagonal form: an RX- or RY-form rotation or a
// diagonal with |d0| = |d1| (what scale_pass below rewrites).
bool scalable_1q(const double2 m[4]) {
    if (rotation_form(m) != 0) return true;
    if (m[1].x != 0.0 || m[1].y != 0.0 || m[2].x != 0.0 || m[2].y != 0.0) return false;
    const double a0 = std::hypot(m[0].x, m[0].y), a3 = std::hypot(m[3].x, m[3].y);
    return a0 > 0.0 && std::fabs(a0 - a3) <= 1e-14 * a0;
}

double2 cmulh(double2 a, double2 b) {
    return make_double2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

// Scaled pass (compiled kernels; FOp::sform/sgrad/soff, Step::scaled/sfin). A Pauli rotation or
// a unitary one-qubit diagonal is f * M with M's diagonal 1 (RY: c [[1, -t], [t, 1]], t = s/c;
// RX: c [[1, -it], [-it, 1]]; diag(d0, d1) = f diag(1 - i tau, 1 + i tau) with
// tau = tan(arg(d1/d0) / 2), f = d0 cos(g) e^{ig}), so applying M costs one FMA per component
// (2 FP64 instructions per amplitude instead of 4) and the factors f collect in one scalar sigma
// per pass: true state = sigma * stored state. psi and lambda of an adjoint pass get the same
// daggered ops, so they carry the same sigma and <lam|P|psi> = |sigma|^2 <lam~|P|psi~>: each
// gradient is multiplied by 0.5 |sigma|^2 at its op instead of 0.5. Ops without such a form run
// as they are (a scalar commutes with every linear op). The growth of 1/|sigma| is capped at
// 2^300 per pass (and 2^30 per op), far from the f64 range even for the squared factor.
void scale_pass(Step &st, bool adjoint) {
    if (!scaled_passes()) return;
    for (const SubBlock &sb : st.subs)
        if (!(sb.flags & SB_JIT_FAST)) return;  // runs on the table-driven kernel
    const size_t base = st.mats.size();
    std::vector<double2> extra;
    double2 sigma = make_double2(1.0, 0.0);
    double growth = 0.0;  // log2(1 / |sigma|)
    bool any = false;
    for (FOp &o : st.ops) {
        const double2 *m = st.mats.data() + o.moff;
        bool sc = false;
        double tau = 0.0;
        double2 f = make_double2(1.0, 0.0);
        // a generic slot gradient is taken on U^dagger psi: its op keeps the plain form
        const bool keep = o.gkind == GK_GENERIC;
        if (!keep && (o.code == FC_RX || o.code == FC_RY) && m[0].x != 0.0) {
            tau = m[0].y / m[0].x;
            f = make_double2(m[0].x, 0.0);
            sc = true;
        } else if (!keep && (o.code == FC_D1_REG || o.code == FC_D1_UNI)) {
            const double a0 = std::hypot(m[0].x, m[0].y), a1 = std::hypot(m[1].x, m[1].y);
            if (a0 > 0.0 && std::fabs(a0 - a1) <= 1e-14 * a0) {
                // r = d1 / d0 = e^{2ig}
                const double2 r = make_double2((m[1].x * m[0].x + m[1].y * m[0].y) / (a0 * a0),
                                               (m[1].y * m[0].x - m[1].x * m[0].y) / (a0 * a0));
                const double g = 0.5 * std::atan2(r.y, r.x);
                tau = std::tan(g);
                f = cmulh(m[0], make_double2(std::cos(g) * std::cos(g), std::cos(g) * std::sin(g)));
                sc = true;
            }
        }
        if (sc) {
            const double gr = -std::log2(std::hypot(f.x, f.y));
            if (!std::isfinite(tau) || !(gr <= 30.0) || growth + gr > 300.0) sc = false;
            else growth += gr;
        }
        const bool grad = adjoint && o.gkind != GK_NONE;
        o.sform = sc ? 1 : 0;
        o.sgrad = grad ? 1 : 0;
        o.soff = 0;
        if (sc || grad) {
            o.soff = uint32_t(base + extra.size());
            extra.push_back(make_double2(tau, 0.5 * (sigma.x * sigma.x + sigma.y * sigma.y)));
        }
        if (sc) {
            sigma = cmulh(sigma, f);
            any = true;
        }
    }
    if (!any || base + extra.size() + 1 > size_t(kMaxPassMats)) {
        for (FOp &o : st.ops) o.sform = o.sgrad = 0, o.soff = 0;
        return;
    }
    st.sfin = uint32_t(base + extra.size());
    extra.push_back(sigma);
    st.mats.insert(st.mats.end(), extra.begin(), extra.end());
    st.scaled = true;
}

bool is_x(const std::vector<double2> &m) {
    return m.size() == 4 && m[0].x == 0 && m[0].y == 0 && m[1].x == 1 && m[1].y == 0 &&
           m[2].x == 1 && m[2].y == 0 && m[3].x == 0 && m[3].y == 0;
}

// Chooses the op's specialised device path (fused.h FastCode). reg_of(q) is the register bit
// of qubit q in the current sub-block (0xFF if none); lpos[q] its tile bit (-1 if outside).
template <class RegOf>
void classify(FOp &o, const PGate &g, const RegOf &reg_of, const int *lpos) {
    const bool plain = o.lcmask == 0 && o.gcmask == 0;
    const size_t nt = g.targets.size();
    auto put = [&](int slot, uint32_t q) {
        o.dq_in_tile[slot] = lpos[q] >= 0 ? 1 : 0;
        o.dq_pos[slot] = uint8_t(lpos[q] >= 0 ? lpos[q] : int(q));
    };
    o.code = FC_GENERIC;
    if (!g.diag && fast_cnot() && nt == 1 && is_x(g.m)) {
        if (plain) {
            o.code = FC_X;
            return;
        }
        if (g.controls.size() == 1) {
            const uint32_t c = g.controls[0];
            const uint8_t rc = reg_of(c);
            if (rc != 0xFF) {
                o.code = FC_CX_RR;
                o.rb1 = rc;
            } else {
                o.code = FC_CX_CR;
                put(0, c);
            }
            return;
        }
    }
    if (!g.diag) {
        if (plain && nt == 1)
            o.code = o.kind == FK_RX ? FC_RX : (o.kind == FK_RY ? FC_RY : FC_M2);
        else if (plain && nt == 2)
            o.code = FC_M4;
        else if (fast_diag() && nt == 1)
            o.code = FC_CM2;
        return;
    }
    if (nt != 1) {
        if (fast_diag()) o.code = FC_DIAG;
        return;
    }
    const uint32_t t = g.targets[0];
    if (plain) {
        const uint8_t r = reg_of(t);
        if (r != 0xFF) {
            o.code = FC_D1_REG;
            o.rb0 = r;
        } else {
            o.code = FC_D1_UNI;
        }
        return;
    }
    const double2 d0 = g.m[0], d1 = g.m[3];
    const bool sign = d0.x == 1.0 && d0.y == 0.0 && d1.x == -1.0 && d1.y == 0.0;
    if (!sign || g.controls.size() != 1) {
        if (fast_diag()) o.code = FC_DIAG;
        return;
    }
    const uint32_t c = g.controls[0];  // CZ-like: -1 where both c and t are 1
    const uint8_t rc = reg_of(c), rt = reg_of(t);
    if (rc != 0xFF && rt != 0xFF) {
        o.code = FC_SIGN_RR;
        o.rb0 = rc;
        o.rb1 = rt;
    } else if (rt != 0xFF) {
        o.code = FC_SIGN_RC;
        o.rb0 = rt;
        put(0, c);
    } else if (rc != 0xFF) {
        o.code = FC_SIGN_RC;
        o.rb0 = rc;
        put(0, t);
    } else {
        o.code = FC_SIGN_CC;
        put(0, c);
        put(1, t);
    }
}

// Whether the device runs op o without its generic (out-of-line) path: the forward pass needs
// a fast apply; the adjoint pass also needs the gradient, if any, on the same fast path.
bool has_fast_path(const FOp &o, bool adjoint) {
    if (o.code == FC_GENERIC) return false;
    if (o.code == FC_X || o.code == FC_CX_RR || o.code == FC_CX_CR) return false;
    if (o.code == FC_DIAG || o.code == FC_CM2) return false;
    if (!adjoint || o.gkind == GK_NONE) return true;
    return (o.code == FC_RX && o.gcode == GF_X) || (o.code == FC_RY && o.gcode == GF_Y) ||
           (o.code == FC_D1_REG && o.gcode == GF_Z_REG) || (o.code == FC_D1_UNI && o.gcode == GF_Z_UNI);
}

// Unless ARCQML_FAST_DIAG=0, the run-time compiled kernels also run diagonal gates with controls,
// two-qubit diagonals and controlled one-target gates (FC_DIAG / FC_CM2), Pauli-rotation
// gradients with controls or on dense 2x2 forms, and every generic slot gradient of a one- or
// two-qubit diagonal, a one-target gate or an uncontrolled 4x4 (jit.cpp writes each as its
// register arithmetic).
bool has_jit_general_path(const FOp &o, bool adjoint) {
    const bool diag = o.kind == FK_D1 || o.kind == FK_D2;
    const bool one = o.kind == FK_RX || o.kind == FK_RY || o.kind == FK_M2;
    switch (o.code) {
    case FC_DIAG: if (!diag) return false; break;
    case FC_CM2: if (!one) return false; break;
    case FC_D1_REG: case FC_D1_UNI: case FC_RX: case FC_RY: case FC_M2: case FC_M4: break;
    default: return false;
    }
    if (!adjoint || o.gkind == GK_NONE) return true;
    if (o.gkind == GK_GENERIC) return true;
    if (o.gkind == GK_PZ) return o.kind == FK_D1;
    return one && (o.gkind == GK_PX || o.gkind == GK_PY);
}

// The run-time compiled kernels also have fast paths for X and CNOT on register bits
// (register exchanges); the table-driven kernel runs those through its generic path.
bool has_jit_fast_path(const FOp &o, bool adjoint) {
    if (o.code == FC_X || o.code == FC_CX_RR || o.code == FC_CX_CR) return o.gkind == GK_NONE;
    if (fast_diag() && has_jit_general_path(o, adjoint)) return true;
    return has_fast_path(o, adjoint);
}

// Residue of a tile bit under the shared-memory swizzle (fold of 3-bit groups).
inline int residue(int bit) { return bit % 3; }

// Whether `lanes` (a tile-bit mask) holds bits of all three swizzle residues (lane bits 0-2 then
// hit distinct 16-byte bank groups: conflict-free 128-bit shared-memory accesses).
bool all_residues(uint32_t lanes) {
    bool seen[3] = {false, false, false};
    for (int b = 0; b < 32; ++b)
        if ((lanes >> b) & 1u) seen[residue(b)] = true;
    return seen[0] && seen[1] && seen[2];
}

// Splits a pass's sub-blocks (register-bit masks R over k tile bits) into runs of consecutive
// sub-blocks that share one set W of warp bits (k - rb - 5 tile bits outside every R of the
// run, chosen so that each sub-block's lane bits keep all three residues). runW[sb] = W (0: the
// sub-block is alone), warp_next[sb]: the next sub-block is in the same run.
void plan_warp_runs(const std::vector<uint32_t> &R, uint32_t k, uint32_t rb,
                    std::vector<uint32_t> &runW, std::vector<bool> &warp_next) {
    const uint32_t tbits = k - rb;
    if (tbits <= 5) return;
    const uint32_t wbits = tbits - 5;
    const uint32_t all = (k >= 32) ? 0xffffffffu : ((1u << k) - 1);
    // a warp-bit set valid for sub-blocks [a, b], or 0
    auto pick = [&](size_t a, size_t b) -> uint32_t {
        uint32_t uni = 0;
        for (size_t i = a; i <= b; ++i) uni |= R[i];
        const uint32_t free = all & ~uni;
        if (uint32_t(__builtin_popcount(free)) < wbits) return 0u;
        // smallest subsets first: enumerate wbits-subsets of `free` in increasing order
        for (uint32_t m = free; m; m = (m - 1) & free) {
            if (uint32_t(__builtin_popcount(m)) != wbits) continue;
            bool ok = true;
            for (size_t i = a; i <= b && ok; ++i) ok = all_residues(all & ~R[i] & ~m);
            if (ok) return m;
        }
        return 0u;
    };
    size_t a = 0;
    while (a < R.size()) {
        size_t b = a;
        uint32_t W = pick(a, a);
        while (W && b + 1 < R.size()) {
            const uint32_t W2 = pick(a, b + 1);
            if (!W2) break;
            W = W2;
            ++b;
        }
        if (W && b > a) {
            for (size_t i = a; i <= b; ++i) runW[i] = W;
            for (size_t i = a; i < b; ++i) warp_next[i] = true;
        }
        a = b + 1;
    }
}

}  // namespace

bool scaled_passes() {
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_SCALED");
        return !(e && e[0] == '0');
    }();
    return on;
}

// Gates per pass: kMaxPassOps, or fewer with ARCQML_PASS_OPS=<count> (smaller compiled kernels).
size_t pass_op_cap() {
    static const size_t cap = [] {
        const char *e = std::getenv("ARCQML_PASS_OPS");
        const long v = e ? std::strtol(e, nullptr, 10) : 0;
        return (v > 0 && v < kMaxPassOps) ? size_t(v) : size_t(kMaxPassOps);
    }();
    return cap;
}

namespace {

// Sub-blocks of a pass's members with commuting gates reordered (on unless ARCQML_SUBBLOCK_REORDER=0).
// Two gates commute when every qubit they share is acted on diagonally by both (a diagonal
// gate, or a control): then no shared qubit is a non-diagonal target (`needs`) of either. Each
// sub-block first takes every ready gate (all non-commuting earlier gates placed) whose
// non-diagonal targets already are register bits, and grows its register bits by the first
// ready gate that fits only when none is left, so the tile goes through shared memory fewer
// times than in circuit order.
void pack_subblocks(const std::vector<PGate> &gates, const std::vector<size_t> &members,
                    const int *lpos, uint32_t rb, std::vector<std::vector<size_t>> &subs,
                    std::vector<uint32_t> &sub_R) {
    const size_t m = members.size();
    std::vector<uint32_t> need(m, 0);
    std::vector<std::vector<uint32_t>> deps(m);
    for (size_t b = 0; b < m; ++b) {
        const PGate &B = gates[members[b]];
        if (!B.diag)
            for (uint32_t t : B.targets) need[b] |= 1u << lpos[t];
        for (size_t a = 0; a < b; ++a) {
            const PGate &A = gates[members[a]];
            if ((A.touched & B.touched) & (A.needs | B.needs)) deps[b].push_back(uint32_t(a));
        }
    }
    std::vector<char> placed(m, 0);
    auto ready = [&](size_t b) {
        for (uint32_t a : deps[b])
            if (!placed[a]) return false;
        return true;
    };
    size_t left = m;
    while (left) {
        uint32_t R = 0;
        std::vector<size_t> cur;
        while (true) {
            bool took = false;
            for (size_t b = 0; b < m; ++b)
                if (!placed[b] && (need[b] & ~R) == 0 && ready(b)) {
                    cur.push_back(members[b]);
                    placed[b] = 1;
                    --left;
                    took = true;
                }
            if (took) continue;
            for (size_t b = 0; b < m && !took; ++b)
                if (!placed[b] && uint32_t(__builtin_popcount(R | need[b])) <= rb && ready(b)) {
                    R |= need[b];
                    cur.push_back(members[b]);
                    placed[b] = 1;
                    --left;
                    took = true;
                }
            if (!took) break;
        }
        subs.push_back(cur);
        sub_R.push_back(R);
    }
}

}  // namespace

uint32_t adjoint_tile_cap() {
    static const uint32_t cap = [] {
        const char *e = std::getenv("ARCQML_ADJ_TILE");
        return (e && e[0] == '1' && e[1] == '0' && !e[2]) ? 10u : 11u;
    }();
    return cap;
}

uint32_t forward_tile_cap() {
    static const uint32_t cap = [] {
        const char *e = std::getenv("ARCQML_FWD_TILE");
        return (e && e[0] == '1' && e[1] == '1' && !e[2]) ? 11u : 12u;
    }();
    return cap;
}

bool warp_local_exchanges() {
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_WARP_LOCAL");
        return !(e && e[0] == '0');
    }();
    return on;
}

bool fast_cnot() {
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_FAST_CNOT");
        return !(e && e[0] == '0');
    }();
    return on;
}

bool fast_diag() {
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_FAST_DIAG");
        return !(e && e[0] == '0');
    }();
    return on;
}

bool lookahead_tiles() {
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_LOOKAHEAD");
        return !(e && e[0] == '0');
    }();
    return on;
}

bool subblock_reorder() {
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_SUBBLOCK_REORDER");
        return !(e && e[0] == '0');
    }();
    return on;
}

bool rotation_merge() {
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_ROT_MERGE");
        return !(e && e[0] == '0');
    }();
    return on;
}

namespace {

// Passes merge a Pauli rotation exp(-i a P / 2) into the previous rotation about the same axis
// on its qubit when nothing in between fails to commute with P: one rotation by the summed
// angle (on psi, and on lambda in the adjoint sweep), and there one gradient sum for both
// parameters. Both are exact:
// the rotations commute with P, so <lam|P|psi> is the same on either side of one of them (the
// gradient of each is that sum), and moving the later rotation back past gates that commute
// with it changes neither the states nor their gradients. Between two RX or RY rotations no
// gate may touch the qubit; between two RZ rotations gates acting diagonally on it (diagonal
// gates, controls) may stand.
//
// The axis (ARCQML_OP_RX/RY/RZ) of a gate that can take part in such a merge, else 0.
uint32_t merge_axis(const PGate &g) {
    if (g.noop || g.dense_barrier || !g.controls.empty() || g.targets.size() != 1) return 0;
    if (g.parents.size() > 1 || g.gkind == GK_GENERIC || g.m.size() != 4) return 0;
    const uint32_t o = g.op->opcode;
    if (o == ARCQML_OP_RZ) return g.diag ? o : 0;
    // an RX or RY at angle 0 is the identity: it is emitted as a diagonal, not a rotation form
    if (g.diag) return 0;
    if (o == ARCQML_OP_RX) return rotation_form(g.m.data()) == FK_RX ? o : 0;
    if (o == ARCQML_OP_RY) return rotation_form(g.m.data()) == FK_RY ? o : 0;
    return 0;
}

// Per qubit, the axis of the rotation later rotations may merge into (0: none).
struct MergeChain {
    uint32_t axis = 0;
    int op = -1;       // its op in the pass (emission)
    bool row = false;  // it has a gradient row (member selection)
};

// A gate g that is not merged ends the chains it does not commute with.
void end_chains(MergeChain *chain, const PGate &g) {
    for (uint32_t q = 0; q < 64; ++q) {
        if (!((g.touched >> q) & 1) || chain[q].axis == 0) continue;
        if (chain[q].axis == ARCQML_OP_RZ && !((g.needs >> q) & 1)) continue;
        chain[q] = MergeChain{};
    }
}

uint8_t pauli_grad_code(const FOp &o) {
    if (o.lcmask != 0 || o.gcmask != 0) return GF_GENERIC;
    if (o.gkind == GK_PX) return GF_X;
    if (o.gkind == GK_PY) return GF_Y;
    if (o.gkind == GK_PZ) return o.code == FC_D1_REG ? GF_Z_REG : GF_Z_UNI;
    return GF_GENERIC;
}

}  // namespace

Schedule build_schedule(const Plan &plan, uint32_t n, bool adjoint, const uint8_t *req,
                        bool grads, uint32_t k, uint32_t rb) {
    Schedule sch;
    sch.k = k;
    sch.rb = rb;
    // Gates in execution order (reversed and daggered for the adjoint sweep).
    std::vector<PGate> gates;
    gates.reserve(plan.ops.size());
    if (!adjoint) {
        for (const auto &op : plan.ops) gates.push_back(make_pgate(op, false, req, false));
    } else {
        for (size_t i = plan.ops.size(); i-- > 0;)
            gates.push_back(make_pgate(plan.ops[i], true, req, grads));
    }
    const uint32_t L = std::min<uint32_t>(kLowFixed, k);
    const uint64_t low_mask = (uint64_t(1) << L) - 1;

    std::vector<char> done(gates.size(), 0);
    for (size_t i = 0; i < gates.size(); ++i) done[i] = gates[i].noop ? 1 : 0;
    size_t first = 0;
    uint32_t acc_total = 0;
    const bool merge_rot = rotation_merge();
    // Tile choices of an earlier schedule of this plan with the same gate structure (what the
    // member walk below reads of each gate: its qubits, non-diagonal targets, table size, rows,
    // merge axis) are taken again instead of searched.
    std::vector<uint64_t> sig;
    sig.reserve(3 * gates.size());
    for (const PGate &g : gates) {
        sig.push_back(g.touched);
        sig.push_back(g.needs);
        sig.push_back(uint64_t(g.noop) | uint64_t(g.dense_barrier) << 1 |
                      uint64_t(g.parents.size()) << 2 | uint64_t(merge_rot ? merge_axis(g) : 0) << 8 |
                      uint64_t(mat_entries(g)) << 16 | uint64_t(g.targets.empty() ? 0 : g.targets[0]) << 40);
    }
    const uint64_t ckey = uint64_t(n) | uint64_t(k) << 8 | uint64_t(rb) << 16 |
                          uint64_t(adjoint) << 24 | uint64_t(lookahead_tiles()) << 25;
    std::vector<std::pair<uint64_t, uint32_t>> cached, chosen;
    {
        std::lock_guard<std::mutex> lock(plan.tiles_mu);
        for (const TileChoices &t : plan.tiles)
            if (t.key == ckey && t.signature == sig) cached = t.take;
    }
    while (true) {
        while (first < gates.size() && done[first]) ++first;
        if (first >= gates.size()) break;
        if (gates[first].dense_barrier) {
            Step st;
            st.dense_op = gates[first].op;
            st.is_pass = false;
            sch.steps.push_back(std::move(st));
            done[first] = 1;
            continue;
        }
        // --- choose S and collect the pass's gates. take(S0, free0) walks the remaining gates
        // in order from tile qubits S0, adding the non-diagonal targets of a gate while free0
        // qubits are left, and takes every gate the tile holds that no skipped gate blocks.
        auto take = [&](uint64_t S0, uint32_t free0, std::vector<size_t> &mem) -> uint64_t {
            uint64_t S = S0, blocked = 0;
            uint32_t free_slots = free0;
            size_t pass_acc = 0, pass_mats = 0;
            MergeChain chain[64];  // the merges the emission below makes, for the row count
            mem.clear();
            const uint64_t all = n >= 64 ? ~uint64_t(0) : (uint64_t(1) << n) - 1;
            for (size_t i = first; i < gates.size(); ++i) {
                if (blocked == all) break;  // every later gate is blocked
                if (done[i]) continue;
                const PGate &g = gates[i];
                const uint32_t ax = merge_rot ? merge_axis(g) : 0;
                const bool merges = ax != 0 && chain[g.targets[0]].axis == ax;
                const size_t rows = (merges && chain[g.targets[0]].row) ? 0 : g.parents.size();
                if (pass_acc + rows > size_t(kMaxPassAcc)) break;
                if (pass_mats + mat_entries(g) > size_t(kMaxPassMats)) break;
                if (g.dense_barrier || (g.touched & blocked)) {
                    blocked |= g.touched;
                    continue;
                }
                const uint64_t extra = g.needs & ~S;
                const uint32_t cnt = uint32_t(__builtin_popcountll(extra));
                if (cnt <= free_slots) {
                    S |= extra;
                    free_slots -= cnt;
                    mem.push_back(i);
                    pass_acc += rows;
                    pass_mats += mat_entries(g);
                    if (merges) {
                        chain[g.targets[0]].row = chain[g.targets[0]].row || !g.parents.empty();
                    } else if (merge_rot) {
                        end_chains(chain, g);
                        if (ax) chain[g.targets[0]] = MergeChain{ax, -1, !g.parents.empty()};
                    }
                    if (mem.size() >= pass_op_cap()) break;
                } else {
                    blocked |= g.touched;
                }
            }
            return S;
        };
        std::vector<size_t> members;
        uint64_t S;
        if (chosen.size() < cached.size()) {  // as an earlier schedule of this structure
            chosen.push_back(cached[chosen.size()]);
            S = take(chosen.back().first, chosen.back().second, members);
        } else {  // search: first come, then lookahead
            chosen.push_back({low_mask, k - L});
            S = take(low_mask, k - L, members);  // first come: targets in gate order
            if (lookahead_tiles() && n > k) {
                // Lookahead: the qubits beyond the low ones one at a time, each the one whose tile
                // (the low qubits, those picked so far and it) holds the most of the remaining
                // gates; the pass keeps the choice that takes more gates.
                const uint64_t all = n >= 64 ? ~uint64_t(0) : (uint64_t(1) << n) - 1;
                auto held = [&](uint64_t Sx) {
                    uint64_t blk = 0;
                    size_t cnt = 0, acc = 0, mats = 0;
                    for (size_t i = first; i < gates.size(); ++i) {
                        if (blk == all) break;  // every later gate is blocked
                        if (done[i]) continue;
                        const PGate &g = gates[i];
                        if (acc + g.parents.size() > size_t(kMaxPassAcc)) break;
                        if (mats + mat_entries(g) > size_t(kMaxPassMats)) break;
                        if (g.dense_barrier || (g.touched & blk) || (g.needs & ~Sx)) {
                            blk |= g.touched;
                            continue;
                        }
                        ++cnt;
                        acc += g.parents.size();
                        mats += mat_entries(g);
                    }
                    return cnt;
                };
                uint64_t SL = low_mask;
                for (uint32_t pick = L; pick < k; ++pick) {
                    int best = -1;
                    size_t best_n = 0;
                    for (uint32_t q = L; q < n; ++q) {
                        if ((SL >> q) & 1) continue;
                        const size_t c = held(SL | (uint64_t(1) << q));
                        if (best < 0 || c > best_n) {
                            best = int(q);
                            best_n = c;
                        }
                    }
                    SL |= uint64_t(1) << best;
                }
                std::vector<size_t> alt;
                take(SL, 0, alt);
                if (alt.size() > members.size()) {
                    members.swap(alt);
                    S = SL;
                    chosen.back() = {SL, 0u};
                }
            }
        }
        // fill S up to k bits with the lowest unused qubits (keeps runs long)
        for (uint32_t q = 0; q < n && uint32_t(__builtin_popcountll(S)) < k; ++q) S |= uint64_t(1) << q;

        Step st;
        st.is_pass = true;
        PassHeader &h = st.header;
        std::memset(&h, 0, sizeof(h));
        h.k = k;
        h.rb = rb;
        int lpos[64];
        for (int q = 0; q < 64; ++q) lpos[q] = -1;
        {
            uint32_t j = 0;
            for (uint32_t q = 0; q < n; ++q)
                if ((S >> q) & 1) {
                    h.S[j] = uint8_t(q);
                    lpos[q] = int(j);
                    ++j;
                }
        }
        // --- sub-blocks (consecutive members whose non-diagonal targets fit in rb bits)
        std::vector<std::vector<size_t>> subs;
        std::vector<uint32_t> sub_R;  // bitmask over tile bits
        if (subblock_reorder()) {
            pack_subblocks(gates, members, lpos, rb, subs, sub_R);
        } else {
            uint32_t R = 0;
            std::vector<size_t> cur;
            for (size_t i : members) {
                uint32_t need = 0;
                if (!gates[i].diag)
                    for (uint32_t t : gates[i].targets) need |= 1u << lpos[t];
                if (uint32_t(__builtin_popcount(R | need)) > rb) {
                    subs.push_back(cur);
                    sub_R.push_back(R);
                    cur.clear();
                    R = 0;
                }
                R |= need;
                cur.push_back(i);
            }
            if (!cur.empty()) {
                subs.push_back(cur);
                sub_R.push_back(R);
            }
        }
        // --- register bits of each sub-block, padded to exactly rb
        std::vector<uint32_t> padR(subs.size());
        for (size_t sb = 0; sb < subs.size(); ++sb) {
            uint32_t R = sub_R[sb];
            for (int b = int(k) - 1; b >= 0 && uint32_t(__builtin_popcount(R)) < rb; --b)
                R |= 1u << b;
            padR[sb] = R;
        }
        // --- warp-local runs: consecutive sub-blocks that leave the same tile bits free for the
        // warp bits (thread bits 5 and up) hold every element in the same warp throughout, so
        // the exchanges between them need only __syncwarp
        std::vector<uint32_t> runW(subs.size(), 0);
        std::vector<bool> warp_next(subs.size(), false);
        if (warp_local_exchanges())
            plan_warp_runs(padR, k, rb, runW, warp_next);
        // --- emit sub-blocks, ops and matrices
        MergeChain echain[64];  // rotation merges (over the whole pass)
        for (size_t sb = 0; sb < subs.size(); ++sb) {
            const uint32_t R = padR[sb];
            SubBlock s;
            std::memset(&s, 0, sizeof(s));
            int ri = 0;
            for (uint32_t b = 0; b < k; ++b)
                if ((R >> b) & 1) s.R[ri++] = uint8_t(b);
            if (warp_next[sb]) s.flags |= SB_WARP_NEXT;
            // thread bits: three lane bits with distinct swizzle residues first, then the rest;
            // in a warp-local run the run's warp bits come last, in the same order every time
            const uint32_t W = runW[sb];
            std::vector<int> rest;
            for (uint32_t b = 0; b < k; ++b)
                if (!((R >> b) & 1) && !((W >> b) & 1)) rest.push_back(int(b));
            std::vector<int> order;
            bool used_res[3] = {false, false, false};
            for (int want = 0; want < 3; ++want)
                for (size_t i = 0; i < rest.size(); ++i) {
                    const int b = rest[i];
                    if (b < 0 || used_res[residue(b)]) continue;
                    used_res[residue(b)] = true;
                    order.push_back(b);
                    rest[i] = -1;
                    break;
                }
            for (int b : rest)
                if (b >= 0) order.push_back(b);
            for (uint32_t b = 0; b < k; ++b)
                if ((W >> b) & 1) order.push_back(int(b));
            for (size_t i = 0; i < order.size(); ++i) s.perm[i] = uint8_t(order[i]);
            s.op_begin = uint16_t(st.ops.size());
            auto reg_of = [&](uint32_t q) -> uint8_t {
                const int lp = lpos[q];
                for (int r = 0; r < int(rb); ++r)
                    if (s.R[r] == lp) return uint8_t(r);
                return 0xFF;
            };
            // Forward passes merge consecutive uncontrolled single-qubit gates on the same qubit
            // (nothing else touching it in between) into one 2x2: same arithmetic, fewer ops —
            // except two rotation-like gates in scaled passes (2 + 2 FP64 instructions per
            // amplitude apart, 8 as one dense 2x2) unless they make a diagonal.
            int last1q[64];
            for (int q = 0; q < 64; ++q) last1q[q] = -1;
            for (size_t gi : subs[sb]) {
                const PGate &g = gates[gi];
                const uint32_t ax = merge_rot ? merge_axis(g) : 0;
                if (ax && echain[g.targets[0]].axis == ax) {
                    FOp &e = st.ops[size_t(echain[g.targets[0]].op)];
                    double2 ue[4], un[4], p[4];
                    op_matrix2(e, st.mats, ue);
                    for (int i = 0; i < 4; ++i) un[i] = g.m[i];
                    mul2(un, ue, p);  // the earlier rotation acts first
                    e.moff = uint32_t(st.mats.size());
                    if (e.kind == FK_D1) {
                        if (p[1].x != 0 || p[1].y != 0 || p[2].x != 0 || p[2].y != 0)
                            fail("internal: merged diagonal rotation is not diagonal");
                        st.mats.push_back(p[0]);
                        st.mats.push_back(p[3]);
                    } else {
                        // (two rotations about one axis make one about it, the identity included)
                        if (!has_rotation_form(p, e.kind))
                            fail("internal: merged rotation lost its form");
                        st.mats.push_back(make_double2(p[0].x, e.kind == FK_RX ? -p[1].y : p[2].x));
                    }
                    if (!g.parents.empty()) {
                        if (e.gkind != GK_NONE) {
                            st.alias.push_back({e.acc[0], g.parents[0]});
                        } else {
                            e.gkind = g.gkind;
                            e.gcode = pauli_grad_code(e);
                            e.nslots = 1;
                            e.acc[0] = uint32_t(st.parents.size());
                            st.parents.push_back(g.parents[0]);
                        }
                    }
                    continue;
                }
                if (merge_rot) end_chains(echain, g);
                const bool mergeable = !adjoint && g.controls.empty() && g.targets.size() == 1 &&
                                       g.gkind == GK_NONE;
                bool merge = mergeable && last1q[g.targets[0]] >= 0;
                double2 ue[4], un[4], p[4];
                bool pdiag = false;
                if (merge) {
                    op_matrix2(st.ops[size_t(last1q[g.targets[0]])], st.mats, ue);
                    for (int i = 0; i < 4; ++i) un[i] = g.m[i];
                    mul2(un, ue, p);  // the earlier gate acts first
                    pdiag = p[1].x == 0 && p[1].y == 0 && p[2].x == 0 && p[2].y == 0;
                    const bool to_diag = pdiag &&
                                         st.ops[size_t(last1q[g.targets[0]])].kind == FK_D1;
                    if (scaled_passes() && !to_diag && rotation_form(p) == 0 &&
                        scalable_1q(ue) && scalable_1q(un))
                        merge = false;
                    // an X on the fast path is a register exchange: keep it out of a dense 2x2
                    if (fast_cnot() && (is_x(std::vector<double2>(ue, ue + 4)) ||
                                        is_x(std::vector<double2>(un, un + 4))))
                        merge = false;
                }
                if (merge) {
                    FOp &e = st.ops[size_t(last1q[g.targets[0]])];
                    e.moff = uint32_t(st.mats.size());
                    const int rot = e.kind == FK_D1 ? 0 : rotation_form(p);
                    if (pdiag && e.kind == FK_D1) {
                        st.mats.push_back(p[0]);
                        st.mats.push_back(p[3]);
                    } else if (rot != 0) {  // RX(a) RX(b), RY(a) RY(b): one rotation again
                        e.kind = uint8_t(rot);
                        e.code = rot == FK_RX ? FC_RX : FC_RY;
                        e.rb0 = reg_of(g.targets[0]);
                        if (e.rb0 == 0xFF) fail("internal: merged gate without a register target");
                        st.mats.push_back(make_double2(p[0].x, rot == FK_RX ? -p[1].y : p[2].x));
                    } else {
                        const uint8_t r = reg_of(g.targets[0]);
                        if (r == 0xFF) fail("internal: merged gate without a register target");
                        e.kind = FK_M2;
                        e.code = FC_M2;
                        e.rb0 = r;
                        for (int i = 0; i < 4; ++i) st.mats.push_back(p[i]);
                    }
                    continue;
                }
                for (uint32_t q = 0; q < 64; ++q)
                    if ((g.touched >> q) & 1) last1q[q] = -1;
                if (mergeable) last1q[g.targets[0]] = int(st.ops.size());
                FOp o;
                std::memset(&o, 0, sizeof(o));
                for (uint32_t c : g.controls) {
                    if (lpos[c] >= 0) o.lcmask |= uint16_t(1u << lpos[c]);
                    else o.gcmask |= uint64_t(1) << c;
                }
                o.moff = uint32_t(st.mats.size());
                const size_t nt = g.targets.size();
                if (g.diag) {
                    o.kind = nt == 1 ? FK_D1 : FK_D2;
                    for (size_t t = 0; t < nt; ++t) {
                        const uint32_t q = g.targets[t];
                        o.dq_in_tile[t] = lpos[q] >= 0 ? 1 : 0;
                        o.dq_pos[t] = uint8_t(lpos[q] >= 0 ? lpos[q] : int(q));
                    }
                    const size_t dim = size_t(1) << nt;
                    for (size_t i = 0; i < dim; ++i) st.mats.push_back(g.m[i * dim + i]);
                } else if (nt == 1) {
                    o.rb0 = reg_of(g.targets[0]);
                    const double2 *m = g.m.data();
                    const bool same_diag = eq(m[0], m[3]) && m[0].y == 0.0;
                    if (same_diag && m[1].x == 0.0 && eq(m[1], m[2])) {
                        o.kind = FK_RX;  // [[c, -is], [-is, c]] with m01 = (0, -s)
                        st.mats.push_back(make_double2(m[0].x, -m[1].y));
                    } else if (same_diag && m[1].y == 0.0 && m[2].y == 0.0 && m[1].x == -m[2].x) {
                        o.kind = FK_RY;  // [[c, -s], [s, c]]
                        st.mats.push_back(make_double2(m[0].x, m[2].x));
                    } else {
                        o.kind = FK_M2;
                        for (int i = 0; i < 4; ++i) st.mats.push_back(m[i]);
                    }
                } else {
                    o.kind = FK_M4;
                    o.rb0 = reg_of(g.targets[0]);
                    o.rb1 = reg_of(g.targets[1]);
                    for (int i = 0; i < 16; ++i) st.mats.push_back(g.m[i]);
                }
                classify(o, g, reg_of, lpos);
                o.gkind = g.gkind;
                if (g.gkind != GK_NONE) {
                    o.gcode = pauli_grad_code(o);
                    o.nslots = uint16_t(g.parents.size());
                    if (g.gkind == GK_GENERIC) {
                        // a diagonal gate's derivative is diagonal: store its diagonal only,
                        // in the same layout as the gate's own phases
                        const size_t dim = size_t(1) << nt;
                        for (const auto &d : g.dm) {
                            if (g.diag)
                                for (size_t i = 0; i < dim; ++i) st.mats.push_back(d[i * dim + i]);
                            else
                                for (const auto &x : d) st.mats.push_back(x);
                        }
                    }
                    for (size_t s2 = 0; s2 < g.parents.size(); ++s2) {
                        o.acc[s2] = uint32_t(st.parents.size());
                        st.parents.push_back(g.parents[s2]);
                    }
                }
                // the op must carry the axis's form (merges above rewrite it as that form)
                const uint8_t want = ax == ARCQML_OP_RZ ? FK_D1 : ax == ARCQML_OP_RX ? FK_RX : FK_RY;
                if (ax && o.kind != want) fail("internal: rotation emitted without its form");
                if (ax) echain[g.targets[0]] = MergeChain{ax, int(st.ops.size()), false};
                st.ops.push_back(o);
            }
            s.op_end = uint16_t(st.ops.size());
            st.subs.push_back(s);
        }
        // fast-path flags once every op is final (a merge can give an earlier op a gradient)
        for (SubBlock &s : st.subs) {
            s.flags |= SB_ALL_FAST | SB_JIT_FAST;
            for (size_t oi = s.op_begin; oi < s.op_end; ++oi) {
                if (!has_fast_path(st.ops[oi], adjoint)) s.flags &= ~SB_ALL_FAST;
                if (!has_jit_fast_path(st.ops[oi], adjoint)) s.flags &= ~SB_JIT_FAST;
            }
        }
        scale_pass(st, adjoint);
        h.nsub = uint32_t(st.subs.size());
        h.nops = uint32_t(st.ops.size());
        h.nmat = uint32_t(st.mats.size());
        h.nacc = uint32_t(st.parents.size());
        h.acc_base = acc_total;
        acc_total += h.nacc;
        for (size_t i : members) done[i] = 1;
        sch.steps.push_back(std::move(st));
    }
    sch.total_acc = acc_total;
    if (cached.empty()) {
        std::lock_guard<std::mutex> lock(plan.tiles_mu);
        bool stored = false;
        for (TileChoices &t : plan.tiles)
            if (t.key == ckey) {
                t.signature = sig;
                t.take = chosen;
                stored = true;
            }
        if (!stored) {
            if (plan.tiles.size() >= 8) plan.tiles.erase(plan.tiles.begin());
            plan.tiles.push_back(TileChoices{ckey, sig, chosen});
        }
    }
    return sch;
}

}  // namespace arcqml
