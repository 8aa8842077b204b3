// jit.cpp — per-pass fused kernels compiled at run time.
//
// The precompiled pass kernel (fused.cu) interprets the pass's op table: per op it loads the op
// descriptor, branches on its kind and register bits, and only then does the arithmetic, so the
// dependent-latency chains of consecutive gates cannot overlap. Here each pass whose ops all have
// fast paths becomes its own kernel: the same tile loop (fused_body in fused_core.cuh) with the
// pass's gates written out in order, register bits as template constants and matrix offsets as
// literals. The compiler then schedules across gates. Parameter values stay in the uploaded
// matrix table, so a kernel is reused for every parameter vector of the same circuit structure
// (kernels are cached by their source text, per device, and by the pass's structure).
//
// Compilation goes through NVRTC (loaded on first use) for sm_100a; the cubin is loaded with the
// driver API reached through cudaGetDriverEntryPoint, so the library links no driver or NVRTC
// import at build time. ARCQML_JIT=0 turns the path off; a pass that fails to compile runs on the
// precompiled kernel and the failure is reported by arcqml_rt_v2_jit_info.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nvrtc.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <functional>
#include <mutex>
#include <sstream>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "fused.h"
#include "jit.h"
#include "planner.h"
#include "rt_internal.h"

#include "jit_source.inc"

namespace arcqml {
namespace {

// Largest matrix table passed by value: kernel parameters may total 32764 bytes (sm_70 and
// later, CUDA 12.1 and later); the other arguments take under 100.
constexpr size_t kJitMaxParamMats = 32000;

// ---------------------------------------------------------------- NVRTC and driver entry points

struct Nvrtc {
    bool tried = false, ok = false;
    std::string why;
    nvrtcResult (*create)(nvrtcProgram *, const char *, const char *, int, const char *const *,
                          const char *const *) = nullptr;
    nvrtcResult (*compile)(nvrtcProgram, int, const char *const *) = nullptr;
    nvrtcResult (*log_size)(nvrtcProgram, size_t *) = nullptr;
    nvrtcResult (*log)(nvrtcProgram, char *) = nullptr;
    nvrtcResult (*cubin_size)(nvrtcProgram, size_t *) = nullptr;
    nvrtcResult (*cubin)(nvrtcProgram, char *) = nullptr;
    nvrtcResult (*destroy)(nvrtcProgram *) = nullptr;
};

struct Driver {
    bool tried = false, ok = false;
    std::string why;
    CUresult (*load)(CUmodule *, const void *) = nullptr;
    CUresult (*get)(CUfunction *, CUmodule, const char *) = nullptr;
    CUresult (*set_attr)(CUfunction, CUfunction_attribute, int) = nullptr;
    CUresult (*get_attr)(int *, CUfunction_attribute, CUfunction) = nullptr;
    CUresult (*occupancy)(int *, CUfunction, int, size_t) = nullptr;
    CUresult (*launch)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                       unsigned, CUstream, void **, void **) = nullptr;
};

std::mutex g_mu;
Nvrtc g_nvrtc;
Driver g_drv;

template <class F>
bool sym(void *lib, const char *name, F &out) {
    out = reinterpret_cast<F>(dlsym(lib, name));
    return out != nullptr;
}

bool load_nvrtc() {
    if (g_nvrtc.tried) return g_nvrtc.ok;
    g_nvrtc.tried = true;
    void *lib = dlopen("libnvrtc.so.12", RTLD_NOW | RTLD_LOCAL);
    if (!lib) lib = dlopen("/usr/local/cuda/lib64/libnvrtc.so.12", RTLD_NOW | RTLD_LOCAL);
    if (!lib) {
        g_nvrtc.why = "libnvrtc.so.12 not found";
        return false;
    }
    g_nvrtc.ok = sym(lib, "nvrtcCreateProgram", g_nvrtc.create) &&
                 sym(lib, "nvrtcCompileProgram", g_nvrtc.compile) &&
                 sym(lib, "nvrtcGetProgramLogSize", g_nvrtc.log_size) &&
                 sym(lib, "nvrtcGetProgramLog", g_nvrtc.log) &&
                 sym(lib, "nvrtcGetCUBINSize", g_nvrtc.cubin_size) &&
                 sym(lib, "nvrtcGetCUBIN", g_nvrtc.cubin) &&
                 sym(lib, "nvrtcDestroyProgram", g_nvrtc.destroy);
    if (!g_nvrtc.ok) g_nvrtc.why = "libnvrtc.so.12 lacks a needed entry point";
    return g_nvrtc.ok;
}

template <class F>
bool entry(const char *name, F &out) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !p)
        return false;
    out = reinterpret_cast<F>(p);
    return true;
}

bool load_driver() {
    if (g_drv.tried) return g_drv.ok;
    g_drv.tried = true;
    g_drv.ok = entry("cuModuleLoadData", g_drv.load) && entry("cuModuleGetFunction", g_drv.get) &&
               entry("cuFuncSetAttribute", g_drv.set_attr) &&
               entry("cuFuncGetAttribute", g_drv.get_attr) &&
               entry("cuOccupancyMaxActiveBlocksPerMultiprocessor", g_drv.occupancy) &&
               entry("cuLaunchKernel", g_drv.launch);
    if (!g_drv.ok) g_drv.why = "driver entry points unavailable";
    return g_drv.ok;
}

// ---------------------------------------------------------------- code generation

bool adjoint_per_warp();
// Adjoint kernels with 4 register bits (tiles of 12 qubits) keep one accumulator column per warp
// so that psi, lambda and the accumulators fit one CTA's shared memory.
bool acc_per_warp(bool adj, uint32_t rb) { return adj && (adjoint_per_warp() || rb == 4); }

bool adjoint_two_ctas();
// Adjoint kernels on 3 register bits at two CTAs per SM (unless ARCQML_ADJ_2CTA=0) keep one
// accumulator column per four lanes, so that two CTAs' tiles and columns fit one SM.
uint32_t acc_lanes(bool adj, uint32_t rb) {
    if (acc_per_warp(adj, rb)) return 32u;
    return (adj && rb == 3 && adjoint_two_ctas()) ? 4u : 1u;
}

// Compiled adjoint kernels with 3 register bits ask for two CTAs per SM (ARCQML_ADJ_2CTA=0:
// one CTA with a column per thread; two measured 4 % faster at 30 qubits).
bool adjoint_two_ctas() {
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_ADJ_2CTA");
        return !(e && e[0] == '0');
    }();
    return on;
}

// ARCQML_JIT_ADJ_WARP=1: adjoint kernels reduce each gradient over the warp (one accumulator
// column per warp instead of per thread) and ask for two resident CTAs per SM.
bool adjoint_per_warp() {
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_JIT_ADJ_WARP");
        return e && e[0] == '1';
    }();
    return on;
}

}  // namespace

// Compiled forward kernels keep one tile buffer and ask for
// two resident CTAs per SM, so that one CTA's loads and shared-memory exchanges overlap the
// other's arithmetic (ARCQML_FWD_SINGLE=0: two buffers, one CTA per SM).
bool jit_forward_single() {
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_FWD_SINGLE");
        return !(e && e[0] == '0');
    }();
    return on;
}

bool jit_mats_in_params(bool adjoint) {
    (void)adjoint;  // forward and adjoint kernels alike
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_JIT_MATS_SMEM");
        return !(e && e[0] == '1');
    }();
    return on;
}

namespace {

// Host copy of the shared-memory swizzle of fused_core.cuh (phys): j ^ fold of its 3-bit groups.
uint32_t swizzle(uint32_t j) { return j ^ (((j >> 3) ^ (j >> 6) ^ (j >> 9)) & 7u); }

// Per-thread value of the op's qubit `slot` when it is not a register bit (fast paths D1_UNI and
// the sign flips): a tile bit of the thread's base index, or a bit of the tile's global base.
std::string const_bit(const FOp &o, int slot, const SubBlock &S, uint32_t thread_bits) {
    std::ostringstream e;
    if (o.dq_in_tile[slot]) {
        int bit = -1;
        for (uint32_t i = 0; i < thread_bits; ++i)
            if (S.perm[i] == o.dq_pos[slot]) bit = int(i);
        if (bit < 0) return std::string();
        e << "((tid >> " << bit << ") & 1u)";
    } else {
        e << "uint32_t((gbase >> " << int(o.dq_pos[slot]) << ") & 1ull)";
    }
    return e.str();
}

// ---------------------------------------------------------------- ops on general bit positions
//
// On unless ARCQML_FAST_DIAG=0 (FC_DIAG, FC_CM2 and the generic gradients): every qubit of the op — a
// diagonal index bit or a control — is a register bit of the sub-block, known per register
// element when the code is generated, or a per-thread 0/1 value (a thread bit of the tile, or
// a bit of the tile's global base). Register controls select the elements the code lists;
// per-thread controls become one condition around them.

struct BitPos {
    int reg = -1;     // register bit, or -1
    std::string val;  // otherwise the per-thread value ("" if the bit is neither)
};

BitPos tile_bit_pos(uint32_t lb, const SubBlock &S, uint32_t rb, uint32_t tbits) {
    BitPos p;
    for (uint32_t r = 0; r < rb; ++r)
        if (S.R[r] == lb) {
            p.reg = int(r);
            return p;
        }
    for (uint32_t i = 0; i < tbits; ++i)
        if (S.perm[i] == lb) {
            p.val = "((tid >> " + std::to_string(i) + ") & 1u)";
            return p;
        }
    return p;
}

BitPos global_bit_pos(uint32_t q) {
    BitPos p;
    p.val = "uint32_t((gbase >> " + std::to_string(q) + ") & 1ull)";
    return p;
}

struct OpBits {
    bool ok = true;
    uint32_t creg = 0;  // register bits every control of which must be 1
    std::string cond;   // per-thread control condition ("" if none)
    int nslot = 0;      // diagonal ops: entry index = sum over slots s of bit(s) << s
    BitPos slot[2];
    std::string uval;   // per-thread part of the entry index ("" if none)

    bool active(uint32_t e) const { return (e & creg) == creg; }
    uint32_t entry(uint32_t e) const {  // register part of element e's entry index
        uint32_t x = 0;
        for (int s = 0; s < nslot; ++s)
            if (slot[s].reg >= 0) x |= ((e >> slot[s].reg) & 1u) << s;
        return x;
    }
    std::string open() const { return cond.empty() ? "{ " : "if (" + cond + ") { "; }
    // matrix-table element of entry x (its per-thread part in `u`)
    std::string at(uint32_t base, uint32_t x) const {
        std::ostringstream e;
        if (uval.empty()) e << "M[" << base + x << "]";
        else e << "M[" << base << "u + (u | " << x << "u)]";
        return e.str();
    }
    std::string decl_u() const { return uval.empty() ? "" : "const uint32_t u = " + uval + "; "; }
};

OpBits op_bits(const FOp &o, const SubBlock &S, uint32_t rb, uint32_t tbits) {
    OpBits b;
    std::vector<std::string> conds;
    for (uint32_t t = 0; t < 16; ++t) {
        if (!((o.lcmask >> t) & 1u)) continue;
        const BitPos p = tile_bit_pos(t, S, rb, tbits);
        if (p.reg >= 0) b.creg |= 1u << p.reg;
        else if (!p.val.empty()) conds.push_back(p.val);
        else b.ok = false;
    }
    for (uint32_t q = 0; q < 64; ++q)
        if ((o.gcmask >> q) & 1u) conds.push_back(global_bit_pos(q).val);
    for (size_t i = 0; i < conds.size(); ++i) b.cond += (i ? " & " : "") + conds[i];
    if (o.kind == FK_D1 || o.kind == FK_D2) {
        b.nslot = o.kind == FK_D1 ? 1 : 2;
        for (int s = 0; s < b.nslot; ++s) {
            b.slot[s] = o.dq_in_tile[s] ? tile_bit_pos(o.dq_pos[s], S, rb, tbits)
                                        : global_bit_pos(o.dq_pos[s]);
            const BitPos &p = b.slot[s];
            if (p.reg >= 0) continue;
            if (p.val.empty()) b.ok = false;
            if (!b.uval.empty()) b.uval += " | ";
            b.uval += s ? "(" + p.val + " << 1)" : p.val;
        }
    }
    return b;
}

// U (or U^dagger) of an FC_DIAG or FC_CM2 op on the register array `r`.
bool emit_general_apply(std::ostringstream &c, const FOp &o, const char *r, uint32_t rb,
                        const SubBlock &S, uint32_t tbits) {
    const OpBits b = op_bits(o, S, rb, tbits);
    if (!b.ok) return false;
    const uint32_t N = 1u << rb, m = o.moff;
    if (o.code == FC_DIAG) {
        if (b.nslot == 0) return false;
        c << "{ " << b.decl_u() << b.open();
        bool need[4] = {false, false, false, false};
        for (uint32_t e = 0; e < N; ++e)
            if (b.active(e)) need[b.entry(e)] = true;
        for (uint32_t x = 0; x < 4; ++x)
            if (need[x]) c << "const double2 d" << x << " = " << b.at(m, x) << "; ";
        for (uint32_t e = 0; e < N; ++e)
            if (b.active(e))
                c << r << "[" << e << "] = cmul(d" << b.entry(e) << ", " << r << "[" << e << "]); ";
        c << "} }";
        return true;
    }
    if (o.code != FC_CM2) return false;
    const uint32_t t = 1u << o.rb0;
    if (o.rb0 >= rb || (b.creg & t)) return false;
    c << "{ " << b.open();
    for (uint32_t e = 0; e < N; ++e) {
        if ((e & t) || !b.active(e)) continue;
        const std::string x0 = std::string(r) + "[" + std::to_string(e) + "]";
        const std::string x1 = std::string(r) + "[" + std::to_string(e | t) + "]";
        if (o.kind == FK_RX) c << "p_rx(" << x0 << ", " << x1 << ", M[" << m << "].x, M[" << m << "].y); ";
        else if (o.kind == FK_RY) c << "p_ry(" << x0 << ", " << x1 << ", M[" << m << "].x, M[" << m << "].y); ";
        else if (o.kind == FK_M2) c << "p_m2(" << x0 << ", " << x1 << ", M + " << m << "); ";
        else return false;
    }
    c << "} }";
    return true;
}

// The fast path of op o on the register array `r` (U in forward passes, U^dagger in adjoint
// passes: the planner stores the daggered matrices). False for a combination without one.
bool emit_apply(std::ostringstream &c, const FOp &o, const char *r, uint32_t rb,
                const SubBlock &S, uint32_t tbits) {
    if (o.code == FC_DIAG || o.code == FC_CM2) return emit_general_apply(c, o, r, rb, S, tbits);
    const int b0 = o.rb0, b1 = o.rb1;
    const std::string bit0 = (o.code == FC_D1_UNI || o.code == FC_SIGN_RC || o.code == FC_SIGN_CC ||
                              o.code == FC_CX_CR)
                                 ? const_bit(o, 0, S, tbits) : std::string("0u");
    const std::string bit1 = o.code == FC_SIGN_CC ? const_bit(o, 1, S, tbits) : std::string("0u");
    if (bit0.empty() || bit1.empty()) return false;
    const uint32_t m = o.moff;
    const bool uses_b0 = o.code != FC_D1_UNI && o.code != FC_SIGN_CC;
    const bool uses_b1 = o.code == FC_SIGN_RR || o.code == FC_M4 || o.code == FC_CX_RR;
    if ((uses_b0 && b0 >= int(rb)) || (uses_b1 && b1 >= int(rb))) return false;
    const uint32_t so = o.soff;
    if (o.sform) {  // scaled unit-diagonal form (mats[soff].x = t or tau)
        switch (o.code) {
        case FC_RX: c << "fs_rx<RB, " << b0 << ">(" << r << ", M[" << so << "].x);"; return true;
        case FC_RY: c << "fs_ry<RB, " << b0 << ">(" << r << ", M[" << so << "].x);"; return true;
        case FC_D1_REG:
            c << "fs_d1_reg<RB, " << b0 << ">(" << r << ", M[" << so << "].x);";
            return true;
        case FC_D1_UNI:
            c << "fs_d1_uni<RB>(" << r << ", " << bit0 << " ? M[" << so << "].x : -M[" << so
              << "].x);";
            return true;
        default: return false;
        }
    }
    switch (o.code) {
    case FC_RX:
        c << "f_rx<RB, " << b0 << ">(" << r << ", M[" << m << "].x, M[" << m << "].y);";
        break;
    case FC_RY:
        c << "f_ry<RB, " << b0 << ">(" << r << ", M[" << m << "].x, M[" << m << "].y);";
        break;
    case FC_M2: c << "f_m2<RB, " << b0 << ">(" << r << ", M + " << m << ");"; break;
    case FC_D1_REG:
        c << "f_d1_reg<RB, " << b0 << ">(" << r << ", M[" << m << "], M[" << m + 1 << "]);";
        break;
    case FC_D1_UNI:
        c << "f_d1_uni<RB>(" << r << ", " << bit0 << " ? M[" << m + 1 << "] : M[" << m
          << "]);";
        break;
    case FC_SIGN_RR: c << "f_sign_rr<RB, " << b0 << ", " << b1 << ">(" << r << ");"; break;
    case FC_SIGN_RC:
        c << "f_sign_rc<RB, " << b0 << ">(" << r << ", " << bit0
          << " ? 0x80000000u : 0u);";
        break;
    case FC_SIGN_CC:
        c << "f_sign_cc<RB>(" << r << ", (" << bit0 << " & " << bit1
          << ") ? 0x80000000u : 0u);";
        break;
    case FC_M4: c << "f_m4<RB, " << b0 << ", " << b1 << ">(" << r << ", M + " << m << ");"; break;
    case FC_X: c << "f_x<RB, " << b0 << ">(" << r << ");"; break;
    case FC_CX_RR: c << "f_cx_rr<RB, " << b1 << ", " << b0 << ">(" << r << ");"; break;
    case FC_CX_CR: c << "f_cx_cr<RB, " << b0 << ">(" << r << ", " << bit0 << ");"; break;
    default: return false;
    }
    return true;
}

// Per pass-local accumulator row, the factor its total is multiplied by (an expression in the
// pass's matrix table M): rows are summed unscaled, the factor applied once per row per CTA.
using RowFactors = std::vector<std::string>;
void set_factor(RowFactors &rf, uint32_t row, const std::string &f) {
    if (rf.size() <= row) rf.resize(row + 1, "1.0");
    rf[row] = f;
}

// Where the generated code puts a gradient sum `z` of accumulator row `row`. With one column per
// four lanes, sums are paired: the first of a pair waits in zp[0], the second triggers
// accumulate_quad2 (one shuffle round halves the pair over lane bit 0, a second sums over bit 1);
// a sum left unpaired at the end of a sub-block goes through accumulate_quad alone.
struct AccSink {
    RowFactors rf;
    uint32_t lanes = 1;
    int pending = -1;  // row waiting in zp[0], or -1
};
void emit_acc(std::ostringstream &c, AccSink &a, uint32_t row) {
    if (a.lanes != 4u) {
        c << (a.lanes == 32u ? "accumulate_warp" : "accumulate") << "(sacc, " << row
          << "u * kCols, z); ";
        return;
    }
    if (a.pending < 0) {
        c << "zp[0] = z; ";
        a.pending = int(row);
        return;
    }
    c << "accumulate_quad2(sacc, zp[0], z, " << a.pending << "u * kCols, " << row
      << "u * kCols); ";
    a.pending = -1;
}
void flush_acc(std::ostringstream &c, AccSink &a) {
    if (a.pending < 0) return;
    c << "        accumulate_quad(sacc, " << a.pending << "u * kCols, zp[0]);\n";
    a.pending = -1;
}

// Gradients on general bit positions (on unless ARCQML_FAST_DIAG=0), in the order of the table-driven
// kernel: a Pauli-rotation gradient Im<lam|P|psi> on psi before U^dagger (X / Y over the
// target pairs whose controls are set, Z with the sign of the target bit), then U^dagger on
// psi, then each generic slot gradient Re<lam| dU_s |U^dagger psi>, then U^dagger on lambda.
// In a scaled pass psi and lambda carry the pass factor sigma from before the op (which keeps
// its plain form), so each sum is multiplied by |sigma|^2 = 2 * mats[soff].y.
bool emit_adjoint_general(std::ostringstream &c, const FOp &o, uint32_t rb, const SubBlock &S,
                          uint32_t tbits, AccSink &acc) {
    const OpBits b = op_bits(o, S, rb, tbits);
    if (!b.ok) return false;
    const bool diag = o.kind == FK_D1 || o.kind == FK_D2;
    const bool one = o.kind == FK_RX || o.kind == FK_RY || o.kind == FK_M2;
    const bool four = o.kind == FK_M4;
    const uint32_t N = 1u << rb, t0 = 1u << o.rb0, t1 = 1u << o.rb1;
    if ((one || four) && (o.rb0 >= rb || (b.creg & t0))) return false;
    if (four && (o.rb1 >= rb || o.rb1 == o.rb0 || b.creg || !b.cond.empty())) return false;
    const std::string so = std::to_string(o.soff);
    // the sum goes into the row unscaled; its factor is applied once to the row's total
    auto put_acc = [&](uint32_t slot, bool pauli) {
        emit_acc(c, acc, o.acc[slot]);
        if (pauli) set_factor(acc.rf, o.acc[slot], o.sgrad ? "M[" + so + "].y" : "0.5");
        else set_factor(acc.rf, o.acc[slot], o.sgrad ? "2.0 * M[" + so + "].y" : "1.0");
    };
    auto apply_to = [&](const char *r) {
        c << "\n        ";
        if (!emit_apply(c, o, r, rb, S, tbits)) return false;
        c << "\n        ";
        return true;
    };
    auto apply_both = [&]() { return apply_to("v") && apply_to("w"); };
    auto reg = [](const char *a, uint32_t e) { return std::string(a) + "[" + std::to_string(e) + "]"; };
    if (o.gkind == GK_PX || o.gkind == GK_PY) {
        if (!one) return false;
        c << "{ double z = 0.0; " << b.open();
        for (uint32_t e = 0; e < N; ++e) {
            if ((e & t0) || !b.active(e)) continue;
            const uint32_t f = e | t0;
            c << "z += " << (o.gkind == GK_PX ? "p_gx(" : "p_gy(") << reg("v", e) << ", "
              << reg("v", f) << ", " << reg("w", e) << ", " << reg("w", f) << "); ";
        }
        c << "}";
        if (!apply_both()) return false;
        put_acc(0, true);
        c << "}";
        return true;
    }
    if (o.gkind == GK_PZ) {
        if (o.kind != FK_D1) return false;
        const BitPos &q = b.slot[0];
        c << "{ double z = 0.0; " << b.open();
        for (uint32_t e = 0; e < N; ++e) {
            if (!b.active(e)) continue;
            const bool neg = q.reg >= 0 && ((e >> q.reg) & 1u);
            c << "z " << (neg ? "-" : "+") << "= icm(" << reg("w", e) << ", " << reg("v", e) << "); ";
        }
        c << "} ";
        if (q.reg < 0) c << "if (" << q.val << ") z = -z;";
        if (!apply_both()) return false;
        put_acc(0, true);
        c << "}";
        return true;
    }
    if (o.gkind != GK_GENERIC) return false;
    // U's entries, then nslots derivative blocks of the same shape (diagonals: their diagonal)
    const uint32_t ulen = o.kind == FK_RX || o.kind == FK_RY ? 1u
                          : o.kind == FK_M2 ? 4u : o.kind == FK_D1 ? 2u : o.kind == FK_D2 ? 4u : 16u;
    const uint32_t dlen = o.kind == FK_D1 ? 2u : o.kind == FK_M4 ? 16u : 4u;
    if (o.nslots < 1 || o.nslots > 3) return false;
    c << "{";
    if (!apply_to("v")) return false;
    if (diag) {
        // s_x = sum of conj(lambda) psi over the elements on diagonal entry x (once for all
        // slots), then each slot's sum is Re(sum_x d_s[x] s_x)
        bool need[4] = {false, false, false, false};
        for (uint32_t e = 0; e < N; ++e)
            if (b.active(e)) need[b.entry(e)] = true;
        c << "{ " << b.decl_u();
        for (uint32_t x = 0; x < 4; ++x)
            if (need[x]) c << "double2 s" << x << " = make_double2(0.0, 0.0); ";
        c << b.open();
        for (uint32_t e = 0; e < N; ++e)
            if (b.active(e))
                c << "acc_cw(s" << b.entry(e) << ", " << reg("w", e) << ", " << reg("v", e) << "); ";
        c << "}";
        for (uint32_t s = 0; s < o.nslots; ++s) {
            const uint32_t d = o.moff + ulen + s * dlen;
            c << "\n        { double z = 0.0; ";
            for (uint32_t x = 0; x < 4; ++x)
                if (need[x])
                    c << "{ const double2 g = " << b.at(d, x) << "; z = fma(g.x, s" << x
                      << ".x, fma(-g.y, s" << x << ".y, z)); } ";
            put_acc(s, false);
            c << "}";
        }
        c << " }";
        if (!apply_to("w")) return false;
        c << "}";
        return true;
    }
    if (one) {
        // s_ij = sum over the target pairs of conj(lambda_i) psi_j (once for all slots), then
        // each slot's sum is Re(sum_ij dU_s[i][j] s_ij)
        c << "{ double2 s00 = make_double2(0.0, 0.0), s01 = s00, s10 = s00, s11 = s00; "
          << b.open();
        for (uint32_t e = 0; e < N; ++e) {
            if ((e & t0) || !b.active(e)) continue;
            const std::string v0 = reg("v", e), v1 = reg("v", e | t0);
            const std::string w0 = reg("w", e), w1 = reg("w", e | t0);
            c << "acc_cw(s00, " << w0 << ", " << v0 << "); acc_cw(s01, " << w0 << ", " << v1
              << "); acc_cw(s10, " << w1 << ", " << v0 << "); acc_cw(s11, " << w1 << ", " << v1
              << "); ";
        }
        c << "}";
        for (uint32_t s = 0; s < o.nslots; ++s) {
            const uint32_t d = o.moff + ulen + s * dlen;
            c << "\n        { const double2 *g = M + " << d << "; double z = 0.0; ";
            const char *sij[4] = {"s00", "s01", "s10", "s11"};
            for (int i = 0; i < 4; ++i)
                c << "z = fma(g[" << i << "].x, " << sij[i] << ".x, fma(-g[" << i << "].y, "
                  << sij[i] << ".y, z)); ";
            put_acc(s, false);
            c << "}";
        }
        c << " }";
        if (!apply_to("w")) return false;
        c << "}";
        return true;
    }
    // an uncontrolled dense 4x4: Re<lam| dU_s |psi> group by group
    for (uint32_t s = 0; s < o.nslots; ++s) {
        const uint32_t d = o.moff + ulen + s * dlen;
        c << "{ double z = 0.0; ";
        for (uint32_t e = 0; e < N; ++e) {
            if (e & (t0 | t1)) continue;
            const uint32_t i[4] = {e, e | t0, e | t1, e | t0 | t1};
            c << "z += q_gm4(M + " << d;
            for (const char *a : {"v", "w"})
                for (uint32_t j : i) c << ", " << reg(a, j);
            c << "); ";
        }
        put_acc(s, false);
        c << "}";
    }
    if (!apply_to("w")) return false;
    c << "}";
    return true;
}

// Gradient then U^dagger on psi and lambda, as adj_fast does it.
bool emit_adjoint(std::ostringstream &c, const FOp &o, uint32_t rb, const SubBlock &S,
                  uint32_t tbits, AccSink &acc) {
    if (o.gkind == GK_NONE) {
        if (!emit_apply(c, o, "v", rb, S, tbits)) return false;
        c << "\n        ";
        return emit_apply(c, o, "w", rb, S, tbits);
    }
    const bool pauli_fast = (o.code == FC_RX && o.gcode == GF_X) ||
                            (o.code == FC_RY && o.gcode == GF_Y) ||
                            (o.code == FC_D1_REG && o.gcode == GF_Z_REG) ||
                            (o.code == FC_D1_UNI && o.gcode == GF_Z_UNI);
    if (!pauli_fast) return fast_diag() && emit_adjoint_general(c, o, rb, S, tbits, acc);
    const int b0 = o.rb0;
    if (b0 >= int(rb) && o.code != FC_D1_UNI) return false;
    c << "{ double z; ";
    if (o.code == FC_RX && o.gcode == GF_X) c << "z = g_x<RB, " << b0 << ">(v, w);";
    else if (o.code == FC_RY && o.gcode == GF_Y) c << "z = g_y<RB, " << b0 << ">(v, w);";
    else if (o.code == FC_D1_REG && o.gcode == GF_Z_REG) c << "z = g_z<RB, " << b0 << ">(v, w);";
    else if (o.code == FC_D1_UNI && o.gcode == GF_Z_UNI) {
        const std::string bit = const_bit(o, 0, S, tbits);
        if (bit.empty()) return false;
        c << "z = g_z_uni<RB>(v, w); if (" << bit << ") z = -z;";
    } else {
        return false;
    }
    c << "\n        ";
    if (!emit_apply(c, o, "v", rb, S, tbits)) return false;
    c << "\n        ";
    if (!emit_apply(c, o, "w", rb, S, tbits)) return false;
    // the row's factor, applied to its total: 0.5, times |sigma|^2 in a scaled pass
    c << "\n        ";
    emit_acc(c, acc, o.acc[0]);
    c << "}";
    set_factor(acc.rf, o.acc[0], o.sgrad ? "M[" + std::to_string(o.soff) + "].y" : "0.5");
    return true;
}

// Source of the kernel `arcqml_pass` for one pass; empty when some op has no fast path.
std::string pass_source(const Step &st, bool adj, uint32_t rb) {
    std::ostringstream c;
    const uint32_t threads = 1u << (st.header.k - rb);
    const uint32_t cols = acc_row_stride(threads / acc_lanes(adj, rb), acc_lanes(adj, rb));
    const bool single = !adj && jit_forward_single();
    const bool params = jit_mats_in_params(adj);
    // the pass's matrix table as one by-value kernel parameter (constant-bank operands)
    const size_t nmats = st.mats.empty() ? 1 : st.mats.size();
    if (params && nmats * sizeof(double2) > kJitMaxParamMats) return std::string();
    if (params) c << "struct PassMats { double2 m[" << nmats << "]; };\n";
    AccSink acc;
    acc.lanes = adj ? acc_lanes(adj, rb) : 1u;
    c << "struct PassOps {\n"
         "    static constexpr int kAccLanes = " << acc_lanes(adj, rb) << ";\n"
         "    static constexpr bool kSingleBuffer = " << (single ? "true" : "false") << ";\n"
         "    static constexpr bool kOpsInSmem = false;\n"
         "    static constexpr bool kMatsInSmem = " << (params ? "false" : "true") << ";\n"
         // the next tile into L2 while this one is computed: adjoint kernels only (32 qubits:
         // adjoint passes 0.7 % faster with it, forward passes 1 % faster without)
         "    static constexpr bool kPrefetch = " << (adj ? "true" : "false") << ";\n"
         "    template <int RB, bool ADJ, class MT>\n"
         "    __device__ static __forceinline__ void run(uint32_t sb, uint32_t, double2 *tp,\n"
         "            double2 *tl, const FOp *, const MT &MS, const SubBlock *, double *sacc,\n"
         "            uint32_t nthreads, uint64_t gbase) {\n"
         "        const auto &M = mats_of(MS);\n"
         "        double2 v[1 << RB], w[1 << RB];\n"
         "        double zp[1];  // a gradient sum waiting for its pair (accumulate_quad2)\n"
         "        (void)zp;\n"
         "        constexpr uint32_t kCols = " << cols << "u;  // accumulator row stride\n"
         "        const uint32_t tid = threadIdx.x;\n"
         "        uint32_t p;\n"
         "        switch (sb) {\n";
    for (size_t sb = 0; sb < st.subs.size(); ++sb) {
        const SubBlock &S = st.subs[sb];
        if (!(S.flags & SB_JIT_FAST)) return std::string();
        // Swizzled shared-memory slot of register element e: phys is linear over XOR and tb
        // shares no bit with the element's register bits, so slot = phys(tb) ^ phys(bits of e).
        std::vector<uint32_t> slot(size_t(1) << rb);
        for (uint32_t e = 0; e < slot.size(); ++e) {
            uint32_t x = 0;
            for (uint32_t r = 0; r < rb; ++r)
                if ((e >> r) & 1u) x |= 1u << S.R[r];
            slot[e] = swizzle(x);
        }
        c << "        case " << sb << ":\n";
        // the thread's swizzled base: thread bit i is tile bit S.perm[i]
        const uint32_t kb = st.header.k - rb;
        c << "        p = 0u";
        for (uint32_t i = 0; i < kb; ++i)
            c << " ^ (((tid >> " << i << ") & 1u) * " << swizzle(1u << S.perm[i]) << "u)";
        c << ";\n";
        for (uint32_t e = 0; e < slot.size(); ++e) {
            c << "        v[" << e << "] = tp[p ^ " << slot[e] << "u];";
            if (adj) c << " w[" << e << "] = tl[p ^ " << slot[e] << "u];";
            c << "\n";
        }
        for (uint32_t oi = S.op_begin; oi < S.op_end; ++oi) {
            c << "        ";
            const bool ok = adj ? emit_adjoint(c, st.ops[oi], rb, S, kb, acc)
                                : emit_apply(c, st.ops[oi], "v", rb, S, kb);
            if (!ok) return std::string();
            c << "\n";
        }
        flush_acc(c, acc);  // a sum left unpaired: before the registers leave the sub-block
        if (st.scaled && sb + 1 == st.subs.size()) {
            c << "        fs_scale<RB>(v, M[" << st.sfin << "]);";
            if (adj) c << " fs_scale<RB>(w, M[" << st.sfin << "]);";
            c << "\n";
        }
        for (uint32_t e = 0; e < slot.size(); ++e) {
            c << "        tp[p ^ " << slot[e] << "u] = v[" << e << "];";
            if (adj) c << " tl[p ^ " << slot[e] << "u] = w[" << e << "];";
            c << "\n";
        }
        c << "        break;\n";
    }
    c << "        }\n"
         "    }\n";
    // sub-blocks whose successor keeps every element in the same warp
    c << "    __device__ static __forceinline__ bool warp_next(uint32_t sb) {\n"
         "        switch (sb) {\n";
    for (size_t sb = 0; sb < st.subs.size(); ++sb)
        if (st.subs[sb].flags & SB_WARP_NEXT) c << "        case " << sb << ":\n";
    c << "            return true;\n"
         "        default: return false;\n"
         "        }\n"
         "    }\n";
    // factors of the accumulator rows (adjoint), applied to each row's total
    c << "    template <class MT>\n"
         "    __device__ static __forceinline__ double row_factor(uint32_t a, const MT &MS) {\n"
         "        const auto &M = mats_of(MS);\n"
         "        (void)M;\n"
         "        switch (a) {\n";
    for (size_t r = 0; r < acc.rf.size(); ++r)
        c << "        case " << r << ": return " << acc.rf[r] << ";\n";
    c << "        default: return 1.0;\n"
         "        }\n"
         "    }\n"
         "};\n";
    // Kernels made for several CTAs per SM ask for that many resident CTAs: adjoint kernels
    // 512 resident threads per SM (two CTAs of 256, four of 128: 128 registers); forward kernels
    // two CTAs of 256 threads, and 1024 threads per SM in smaller CTAs (64 registers: the
    // small-state forward passes, e.g. the batched QNN's rows, run faster with more warps than
    // with more registers). The others run one CTA per SM.
    const bool multi_adj = adj && (adjoint_per_warp() || adjoint_two_ctas()) && rb == 3;
    const bool multi_fwd = single && threads <= 256;
    const uint32_t per_sm = multi_adj ? 512u : (threads >= 256 ? 512u : 1024u);
    const bool multi = multi_adj || multi_fwd;
    const int bound = multi ? int(threads) : ((adj || rb == 4) ? 256 : 512);
    const int min_blocks = multi ? int(per_sm / threads) : 1;
    c << "extern \"C\" __global__ void __launch_bounds__(" << bound << ", " << min_blocks << ")\n"
         "arcqml_pass(double2 *__restrict__ psi, double2 *__restrict__ lam, uint32_t n,\n"
         "            uint32_t tiles_log, uint64_t total_tiles, const PassHeader *__restrict__ hdr,\n"
         "            const SubBlock *__restrict__ subs, const FOp *__restrict__ gops,\n"
      << (params ? "            const __grid_constant__ PassMats pm,"
                 : "            const double2 *__restrict__ gmats,")
      << " double *__restrict__ partials,\n"
         "            uint32_t stride) {\n"
         "    fused_body<" << rb << ", " << (adj ? "true" : "false")
      << ", PassOps, " << st.header.k << ">(psi, lam, n, tiles_log, total_tiles, hdr, subs, gops, "
      << (params ? "pm" : "gmats") << ", partials, stride);\n}\n";
    return c.str();
}

std::string full_source(const std::string &pass) {
    std::string s =
        "#ifdef __CUDACC_RTC__\n"
        "typedef unsigned char uint8_t;\ntypedef unsigned short uint16_t;\n"
        "typedef unsigned int uint32_t;\ntypedef unsigned long long uint64_t;\n"
        "typedef decltype(sizeof(0)) size_t;\n"
        "#endif\n";
    s += kJitFusedH;
    s += "\nnamespace arcqml {\n";
    s += kJitCore;
    s += "\n";
    s += pass;
    s += "}  // namespace arcqml\n";
    return s;
}

// ---------------------------------------------------------------- compilation and cache

struct Compiled {
    std::vector<char> cubin;
    std::string error;
};

// ARCQML_JIT_DUMP=<dir> writes every generated source there (inspection with nvcc -Xptxas -v).
void dump_source(const std::string &src) {
    const char *dir = std::getenv("ARCQML_JIT_DUMP");
    if (!dir || !*dir) return;
    const std::string path = std::string(dir) + "/pass_" +
                             std::to_string(std::hash<std::string>()(src)) + ".cu";
    if (FILE *f = std::fopen(path.c_str(), "w")) {
        std::fwrite(src.data(), 1, src.size(), f);
        std::fclose(f);
    }
}

Compiled compile(const std::string &src) {
    Compiled out;
    dump_source(src);
    nvrtcProgram prog = nullptr;
    if (g_nvrtc.create(&prog, src.c_str(), "arcqml_pass.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS) {
        out.error = "nvrtcCreateProgram failed";
        return out;
    }
    const char *opts[] = {"--gpu-architecture=sm_100a", "-std=c++17"};
    const nvrtcResult r = g_nvrtc.compile(prog, 2, opts);
    if (r != NVRTC_SUCCESS) {
        size_t n = 0;
        g_nvrtc.log_size(prog, &n);
        std::string log(n, '\0');
        if (n) g_nvrtc.log(prog, &log[0]);
        out.error = "pass kernel compile failed: " + log.substr(0, 2000);
    } else {
        size_t n = 0;
        g_nvrtc.cubin_size(prog, &n);
        out.cubin.resize(n);
        g_nvrtc.cubin(prog, out.cubin.data());
    }
    g_nvrtc.destroy(&prog);
    return out;
}

// Per device: source -> kernel (nullptr: the source failed to compile or load; not retried).
std::unordered_map<int, std::unordered_map<std::string, CUfunction>> g_cache;
// Per device: a pass's structure (struct_key) -> its kernel, so that a pass seen before skips
// writing its source (the source is a function of these bytes and the process's switches; the
// matrix values it reads at run time are not part of it).
std::unordered_map<int, std::unordered_map<std::string, CUfunction>> g_struct_cache;

std::string struct_key(const Step &st, bool adj) {
    PassHeader h = st.header;
    h.acc_base = 0;  // read from the header at run time
    std::string k;
    k.reserve(16 + sizeof(h) + st.subs.size() * sizeof(SubBlock) + st.ops.size() * sizeof(FOp));
    const uint32_t misc[4] = {adj ? 1u : 0u, st.scaled ? 1u : 0u, st.sfin,
                              uint32_t(st.mats.size())};
    k.append(reinterpret_cast<const char *>(misc), sizeof(misc));
    k.append(reinterpret_cast<const char *>(&h), sizeof(h));
    k.append(reinterpret_cast<const char *>(st.subs.data()), st.subs.size() * sizeof(SubBlock));
    k.append(reinterpret_cast<const char *>(st.ops.data()), st.ops.size() * sizeof(FOp));
    return k;
}
std::atomic<uint64_t> g_compiled{0}, g_jit_launches{0}, g_fallbacks{0};
std::string g_last_error;

}  // namespace

std::string jit_pass_code(const Step &st, bool adjoint) {
    return st.is_pass ? pass_source(st, adjoint, st.header.rb) : std::string();
}

bool jit_enabled() {
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_JIT");
        return !(e && e[0] == '0');
    }();
    return on;
}

std::vector<void *> jit_kernels(const Schedule &sch, bool adj) {
    std::vector<void *> fns(sch.steps.size(), nullptr);
    if (!jit_enabled()) return fns;
    int dev = 0;
    check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    std::vector<std::string> keys(sch.steps.size());
    std::vector<char> known(sch.steps.size(), 0);
    for (size_t i = 0; i < sch.steps.size(); ++i)
        if (sch.steps[i].is_pass) keys[i] = struct_key(sch.steps[i], adj);
    {
        std::lock_guard<std::mutex> lock(g_mu);
        auto &sc = g_struct_cache[dev];
        for (size_t i = 0; i < keys.size(); ++i) {
            if (keys[i].empty()) continue;
            auto it = sc.find(keys[i]);
            if (it == sc.end()) continue;
            known[i] = 1;
            fns[i] = it->second;
            if (!fns[i]) ++g_fallbacks;
        }
    }
    std::vector<std::string> srcs(sch.steps.size());
    bool any = false;
    for (size_t i = 0; i < sch.steps.size(); ++i)
        if (sch.steps[i].is_pass && !known[i]) {
            const std::string pass = pass_source(sch.steps[i], adj, sch.steps[i].header.rb);
            if (!pass.empty()) srcs[i] = full_source(pass);
            any = true;
        }
    if (!any) return fns;
    std::lock_guard<std::mutex> lock(g_mu);
    auto &cache = g_cache[dev];
    auto &sc = g_struct_cache[dev];
    std::vector<size_t> todo;
    for (size_t i = 0; i < srcs.size(); ++i) {
        if (srcs[i].empty()) continue;
        auto it = cache.find(srcs[i]);
        if (it != cache.end()) {
            fns[i] = it->second;
            sc[keys[i]] = it->second;
            if (!fns[i]) ++g_fallbacks;
        } else {
            bool dup = false;
            for (size_t j : todo) dup = dup || srcs[j] == srcs[i];
            if (!dup) todo.push_back(i);
        }
    }
    if (!todo.empty()) {
        if (!load_nvrtc() || !load_driver()) {
            g_last_error = !g_nvrtc.ok ? g_nvrtc.why : g_drv.why;
            g_fallbacks += todo.size();
            return fns;
        }
        std::vector<Compiled> out(todo.size());
        std::atomic<size_t> next{0};
        const unsigned hw = std::thread::hardware_concurrency();
        const size_t nthreads = std::min<size_t>(todo.size(), hw ? std::min(hw, 16u) : 4u);
        std::vector<std::thread> pool;
        for (size_t t = 0; t < nthreads; ++t)
            pool.emplace_back([&] {
                for (size_t j; (j = next++) < todo.size();) out[j] = compile(srcs[todo[j]]);
            });
        for (auto &th : pool) th.join();
        int optin = 0;
        check_cuda(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev),
                   "cudaDeviceGetAttribute");
        for (size_t j = 0; j < todo.size(); ++j) {
            cache[srcs[todo[j]]] = nullptr;
            if (!out[j].error.empty()) {
                g_last_error = out[j].error;
                ++g_fallbacks;
                continue;
            }
            CUmodule mod = nullptr;
            CUfunction fn = nullptr;
            int static_smem = 0;
            CUresult r = g_drv.load(&mod, out[j].cubin.data());
            const char *what = "cuModuleLoadData";
            if (r == CUDA_SUCCESS) {
                r = g_drv.get(&fn, mod, "arcqml_pass");
                what = "cuModuleGetFunction";
            }
            if (r == CUDA_SUCCESS) {
                r = g_drv.get_attr(&static_smem, CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, fn);
                what = "cuFuncGetAttribute";
            }
            if (r == CUDA_SUCCESS) {
                // dynamic shared memory may use what the static part leaves of the opt-in limit
                r = g_drv.set_attr(fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                   optin - static_smem);
                what = "cuFuncSetAttribute";
            }
            if (r != CUDA_SUCCESS) {
                std::ostringstream m;
                m << "loading a compiled pass kernel failed: " << what << " returned " << int(r);
                g_last_error = m.str();
                ++g_fallbacks;
                continue;
            }
            cache[srcs[todo[j]]] = fn;
            ++g_compiled;
        }
        for (size_t i = 0; i < srcs.size(); ++i)
            if (!srcs[i].empty() && !fns[i]) {
                auto it = cache.find(srcs[i]);
                if (it != cache.end()) {
                    fns[i] = it->second;
                    sc[keys[i]] = it->second;
                }
            }
    }
    return fns;
}

uint32_t jit_acc_lanes(bool adjoint, uint32_t rb) { return acc_lanes(adjoint, rb); }

bool jit_schedule_compiles(const Schedule &sch, bool adjoint) {
    const std::vector<void *> fns = jit_kernels(sch, adjoint);
    for (size_t i = 0; i < sch.steps.size(); ++i)
        if (sch.steps[i].is_pass && !fns[i]) return false;
    return true;
}

bool adjoint_wide_tiles() {
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_ADJ_WIDE");
        return e && e[0] == '1';
    }();
    return on && jit_enabled();
}

uint32_t jit_grid_blocks(void *fn, uint32_t threads, size_t smem) {
    int per_sm = 0, dev = 0, sms = 0;
    check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev),
               "cudaDeviceGetAttribute");
    if (g_drv.occupancy(&per_sm, static_cast<CUfunction>(fn), int(threads), smem) != CUDA_SUCCESS ||
        per_sm < 1)
        per_sm = 1;
    return uint32_t(sms * per_sm);
}

void jit_launch(void *fn, unsigned grid, unsigned threads, size_t smem, cudaStream_t s,
                void **args) {
    const CUresult r = g_drv.launch(static_cast<CUfunction>(fn), grid, 1, 1, threads, 1, 1,
                                    unsigned(smem), reinterpret_cast<CUstream>(s), args, nullptr);
    if (r != CUDA_SUCCESS) {
        std::ostringstream m;
        m << "compiled pass kernel launch failed (CUresult " << int(r) << ")";
        fail(m.str());
    }
    ++g_jit_launches;
}

size_t jit_compile_check(const Schedule &sch, bool adj, size_t *eligible, std::string *err) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!load_nvrtc()) {
        if (err) *err = g_nvrtc.why;
        if (eligible) *eligible = 0;
        return 0;
    }
    std::vector<std::string> srcs;
    for (const auto &st : sch.steps) {
        if (!st.is_pass) continue;
        const std::string pass = pass_source(st, adj, st.header.rb);
        if (!pass.empty()) srcs.push_back(full_source(pass));
    }
    // compiled on parallel host threads, as jit_kernels does
    std::vector<Compiled> out(srcs.size());
    std::atomic<size_t> next{0};
    const unsigned hw = std::thread::hardware_concurrency();
    const size_t nthreads = std::min<size_t>(srcs.size(), hw ? std::min(hw, 16u) : 4u);
    std::vector<std::thread> pool;
    for (size_t t = 0; t < nthreads; ++t)
        pool.emplace_back([&] {
            for (size_t j; (j = next++) < srcs.size();) out[j] = compile(srcs[j]);
        });
    for (auto &th : pool) th.join();
    size_t ok = 0;
    for (const Compiled &c : out) {
        if (c.error.empty() && !c.cubin.empty()) ++ok;
        else if (err && err->empty()) *err = c.error;
    }
    if (eligible) *eligible = srcs.size();
    return ok;
}

void jit_info(uint64_t *compiled, uint64_t *launches, uint64_t *fallbacks, std::string *last) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (compiled) *compiled = g_compiled;
    if (launches) *launches = g_jit_launches;
    if (fallbacks) *fallbacks = g_fallbacks;
    if (last) *last = g_last_error;
}

}  // namespace arcqml
