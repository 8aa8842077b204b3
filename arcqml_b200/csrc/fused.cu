// fused.cu — fused multi-gate passes for sm_100a (layouts in fused.h, schedules in planner.cpp).
//
// One persistent launch per pass. Each CTA (256 threads) loops over tiles: it streams the
// tile's 2^k amplitudes (psi, and lambda for the adjoint sweep) from HBM into swizzled shared
// memory, runs the pass's sub-blocks — each thread gathers 2^RB amplitudes into registers,
// applies the sub-block's gates there, scatters them back — and streams the tile out. HBM sees
// one read and one write per amplitude per pass; the arithmetic runs from registers.
//
// Adjoint passes apply U^dagger to psi and lambda and accumulate, per bound parameter slot,
// Re<lambda_k| dU/dp |psi_{k-1}> (for Pauli rotations as Im<lambda_k|P|psi_k> / 2) into the
// thread's own shared-memory column; columns are summed per CTA at the end into
// partials[acc][block] (fixed order, deterministic).
//
// The tile loop and the fast gate paths live in fused_core.cuh. The kernels here interpret the
// pass's op table (one dispatch per op); jit.cpp compiles per-pass kernels in which the same
// fast paths are inlined in the pass's op order.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <tuple>
#include <vector>

#include "fused.h"
#include "jit.h"
#include "launch.h"
#include "planner.h"
#include "profile.h"

namespace arcqml {

namespace {

#include "fused_core.cuh"

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ void load_op(const FOp *src, FOp &dst) {
    const uint4 *s = reinterpret_cast<const uint4 *>(src);
    uint4 *d = reinterpret_cast<uint4 *>(&dst);
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = s[i];
}

struct OpEnv {
    bool tile_ok;        // controls outside the tile satisfied
    bool plain;          // no controls at all
    uint32_t lcmask;
    uint64_t gbase;      // global index bits outside the tile
};

template <int RB>
__device__ __forceinline__ bool ctrl_ok(const OpEnv &E, const uint32_t (&Le)[1 << RB], int e) {
    return E.plain || (E.tile_ok && ((Le[e] & E.lcmask) == E.lcmask));
}

// ---------------------------------------------------------------- 1-target gates on bit B

template <int RB, int B>
__device__ __forceinline__ void apply_1t(uint8_t kind, const double2 *mt, double2 (&v)[1 << RB],
                                         const uint32_t (&Le)[1 << RB], const OpEnv &E) {
    constexpr int N = 1 << RB;
    if (kind == FK_RX || kind == FK_RY) {
        const double2 cs = ld(mt);
        const double c = cs.x, s = cs.y;
#pragma unroll
        for (int e = 0; e < N; ++e) {
            if (e & (1 << B)) continue;
            const int f = e | (1 << B);
            const double2 x0 = v[e], x1 = v[f];
            double2 y0, y1;
            if (kind == FK_RX) {
                y0 = make_double2(fma(c, x0.x, s * x1.y), fma(c, x0.y, -s * x1.x));
                y1 = make_double2(fma(c, x1.x, s * x0.y), fma(c, x1.y, -s * x0.x));
            } else {
                y0 = make_double2(fma(c, x0.x, -s * x1.x), fma(c, x0.y, -s * x1.y));
                y1 = make_double2(fma(s, x0.x, c * x1.x), fma(s, x0.y, c * x1.y));
            }
            const bool ok = ctrl_ok<RB>(E, Le, e);
            v[e] = ok ? y0 : x0;
            v[f] = ok ? y1 : x1;
        }
    } else {  // FK_M2
        const double2 m0 = ld(mt), m1 = ld(mt + 1), m2 = ld(mt + 2), m3 = ld(mt + 3);
#pragma unroll
        for (int e = 0; e < N; ++e) {
            if (e & (1 << B)) continue;
            const int f = e | (1 << B);
            const double2 x0 = v[e], x1 = v[f];
            const double2 y0 = cfma(m0, x0, cmul(m1, x1));
            const double2 y1 = cfma(m2, x0, cmul(m3, x1));
            const bool ok = ctrl_ok<RB>(E, Le, e);
            v[e] = ok ? y0 : x0;
            v[f] = ok ? y1 : x1;
        }
    }
}

template <int RB>
__device__ __forceinline__ void apply_1t_dispatch(int b, uint8_t kind, const double2 *mt,
                                                  double2 (&v)[1 << RB],
                                                  const uint32_t (&Le)[1 << RB], const OpEnv &E) {
    switch (b) {
    case 0: apply_1t<RB, 0>(kind, mt, v, Le, E); break;
    case 1: apply_1t<RB, 1>(kind, mt, v, Le, E); break;
    case 2: apply_1t<RB, 2>(kind, mt, v, Le, E); break;
    default:
        if constexpr (RB > 3) apply_1t<RB, 3>(kind, mt, v, Le, E);
        break;
    }
}

// ---------------------------------------------------------------- 2-target dense on (B0, B1)

template <int RB, int B0, int B1>
__device__ __forceinline__ void apply_m4(const double2 *mt, double2 (&v)[1 << RB],
                                         const uint32_t (&Le)[1 << RB], const OpEnv &E) {
    constexpr int N = 1 << RB;
#pragma unroll
    for (int e = 0; e < N; ++e) {
        if (e & ((1 << B0) | (1 << B1))) continue;
        const int idx[4] = {e, e | (1 << B0), e | (1 << B1), e | (1 << B0) | (1 << B1)};
        double2 x[4], y[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = v[idx[j]];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            double2 acc = cmul(ld(mt + i * 4), x[0]);
            acc = cfma(ld(mt + i * 4 + 1), x[1], acc);
            acc = cfma(ld(mt + i * 4 + 2), x[2], acc);
            acc = cfma(ld(mt + i * 4 + 3), x[3], acc);
            y[i] = acc;
        }
        const bool ok = ctrl_ok<RB>(E, Le, e);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[idx[j]] = ok ? y[j] : x[j];
    }
}

template <int RB, int B0>
__device__ __forceinline__ void apply_m4_b1(int b1, const double2 *mt, double2 (&v)[1 << RB],
                                            const uint32_t (&Le)[1 << RB], const OpEnv &E) {
    switch (b1) {
    case 0: if constexpr (B0 != 0) apply_m4<RB, B0, 0>(mt, v, Le, E); break;
    case 1: if constexpr (B0 != 1) apply_m4<RB, B0, 1>(mt, v, Le, E); break;
    case 2: if constexpr (B0 != 2) apply_m4<RB, B0, 2>(mt, v, Le, E); break;
    default:
        if constexpr (RB > 3 && B0 != 3) apply_m4<RB, B0, 3>(mt, v, Le, E);
        break;
    }
}

template <int RB>
__device__ __forceinline__ void apply_m4_dispatch(int b0, int b1, const double2 *mt,
                                                  double2 (&v)[1 << RB],
                                                  const uint32_t (&Le)[1 << RB], const OpEnv &E) {
    switch (b0) {
    case 0: apply_m4_b1<RB, 0>(b1, mt, v, Le, E); break;
    case 1: apply_m4_b1<RB, 1>(b1, mt, v, Le, E); break;
    case 2: apply_m4_b1<RB, 2>(b1, mt, v, Le, E); break;
    default:
        if constexpr (RB > 3) apply_m4_b1<RB, 3>(b1, mt, v, Le, E);
        break;
    }
}

// ---------------------------------------------------------------- diagonal gates

template <int RB>
__device__ __forceinline__ uint32_t dbit(const FOp &o, int t, const uint32_t (&Le)[1 << RB], int e,
                                         uint64_t gbase) {
    return o.dq_in_tile[t] ? ((Le[e] >> o.dq_pos[t]) & 1u) : uint32_t((gbase >> o.dq_pos[t]) & 1u);
}

template <int RB>
__device__ __forceinline__ void apply_diag(const FOp &o, const double2 *mt, double2 (&v)[1 << RB],
                                           const uint32_t (&Le)[1 << RB], const OpEnv &E) {
    constexpr int N = 1 << RB;
    if (o.kind == FK_D1) {
        const double2 d0 = ld(mt), d1 = ld(mt + 1);
#pragma unroll
        for (int e = 0; e < N; ++e) {
            const double2 d = dbit<RB>(o, 0, Le, e, E.gbase) ? d1 : d0;
            const double2 y = cmul(d, v[e]);
            v[e] = ctrl_ok<RB>(E, Le, e) ? y : v[e];
        }
    } else {
        const double2 d0 = ld(mt), d1 = ld(mt + 1), d2 = ld(mt + 2), d3 = ld(mt + 3);
#pragma unroll
        for (int e = 0; e < N; ++e) {
            const uint32_t b = dbit<RB>(o, 0, Le, e, E.gbase) | (dbit<RB>(o, 1, Le, e, E.gbase) << 1);
            const double2 d = b == 0 ? d0 : (b == 1 ? d1 : (b == 2 ? d2 : d3));
            const double2 y = cmul(d, v[e]);
            v[e] = ctrl_ok<RB>(E, Le, e) ? y : v[e];
        }
    }
}

template <int RB>
__device__ __forceinline__ void apply_op(const FOp &o, const double2 *mt, double2 (&v)[1 << RB],
                                         const uint32_t (&Le)[1 << RB], const OpEnv &E) {
    switch (o.kind) {
    case FK_RX:
    case FK_RY:
    case FK_M2: apply_1t_dispatch<RB>(o.rb0, o.kind, mt, v, Le, E); break;
    case FK_D1:
    case FK_D2: apply_diag<RB>(o, mt, v, Le, E); break;
    case FK_M4: apply_m4_dispatch<RB>(o.rb0, o.rb1, mt, v, Le, E); break;
    default: break;
    }
}

// ---------------------------------------------------------------- adjoint gradients

// Im<lam|X|psi> or Im<lam|Y|psi> over pairs on register bit B (psi = psi_k, before U^dag).
template <int RB, int B>
__device__ __forceinline__ double grad_xy(bool is_y, const double2 (&v)[1 << RB],
                                          const double2 (&w)[1 << RB],
                                          const uint32_t (&Le)[1 << RB], const OpEnv &E) {
    constexpr int N = 1 << RB;
    double z = 0.0;
#pragma unroll
    for (int e = 0; e < N; ++e) {
        if (e & (1 << B)) continue;
        const int f = e | (1 << B);
        // X: Im(conj(l0) x1) + Im(conj(l1) x0);  Y: -Re(conj(l0) x1) + Re(conj(l1) x0)
        const double t = is_y ? (rcm(w[f], v[e]) - rcm(w[e], v[f])) : (icm(w[e], v[f]) + icm(w[f], v[e]));
        z += ctrl_ok<RB>(E, Le, e) ? t : 0.0;
    }
    return z;
}

template <int RB>
__device__ __forceinline__ double grad_xy_dispatch(int b, bool is_y, const double2 (&v)[1 << RB],
                                                   const double2 (&w)[1 << RB],
                                                   const uint32_t (&Le)[1 << RB], const OpEnv &E) {
    switch (b) {
    case 0: return grad_xy<RB, 0>(is_y, v, w, Le, E);
    case 1: return grad_xy<RB, 1>(is_y, v, w, Le, E);
    case 2: return grad_xy<RB, 2>(is_y, v, w, Le, E);
    default:
        if constexpr (RB > 3) return grad_xy<RB, 3>(is_y, v, w, Le, E);
        return 0.0;
    }
}

// Im<lam|Z_q|psi> for the op's diagonal qubit q.
template <int RB>
__device__ __forceinline__ double grad_z(const FOp &o, const double2 (&v)[1 << RB],
                                         const double2 (&w)[1 << RB], const uint32_t (&Le)[1 << RB],
                                         const OpEnv &E) {
    constexpr int N = 1 << RB;
    double z = 0.0;
#pragma unroll
    for (int e = 0; e < N; ++e) {
        const double t = icm(w[e], v[e]);
        const double st = dbit<RB>(o, 0, Le, e, E.gbase) ? -t : t;
        z += ctrl_ok<RB>(E, Le, e) ? st : 0.0;
    }
    return z;
}

// Re<lam| D |psi'> for a small matrix D of the op's shape, psi' already U^dag psi.
template <int RB, int B>
__device__ __forceinline__ double grad_m2(const double2 *d, const double2 (&v)[1 << RB],
                                          const double2 (&w)[1 << RB],
                                          const uint32_t (&Le)[1 << RB], const OpEnv &E) {
    constexpr int N = 1 << RB;
    const double2 m0 = ld(d), m1 = ld(d + 1), m2 = ld(d + 2), m3 = ld(d + 3);
    double z = 0.0;
#pragma unroll
    for (int e = 0; e < N; ++e) {
        if (e & (1 << B)) continue;
        const int f = e | (1 << B);
        const double2 y0 = cfma(m0, v[e], cmul(m1, v[f]));
        const double2 y1 = cfma(m2, v[e], cmul(m3, v[f]));
        const double t = rcm(w[e], y0) + rcm(w[f], y1);
        z += ctrl_ok<RB>(E, Le, e) ? t : 0.0;
    }
    return z;
}

template <int RB, int B0, int B1>
__device__ __forceinline__ double grad_m4(const double2 *d, const double2 (&v)[1 << RB],
                                          const double2 (&w)[1 << RB],
                                          const uint32_t (&Le)[1 << RB], const OpEnv &E) {
    constexpr int N = 1 << RB;
    double z = 0.0;
#pragma unroll
    for (int e = 0; e < N; ++e) {
        if (e & ((1 << B0) | (1 << B1))) continue;
        const int idx[4] = {e, e | (1 << B0), e | (1 << B1), e | (1 << B0) | (1 << B1)};
        double t = 0.0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            double2 acc = cmul(ld(d + i * 4), v[idx[0]]);
            acc = cfma(ld(d + i * 4 + 1), v[idx[1]], acc);
            acc = cfma(ld(d + i * 4 + 2), v[idx[2]], acc);
            acc = cfma(ld(d + i * 4 + 3), v[idx[3]], acc);
            t += rcm(w[idx[i]], acc);
        }
        z += ctrl_ok<RB>(E, Le, e) ? t : 0.0;
    }
    return z;
}

template <int RB, int B0>
__device__ __forceinline__ double grad_m4_b1(int b1, const double2 *d, const double2 (&v)[1 << RB],
                                             const double2 (&w)[1 << RB],
                                             const uint32_t (&Le)[1 << RB], const OpEnv &E) {
    switch (b1) {
    case 0: if constexpr (B0 != 0) return grad_m4<RB, B0, 0>(d, v, w, Le, E); break;
    case 1: if constexpr (B0 != 1) return grad_m4<RB, B0, 1>(d, v, w, Le, E); break;
    case 2: if constexpr (B0 != 2) return grad_m4<RB, B0, 2>(d, v, w, Le, E); break;
    default:
        if constexpr (RB > 3 && B0 != 3) return grad_m4<RB, B0, 3>(d, v, w, Le, E);
        break;
    }
    return 0.0;
}

template <int RB>
__device__ __forceinline__ double grad_generic(const FOp &o, const double2 *d,
                                               const double2 (&v)[1 << RB],
                                               const double2 (&w)[1 << RB],
                                               const uint32_t (&Le)[1 << RB], const OpEnv &E) {
    constexpr int N = 1 << RB;
    if (o.kind == FK_D1 || o.kind == FK_D2) {
        double z = 0.0;
        const bool two = o.kind == FK_D2;
        const double2 d0 = ld(d), d1 = ld(d + 1);
        const double2 d2 = two ? ld(d + 2) : d0, d3 = two ? ld(d + 3) : d1;
#pragma unroll
        for (int e = 0; e < N; ++e) {
            uint32_t b = dbit<RB>(o, 0, Le, e, E.gbase);
            if (two) b |= dbit<RB>(o, 1, Le, e, E.gbase) << 1;
            const double2 dd = b == 0 ? d0 : (b == 1 ? d1 : (b == 2 ? d2 : d3));
            const double t = rcm(w[e], cmul(dd, v[e]));
            z += ctrl_ok<RB>(E, Le, e) ? t : 0.0;
        }
        return z;
    }
    if (o.kind == FK_M4) {
        switch (o.rb0) {
        case 0: return grad_m4_b1<RB, 0>(o.rb1, d, v, w, Le, E);
        case 1: return grad_m4_b1<RB, 1>(o.rb1, d, v, w, Le, E);
        case 2: return grad_m4_b1<RB, 2>(o.rb1, d, v, w, Le, E);
        default:
            if constexpr (RB > 3) return grad_m4_b1<RB, 3>(o.rb1, d, v, w, Le, E);
            return 0.0;
        }
    }
    switch (o.rb0) {
    case 0: return grad_m2<RB, 0>(d, v, w, Le, E);
    case 1: return grad_m2<RB, 1>(d, v, w, Le, E);
    case 2: return grad_m2<RB, 2>(d, v, w, Le, E);
    default:
        if constexpr (RB > 3) return grad_m2<RB, 3>(d, v, w, Le, E);
        return 0.0;
    }
}

// Matrix entries of the op's U (to skip over to the derivative matrices) and of one dU.
__device__ __forceinline__ int umat_len(uint8_t kind) {
    switch (kind) {
    case FK_RX: case FK_RY: return 1;
    case FK_M2: return 4;
    case FK_D1: return 2;
    case FK_D2: return 4;
    default: return 16;
    }
}
__device__ __forceinline__ int dmat_len(uint8_t kind) {
    switch (kind) {
    case FK_D1: return 2;
    case FK_D2: return 4;
    case FK_M4: return 16;
    default: return 4;
    }
}

// Dispatch a template over a runtime register bit b (< RB).
#define ARCQML_BITS(b, CALL)                          \
    switch (b) {                                      \
    case 0: CALL(0); break;                           \
    case 1: CALL(1); break;                           \
    case 2: CALL(2); break;                           \
    default:                                          \
        if constexpr (RB > 3) { CALL(3); }            \
        break;                                        \
    }


// Applies op o (U or U^dagger) to the registers through its fast path; false if the op
// needs the generic path.
template <int RB>
__device__ __forceinline__ bool apply_fast(const FOp &o, const double2 *mt, double2 (&v)[1 << RB],
                                           uint32_t tb, uint64_t gbase) {
    switch (o.code) {
    case FC_RX: {
        const double2 cs = mt[0];
#define C_(B) f_rx<RB, B>(v, cs.x, cs.y)
        ARCQML_BITS(o.rb0, C_)
#undef C_
        return true;
    }
    case FC_RY: {
        const double2 cs = mt[0];
#define C_(B) f_ry<RB, B>(v, cs.x, cs.y)
        ARCQML_BITS(o.rb0, C_)
#undef C_
        return true;
    }
    case FC_M2: {
#define C_(B) f_m2<RB, B>(v, mt)
        ARCQML_BITS(o.rb0, C_)
#undef C_
        return true;
    }
    case FC_D1_REG: {
        const double2 d0 = mt[0], d1 = mt[1];
#define C_(B) f_d1_reg<RB, B>(v, d0, d1)
        ARCQML_BITS(o.rb0, C_)
#undef C_
        return true;
    }
    case FC_D1_UNI:
        f_d1_uni<RB>(v, const_bit(o, 0, tb, gbase) ? mt[1] : mt[0]);
        return true;
    case FC_SIGN_RR: {
#define C1_(B0, B1) f_sign_rr<RB, B0, B1>(v)
#define C_(B1)                                 \
    switch (o.rb0) {                           \
    case 0: C1_(0, B1); break;                 \
    case 1: C1_(1, B1); break;                 \
    case 2: C1_(2, B1); break;                 \
    default:                                   \
        if constexpr (RB > 3) { C1_(3, B1); }  \
        break;                                 \
    }
        ARCQML_BITS(o.rb1, C_)
#undef C_
#undef C1_
        return true;
    }
    case FC_SIGN_RC: {
        const uint32_t m = const_bit(o, 0, tb, gbase) ? 0x80000000u : 0u;
#define C_(B) f_sign_rc<RB, B>(v, m)
        ARCQML_BITS(o.rb0, C_)
#undef C_
        return true;
    }
    case FC_SIGN_CC:
        f_sign_cc<RB>(v, (const_bit(o, 0, tb, gbase) & const_bit(o, 1, tb, gbase)) ? 0x80000000u : 0u);
        return true;
    case FC_M4: {
#define C1_(B0, B1) f_m4<RB, B0, B1>(v, mt)
#define C_(B1)                                                   \
    switch (o.rb0) {                                             \
    case 0: if constexpr (B1 != 0) { C1_(0, B1); } break;        \
    case 1: if constexpr (B1 != 1) { C1_(1, B1); } break;        \
    case 2: if constexpr (B1 != 2) { C1_(2, B1); } break;        \
    default:                                                     \
        if constexpr (RB > 3 && B1 != 3) { C1_(3, B1); }         \
        break;                                                   \
    }
        ARCQML_BITS(o.rb1, C_)
#undef C_
#undef C1_
        return true;
    }
    default:
        return false;
    }
}

// Fast Pauli-rotation gradients (half-gradient units: Im<lam|P|psi> / 2 with psi = psi_k).
template <int RB>
__device__ __forceinline__ bool grad_fast(const FOp &o, const double2 (&v)[1 << RB],
                                          const double2 (&w)[1 << RB], uint32_t tb, uint64_t gbase,
                                          double &z) {
    switch (o.gcode) {
    case GF_X: {
#define C_(B) z = g_x<RB, B>(v, w)
        ARCQML_BITS(o.rb0, C_)
#undef C_
        return true;
    }
    case GF_Y: {
#define C_(B) z = g_y<RB, B>(v, w)
        ARCQML_BITS(o.rb0, C_)
#undef C_
        return true;
    }
    case GF_Z_REG: {
#define C_(B) z = g_z<RB, B>(v, w)
        ARCQML_BITS(o.rb0, C_)
#undef C_
        return true;
    }
    case GF_Z_UNI: {
        const double t = g_z_uni<RB>(v, w);
        z = const_bit(o, 0, tb, gbase) ? -t : t;
        return true;
    }
    default:
        return false;
    }
}

// ---------------------------------------------------------------- generic path (out of line)
//
// Gates without a fast path (controlled gates other than CZ, two-qubit diagonals, controlled
// rotations' gradients, ...) run through these non-inlined functions, so their per-element
// index and control logic never mixes into the hot loop of the fast paths. The caller copies
// the thread's registers into a local array around the call.

template <int RB>
__device__ __forceinline__ void rebuild(uint32_t tb, const uint32_t *rm, uint64_t gbase,
                                        const FOp &o, uint32_t (&Le)[1 << RB], OpEnv &E) {
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) {
        uint32_t x = tb;
#pragma unroll
        for (int r = 0; r < RB; ++r)
            if ((e >> r) & 1) x |= rm[r];
        Le[e] = x;
    }
    E.lcmask = o.lcmask;
    E.gbase = gbase;
    E.tile_ok = (gbase & o.gcmask) == o.gcmask;
    E.plain = (o.lcmask == 0) && (o.gcmask == 0);
}

// The op is read from its shared-memory table entry and the register bits from the sub-block
// descriptor, so the hot loop passes only pointers (nothing of it is spilled for these calls).
template <int RB>
__device__ __forceinline__ void slow_setup(const FOp *op, const SubBlock *sbp, uint32_t tb,
                                           uint64_t gbase, FOp &o, uint32_t (&Le)[1 << RB],
                                           OpEnv &E) {
    load_op(op, o);
    uint32_t rm[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) rm[r] = 1u << sbp->R[r];
    rebuild<RB>(tb, rm, gbase, o, Le, E);
}

template <int RB>
__device__ __noinline__ void slow_apply(const FOp *op, const double2 *mt, double2 *vp, uint32_t tb,
                                        const SubBlock *sbp, uint64_t gbase) {
    FOp o;
    uint32_t Le[1 << RB];
    OpEnv E;
    slow_setup<RB>(op, sbp, tb, gbase, o, Le, E);
    apply_op<RB>(o, mt, *reinterpret_cast<double2(*)[1 << RB]>(vp), Le, E);
}

// d == nullptr: Pauli gradient (gkind X/Y/Z) before U^dag; else generic slot gradient with the
// derivative matrix d after U^dag.
template <int RB>
__device__ __noinline__ double slow_grad(const FOp *op, const double2 *d, const double2 *vp,
                                         const double2 *wp, uint32_t tb, const SubBlock *sbp,
                                         uint64_t gbase) {
    FOp o;
    uint32_t Le[1 << RB];
    OpEnv E;
    slow_setup<RB>(op, sbp, tb, gbase, o, Le, E);
    const auto &v = *reinterpret_cast<const double2(*)[1 << RB]>(vp);
    const auto &w = *reinterpret_cast<const double2(*)[1 << RB]>(wp);
    if (d) return grad_generic<RB>(o, d, v, w, Le, E);
    if (o.gkind == GK_PZ) return grad_z<RB>(o, v, w, Le, E);
    return grad_xy_dispatch<RB>(o.rb0, o.gkind == GK_PY, v, w, Le, E);
}


// Adjoint step for the common uncontrolled gates in one dispatch: the Pauli-rotation gradient
// (from psi_k, lambda_k), then U^dagger on psi and on lambda. Returns false when the op needs
// the general sequence (controlled gates, generic gradients).
template <int RB>
__device__ __forceinline__ bool adj_fast(const FOp &o, const double2 *mt, double2 (&v)[1 << RB],
                                         double2 (&w)[1 << RB], uint32_t tb, uint64_t gbase,
                                         double &z) {
    const bool none = o.gkind == GK_NONE;
    switch (o.code) {
    case FC_RX: {
        if (!none && o.gcode != GF_X) return false;
        const double2 cs = mt[0];
#define C_(B)                                   \
    {                                           \
        if (!none) z = g_x<RB, B>(v, w);        \
        f_rx<RB, B>(v, cs.x, cs.y);             \
        f_rx<RB, B>(w, cs.x, cs.y);             \
    }
        ARCQML_BITS(o.rb0, C_)
#undef C_
        return true;
    }
    case FC_RY: {
        if (!none && o.gcode != GF_Y) return false;
        const double2 cs = mt[0];
#define C_(B)                                   \
    {                                           \
        if (!none) z = g_y<RB, B>(v, w);        \
        f_ry<RB, B>(v, cs.x, cs.y);             \
        f_ry<RB, B>(w, cs.x, cs.y);             \
    }
        ARCQML_BITS(o.rb0, C_)
#undef C_
        return true;
    }
    case FC_D1_REG: {
        if (!none && o.gcode != GF_Z_REG) return false;
        const double2 d0 = mt[0], d1 = mt[1];
#define C_(B)                                   \
    {                                           \
        if (!none) z = g_z<RB, B>(v, w);        \
        f_d1_reg<RB, B>(v, d0, d1);             \
        f_d1_reg<RB, B>(w, d0, d1);             \
    }
        ARCQML_BITS(o.rb0, C_)
#undef C_
        return true;
    }
    case FC_D1_UNI: {
        if (!none && o.gcode != GF_Z_UNI) return false;
        const bool bit = const_bit(o, 0, tb, gbase) != 0;
        if (!none) {
            const double t = g_z_uni<RB>(v, w);
            z = bit ? -t : t;
        }
        const double2 d = bit ? mt[1] : mt[0];
        f_d1_uni<RB>(v, d);
        f_d1_uni<RB>(w, d);
        return true;
    }
    default:
        if (!none) return false;
        if (!apply_fast<RB>(o, mt, v, tb, gbase)) return false;
        apply_fast<RB>(o, mt, w, tb, gbase);
        return true;
    }
}

// A sub-block with at least one op on the generic path, out of line so that the fast loop
// above keeps a register allocation of its own.
template <int RB, bool ADJ>
__device__ __noinline__ void general_subblock(const SubBlock &S, uint32_t sb, double2 *tp,
                                              double2 *tl, const FOp *ops, const double2 *mats,
                                              const SubBlock *subs, double *sacc,
                                              uint32_t nthreads, uint32_t tb, uint64_t gbase) {
    constexpr int N = 1 << RB;
    uint32_t rm[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) rm[r] = 1u << S.R[r];
    double2 v[N], w[N];
#pragma unroll
    for (int e = 0; e < N; ++e) {
        const uint32_t x = sub_index<RB>(tb, rm, e);
        v[e] = tp[phys(x)];
        if (ADJ) w[e] = tl[phys(x)];
    }
    for (uint32_t oi = S.op_begin; oi < S.op_end; ++oi) {
        FOp o;
        load_op(ops + oi, o);
        const double2 *mt = mats + o.moff;
        if constexpr (ADJ) {
            // one dispatch: Pauli gradient (if any), then U^dagger on psi and lambda
            double z = 0.0;
            if (adj_fast<RB>(o, mt, v, w, tb, gbase, z)) {
                if (o.gkind != GK_NONE) accumulate(sacc, o.acc[0] * nthreads, 0.5 * z);
                continue;
            }
            if (o.gkind != GK_NONE && o.gkind != GK_GENERIC) {
                if (!grad_fast<RB>(o, v, w, tb, gbase, z)) {
                    double2 tv[N], tw[N];
#pragma unroll
                    for (int e = 0; e < N; ++e) {
                        tv[e] = v[e];
                        tw[e] = w[e];
                    }
                    z = slow_grad<RB>(ops + oi, nullptr, tv, tw, tb, subs + sb, gbase);
                }
                accumulate(sacc, o.acc[0] * nthreads, 0.5 * z);
            }
        }
        const bool fast = apply_fast<RB>(o, mt, v, tb, gbase);
        if (!fast) {
            double2 tv[N];
#pragma unroll
            for (int e = 0; e < N; ++e) tv[e] = v[e];
            slow_apply<RB>(ops + oi, mt, tv, tb, subs + sb, gbase);
#pragma unroll
            for (int e = 0; e < N; ++e) v[e] = tv[e];
        }
        if constexpr (ADJ) {
            if (o.gkind == GK_GENERIC) {
                const double2 *d = mt + umat_len(o.kind);
                const int dl = dmat_len(o.kind);
                double2 tv[N], tw[N];
#pragma unroll
                for (int e = 0; e < N; ++e) {
                    tv[e] = v[e];
                    tw[e] = w[e];
                }
                for (int s = 0; s < int(o.nslots); ++s)
                    accumulate(sacc, o.acc[s] * nthreads,
                               slow_grad<RB>(ops + oi, d + s * dl, tv, tw, tb, subs + sb, gbase));
            }
            if (fast) {
                apply_fast<RB>(o, mt, w, tb, gbase);
            } else {
                double2 tw[N];
#pragma unroll
                for (int e = 0; e < N; ++e) tw[e] = w[e];
                slow_apply<RB>(ops + oi, mt, tw, tb, subs + sb, gbase);
#pragma unroll
                for (int e = 0; e < N; ++e) w[e] = tw[e];
            }
        }
    }
#pragma unroll
    for (int e = 0; e < N; ++e) {
        const uint32_t x = sub_index<RB>(tb, rm, e);
        tp[phys(x)] = v[e];
        if (ADJ) tl[phys(x)] = w[e];
    }
}

// ---------------------------------------------------------------- the pass kernel



// ---------------------------------------------------------------- the precompiled pass kernel

// Applies sub-block sb by interpreting its op table: sub-blocks whose ops all have fast paths
// run an inline loop with one dispatch per op, the others the out-of-line general routine.
struct TableRunner {
    static constexpr int kAccLanes = 1;
    static constexpr bool kSingleBuffer = false;
    static constexpr bool kOpsInSmem = true;
    static constexpr bool kMatsInSmem = true;
    static constexpr bool kPrefetch = true;
    // every exchange of the table-driven kernel is a CTA barrier
    __device__ static __forceinline__ bool warp_next(uint32_t) { return false; }
    // the table-driven kernel scales each gradient term as it adds it
    template <class MT>
    __device__ static __forceinline__ double row_factor(uint32_t, const MT &) { return 1.0; }
    template <int RB, bool ADJ>
    __device__ static __forceinline__ void run(uint32_t sb, uint32_t k, double2 *tp, double2 *tl,
                                               const FOp *ops, const double2 *mats,
                                               const SubBlock *subs, double *sacc,
                                               uint32_t nthreads, uint64_t gbase) {
        const SubBlock S = load_subblock(subs, sb);
        const uint32_t tb = thread_base<RB>(S, k);
        if (!(S.flags & SB_ALL_FAST)) {
            general_subblock<RB, ADJ>(S, sb, tp, tl, ops, mats, subs, sacc, nthreads, tb, gbase);
            return;
        }
        double2 v[1 << RB], w[1 << RB];
        load_regs<RB, ADJ>(S, tb, tp, tl, v, w);
        for (uint32_t oi = S.op_begin; oi < S.op_end; ++oi) {
            FOp o;
            load_op(ops + oi, o);
            const double2 *mt = mats + o.moff;
            if constexpr (ADJ) {
                double z = 0.0;
                adj_fast<RB>(o, mt, v, w, tb, gbase, z);
                if (o.gkind != GK_NONE) accumulate(sacc, o.acc[0] * nthreads, 0.5 * z);
            } else {
                apply_fast<RB>(o, mt, v, tb, gbase);
            }
        }
        store_regs<RB, ADJ>(S, tb, tp, tl, v, w);
    }
};

template <int RB, bool ADJ>
__global__ void __launch_bounds__((ADJ || RB == 4) ? 256 : 512)
    k_fused(double2 *__restrict__ psi, double2 *__restrict__ lam, uint32_t n, uint32_t tiles_log,
            uint64_t total_tiles, const PassHeader *__restrict__ hdr,
            const SubBlock *__restrict__ subs, const FOp *__restrict__ gops,
            const double2 *__restrict__ gmats, double *__restrict__ partials, uint32_t stride) {
    fused_body<RB, ADJ, TableRunner>(psi, lam, n, tiles_log, total_tiles, hdr, subs, gops, gmats,
                                     partials, stride);
}

size_t fused_smem(bool adj, uint32_t k, uint32_t nacc, uint32_t nops, uint32_t nmat,
                  uint32_t acc_cols, bool single = false) {
    return smem_layout(adj, k, nacc, nops, nmat, acc_cols, single).total;
}

using FusedKernel = void (*)(double2 *, double2 *, uint32_t, uint32_t, uint64_t,
                             const PassHeader *, const SubBlock *, const FOp *, const double2 *,
                             double *, uint32_t);

FusedKernel fused_kernel(bool adj, uint32_t rb) {
    if (adj) return k_fused<3, true>;
    return rb == 4 ? k_fused<4, false> : k_fused<3, false>;
}

// Resident CTAs per device for each (adjoint, k, rb) launch shape, computed once.
struct GridKey {
    int dev;
    bool adj;
    uint32_t k, rb;
};
std::mutex g_grid_mu;
std::vector<std::pair<GridKey, uint32_t>> g_grid;
// Largest dynamic shared memory allowed so far per (device, kernel): the attribute belongs to
// the kernel function, which serves several tile sizes, so it may only grow.
std::vector<std::tuple<int, FusedKernel, size_t>> g_smem_max;

}  // namespace

uint32_t fused_threads(uint32_t k, uint32_t rb) { return 1u << (k - rb); }

uint32_t fused_grid_blocks(bool adjoint, uint32_t k, uint32_t rb) {
    int dev = 0;
    check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lock(g_grid_mu);
    for (const auto &e : g_grid)
        if (e.first.dev == dev && e.first.adj == adjoint && e.first.k == k && e.first.rb == rb)
            return e.second;
    int sms = 0;
    check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev),
               "cudaDeviceGetAttribute");
    // occupancy for the largest pass the planner emits (its tables are capped)
    const uint32_t threads = fused_threads(k, rb);
    const uint32_t cols = (adjoint && rb == 4) ? threads / 32u : threads;
    const size_t smem = fused_smem(adjoint, k, adjoint ? kMaxPassAcc : 0, kMaxPassOps, kMaxPassMats,
                                   cols);
    if (smem > 227 * 1024) fail("internal: fused pass shared memory exceeds 227 KB");
    FusedKernel kern = fused_kernel(adjoint, rb);
    size_t allowed = 0;
    for (const auto &e : g_smem_max)
        if (std::get<0>(e) == dev && std::get<1>(e) == kern) allowed = std::get<2>(e);
    if (smem > allowed) {
        check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(smem)),
                   "cudaFuncSetAttribute");
        bool found = false;
        for (auto &e : g_smem_max)
            if (std::get<0>(e) == dev && std::get<1>(e) == kern) {
                std::get<2>(e) = smem;
                found = true;
            }
        if (!found) g_smem_max.emplace_back(dev, kern, smem);
    }
    int per_sm = 0;
    check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern,
                                                             int(fused_threads(k, rb)), smem),
               "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    const uint32_t blocks = uint32_t(sms * (per_sm < 1 ? 1 : per_sm));
    g_grid.push_back({GridKey{dev, adjoint, k, rb}, blocks});
    return blocks;
}

void run_schedule(const Schedule &sch, double2 *psi, double2 *lam, size_t batch, uint32_t n,
                  double *partials, uint32_t partial_stride, ThreadContext &ctx, cudaStream_t s) {
    const bool adj = lam != nullptr;
    // Compiled kernels of the passes that have one (compiled once per circuit structure).
    const std::vector<void *> jit = jit_kernels(sch, adj);
    // Upload every pass's tables into one device blob (16-byte aligned sections).
    struct Off {
        size_t hdr, subs, ops, mats;
    };
    std::vector<Off> offs;
    size_t total = 0;
    auto align = [](size_t x) { return (x + 15) & ~size_t(15); };
    for (const auto &st : sch.steps) {
        Off o{0, 0, 0, 0};
        if (st.is_pass) {
            o.hdr = total;
            total = align(total + sizeof(PassHeader));
            o.subs = total;
            total = align(total + st.subs.size() * sizeof(SubBlock));
            o.ops = total;
            total = align(total + st.ops.size() * sizeof(FOp));
            o.mats = total;
            total = align(total + st.mats.size() * sizeof(double2));
        }
        offs.push_back(o);
    }
    std::vector<char> blob(total);
    for (size_t i = 0; i < sch.steps.size(); ++i) {
        const auto &st = sch.steps[i];
        if (!st.is_pass) continue;
        std::memcpy(blob.data() + offs[i].hdr, &st.header, sizeof(PassHeader));
        std::memcpy(blob.data() + offs[i].subs, st.subs.data(), st.subs.size() * sizeof(SubBlock));
        std::memcpy(blob.data() + offs[i].ops, st.ops.data(), st.ops.size() * sizeof(FOp));
        std::memcpy(blob.data() + offs[i].mats, st.mats.data(), st.mats.size() * sizeof(double2));
    }
    char *dev = nullptr;
    if (total) {
        dev = static_cast<char *>(ctx_buffer(ctx, 4, total));
        check_cuda(cudaMemcpyAsync(dev, blob.data(), total, cudaMemcpyHostToDevice, s),
                   "cudaMemcpyAsync (pass tables)");
    }
    for (size_t i = 0; i < sch.steps.size(); ++i) {
        const auto &st = sch.steps[i];
        if (!st.is_pass) {
            const OpRecord &op = *st.dense_op;
            std::vector<double2> m = op.custom;
            if (adj) {
                const size_t dim = size_t(1) << op.qubits.size();
                for (size_t a = 0; a < dim; ++a)
                    for (size_t b = 0; b < dim; ++b)
                        m[b * dim + a] = make_double2(op.custom[a * dim + b].x, -op.custom[a * dim + b].y);
            }
            DevGate g = lower(op, LOWER_FORWARD, 0);
            std::vector<const std::vector<double2> *> refs{&m};
            g.dense = upload_tables(refs, ctx, s)[0];
            launch_gate(psi, batch, n, g, s);
            if (adj) launch_gate(lam, batch, n, g, s);
            continue;
        }
        const uint32_t k = st.header.k;
        const uint32_t tiles_log = n - k;
        const uint64_t total_tiles = uint64_t(batch) << tiles_log;
        const size_t smem = fused_smem(adj, k, st.header.nacc, st.header.nops, st.header.nmat,
                                       fused_threads(k, st.header.rb));
        const auto *hdr = reinterpret_cast<const PassHeader *>(dev + offs[i].hdr);
        const auto *sub = reinterpret_cast<const SubBlock *>(dev + offs[i].subs);
        const auto *ops = reinterpret_cast<const FOp *>(dev + offs[i].ops);
        const auto *mats = reinterpret_cast<const double2 *>(dev + offs[i].mats);
        const uint32_t threads = fused_threads(k, st.header.rb);
        uint32_t blocks = fused_grid_blocks(adj, k, st.header.rb);
        size_t launch_smem = smem;
        if (jit[i]) {
            // compiled kernels: the op table is inlined (none in shared memory)
            const uint32_t lanes = jit_acc_lanes(adj, st.header.rb);
            launch_smem = fused_smem(adj, k, st.header.nacc, 0,
                                     jit_mats_in_params(adj) ? 0 : st.header.nmat,
                                     acc_row_stride(threads / lanes, lanes),
                                     !adj && jit_forward_single());
            blocks = jit_grid_blocks(jit[i], threads, launch_smem);
        }
        if (!jit[i] && adj && st.header.rb == 4)
            fail("internal: adjoint pass with 4 register bits has no compiled kernel");
        if (adj && blocks > partial_stride) blocks = partial_stride;
        const unsigned grid = unsigned(total_tiles < blocks ? total_tiles : blocks);
        // algorithmic traffic: psi (and lambda) read and written once per pass
        const double bytes = (adj ? 64.0 : 32.0) * double(uint64_t(batch) << n);
        const ProfToken tok = prof_begin(adj ? PROF_FUSED_ADJ : PROF_FUSED_FWD, s);
        if (jit[i]) {
            double2 *a_psi = psi, *a_lam = adj ? lam : nullptr;
            uint32_t a_n = n, a_tl = tiles_log, a_stride = adj ? partial_stride : 0;
            uint64_t a_tt = total_tiles;
            const PassHeader *a_h = hdr;
            const SubBlock *a_sub = sub;
            const FOp *a_ops = ops;
            const double2 *a_mats = mats;
            double *a_part = adj ? partials : nullptr;
            // by value: the pass's matrix table itself is the kernel parameter (copied at launch)
            static const double2 kNoMats[1] = {};
            void *mats_arg = jit_mats_in_params(adj)
                                 ? const_cast<double2 *>(st.mats.empty() ? kNoMats : st.mats.data())
                                 : static_cast<void *>(&a_mats);
            void *args[] = {&a_psi, &a_lam, &a_n, &a_tl, &a_tt, &a_h, &a_sub, &a_ops, mats_arg,
                            &a_part, &a_stride};
            jit_launch(jit[i], grid, threads, launch_smem, s, args);
        } else {
            fused_kernel(adj, st.header.rb)<<<grid, fused_threads(k, st.header.rb), smem, s>>>(
                psi, adj ? lam : nullptr, n, tiles_log, total_tiles, hdr, sub, ops, mats,
                adj ? partials : nullptr, adj ? partial_stride : 0);
        }
        prof_end(tok, s, bytes);
        check_cuda(cudaGetLastError(), "fused pass launch");
    }
}

}  // namespace arcqml
