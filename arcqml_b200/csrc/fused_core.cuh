// fused_core.cuh — device code shared by the precompiled fused-pass kernels (fused.cu) and the
// per-pass kernels compiled at run time (jit.cpp embeds this file's text).
//
// Included inside namespace arcqml after fused.h. Compiles under nvcc and NVRTC alike: it uses
// no standard headers. With ARCQML_HOST_RUN defined, the parts that only a GPU can run
// (asynchronous copies, warp shuffles, the tile loop) are left out, so that a host build of a
// compiled pass's code can be executed on the CPU by a test.
#pragma once

__device__ __forceinline__ uint32_t phys(uint32_t j) {
    return j ^ (((j >> 3) ^ (j >> 6) ^ (j >> 9)) & 7u);
}

__device__ __forceinline__ double2 cmul(double2 a, double2 b) {
    return make_double2(fma(a.x, b.x, -a.y * b.y), fma(a.x, b.y, a.y * b.x));
}
__device__ __forceinline__ double2 cfma(double2 a, double2 b, double2 c) {
    return make_double2(fma(a.x, b.x, fma(-a.y, b.y, c.x)), fma(a.x, b.y, fma(a.y, b.x, c.y)));
}
// Re(conj(a) b) and Im(conj(a) b)
__device__ __forceinline__ double rcm(double2 a, double2 b) { return fma(a.x, b.x, a.y * b.y); }
__device__ __forceinline__ double icm(double2 a, double2 b) { return fma(a.x, b.y, -a.y * b.x); }


__device__ __forceinline__ double2 ld(const double2 *p) { return *p; }

// The matrix table a compiled pass indexes as M[...]: a pointer (shared memory, or a host buffer
// in host runs of the pass code), or the m member of the kernel's by-value parameter struct.
__device__ __forceinline__ const double2 *mats_of(const double2 *p) { return p; }
template <class T>
__device__ __forceinline__ const auto &mats_of(const T &params) { return params.m; }

#ifndef ARCQML_HOST_RUN  // device-only: not in host builds of the pass code (tests)
// 16-byte asynchronous global -> shared copy (LDGSTS); completion via commit/wait groups.
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}


// Adds the warp's sum of z into its own column of accumulator row `row` (= acc * warps).
__device__ __forceinline__ void accumulate_warp(double *sacc, uint32_t row, double z) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
    if ((threadIdx.x & 31u) == 0) sacc[row + (threadIdx.x >> 5)] += z;
}

// Adds the sum of z over each group of four lanes into that group's column of accumulator row
// `row` (= acc * blockDim.x / 4): a quarter of the per-thread columns' shared memory, for kernels
// that run two CTAs per SM. Every lane of the warp calls it.
__device__ __forceinline__ void accumulate_quad(double *sacc, uint32_t row, double z) {
    z += __shfl_xor_sync(0xffffffffu, z, 1);
    z += __shfl_xor_sync(0xffffffffu, z, 2);
    if ((threadIdx.x & 3u) == 0) sacc[row + (threadIdx.x >> 2)] += z;
}

// Two gradient sums z0 (row r0) and z1 (row r1) of this thread, each summed over its group of
// four lanes: one shuffle round leaves lane l with the pair's partial of z(l & 1), a second sums
// it over lane bit 1; lanes 0 and 1 of the quad add the results into rows r0 and r1. Every lane
// of the warp calls it.
__device__ __forceinline__ void accumulate_quad2(double *sacc, double z0, double z1, uint32_t r0,
                                                 uint32_t r1) {
    const bool odd = threadIdx.x & 1u;
    double keep = odd ? z1 : z0;
    keep += __shfl_xor_sync(0xffffffffu, odd ? z0 : z1, 1);
    keep += __shfl_xor_sync(0xffffffffu, keep, 2);
    if ((threadIdx.x & 2u) == 0) sacc[(odd ? r1 : r0) + (threadIdx.x >> 2)] += keep;
}
#else
// Host runs execute the threads one after another: the group's column takes each lane's z.
__device__ __forceinline__ void accumulate_quad(double *sacc, uint32_t row, double z) {
    sacc[row + (threadIdx.x >> 2)] += z;
}
__device__ __forceinline__ void accumulate_quad2(double *sacc, double z0, double z1, uint32_t r0,
                                                 uint32_t r1) {
    sacc[r0 + (threadIdx.x >> 2)] += z0;
    sacc[r1 + (threadIdx.x >> 2)] += z1;
}
#endif

// Adds z into this thread's own column of accumulator row `row` (= acc * blockDim.x): no
// cross-lane traffic per gate; the columns are summed once per pass at the end of the kernel.
__device__ __forceinline__ void accumulate(double *sacc, uint32_t row, double z) {
    sacc[row + threadIdx.x] += z;
}

// ---------------------------------------------------------------- specialised fast paths
//
// Uncontrolled gates with compile-time register bits: pure FP64 arithmetic on the thread's
// registers, no per-element index or control logic. Sign flips (CZ, Z) toggle the sign bit
// of the high word with an integer XOR instead of using the FP64 pipe.

__device__ __forceinline__ double flip(double x, uint32_t m) {
    return __hiloint2double(__double2hiint(x) ^ int(m), __double2loint(x));
}
__device__ __forceinline__ double2 flip2(double2 a, uint32_t m) {
    return make_double2(flip(a.x, m), flip(a.y, m));
}

template <int RB, int B>
__device__ __forceinline__ void f_rx(double2 (&v)[1 << RB], double c, double s) {
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) {
        if (e & (1 << B)) continue;
        const int f = e | (1 << B);
        const double2 x0 = v[e], x1 = v[f];
        v[e] = make_double2(fma(c, x0.x, s * x1.y), fma(c, x0.y, -s * x1.x));
        v[f] = make_double2(fma(c, x1.x, s * x0.y), fma(c, x1.y, -s * x0.x));
    }
}

template <int RB, int B>
__device__ __forceinline__ void f_ry(double2 (&v)[1 << RB], double c, double s) {
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) {
        if (e & (1 << B)) continue;
        const int f = e | (1 << B);
        const double2 x0 = v[e], x1 = v[f];
        v[e] = make_double2(fma(c, x0.x, -s * x1.x), fma(c, x0.y, -s * x1.y));
        v[f] = make_double2(fma(s, x0.x, c * x1.x), fma(s, x0.y, c * x1.y));
    }
}

template <int RB, int B>
__device__ __forceinline__ void f_m2(double2 (&v)[1 << RB], const double2 *mt) {
    const double2 m0 = mt[0], m1 = mt[1], m2 = mt[2], m3 = mt[3];
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) {
        if (e & (1 << B)) continue;
        const int f = e | (1 << B);
        const double2 x0 = v[e], x1 = v[f];
        v[e] = cfma(m0, x0, cmul(m1, x1));
        v[f] = cfma(m2, x0, cmul(m3, x1));
    }
}

template <int RB, int B>
__device__ __forceinline__ void f_d1_reg(double2 (&v)[1 << RB], double2 d0, double2 d1) {
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) v[e] = cmul((e >> B) & 1 ? d1 : d0, v[e]);
}

template <int RB>
__device__ __forceinline__ void f_d1_uni(double2 (&v)[1 << RB], double2 d) {
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) v[e] = cmul(d, v[e]);
}

template <int RB, int B0, int B1>
__device__ __forceinline__ void f_sign_rr(double2 (&v)[1 << RB]) {
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e)
        if (((e >> B0) & 1) && ((e >> B1) & 1)) v[e] = flip2(v[e], 0x80000000u);
}

template <int RB, int B>
__device__ __forceinline__ void f_sign_rc(double2 (&v)[1 << RB], uint32_t m) {
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e)
        if ((e >> B) & 1) v[e] = flip2(v[e], m);
}

template <int RB>
__device__ __forceinline__ void f_sign_cc(double2 (&v)[1 << RB], uint32_t m) {
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) v[e] = flip2(v[e], m);
}

// X on register bit B: the pairs exchange registers (no arithmetic once unrolled).
template <int RB, int B>
__device__ __forceinline__ void f_x(double2 (&v)[1 << RB]) {
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) {
        if (e & (1 << B)) continue;
        const double2 t = v[e];
        v[e] = v[e | (1 << B)];
        v[e | (1 << B)] = t;
    }
}

// CNOT with control register bit BC and target register bit BT.
template <int RB, int BC, int BT>
__device__ __forceinline__ void f_cx_rr(double2 (&v)[1 << RB]) {
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) {
        if ((e & (1 << BT)) || !(e & (1 << BC))) continue;
        const double2 t = v[e];
        v[e] = v[e | (1 << BT)];
        v[e | (1 << BT)] = t;
    }
}

// CNOT whose control is the same for all of the thread's elements (a thread or tile bit).
template <int RB, int B>
__device__ __forceinline__ void f_cx_cr(double2 (&v)[1 << RB], uint32_t on) {
    if (on) f_x<RB, B>(v);
}

template <int RB, int B0, int B1>
__device__ __forceinline__ void f_m4(double2 (&v)[1 << RB], const double2 *mt) {
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) {
        if (e & ((1 << B0) | (1 << B1))) continue;
        const int idx[4] = {e, e | (1 << B0), e | (1 << B1), e | (1 << B0) | (1 << B1)};
        double2 x[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = v[idx[j]];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            double2 acc = cmul(mt[i * 4], x[0]);
            acc = cfma(mt[i * 4 + 1], x[1], acc);
            acc = cfma(mt[i * 4 + 2], x[2], acc);
            acc = cfma(mt[i * 4 + 3], x[3], acc);
            v[idx[i]] = acc;
        }
    }
}

// Scaled unit-diagonal forms (compiled scaled passes; the factor the planner took out of each
// op is carried by the pass as one scalar): one FMA per component.
// RX-form c [[1, -it], [-it, 1]]
template <int RB, int B>
__device__ __forceinline__ void fs_rx(double2 (&v)[1 << RB], double t) {
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) {
        if (e & (1 << B)) continue;
        const int f = e | (1 << B);
        const double2 x0 = v[e], x1 = v[f];
        v[e] = make_double2(fma(t, x1.y, x0.x), fma(-t, x1.x, x0.y));
        v[f] = make_double2(fma(t, x0.y, x1.x), fma(-t, x0.x, x1.y));
    }
}

// RY-form c [[1, -t], [t, 1]]
template <int RB, int B>
__device__ __forceinline__ void fs_ry(double2 (&v)[1 << RB], double t) {
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) {
        if (e & (1 << B)) continue;
        const int f = e | (1 << B);
        const double2 x0 = v[e], x1 = v[f];
        v[e] = make_double2(fma(-t, x1.x, x0.x), fma(-t, x1.y, x0.y));
        v[f] = make_double2(fma(t, x0.x, x1.x), fma(t, x0.y, x1.y));
    }
}

// x (1 + i t)
__device__ __forceinline__ double2 one_plus_it(double2 x, double t) {
    return make_double2(fma(-t, x.y, x.x), fma(t, x.x, x.y));
}

// diag(1 - i tau, 1 + i tau) on register bit B
template <int RB, int B>
__device__ __forceinline__ void fs_d1_reg(double2 (&v)[1 << RB], double tau) {
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) v[e] = one_plus_it(v[e], ((e >> B) & 1) ? tau : -tau);
}

// (1 + i t) on every element (t = +-tau by the thread's bit of the qubit)
template <int RB>
__device__ __forceinline__ void fs_d1_uni(double2 (&v)[1 << RB], double t) {
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) v[e] = one_plus_it(v[e], t);
}

// The pass's factor sigma, multiplied in once before the tile is written back.
template <int RB>
__device__ __forceinline__ void fs_scale(double2 (&v)[1 << RB], double2 sigma) {
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) v[e] = cmul(sigma, v[e]);
}

// Gradient sums Im<lam|P|psi> and Re-forms over the thread's elements: one FMA per product
// term (2 FP64 instructions per amplitude), two partial sums (one addition to close them).
template <int RB, int B>
__device__ __forceinline__ double g_x(const double2 (&v)[1 << RB], const double2 (&w)[1 << RB]) {
    double a = 0.0, b = 0.0;
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) {
        if (e & (1 << B)) continue;
        const int f = e | (1 << B);
        a = fma(w[e].x, v[f].y, a);
        a = fma(-w[e].y, v[f].x, a);
        b = fma(w[f].x, v[e].y, b);
        b = fma(-w[f].y, v[e].x, b);
    }
    return a + b;
}

template <int RB, int B>
__device__ __forceinline__ double g_y(const double2 (&v)[1 << RB], const double2 (&w)[1 << RB]) {
    double a = 0.0, b = 0.0;
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) {
        if (e & (1 << B)) continue;
        const int f = e | (1 << B);
        a = fma(w[f].x, v[e].x, a);
        a = fma(w[f].y, v[e].y, a);
        b = fma(-w[e].x, v[f].x, b);
        b = fma(-w[e].y, v[f].y, b);
    }
    return a + b;
}

template <int RB, int B>
__device__ __forceinline__ double g_z(const double2 (&v)[1 << RB], const double2 (&w)[1 << RB]) {
    double z[2] = {0.0, 0.0};
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) {
        const bool neg = (e >> B) & 1;  // compile-time: folds into the FMA operands
        double &a = z[e & 1];
        a = fma(neg ? -w[e].x : w[e].x, v[e].y, a);
        a = fma(neg ? w[e].y : -w[e].y, v[e].x, a);
    }
    return z[0] + z[1];
}

template <int RB>
__device__ __forceinline__ double g_z_uni(const double2 (&v)[1 << RB], const double2 (&w)[1 << RB]) {
    double z[2] = {0.0, 0.0};
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) {
        double &a = z[e & 1];
        a = fma(w[e].x, v[e].y, a);
        a = fma(-w[e].y, v[e].x, a);
    }
    return z[0] + z[1];
}

// One-target gates and gradient terms on one register pair (x0 / v0 / w0: target bit 0), for
// controlled gates in compiled passes, whose code lists the pairs with every control set.
__device__ __forceinline__ void p_rx(double2 &x0, double2 &x1, double c, double s) {
    const double2 a = x0, b = x1;
    x0 = make_double2(fma(c, a.x, s * b.y), fma(c, a.y, -s * b.x));
    x1 = make_double2(fma(c, b.x, s * a.y), fma(c, b.y, -s * a.x));
}
__device__ __forceinline__ void p_ry(double2 &x0, double2 &x1, double c, double s) {
    const double2 a = x0, b = x1;
    x0 = make_double2(fma(c, a.x, -s * b.x), fma(c, a.y, -s * b.y));
    x1 = make_double2(fma(s, a.x, c * b.x), fma(s, a.y, c * b.y));
}
__device__ __forceinline__ void p_m2(double2 &x0, double2 &x1, const double2 *mt) {
    const double2 a = x0, b = x1;
    x0 = cfma(mt[0], a, cmul(mt[1], b));
    x1 = cfma(mt[2], a, cmul(mt[3], b));
}
// Im<lam|X|psi> and Im<lam|Y|psi> over one pair (psi v, lambda w)
__device__ __forceinline__ double p_gx(double2 v0, double2 v1, double2 w0, double2 w1) {
    return icm(w0, v1) + icm(w1, v0);
}
__device__ __forceinline__ double p_gy(double2 v0, double2 v1, double2 w0, double2 w1) {
    return rcm(w1, v0) - rcm(w0, v1);
}
// s += conj(w) v (two FMAs per component): sums that a diagonal's entries multiply afterwards
__device__ __forceinline__ void acc_cw(double2 &s, double2 w, double2 v) {
    s = make_double2(fma(w.x, v.x, fma(w.y, v.y, s.x)), fma(w.x, v.y, fma(-w.y, v.x, s.y)));
}
// Re<lam| D |psi> over one group of four for a dense 4x4 D (group index bit 0: rb0, bit 1: rb1)
__device__ __forceinline__ double q_gm4(const double2 *d, double2 v0, double2 v1, double2 v2,
                                        double2 v3, double2 w0, double2 w1, double2 w2,
                                        double2 w3) {
    const double2 x[4] = {v0, v1, v2, v3}, l[4] = {w0, w1, w2, w3};
    double t = 0.0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        double2 acc = cmul(d[i * 4], x[0]);
        acc = cfma(d[i * 4 + 1], x[1], acc);
        acc = cfma(d[i * 4 + 2], x[2], acc);
        acc = cfma(d[i * 4 + 3], x[3], acc);
        t += rcm(l[i], acc);
    }
    return t;
}


// Per-thread value of a qubit that is not a register bit: a tile bit lives in the thread's
// base index tb, a qubit outside the tile in the tile's global base.
__device__ __forceinline__ uint32_t const_bit(const FOp &o, int slot, uint32_t tb, uint64_t gbase) {
    return o.dq_in_tile[slot] ? ((tb >> o.dq_pos[slot]) & 1u) : uint32_t((gbase >> o.dq_pos[slot]) & 1u);
}

// Tile-local index of a thread's register element e in the current sub-block.
template <int RB>
__device__ __forceinline__ uint32_t sub_index(uint32_t tb, const uint32_t (&rm)[RB], int e) {
    uint32_t x = tb;
#pragma unroll
    for (int r = 0; r < RB; ++r)
        if ((e >> r) & 1) x |= rm[r];
    return x;
}

// Shared memory: [tile buffers][hioff][accumulators][ops][matrices].
// Forward: two psi buffers; while a CTA computes tile i from one, cp.async streams tile
// i + gridDim into the other. Forward single-buffered (`single`, the compiled kernels that run
// two CTAs per SM): one psi buffer, the other CTA on the SM computing while this one loads.
// Adjoint: one psi and one lambda buffer (the next tile is prefetched into L2 instead) and one
// accumulator column per thread. Kernels that do not read
// the op table from shared memory pass nops = 0.
struct SmemLayout {
    uint32_t tile, hioff, sacc, ops, mats, total;
};

// acc_cols: the accumulator table's row stride in doubles (acc_row_stride).
__host__ __device__ inline SmemLayout smem_layout(bool adj, uint32_t k, uint32_t nacc,
                                                  uint32_t nops, uint32_t nmat, uint32_t acc_cols,
                                                  bool single = false) {
    const uint32_t L = k < uint32_t(kLowFixed) ? k : uint32_t(kLowFixed);
    SmemLayout m;
    m.tile = 0;
    uint32_t off = ((adj || !single) ? 2u : 1u) * (16u << k);
    m.hioff = off;
    off += 8u << (k - L);
    off = (off + 15u) & ~15u;
    m.sacc = off;
    off += adj ? nacc * acc_cols * 8u : 0u;
    off = (off + 15u) & ~15u;
    m.ops = off;
    off += nops * uint32_t(sizeof(FOp));
    m.mats = off;
    off += nmat * 16u;
    m.total = off;
    return m;
}

// Gathers the thread's 2^RB amplitudes of psi (and lambda) for sub-block S.
template <int RB, bool ADJ>
__device__ __forceinline__ void load_regs(const SubBlock &S, uint32_t tb, const double2 *tp,
                                          const double2 *tl, double2 (&v)[1 << RB],
                                          double2 (&w)[1 << RB]) {
    uint32_t rm[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) rm[r] = 1u << S.R[r];
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) {
        const uint32_t x = sub_index<RB>(tb, rm, e);
        v[e] = tp[phys(x)];
        if (ADJ) w[e] = tl[phys(x)];
    }
}

template <int RB, bool ADJ>
__device__ __forceinline__ void store_regs(const SubBlock &S, uint32_t tb, double2 *tp,
                                           double2 *tl, const double2 (&v)[1 << RB],
                                           const double2 (&w)[1 << RB]) {
    uint32_t rm[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) rm[r] = 1u << S.R[r];
#pragma unroll
    for (int e = 0; e < (1 << RB); ++e) {
        const uint32_t x = sub_index<RB>(tb, rm, e);
        tp[phys(x)] = v[e];
        if (ADJ) tl[phys(x)] = w[e];
    }
}

// Thread base index of sub-block S: thread bit i goes to tile bit S.perm[i].
template <int RB>
__device__ __forceinline__ uint32_t thread_base(const SubBlock &S, uint32_t k) {
    uint32_t tb = 0;
#pragma unroll
    for (int i = 0; i < 12 - RB; ++i)
        if (i < int(k) - RB && ((threadIdx.x >> i) & 1)) tb |= 1u << S.perm[i];
    return tb;
}

#ifndef ARCQML_HOST_RUN
// Sub-block sb of the pass table, read through the read-only cache.
__device__ __forceinline__ SubBlock load_subblock(const SubBlock *subs, uint32_t sb) {
    SubBlock S;
    const uint2 *src = reinterpret_cast<const uint2 *>(subs + sb);
    uint2 *d = reinterpret_cast<uint2 *>(&S);
#pragma unroll
    for (int i = 0; i < 3; ++i) d[i] = __ldg(src + i);
    return S;
}

// One pass over all tiles; Runner::run<RB, ADJ>(sb, ...) applies sub-block sb of the pass to
// the tile (it gathers the thread's registers, applies the gates and scatters them back).
// Runner::kSingleBuffer: a forward pass keeps one tile buffer (load, compute, write back), as
// the adjoint does. Runner::kPrefetch: one-buffer loops ask L2 for the next tile while this one
// is computed. Runner::kOpsInSmem: the runner reads
// the op table from shared memory (the table-driven kernel; compiled kernels have it inlined).
// Runner::kMatsInSmem: the matrix table `gmats` (a pointer) is staged in shared memory;
// otherwise `gmats` is the kernel's by-value parameter struct holding the table (member m), which
// the runner indexes directly, so that its entries are constant-bank operands of the arithmetic
// and need no loads or registers of their own.
// fn(j, phys(j)) for every tile element j the calling thread copies between the state and the
// tile: with KT > 0 (blockDim.x = 2^(KT - RB)) 2^RB unrolled accesses whose slots differ from
// phys(threadIdx.x) = ptid by compile-time constants (phys is linear over XOR).
template <int RB, int KT, class F>
__device__ __forceinline__ void tile_elements(uint32_t D, uint32_t ptid, const F &fn) {
    if constexpr (KT > 0) {
#pragma unroll
        for (uint32_t i = 0; i < (1u << RB); ++i) {
            const uint32_t hi = i << (KT - RB);
            fn(threadIdx.x | hi, ptid ^ phys(hi));
        }
    } else {
        for (uint32_t j = threadIdx.x; j < D; j += blockDim.x) fn(j, phys(j));
    }
}

// KT > 0: the tile has KT qubits (the compiled kernels know it), so the copies between the
// state and the tile unroll into 2^RB accesses per thread whose shared-memory slots differ from
// the thread's own by compile-time constants (phys is linear over XOR); KT = 0 reads k from the
// pass header.
template <int RB, bool ADJ, class Runner, int KT = 0, class GM = const double2 *>
__device__ __forceinline__ void fused_body(double2 *__restrict__ psi, double2 *__restrict__ lam,
                                           uint32_t n, uint32_t tiles_log, uint64_t total_tiles,
                                           const PassHeader *__restrict__ hdr,
                                           const SubBlock *__restrict__ subs,
                                           const FOp *__restrict__ gops,
                                           const GM &gmats,
                                           double *__restrict__ partials, uint32_t stride) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ uint8_t sS[16];
    __shared__ uint32_t sk, snsub, snacc, sacc_base, snops, snmat;
    if (threadIdx.x < 16) sS[threadIdx.x] = hdr->S[threadIdx.x];
    if (threadIdx.x == 0) {
        sk = hdr->k;
        snsub = hdr->nsub;
        snacc = hdr->nacc;
        sacc_base = hdr->acc_base;
        snops = hdr->nops;
        snmat = hdr->nmat;
    }
    __syncthreads();
    const uint32_t k = KT > 0 ? uint32_t(KT) : sk;
    const uint32_t D = 1u << k;
    const uint32_t L = k < uint32_t(kLowFixed) ? k : uint32_t(kLowFixed);
    const uint32_t lowmask = (1u << L) - 1;
    // accumulator columns: one per Runner::kAccLanes threads (1, 4 or a warp); row stride
    const uint32_t ncols = blockDim.x / uint32_t(Runner::kAccLanes);
    const uint32_t nthreads = acc_row_stride(ncols, uint32_t(Runner::kAccLanes));
    constexpr bool kSingle = ADJ || Runner::kSingleBuffer;
    const uint32_t nops_smem = Runner::kOpsInSmem ? snops : 0u;
    const uint32_t nmat_smem = Runner::kMatsInSmem ? snmat : 0u;
    const SmemLayout lay =
        smem_layout(ADJ, k, snacc, nops_smem, nmat_smem, nthreads, Runner::kSingleBuffer);
    double2 *bufs = reinterpret_cast<double2 *>(smem + lay.tile);
    uint64_t *hioff = reinterpret_cast<uint64_t *>(smem + lay.hioff);
    double *sacc = reinterpret_cast<double *>(smem + lay.sacc);
    FOp *ops = reinterpret_cast<FOp *>(smem + lay.ops);
    const double2 *smats = reinterpret_cast<const double2 *>(smem + lay.mats);
    // forward: buffer b (always 0 single-buffered); adjoint: state st (0 = psi, 1 = lambda)
    auto tile_buf = [&](int b, int st) { return bufs + size_t(ADJ ? st : b) * D; };

    for (uint32_t h = threadIdx.x; h < (1u << (k - L)); h += blockDim.x) {
        uint64_t off = 0;
        for (uint32_t b = 0; b < k - L; ++b)
            if ((h >> b) & 1) off |= uint64_t(1) << sS[L + b];
        hioff[h] = off;
    }
    {
        const uint4 *src = reinterpret_cast<const uint4 *>(gops);
        uint4 *dst = reinterpret_cast<uint4 *>(ops);
        for (uint32_t i = threadIdx.x; i < nops_smem * 4; i += blockDim.x) dst[i] = src[i];
        if constexpr (Runner::kMatsInSmem) {
            double2 *dst_m = reinterpret_cast<double2 *>(smem + lay.mats);
            for (uint32_t i = threadIdx.x; i < nmat_smem; i += blockDim.x) dst_m[i] = gmats[i];
        }
    }
    if (ADJ)
        for (uint32_t a = threadIdx.x; a < snacc * nthreads; a += blockDim.x) sacc[a] = 0.0;
    __syncthreads();

    const uint32_t ptid = phys(threadIdx.x);

    const uint64_t tmask = (uint64_t(1) << tiles_log) - 1;
    auto tile_base = [&](uint64_t T) {
        uint64_t g = T & tmask;
        for (uint32_t b = 0; b < k; ++b) {
            const uint32_t p = sS[b];
            g = ((g >> p) << (p + 1)) | (g & ((uint64_t(1) << p) - 1));
        }
        return g;
    };
    auto issue_load = [&](uint64_t T, int b) {
        const uint64_t off = ((T >> tiles_log) << n) + tile_base(T);
        const double2 *P = psi + off;
        const double2 *Lm = ADJ ? lam + off : nullptr;
        double2 *tp = tile_buf(b, 0);
        double2 *tl = ADJ ? tile_buf(b, 1) : nullptr;
        tile_elements<RB, KT>(D, ptid, [&](uint32_t j, uint32_t pj) {
            const uint64_t g = (j & lowmask) | hioff[j >> L];
            cp_async16(tp + pj, P + g);
            if (ADJ) cp_async16(tl + pj, Lm + g);
        });
        cp_async_commit();
    };

    // Applies every sub-block of the pass to the tile in buffer b and writes it back.
    auto process_tile = [&](uint64_t T, int b) {
        const uint64_t gbase = tile_base(T);
        double2 *tp = tile_buf(b, 0);
        double2 *tl = ADJ ? tile_buf(b, 1) : nullptr;
        for (uint32_t sb = 0; sb < snsub; ++sb) {
            if constexpr (Runner::kMatsInSmem)
                Runner::template run<RB, ADJ>(sb, k, tp, tl, ops, smats, subs, sacc, nthreads,
                                              gbase);
            else
                Runner::template run<RB, ADJ>(sb, k, tp, tl, ops, gmats, subs, sacc, nthreads,
                                              gbase);
            // the next sub-block reads only elements this warp wrote: the warp's own barrier
            if (Runner::warp_next(sb)) __syncwarp();
            else __syncthreads();
        }
        const uint64_t off = ((T >> tiles_log) << n) + gbase;
        double2 *P = psi + off;
        double2 *Lm = ADJ ? lam + off : nullptr;
        tile_elements<RB, KT>(D, ptid, [&](uint32_t j, uint32_t pj) {
            const uint64_t g = (j & lowmask) | hioff[j >> L];
            P[g] = tp[pj];
            if (ADJ) Lm[g] = tl[pj];
        });
    };

    if constexpr (kSingle) {
        // One buffer: load tile T, ask L2 for tile T + gridDim while T is computed (when
        // Runner::kPrefetch).
        const uint32_t run_bytes = 16u << L;
        const uint32_t lines = run_bytes >= 128u ? run_bytes / 128u : 1u;
        for (uint64_t T = blockIdx.x; T < total_tiles; T += gridDim.x) {
            issue_load(T, 0);
            const uint64_t Tn = T + gridDim.x;
            if (Runner::kPrefetch && Tn < total_tiles) {
                const uint64_t off = ((Tn >> tiles_log) << n) + tile_base(Tn);
                const char *P = reinterpret_cast<const char *>(psi + off);
                const char *Lm = ADJ ? reinterpret_cast<const char *>(lam + off) : nullptr;
                const uint32_t count = lines << (k - L);
                for (uint32_t i = threadIdx.x; i < count; i += blockDim.x) {
                    const size_t o = size_t(hioff[i / lines]) * 16u + size_t(i % lines) * 128u;
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(P + o));
                    if (ADJ) asm volatile("prefetch.global.L2 [%0];" ::"l"(Lm + o));
                }
            }
            cp_async_wait<0>();
            __syncthreads();
            process_tile(T, 0);
            __syncthreads();
        }
    } else {
        if (uint64_t(blockIdx.x) < total_tiles) issue_load(blockIdx.x, 0);
        else cp_async_commit();
        int b = 0;
        for (uint64_t T = blockIdx.x; T < total_tiles; T += gridDim.x, b ^= 1) {
            const uint64_t Tn = T + gridDim.x;
            if (Tn < total_tiles) issue_load(Tn, b ^ 1);
            else cp_async_commit();
            cp_async_wait<1>();
            __syncthreads();
            process_tile(T, b);
            __syncthreads();
        }
    }
    cp_async_wait<0>();
    if (ADJ) {
        // column sums in a fixed order (deterministic)
        for (uint32_t a = threadIdx.x; a < snacc; a += blockDim.x) {
            const double *row = sacc + size_t(a) * nthreads;
            double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
            uint32_t t = 0;
            for (; t + 4 <= ncols; t += 4) {
                s0 += row[t];
                s1 += row[t + 1];
                s2 += row[t + 2];
                s3 += row[t + 3];
            }
            for (; t < ncols; ++t) s0 += row[t];
            double f;  // the row's factor (compiled kernels add their sums unscaled)
            if constexpr (Runner::kMatsInSmem) f = Runner::row_factor(a, smats);
            else f = Runner::row_factor(a, gmats);
            partials[size_t(sacc_base + a) * stride + blockIdx.x] = ((s0 + s1) + (s2 + s3)) * f;
        }
    }
}
#endif  // ARCQML_HOST_RUN
