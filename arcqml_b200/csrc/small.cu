// small.cu — one-kernel run + backward for small single states (n <= kSmallMaxQubits), and the
// device optimizer loop built on it.
//
// A 16-amplitude VQE state is bound by launches and host round trips, not by arithmetic: the
// per-gate path issues ~40 launches and two synchronisations per step. Here one CTA holds psi
// and lambda in shared memory and does the whole step — every gate forward, H psi and <H> (the
// CompiledHamiltonian arithmetic of compiled_hamiltonian.rs:81-182), then the adjoint reverse
// sweep with each bound slot's 2 Re<lambda| dU/dp |psi> summed in a fixed order — and writes
// the value and the gradients in one small block, read back with one copy.
#include <cuda_runtime.h>

#include "launch.h"
#include "profile.h"
#include "rt_internal.h"

namespace arcqml {
namespace {

constexpr int kSmallThreads = 256;

__device__ __forceinline__ double2 s_cmul(double2 a, double2 b) {
    return make_double2(fma(a.x, b.x, -a.y * b.y), fma(a.x, b.y, a.y * b.x));
}
__device__ __forceinline__ double2 s_cfma(double2 a, double2 b, double2 c) {
    return make_double2(fma(a.x, b.x, fma(-a.y, b.y, c.x)), fma(a.x, b.y, fma(a.y, b.x, c.y)));
}

__device__ __forceinline__ uint32_t s_insert_zeros(uint32_t g, const uint8_t *pos, int npos) {
    for (int b = 0; b < npos; ++b) {
        const uint32_t p = pos[b];
        g = ((g >> p) << (p + 1)) | (g & ((1u << p) - 1));
    }
    return g;
}

// Sum over the CTA of one value per thread, fixed order; valid in every thread.
__device__ double s_block_sum(double v, double *red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    double r = 0.0;
    for (int w = 0; w < int(blockDim.x >> 5); ++w) r += red[w];
    __syncthreads();
    return r;
}

// a <- U a for a lowered gate (1Q / 2Q dense or diagonal, optional controls; DENSE up to 4
// targets without controls), every thread taking groups of the gate's targets.
__device__ void s_apply(double2 *a, uint32_t n, const DevGate &g) {
    if (g.kind == KIND_NONE) return;
    const uint32_t groups = 1u << (n - uint32_t(g.npos));
    for (uint32_t gid = threadIdx.x; gid < groups; gid += blockDim.x) {
        const uint32_t base = s_insert_zeros(gid, g.positions, g.npos) |
                              (g.kind == KIND_DENSE ? 0u : uint32_t(g.cmask));
        if (g.kind == KIND_1Q) {
            const uint32_t i1 = base | (1u << g.t[0]);
            const double2 x0 = a[base], x1 = a[i1];
            a[base] = s_cfma(g.m[0], x0, s_cmul(g.m[1], x1));
            a[i1] = s_cfma(g.m[2], x0, s_cmul(g.m[3], x1));
        } else if (g.kind == KIND_2Q) {
            const uint32_t b0 = 1u << g.t[0], b1 = 1u << g.t[1];
            const uint32_t idx[4] = {base, base | b0, base | b1, base | b0 | b1};
            double2 x[4];
            for (int j = 0; j < 4; ++j) x[j] = a[idx[j]];
            for (int i = 0; i < 4; ++i) {
                double2 acc = s_cmul(g.m[i * 4], x[0]);
                for (int c = 1; c < 4; ++c) acc = s_cfma(g.m[i * 4 + c], x[c], acc);
                a[idx[i]] = acc;
            }
        } else if (g.kind == KIND_DIAG1 || g.kind == KIND_DIAG2) {
            // one amplitude per group (the enumeration may already fix a target bit)
            uint32_t b = (base >> g.t[0]) & 1u;
            if (g.kind == KIND_DIAG2) b |= ((base >> g.t[1]) & 1u) << 1;
            a[base] = s_cmul(g.m[b], a[base]);
        } else {  // KIND_DENSE, k <= 4 targets
            const uint32_t k = uint32_t(g.nt), dim = 1u << k;
            double2 x[16];
            for (uint32_t j = 0; j < dim; ++j) {
                uint32_t off = 0;
                for (uint32_t b = 0; b < k; ++b)
                    if ((j >> b) & 1) off |= 1u << g.dense_targets[b];
                x[j] = a[base | off];
            }
            for (uint32_t r = 0; r < dim; ++r) {
                double2 acc = make_double2(0.0, 0.0);
                for (uint32_t c = 0; c < dim; ++c) acc = s_cfma(g.dense[r * dim + c], x[c], acc);
                uint32_t off = 0;
                for (uint32_t b = 0; b < k; ++b)
                    if ((r >> b) & 1) off |= 1u << g.dense_targets[b];
                a[base | off] = acc;
            }
        }
    }
}

// H psi into lam and <psi|H|psi> (tables as k_pauli's: single-term groups, then the others).
__device__ double s_observable(const double2 *psi, double2 *lam, uint32_t n, const PauliTables &T,
                               double *red) {
    const unsigned char *tb = T.base;
    const double2 *sW = reinterpret_cast<const double2 *>(tb + T.s_w);
    const uint64_t *sF = reinterpret_cast<const uint64_t *>(tb + T.s_f);
    const uint64_t *sZ = reinterpret_cast<const uint64_t *>(tb + T.s_z);
    const double2 *mW = reinterpret_cast<const double2 *>(tb + T.m_w);
    const uint64_t *mZ = reinterpret_cast<const uint64_t *>(tb + T.m_z);
    const uint64_t *mF = reinterpret_cast<const uint64_t *>(tb + T.m_f);
    const uint32_t *mE = reinterpret_cast<const uint32_t *>(tb + T.m_e);
    double ev = 0.0;
    for (uint32_t t = threadIdx.x; t < (1u << n); t += blockDim.x) {
        double2 acc = make_double2(0.0, 0.0);
        for (uint32_t i = 0; i < T.ns; ++i) {
            const double2 w = sW[i];
            const double sg = (__popcll(uint64_t(t) & sZ[i]) & 1) ? -1.0 : 1.0;
            acc = s_cfma(make_double2(sg * w.x, sg * w.y), psi[t ^ uint32_t(sF[i])], acc);
        }
        for (uint32_t g = 0; g < T.nm; ++g) {
            double2 w = make_double2(0.0, 0.0);
            for (uint32_t k = mE[g]; k < mE[g + 1]; ++k) {
                const double sg = (__popcll(uint64_t(t) & mZ[k]) & 1) ? -1.0 : 1.0;
                w.x += sg * mW[k].x;
                w.y += sg * mW[k].y;
            }
            acc = s_cfma(w, psi[t ^ uint32_t(mF[g])], acc);
        }
        lam[t] = acc;
        const double2 p = psi[t];
        ev += fma(p.x, acc.x, p.y * acc.y);
    }
    return s_block_sum(ev, red);
}

// The step on psi and lambda in shared memory: psi <- plan |init> (null: |0...0>), lambda <- H psi,
// then the reverse sweep; rows(j, sum) is called in every thread with the block sum of
// Re<lambda| dU/dp |psi> for the j-th (op, slot) of the sweep. Returns <H> (in every thread).
template <class Rows>
__device__ double small_body(double2 *psi, double2 *lam, const double2 *init, uint32_t n,
                             const SmallOp *ops, uint32_t nops, const PauliTables &T, double *red,
                             Rows rows) {
    const uint32_t dim = 1u << n;
    for (uint32_t t = threadIdx.x; t < dim; t += blockDim.x)
        psi[t] = init ? init[t] : make_double2(t == 0 ? 1.0 : 0.0, 0.0);
    __syncthreads();
    for (uint32_t k = 0; k < nops; ++k) {
        s_apply(psi, n, ops[k].u);
        __syncthreads();
    }
    const double value = s_observable(psi, lam, n, T, red);
    __syncthreads();
    uint32_t row = 0;
    for (uint32_t k = nops; k-- > 0;) {
        const SmallOp &o = ops[k];
        if (o.ns == 0) {
            s_apply(psi, n, o.ua);
            s_apply(lam, n, o.ua);
            __syncthreads();
            continue;
        }
        // dense small form of U^dagger (KIND_1Q / KIND_2Q) and dU/dp per slot
        const int D = o.ua.nt == 2 ? 4 : 2;
        const uint32_t groups = 1u << (n - uint32_t(o.ua.npos));
        double acc[3] = {0.0, 0.0, 0.0};
        for (uint32_t gid = threadIdx.x; gid < groups; gid += blockDim.x) {
            const uint32_t base = s_insert_zeros(gid, o.ua.positions, o.ua.npos) |
                                  uint32_t(o.ua.cmask);
            uint32_t idx[4];
            idx[0] = base;
            idx[1] = base | (1u << o.ua.t[0]);
            if (D == 4) {
                idx[2] = base | (1u << o.ua.t[1]);
                idx[3] = idx[1] | (1u << o.ua.t[1]);
            }
            double2 p[4], l[4], q[4];
            for (int j = 0; j < D; ++j) {
                p[j] = psi[idx[j]];
                l[j] = lam[idx[j]];
            }
            for (int i = 0; i < D; ++i) {
                double2 t = make_double2(0.0, 0.0);
                for (int c = 0; c < D; ++c) t = s_cfma(o.ua.m[i * D + c], p[c], t);
                q[i] = t;
            }
            for (int sl = 0; sl < o.ns; ++sl) {
                double v = 0.0;
                for (int i = 0; i < D; ++i) {
                    double2 t = make_double2(0.0, 0.0);
                    for (int c = 0; c < D; ++c) t = s_cfma(o.d[sl][i * D + c], q[c], t);
                    v += fma(l[i].x, t.x, l[i].y * t.y);
                }
                acc[sl] += v;
            }
            for (int i = 0; i < D; ++i) {
                double2 t = make_double2(0.0, 0.0);
                for (int c = 0; c < D; ++c) t = s_cfma(o.ua.m[i * D + c], l[c], t);
                psi[idx[i]] = q[i];
                lam[idx[i]] = t;
            }
        }
        __syncthreads();
        for (int sl = 0; sl < o.ns; ++sl) rows(row++, s_block_sum(acc[sl], red));
    }
    return value;
}

// out[0] = <H>; out[1 + j] = sum over the state of Re<lambda| dU/dp |psi> for the j-th
// (op, slot) of the reverse sweep; lam0 (optional) receives lambda at the start of the circuit.
__global__ void __launch_bounds__(kSmallThreads)
    k_small_step(const double2 *__restrict__ init, uint32_t n, const SmallOp *__restrict__ ops,
                 uint32_t nops, const __grid_constant__ PauliTables T, double *__restrict__ out,
                 double2 *__restrict__ lam0) {
    extern __shared__ __align__(16) double2 s_state[];
    __shared__ double red[kSmallThreads / 32];
    const uint32_t dim = 1u << n;
    double2 *psi = s_state;
    double2 *lam = s_state + dim;
    const double value = small_body(psi, lam, init, n, ops, nops, T, red,
                                    [&](uint32_t row, double sum) {
                                        if (threadIdx.x == 0) out[1 + row] = sum;
                                    });
    if (threadIdx.x == 0) out[0] = value;
    if (lam0)
        for (uint32_t t = threadIdx.x; t < dim; t += blockDim.x) lam0[t] = lam[t];
}

// Adam's update of one parameter, each operation rounded on its own (no contraction), in the
// order of the f64 Adam of crates/arcqml-optim/src/adam.rs:190-240 (coupled L2 weight decay,
// bias-corrected moments): bc1 = 1 - beta1^t, bc2 = 1 - beta2^t come from the host.
__device__ __forceinline__ void adam_update(double &theta, double &m, double &v, double g,
                                            const SmallAdam &h, double bc1, double bc2) {
    const double adj = __dadd_rn(g, __dmul_rn(h.weight_decay, theta));
    m = __dadd_rn(__dmul_rn(h.beta1, m), __dmul_rn(__dsub_rn(1.0, h.beta1), adj));
    v = __dadd_rn(__dmul_rn(h.beta2, v), __dmul_rn(__dmul_rn(__dsub_rn(1.0, h.beta2), adj), adj));
    const double mh = __ddiv_rn(m, bc1), vh = __ddiv_rn(v, bc2);
    theta = __dsub_rn(theta, __ddiv_rn(__dmul_rn(h.lr, mh), __dadd_rn(__dsqrt_rn(vh), h.eps)));
}

// `steps` optimizer steps in one CTA: per step the trained ops' U, U^dagger and dU/dp from the
// current parameters (U = a0 + cos(alpha t) a1 + sin(alpha t) a2), the step of small_body, the
// gradient of every parent summed over its rows (x 2, reverse-sweep order), energies[step] = <H>
// and Adam on the trained parents. theta / adam_m / adam_v are indexed by parent (in and out).
__global__ void __launch_bounds__(kSmallThreads)
    k_small_adam(const double2 *__restrict__ init, uint32_t n, const SmallOp *__restrict__ ops_g,
                 uint32_t nops, const SmallParamOp *__restrict__ pops, uint32_t npops,
                 const uint32_t *__restrict__ row_parent, const uint32_t *__restrict__ trained,
                 uint32_t ntrained, uint32_t nparents, const __grid_constant__ PauliTables T,
                 SmallAdam h, const double *__restrict__ bc, uint32_t steps,
                 double *__restrict__ state, double *__restrict__ energies) {
    extern __shared__ __align__(16) double2 s_state[];
    __shared__ double red[kSmallThreads / 32];
    const uint32_t dim = 1u << n;
    double2 *psi = s_state;
    double2 *lam = s_state + dim;
    SmallOp *ops = reinterpret_cast<SmallOp *>(lam + dim);
    double *th = reinterpret_cast<double *>(ops + nops);  // theta, m, v, grad per parent
    double *am = th + nparents, *av = am + nparents, *gr = av + nparents;
    {
        const uint32_t words = nops * uint32_t(sizeof(SmallOp) / sizeof(double2));
        const double2 *src = reinterpret_cast<const double2 *>(ops_g);
        double2 *dst = reinterpret_cast<double2 *>(ops);
        for (uint32_t i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
        for (uint32_t i = threadIdx.x; i < 3 * nparents; i += blockDim.x) th[i] = state[i];
    }
    __syncthreads();
    for (uint32_t step = 0; step < steps; ++step) {
        for (uint32_t j = threadIdx.x; j < npops; j += blockDim.x) {
            const SmallParamOp &P = pops[j];
            SmallOp &o = ops[P.op];
            double sn, cs;
            sincos(P.alpha * th[P.parent], &sn, &cs);
            const int D = P.dim;
            for (int i = 0; i < D * D; ++i) {
                const double2 a0 = P.a0[i], a1 = P.a1[i], a2 = P.a2[i];
                o.u.m[i] = make_double2(fma(sn, a2.x, fma(cs, a1.x, a0.x)),
                                        fma(sn, a2.y, fma(cs, a1.y, a0.y)));
                o.d[P.slot_row][i] = make_double2(P.alpha * fma(cs, a2.x, -sn * a1.x),
                                                  P.alpha * fma(cs, a2.y, -sn * a1.y));
            }
            for (int r = 0; r < D; ++r)  // U^dagger[r][c] = conj(U[c][r])
                for (int c = 0; c < D; ++c) {
                    const double2 x = o.u.m[c * D + r];
                    o.ua.m[r * D + c] = make_double2(x.x, -x.y);
                }
        }
        for (uint32_t i = threadIdx.x; i < nparents; i += blockDim.x) gr[i] = 0.0;
        __syncthreads();
        const double value = small_body(psi, lam, init, n, ops, nops, T, red,
                                        [&](uint32_t row, double sum) {
                                            if (threadIdx.x == 0)
                                                gr[row_parent[row]] += 2.0 * sum;
                                        });
        if (threadIdx.x == 0) {
            energies[step] = value;
            for (uint32_t i = 0; i < ntrained; ++i) {
                const uint32_t p = trained[i];
                adam_update(th[p], am[p], av[p], gr[p], h, bc[2 * step], bc[2 * step + 1]);
            }
        }
        __syncthreads();
    }
    for (uint32_t i = threadIdx.x; i < 3 * nparents; i += blockDim.x) state[i] = th[i];
}

}  // namespace

// One warp up to 64 amplitudes (half of the groups of a one-qubit gate per thread), then up to
// kSmallThreads threads.
static uint32_t small_threads(uint32_t n) {
    const uint32_t half = n >= 1 ? 1u << (n - 1) : 1u;
    return half < 32u ? 32u : (half > uint32_t(kSmallThreads) ? uint32_t(kSmallThreads) : half);
}

void launch_small_step(const double2 *init, uint32_t n, const SmallOp *ops, uint32_t nops,
                       const PauliTables &tab, double *out, double2 *lam0, cudaStream_t s) {
    if (n > kSmallMaxQubits) fail("internal: state too large for the one-kernel step");
    const size_t smem = size_t(2) * (size_t(1) << n) * sizeof(double2);
    const ProfToken tok = prof_begin(PROF_OTHER, s);
    k_small_step<<<1, small_threads(n), smem, s>>>(init, n, ops, nops, tab, out, lam0);
    prof_end(tok, s, 16.0 * double(size_t(1) << n));
    check_cuda(cudaGetLastError(), "one-kernel step launch");
}

size_t small_adam_smem(uint32_t n, uint32_t nops, uint32_t nparents) {
    return size_t(2) * (size_t(1) << n) * sizeof(double2) + size_t(nops) * sizeof(SmallOp) +
           size_t(4) * nparents * sizeof(double);
}

void launch_small_adam(const double2 *init, uint32_t n, const SmallOp *ops, uint32_t nops,
                       const SmallParamOp *pops, uint32_t npops, const uint32_t *row_parent,
                       const uint32_t *trained, uint32_t ntrained, uint32_t nparents,
                       const PauliTables &tab, const SmallAdam &h, const double *bc,
                       uint32_t steps, double *state, double *energies, cudaStream_t s) {
    if (n > kSmallMaxQubits) fail("internal: state too large for the one-kernel step");
    const size_t smem = small_adam_smem(n, nops, nparents);
    static_assert(sizeof(SmallOp) % sizeof(double2) == 0, "SmallOp copies as double2 words");
    check_cuda(cudaFuncSetAttribute(k_small_adam, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(smem)),
               "cudaFuncSetAttribute (optimizer loop)");
    const ProfToken tok = prof_begin(PROF_OTHER, s);
    k_small_adam<<<1, small_threads(n), smem, s>>>(init, n, ops, nops, pops, npops, row_parent,
                                                   trained, ntrained, nparents, tab, h, bc, steps,
                                                   state, energies);
    prof_end(tok, s, 16.0 * double(size_t(1) << n) * double(steps));
    check_cuda(cudaGetLastError(), "optimizer loop launch");
}

}  // namespace arcqml
