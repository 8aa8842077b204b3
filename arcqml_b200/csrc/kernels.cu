// kernels.cu — per-gate statevector kernels for sm_100a (complex128, HBM-bound).
//
// Every kernel walks "groups": the 2^nt amplitudes a gate mixes, found by inserting zero
// bits at the gate's sorted fixed positions (targets and controls) into a group counter and
// OR-ing the control mask. Consecutive threads take consecutive group counters, so for any
// target above bit 0 a warp reads 32 consecutive 16-byte amplitudes per load (fully
// coalesced 512 B), and for target 0 each thread reads one 32-byte pair (also coalesced).
// Batches [batch, 2^n] are one flat group range: row = counter >> (n - npos).
#include <cuda_runtime.h>

#include "launch.h"
#include "profile.h"
#include "rt_internal.h"

namespace arcqml {

namespace {

__device__ __forceinline__ double2 cmul(double2 a, double2 b) {
    return make_double2(fma(a.x, b.x, -a.y * b.y), fma(a.x, b.y, a.y * b.x));
}
__device__ __forceinline__ double2 cfma(double2 a, double2 b, double2 c) {
    // a*b + c
    return make_double2(fma(a.x, b.x, fma(-a.y, b.y, c.x)), fma(a.x, b.y, fma(a.y, b.x, c.y)));
}
__device__ __forceinline__ double re_conj_mul(double2 a, double2 b) {
    // Re(conj(a) * b)
    return fma(a.x, b.x, a.y * b.y);
}

__device__ __forceinline__ uint64_t insert_zeros(uint64_t g, const uint8_t *pos, int npos) {
    for (int b = 0; b < npos; ++b) {
        const uint32_t p = pos[b];
        const uint64_t low = g & ((uint64_t(1) << p) - 1);
        g = ((g >> p) << (p + 1)) | low;
    }
    return g;
}

constexpr int kThreads = 256;

__device__ __forceinline__ double block_sum(double v, double *smem) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) smem[warp] = v;
    __syncthreads();
    double r = 0.0;
    if (threadIdx.x == 0) {
        for (int w = 0; w < int(blockDim.x >> 5); ++w) r += smem[w];
    }
    return r;  // valid in thread 0
}

// ---------------------------------------------------------------- in-place gate kernels

__global__ void __launch_bounds__(kThreads) k_gate_1q(double2 *__restrict__ a, uint64_t total,
                                                      uint32_t n, uint32_t glog,
                                                      const __grid_constant__ DevGate g) {
    const uint64_t gmask = (uint64_t(1) << glog) - 1;
    const uint64_t tb = uint64_t(1) << g.t[0];
    const double2 m0 = g.m[0], m1 = g.m[1], m2 = g.m[2], m3 = g.m[3];
    for (uint64_t gid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; gid < total;
         gid += uint64_t(gridDim.x) * blockDim.x) {
        double2 *r = a + ((gid >> glog) << n);
        const uint64_t i0 = insert_zeros(gid & gmask, g.positions, g.npos) | g.cmask;
        const uint64_t i1 = i0 | tb;
        const double2 x0 = r[i0], x1 = r[i1];
        r[i0] = cfma(m0, x0, cmul(m1, x1));
        r[i1] = cfma(m2, x0, cmul(m3, x1));
    }
}

__global__ void __launch_bounds__(kThreads) k_gate_2q(double2 *__restrict__ a, uint64_t total,
                                                      uint32_t n, uint32_t glog,
                                                      const __grid_constant__ DevGate g) {
    const uint64_t gmask = (uint64_t(1) << glog) - 1;
    const uint64_t b0 = uint64_t(1) << g.t[0], b1 = uint64_t(1) << g.t[1];
    for (uint64_t gid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; gid < total;
         gid += uint64_t(gridDim.x) * blockDim.x) {
        double2 *r = a + ((gid >> glog) << n);
        const uint64_t i0 = insert_zeros(gid & gmask, g.positions, g.npos) | g.cmask;
        const uint64_t idx[4] = {i0, i0 | b0, i0 | b1, i0 | b0 | b1};
        double2 x[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = r[idx[j]];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            double2 acc = cmul(g.m[i * 4 + 0], x[0]);
            acc = cfma(g.m[i * 4 + 1], x[1], acc);
            acc = cfma(g.m[i * 4 + 2], x[2], acc);
            acc = cfma(g.m[i * 4 + 3], x[3], acc);
            r[idx[i]] = acc;
        }
    }
}

// Diagonal gates: one amplitude per item; the enumeration covers only the controlled
// subspace (and only target=1 when the |0> phase is 1).
__global__ void __launch_bounds__(kThreads) k_gate_diag(double2 *__restrict__ a, uint64_t total,
                                                        uint32_t n, uint32_t glog,
                                                        const __grid_constant__ DevGate g) {
    const uint64_t gmask = (uint64_t(1) << glog) - 1;
    for (uint64_t gid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; gid < total;
         gid += uint64_t(gridDim.x) * blockDim.x) {
        double2 *r = a + ((gid >> glog) << n);
        const uint64_t i = insert_zeros(gid & gmask, g.positions, g.npos) | g.cmask;
        uint32_t b = uint32_t((i >> g.t[0]) & 1);
        if (g.kind == KIND_DIAG2) b |= uint32_t((i >> g.t[1]) & 1) << 1;
        r[i] = cmul(g.m[b], r[i]);
    }
}

// Generic dense k-qubit gate (custom unitaries of arity > 2): one block per group at a time,
// the group staged in shared memory, one output row per thread.
__global__ void __launch_bounds__(kThreads) k_gate_dense(double2 *__restrict__ a, uint64_t groups,
                                                         uint32_t n, uint32_t glog,
                                                         const __grid_constant__ DevGate g) {
    extern __shared__ double2 s_in[];
    const uint32_t k = uint32_t(g.nt);
    const uint32_t dim = 1u << k;
    const uint64_t gmask = (uint64_t(1) << glog) - 1;
    for (uint64_t gid = blockIdx.x; gid < groups; gid += gridDim.x) {
        double2 *r = a + ((gid >> glog) << n);
        const uint64_t base = insert_zeros(gid & gmask, g.positions, g.npos);
        for (uint32_t j = threadIdx.x; j < dim; j += blockDim.x) {
            uint64_t off = 0;
            for (uint32_t b = 0; b < k; ++b)
                if ((j >> b) & 1) off |= uint64_t(1) << g.dense_targets[b];
            s_in[j] = r[base | off];
        }
        __syncthreads();
        for (uint32_t row = threadIdx.x; row < dim; row += blockDim.x) {
            double2 acc = make_double2(0.0, 0.0);
            const double2 *mr = g.dense + size_t(row) * dim;
            for (uint32_t c = 0; c < dim; ++c) acc = cfma(__ldg(&mr[c]), s_in[c], acc);
            uint64_t off = 0;
            for (uint32_t b = 0; b < k; ++b)
                if ((row >> b) & 1) off |= uint64_t(1) << g.dense_targets[b];
            r[base | off] = acc;
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------- out-of-place (derivatives)

// out <- M in where M acts on the targets when every control bit is set; elsewhere out is
// in (gate) or zero (derivative of a controlled gate). Groups enumerate targets only.
__global__ void __launch_bounds__(kThreads) k_gate_out(const double2 *__restrict__ in,
                                                       double2 *__restrict__ out, uint64_t total,
                                                       uint32_t n, uint32_t glog,
                                                       const __grid_constant__ DevGate g) {
    const uint64_t gmask = (uint64_t(1) << glog) - 1;
    const bool diag = g.kind == KIND_DIAG1 || g.kind == KIND_DIAG2;
    const int nt = g.nt;
    uint8_t tpos[2];
    tpos[0] = uint8_t(nt == 2 ? min(g.t[0], g.t[1]) : g.t[0]);
    tpos[1] = uint8_t(nt == 2 ? max(g.t[0], g.t[1]) : 0);
    const uint64_t b0 = uint64_t(1) << g.t[0];
    const uint64_t b1 = nt == 2 ? uint64_t(1) << g.t[1] : 0;
    for (uint64_t gid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; gid < total;
         gid += uint64_t(gridDim.x) * blockDim.x) {
        const size_t roff = size_t(gid >> glog) << n;
        const double2 *ri = in + roff;
        double2 *ro = out + roff;
        const uint64_t i0 = insert_zeros(gid & gmask, tpos, nt);
        const uint32_t cnt = 1u << nt;
        uint64_t idx[4] = {i0, i0 | b0, i0 | b1, i0 | b0 | b1};
        double2 x[4];
        for (uint32_t j = 0; j < cnt; ++j) x[j] = ri[idx[j]];
        for (uint32_t j = 0; j < cnt; ++j) {
            const uint64_t i = idx[j];
            double2 y;
            if ((i & g.cmask) != g.cmask) {
                y = g.zero_uncontrolled ? make_double2(0.0, 0.0) : x[j];
            } else if (diag) {
                y = cmul(g.m[j], x[j]);
            } else {
                y = make_double2(0.0, 0.0);
                for (uint32_t c = 0; c < cnt; ++c) y = cfma(g.m[j * cnt + c], x[c], y);
            }
            ro[i] = y;
        }
    }
}

// ---------------------------------------------------------------- adjoint step

struct AdjArgs {
    DevGate u;               // U^dagger, dense small form (KIND_1Q / KIND_2Q)
    int32_t ns;              // number of derivative slots (0..3)
    double2 d[3][16];        // dU/dp per slot, same targets as u
};

// One pass over the controlled subspace of psi and lambda:
//   psi <- U^dag psi;  acc_s += Re sum conj(lambda) (dU_s psi);  lambda <- U^dag lambda.
// Outside the controlled subspace U is the identity and dU is zero, so nothing is read.
template <int NT>
__global__ void __launch_bounds__(kThreads) k_adjoint(double2 *__restrict__ psi,
                                                      double2 *__restrict__ lam, uint64_t total,
                                                      uint32_t n, uint32_t glog,
                                                      const __grid_constant__ AdjArgs A,
                                                      double *__restrict__ partials,
                                                      uint32_t partial_stride) {
    constexpr int D = 1 << NT;
    __shared__ double s_red[kThreads / 32];
    const uint64_t gmask = (uint64_t(1) << glog) - 1;
    const uint64_t b0 = uint64_t(1) << A.u.t[0];
    const uint64_t b1 = NT == 2 ? uint64_t(1) << A.u.t[1] : 0;
    double acc[3] = {0.0, 0.0, 0.0};
    for (uint64_t gid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; gid < total;
         gid += uint64_t(gridDim.x) * blockDim.x) {
        const size_t roff = size_t(gid >> glog) << n;
        double2 *P = psi + roff;
        double2 *L = lam + roff;
        const uint64_t i0 = insert_zeros(gid & gmask, A.u.positions, A.u.npos) | A.u.cmask;
        uint64_t idx[D];
        idx[0] = i0;
        idx[1] = i0 | b0;
        if constexpr (NT == 2) {
            idx[2] = i0 | b1;
            idx[3] = i0 | b0 | b1;
        }
        double2 p[D], l[D], q[D];
#pragma unroll
        for (int j = 0; j < D; ++j) {
            p[j] = P[idx[j]];
            l[j] = L[idx[j]];
        }
#pragma unroll
        for (int i = 0; i < D; ++i) {
            double2 t = make_double2(0.0, 0.0);
#pragma unroll
            for (int c = 0; c < D; ++c) t = cfma(A.u.m[i * D + c], p[c], t);
            q[i] = t;
        }
#pragma unroll
        for (int s = 0; s < 3; ++s) {
            if (s < A.ns) {
                double v = 0.0;
#pragma unroll
                for (int i = 0; i < D; ++i) {
                    double2 t = make_double2(0.0, 0.0);
#pragma unroll
                    for (int c = 0; c < D; ++c) t = cfma(A.d[s][i * D + c], q[c], t);
                    v += re_conj_mul(l[i], t);
                }
                acc[s] += v;
            }
        }
#pragma unroll
        for (int i = 0; i < D; ++i) {
            double2 t = make_double2(0.0, 0.0);
#pragma unroll
            for (int c = 0; c < D; ++c) t = cfma(A.u.m[i * D + c], l[c], t);
            P[idx[i]] = q[i];
            L[idx[i]] = t;
        }
    }
    for (int s = 0; s < A.ns; ++s) {
        const double r = block_sum(acc[s], s_red);
        if (threadIdx.x == 0) partials[size_t(s) * partial_stride + blockIdx.x] = r;
    }
}

// ---------------------------------------------------------------- reductions, scaling

// sums[j] = sum over blocks of partials[j * nblocks + b], fixed order (deterministic).
__global__ void k_reduce_rows(const double *__restrict__ partials, uint32_t nblocks,
                              double *__restrict__ sums) {
    __shared__ double s_red[kThreads / 32];
    const double *p = partials + size_t(blockIdx.x) * nblocks;
    double v = 0.0;
    for (uint32_t b = threadIdx.x; b < nblocks; b += blockDim.x) v += p[b];
    const double r = block_sum(v, s_red);
    if (threadIdx.x == 0) sums[blockIdx.x] = r;
}

__global__ void k_scale_rows(double2 *__restrict__ a, uint64_t total, uint32_t n,
                             const double *__restrict__ scale) {
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += uint64_t(gridDim.x) * blockDim.x) {
        const double s = scale[i >> n];
        double2 v = a[i];
        a[i] = make_double2(v.x * s, v.y * s);
    }
}

__global__ void k_basis_state(double2 *__restrict__ a, uint64_t total, uint32_t n,
                              uint64_t index) {
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += uint64_t(gridDim.x) * blockDim.x) {
        const uint64_t local = i & ((uint64_t(1) << n) - 1);
        a[i] = make_double2(local == index ? 1.0 : 0.0, 0.0);
    }
}

// Row norms: partials[row * gridDim.x + block] = sum |a|^2 over the block's slice of the row.
__global__ void __launch_bounds__(kThreads) k_norms(const double2 *__restrict__ a, uint64_t dim,
                                                    double *__restrict__ partials) {
    __shared__ double s_red[kThreads / 32];
    const double2 *r = a + size_t(blockIdx.y) * dim;
    double v = 0.0;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < dim;
         i += uint64_t(gridDim.x) * blockDim.x) {
        const double2 x = r[i];
        v = fma(x.x, x.x, fma(x.y, x.y, v));
    }
    const double t = block_sum(v, s_red);
    if (threadIdx.x == 0) partials[size_t(blockIdx.y) * gridDim.x + blockIdx.x] = t;
}

// ---------------------------------------------------------------- Pauli observable

struct PauliArgs {
    // Observable tables, one contiguous block (copied to shared memory when table_bytes > 0),
    // offsets in bytes from its start. Weights fold the group's flip into the phase:
    // w'_k = coefficient * i^(y mod 4) * (-1)^popc(f & z_k), so term k contributes
    // w'_k (-1)^popc(t & z_k) psi[t ^ f] to (H psi)[t].
    //   groups with one term ("singles", ns of them): w' (double2), f (u64), z (u64) arrays;
    //   the other groups (nm of them, ntm terms): w' and z per term, f per group, and the first
    //   term of each group plus one final end index.
    const unsigned char *tables;
    uint32_t s_w, s_f, s_z, m_w, m_z, m_f, m_e;
    uint32_t ns, nm, table_bytes;
    // Traversal order (perm == nullptr: index order). The loop counter's low 6 bits are index
    // bits 0-5; its next (coset_bits - 6) bits are spread over the other qubits of the coset set
    // by tables 0..nb-1, the remaining bits over the complement by tables nb..ntables-1 (256
    // entries each, one per 8 counter bits).
    const uint64_t *perm;
    uint32_t coset_bits, nb, ntables;
};
constexpr uint32_t kMaxPermTables = 8;
constexpr uint32_t kPauliSmemTables = 30 * 1024;  // larger tables are read from global memory
constexpr int kPauliBatch = 4;

__device__ __forceinline__ double flip_sign(double x, uint32_t m) {
    return __hiloint2double(__double2hiint(x) ^ int(m), __double2loint(x));
}

// out[t] = sum_groups sum_terms w_k (-1)^popc((t^f) & z_k) psi[t^f]   (= (H psi)[t])
// partials[row, block] = sum_t Re(conj(psi[t]) out[t]).
//
// Every flip group reads psi once more (psi[t ^ f]); groups go in batches of kPauliBatch whose
// gathers are all issued before any is consumed. Single-term groups (most of a random Pauli sum)
// take a branch-free path: the term's sign is an XOR on the weight's sign bits. The amplitudes
// are visited coset by coset of a qubit set B chosen on the host (the qubits most flips act on,
// plus 0-5 for coalescing, 2^21 amplitudes = 32 MB per coset): a group whose flips all lie in B
// reads inside the coset being visited, which stays in L2.
template <bool SMEM>
__global__ void __launch_bounds__(kThreads) k_pauli(const double2 *__restrict__ psi,
                                                    double2 *__restrict__ out, uint64_t dim,
                                                    const __grid_constant__ PauliArgs P,
                                                    double *__restrict__ partials, int accumulate) {
    __shared__ double s_red[kThreads / 32];
    __shared__ uint64_t s_perm[kMaxPermTables * 256];
    extern __shared__ __align__(16) unsigned char s_tab[];
    if (P.perm)
        for (uint32_t i = threadIdx.x; i < P.ntables * 256; i += blockDim.x) s_perm[i] = P.perm[i];
    if (SMEM) {
        const uint4 *src = reinterpret_cast<const uint4 *>(P.tables);
        uint4 *dst = reinterpret_cast<uint4 *>(s_tab);
        for (uint32_t i = threadIdx.x; i < P.table_bytes / 16; i += blockDim.x) dst[i] = src[i];
    }
    __syncthreads();
    const unsigned char *tb = SMEM ? s_tab : P.tables;
    const double2 *sW = reinterpret_cast<const double2 *>(tb + P.s_w);
    const uint64_t *sF = reinterpret_cast<const uint64_t *>(tb + P.s_f);
    const uint64_t *sZ = reinterpret_cast<const uint64_t *>(tb + P.s_z);
    const double2 *mW = reinterpret_cast<const double2 *>(tb + P.m_w);
    const uint64_t *mZ = reinterpret_cast<const uint64_t *>(tb + P.m_z);
    const uint64_t *mF = reinterpret_cast<const uint64_t *>(tb + P.m_f);
    const uint32_t *mE = reinterpret_cast<const uint32_t *>(tb + P.m_e);
    const size_t roff = size_t(blockIdx.y) * dim;
    const double2 *r = psi + roff;
    double ev = 0.0;
    for (uint64_t c = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; c < dim;
         c += uint64_t(gridDim.x) * blockDim.x) {
        uint64_t t = c;
        if (P.perm) {
            t = c & 63u;
            for (uint32_t j = 0; j < P.nb; ++j) t |= s_perm[j * 256 + ((c >> (6 + 8 * j)) & 255u)];
            for (uint32_t j = P.nb; j < P.ntables; ++j)
                t |= s_perm[j * 256 + ((c >> (P.coset_bits + 8 * (j - P.nb))) & 255u)];
        }
        const double2 pt = r[t];
        double2 acc = make_double2(0.0, 0.0);
        uint32_t i = 0;
        for (; i + kPauliBatch <= P.ns; i += kPauliBatch) {
            double2 ps[kPauliBatch];
#pragma unroll
            for (int j = 0; j < kPauliBatch; ++j) ps[j] = r[t ^ sF[i + j]];
#pragma unroll
            for (int j = 0; j < kPauliBatch; ++j) {
                const uint32_t neg = uint32_t(__popcll(t & sZ[i + j]) & 1) << 31;
                const double2 w = sW[i + j];
                acc = cfma(make_double2(flip_sign(w.x, neg), flip_sign(w.y, neg)), ps[j], acc);
            }
        }
        for (; i < P.ns; ++i) {
            const uint32_t neg = uint32_t(__popcll(t & sZ[i]) & 1) << 31;
            const double2 w = sW[i];
            acc = cfma(make_double2(flip_sign(w.x, neg), flip_sign(w.y, neg)), r[t ^ sF[i]], acc);
        }
        for (uint32_t g = 0; g < P.nm; ++g) {
            const uint64_t f = mF[g];
            const double2 ps = f ? r[t ^ f] : pt;
            double2 w = make_double2(0.0, 0.0);
            for (uint32_t k = mE[g]; k < mE[g + 1]; ++k) {
                const uint32_t neg = uint32_t(__popcll(t & mZ[k]) & 1) << 31;
                const double2 wk = mW[k];
                w.x += flip_sign(wk.x, neg);
                w.y += flip_sign(wk.y, neg);
            }
            acc = cfma(w, ps, acc);
        }
        if (out) {
            if (accumulate) {
                const double2 o = out[roff + t];
                out[roff + t] = make_double2(o.x + acc.x, o.y + acc.y);
            } else {
                out[roff + t] = acc;
            }
        }
        ev += re_conj_mul(pt, acc);
    }
    const double tsum = block_sum(ev, s_red);
    if (threadIdx.x == 0) partials[size_t(blockIdx.y) * gridDim.x + blockIdx.x] = tsum;
}

// ---------------------------------------------------------------- launch helpers

int g_num_sms = 0;

int num_sms() {
    if (g_num_sms == 0) {
        int dev = 0;
        check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
        check_cuda(cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev),
                   "cudaDeviceGetAttribute");
    }
    return g_num_sms;
}

// Blocks for a grid-stride loop over `items`: at most 8 resident 256-thread blocks per SM.
unsigned grid_for(uint64_t items) {
    const uint64_t need = (items + kThreads - 1) / kThreads;
    const uint64_t cap = uint64_t(num_sms()) * 8;
    return unsigned(need < 1 ? 1 : (need < cap ? need : cap));
}


}  // namespace

void launch_gate(double2 *amps, size_t batch, uint32_t n, const DevGate &g, cudaStream_t s) {
    if (g.kind == KIND_NONE) return;
    if (uint32_t(g.npos) > n) fail("internal: gate wider than the state");
    const uint32_t glog = n - uint32_t(g.npos);
    const uint64_t total = uint64_t(batch) << glog;
    // algorithmic traffic: every touched amplitude is read and written once (16 + 16 bytes)
    const int per_group = (g.kind == KIND_DIAG1 || g.kind == KIND_DIAG2) ? 1 : (1 << g.nt);
    const ProfToken tok = prof_begin(PROF_GATE, s);
    switch (g.kind) {
    case KIND_1Q: k_gate_1q<<<grid_for(total), kThreads, 0, s>>>(amps, total, n, glog, g); break;
    case KIND_2Q: k_gate_2q<<<grid_for(total), kThreads, 0, s>>>(amps, total, n, glog, g); break;
    case KIND_DIAG1:
    case KIND_DIAG2:
        k_gate_diag<<<grid_for(total), kThreads, 0, s>>>(amps, total, n, glog, g);
        break;
    case KIND_DENSE: {
        const size_t smem = sizeof(double2) << g.nt;
        const unsigned blocks = unsigned(total < uint64_t(num_sms()) * 8 ? total : uint64_t(num_sms()) * 8);
        if (smem > 48 * 1024)
            check_cuda(cudaFuncSetAttribute(k_gate_dense, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            int(smem)), "cudaFuncSetAttribute");
        k_gate_dense<<<blocks, kThreads, smem, s>>>(amps, total, n, glog, g);
        break;
    }
    default: fail("internal: bad gate kind");
    }
    prof_end(tok, s, 32.0 * double(total) * per_group);
    check_cuda(cudaGetLastError(), "gate kernel launch");
}

void launch_gate_out(const double2 *in, double2 *out, size_t batch, uint32_t n,
                     const DevGate &g, cudaStream_t s) {
    if (g.kind == KIND_DENSE || g.kind == KIND_NONE) fail("internal: unsupported out-of-place gate");
    if (uint32_t(g.nt) > n) fail("internal: gate wider than the state");
    const uint32_t glog = n - uint32_t(g.nt);
    const uint64_t total = uint64_t(batch) << glog;
    const ProfToken tok = prof_begin(PROF_GATE, s);
    k_gate_out<<<grid_for(total), kThreads, 0, s>>>(in, out, total, n, glog, g);
    prof_end(tok, s, 32.0 * double(uint64_t(batch) << n));
    check_cuda(cudaGetLastError(), "derivative kernel launch");
}

// Returns the number of blocks; partials receives [slot][block] with a row stride of
// adjoint_max_blocks() (the reduction reads whole rows; unused tail entries stay zero).
unsigned launch_adjoint_raw(double2 *psi, double2 *lam, size_t batch, uint32_t n,
                            const DevGate &uadj, const double2 (*d)[16], int ns,
                            double *partials, cudaStream_t s) {
    const uint32_t stride = uint32_t(num_sms()) * 8;
    AdjArgs A;
    std::memset(&A, 0, sizeof(A));
    A.u = uadj;
    A.ns = ns;
    const int dim = uadj.nt == 2 ? 16 : 4;
    for (int j = 0; j < ns; ++j)
        for (int i = 0; i < dim; ++i) A.d[j][i] = d[j][i];
    const uint32_t glog = n - uint32_t(uadj.npos);
    const uint64_t total = uint64_t(batch) << glog;
    const unsigned blocks = grid_for(total);
    if (uadj.kind != KIND_1Q && uadj.kind != KIND_2Q)
        fail("internal: adjoint step needs a dense small form");
    const ProfToken tok = prof_begin(PROF_ADJ_STEP, s);
    if (uadj.kind == KIND_1Q)
        k_adjoint<1><<<blocks, kThreads, 0, s>>>(psi, lam, total, n, glog, A, partials, stride);
    else
        k_adjoint<2><<<blocks, kThreads, 0, s>>>(psi, lam, total, n, glog, A, partials, stride);
    prof_end(tok, s, 64.0 * double(total) * (1 << uadj.nt));
    check_cuda(cudaGetLastError(), "adjoint kernel launch");
    return blocks;
}

unsigned adjoint_max_blocks() { return unsigned(num_sms()) * 8; }

void launch_reduce_rows(const double *partials, uint32_t rows, uint32_t nblocks, double *sums,
                        cudaStream_t s) {
    if (rows == 0) return;
    prof_count_launch();
    k_reduce_rows<<<rows, kThreads, 0, s>>>(partials, nblocks, sums);
    check_cuda(cudaGetLastError(), "reduce kernel launch");
}

void launch_scale(double2 *amps, size_t batch, uint32_t n, const double *row_scale_dev,
                  cudaStream_t s) {
    const uint64_t total = uint64_t(batch) << n;
    const ProfToken tok = prof_begin(PROF_OTHER, s);
    k_scale_rows<<<grid_for(total), kThreads, 0, s>>>(amps, total, n, row_scale_dev);
    prof_end(tok, s, 32.0 * double(total));
    check_cuda(cudaGetLastError(), "scale kernel launch");
}

void launch_basis_state(double2 *amps, size_t batch, uint32_t n, uint64_t index, cudaStream_t s) {
    const uint64_t total = uint64_t(batch) << n;
    const ProfToken tok = prof_begin(PROF_OTHER, s);
    k_basis_state<<<grid_for(total), kThreads, 0, s>>>(amps, total, n, index);
    prof_end(tok, s, 16.0 * double(total));
    check_cuda(cudaGetLastError(), "basis-state kernel launch");
}

// Per-row partial sums: grid (bx, batch). Returns bx.
unsigned launch_norms(const double2 *amps, size_t batch, uint32_t n, double *partials,
                      cudaStream_t s) {
    const uint64_t dim = uint64_t(1) << n;
    unsigned bx = grid_for(dim);
    const unsigned cap = unsigned((uint64_t(num_sms()) * 8 + batch - 1) / batch);
    if (bx > cap) bx = cap < 1 ? 1 : cap;
    const ProfToken tok = prof_begin(PROF_OTHER, s);
    k_norms<<<dim3(bx, unsigned(batch)), kThreads, 0, s>>>(amps, dim, partials);
    prof_end(tok, s, 16.0 * double(dim) * double(batch));
    check_cuda(cudaGetLastError(), "norm kernel launch");
    return bx;
}

unsigned launch_pauli(const double2 *psi, double2 *out, size_t batch, uint32_t n,
                      const PauliTables &tab, const PauliTraversal &tr, double *partials,
                      bool accumulate, cudaStream_t s) {
    if (tr.tables && (tr.ntables > kMaxPermTables || tr.coset_bits < 6 || tr.coset_bits > n))
        fail("internal: observable traversal tables out of range");
    const bool smem = tab.bytes <= kPauliSmemTables;
    PauliArgs P{};
    P.tables = tab.base;
    P.s_w = tab.s_w;
    P.s_f = tab.s_f;
    P.s_z = tab.s_z;
    P.m_w = tab.m_w;
    P.m_z = tab.m_z;
    P.m_f = tab.m_f;
    P.m_e = tab.m_e;
    P.ns = tab.ns;
    P.nm = tab.nm;
    P.table_bytes = smem ? uint32_t(tab.bytes) : 0u;
    P.perm = tr.tables;
    P.coset_bits = tr.coset_bits;
    P.nb = tr.nb;
    P.ntables = tr.ntables;
    const uint64_t dim = uint64_t(1) << n;
    unsigned bx = grid_for(dim);
    const unsigned cap = unsigned((uint64_t(num_sms()) * 8 + batch - 1) / batch);
    if (bx > cap) bx = cap < 1 ? 1 : cap;
    // algorithmic traffic: read psi once, write H psi once (when requested)
    const ProfToken tok = prof_begin(PROF_PAULI, s);
    if (smem)
        k_pauli<true><<<dim3(bx, unsigned(batch)), kThreads, P.table_bytes, s>>>(
            psi, out, dim, P, partials, accumulate ? 1 : 0);
    else
        k_pauli<false><<<dim3(bx, unsigned(batch)), kThreads, 0, s>>>(psi, out, dim, P, partials,
                                                                     accumulate ? 1 : 0);
    prof_end(tok, s, (out ? (accumulate ? 48.0 : 32.0) : 16.0) * double(dim) * double(batch));
    check_cuda(cudaGetLastError(), "observable kernel launch");
    return bx;
}

}  // namespace arcqml
