// analysis.cu — analysis of device states (crates/arcqml-analysis/src/statevector): basis
// probabilities, marginal probabilities of a qubit selection, Bloch vectors, <lhs|rhs>, and the
// adjoint cotangents of those outputs (lambda for the reverse sweep).
//
// All of it is HBM-bound elementwise work or reductions. Reductions are deterministic: every
// block sums its part in a fixed order (warp shuffles, then the warps in order) into its own
// partial, and k_reduce_rows adds the partials of a row in block order.
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "analysis.h"
#include "launch.h"
#include "profile.h"
#include "rt_internal.h"

namespace arcqml {
namespace {

constexpr int kAT = 256;

__device__ __forceinline__ double a_block_sum(double v, double *smem) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) smem[warp] = v;
    __syncthreads();
    double r = 0.0;
    if (threadIdx.x == 0)
        for (int w = 0; w < int(blockDim.x >> 5); ++w) r += smem[w];
    return r;  // valid in thread 0
}

// bin of basis index i: the selected bits in display order (disp[0] the most significant);
// every qubit selected in descending order is the identity
__device__ __forceinline__ uint64_t sel_bin(uint64_t i, const Selection &S) {
    if (S.identity) return i;
    uint64_t m = 0;
    for (uint32_t j = 0; j < S.k; ++j) m = (m << 1) | ((i >> S.disp[j]) & 1u);
    return m;
}

// basis index of the o-th member of bin m: o fills the unselected bits in order, m the selected
__device__ __forceinline__ uint64_t sel_index(uint64_t m, uint64_t o, const Selection &S) {
    uint64_t g = o;
    for (uint32_t j = 0; j < S.k; ++j) {
        const uint32_t p = S.asc[j];
        g = ((g >> p) << (p + 1)) | (g & ((uint64_t(1) << p) - 1));
    }
    for (uint32_t j = 0; j < S.k; ++j) g |= ((m >> (S.k - 1 - j)) & 1u) << S.disp[j];
    return g;
}

__device__ __forceinline__ double prob(double2 x) { return fma(x.x, x.x, x.y * x.y); }

__global__ void __launch_bounds__(kAT)
    k_probabilities(const double2 *__restrict__ a, uint64_t total, double *__restrict__ out) {
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride)
        out[i] = prob(a[i]);
}

// Bins with few members: one thread per bin sums its members in order.
__global__ void __launch_bounds__(kAT)
    k_marginal_per_bin(const double2 *__restrict__ a, const __grid_constant__ Selection S,
                       uint64_t bins, uint64_t per_bin, double *__restrict__ out) {
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t m = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; m < bins; m += stride) {
        double v = 0.0;
        for (uint64_t o = 0; o < per_bin; ++o) v += prob(a[sel_index(m, o, S)]);
        out[m] = v;
    }
}

// Bins with many members: block (b, y) sums its chunk of bin bin0 + y into
// partials[y * gridDim.x + b].
__global__ void __launch_bounds__(kAT)
    k_marginal_chunks(const double2 *__restrict__ a, const __grid_constant__ Selection S,
                      uint64_t bin0, uint64_t per_bin, double *__restrict__ partials) {
    __shared__ double red[kAT / 32];
    const uint64_t m = bin0 + blockIdx.y;
    const uint64_t chunk = (per_bin + gridDim.x - 1) / gridDim.x;
    const uint64_t o0 = uint64_t(blockIdx.x) * chunk;
    const uint64_t o1 = o0 + chunk < per_bin ? o0 + chunk : per_bin;
    double v = 0.0;
    for (uint64_t o = o0 + threadIdx.x; o < o1; o += blockDim.x) v += prob(a[sel_index(m, o, S)]);
    const double r = a_block_sum(v, red);
    if (threadIdx.x == 0) partials[uint64_t(blockIdx.y) * gridDim.x + blockIdx.x] = r;
}

// (<X_q>, <Y_q>, <Z_q>) of row blockIdx.y: partials[(row * 3 + c) * gridDim.x + b].
__global__ void __launch_bounds__(kAT)
    k_bloch(const double2 *__restrict__ a, uint32_t n, uint32_t q, double *__restrict__ partials) {
    __shared__ double red[kAT / 32];
    const double2 *r = a + (uint64_t(blockIdx.y) << n);
    const uint64_t pairs = uint64_t(1) << (n - 1), mask = uint64_t(1) << q;
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    double x = 0.0, y = 0.0, z = 0.0;
    for (uint64_t g = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < pairs; g += stride) {
        const uint64_t i0 = ((g >> q) << (q + 1)) | (g & (mask - 1));
        const double2 a0 = r[i0], a1 = r[i0 | mask];
        x += 2.0 * fma(a0.x, a1.x, a0.y * a1.y);
        y += 2.0 * fma(a0.x, a1.y, -a0.y * a1.x);
        z += prob(a0) - prob(a1);
    }
    const double v[3] = {x, y, z};
    for (int c = 0; c < 3; ++c) {
        const double s = a_block_sum(v[c], red);
        if (threadIdx.x == 0) partials[(uint64_t(blockIdx.y) * 3 + c) * gridDim.x + blockIdx.x] = s;
    }
}

// <lhs|rhs> of row blockIdx.y: partials[(row * 2 + c) * gridDim.x + b], c = 0 real, 1 imaginary.
__global__ void __launch_bounds__(kAT)
    k_overlap(const double2 *__restrict__ l, const double2 *__restrict__ r, uint32_t n,
              double *__restrict__ partials) {
    __shared__ double red[kAT / 32];
    const uint64_t dim = uint64_t(1) << n, off = uint64_t(blockIdx.y) << n;
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    double re = 0.0, im = 0.0;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < dim; i += stride) {
        const double2 x = l[off + i], w = r[off + i];
        re += fma(x.x, w.x, x.y * w.y);
        im += fma(x.x, w.y, -x.y * w.x);
    }
    const double v[2] = {re, im};
    for (int c = 0; c < 2; ++c) {
        const double s = a_block_sum(v[c], red);
        if (threadIdx.x == 0) partials[(uint64_t(blockIdx.y) * 2 + c) * gridDim.x + blockIdx.x] = s;
    }
}

// lam_i = g[row * bins + bin(i)] psi_i (the cotangent of sum_m g[m] P(m)).
__global__ void __launch_bounds__(kAT)
    k_probability_cotangent(const double2 *__restrict__ psi, uint64_t total, uint32_t n,
                            const __grid_constant__ Selection S, const double *__restrict__ g,
                            double2 *__restrict__ lam) {
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    const uint64_t mask = (uint64_t(1) << n) - 1, bins = uint64_t(1) << S.k;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const double w = g[(i >> n) * bins + sel_bin(i & mask, S)];
        const double2 x = psi[i];
        lam[i] = make_double2(w * x.x, w * x.y);
    }
}

// out_i = alpha[row] x_i (complex alpha per row).
__global__ void __launch_bounds__(kAT)
    k_scaled_copy(const double2 *__restrict__ x, uint64_t total, uint32_t n,
                  const double2 *__restrict__ alpha, double2 *__restrict__ out) {
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const double2 s = alpha[i >> n], v = x[i];
        out[i] = make_double2(fma(s.x, v.x, -s.y * v.y), fma(s.x, v.y, s.y * v.x));
    }
}

unsigned blocks_for(uint64_t items) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint64_t need = (items + kAT - 1) / kAT, cap = uint64_t(sms) * 8;
    return unsigned(std::max<uint64_t>(1, std::min(need, cap)));
}

void after_launch(const char *what) { check_cuda(cudaGetLastError(), what); }

// One row of sums per (row, component) from `rows` x `nblocks` partials, read back to host.
void reduce_to_host(const double *partials, uint32_t rows, uint32_t nblocks, double *host,
                    ThreadContext &ctx, cudaStream_t s) {
    double *sums = ctx_dgrads(ctx, rows);
    launch_reduce_rows(partials, rows, nblocks, sums, s);
    double *h = ctx_hvals(ctx, rows);
    check_cuda(cudaMemcpyAsync(h, sums, rows * sizeof(double), cudaMemcpyDeviceToHost, s),
               "cudaMemcpyAsync (analysis sums)");
    check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    std::copy(h, h + rows, host);
}

}  // namespace

Selection make_selection(uint32_t n, const std::vector<uint32_t> &qubits) {
    Selection S{};
    S.k = uint32_t(qubits.size());
    std::vector<uint32_t> d(qubits);
    std::sort(d.begin(), d.end(), [](uint32_t a, uint32_t b) { return a > b; });
    for (uint32_t j = 0; j < S.k; ++j) {
        S.disp[j] = uint8_t(d[j]);
        S.asc[j] = uint8_t(d[S.k - 1 - j]);
    }
    S.identity = S.k == n ? 1 : 0;  // all n distinct qubits, descending: the bin is the index
    return S;
}

void probabilities_device(const double2 *a, size_t batch, uint32_t n, double *out,
                          cudaStream_t s) {
    const uint64_t total = uint64_t(batch) << n;
    const ProfToken tok = prof_begin(PROF_OTHER, s);
    k_probabilities<<<blocks_for(total), kAT, 0, s>>>(a, total, out);
    prof_end(tok, s, 24.0 * double(total));
    after_launch("probabilities kernel launch");
}

void marginal_device(const double2 *a, size_t batch, uint32_t n, const Selection &S,
                     double *out, ThreadContext &ctx, cudaStream_t s) {
    const uint64_t bins = uint64_t(1) << S.k, per_bin = uint64_t(1) << (n - S.k);
    for (size_t row = 0; row < batch; ++row) {
        const double2 *r = a + (uint64_t(row) << n);
        double *o = out + row * bins;
        if (per_bin <= 256) {
            const ProfToken tok = prof_begin(PROF_OTHER, s);
            k_marginal_per_bin<<<blocks_for(bins), kAT, 0, s>>>(r, S, bins, per_bin, o);
            prof_end(tok, s, 16.0 * double(uint64_t(1) << n) + 8.0 * double(bins));
            after_launch("marginal kernel launch");
            continue;
        }
        // blocks per bin: about 8 resident blocks per SM in total, at least 4 members a thread
        const uint64_t target = blocks_for(uint64_t(1) << 62) / std::max<uint64_t>(1, bins);
        const uint64_t most = std::max<uint64_t>(1, per_bin / (4 * kAT));
        const unsigned bpb = unsigned(std::max<uint64_t>(1, std::min(target, most)));
        for (uint64_t b0 = 0; b0 < bins; b0 += 32768) {
            const uint32_t nb = uint32_t(std::min<uint64_t>(32768, bins - b0));
            double *partials = ctx_partials(ctx, size_t(nb) * bpb);
            const ProfToken tok = prof_begin(PROF_OTHER, s);
            k_marginal_chunks<<<dim3(bpb, nb), kAT, 0, s>>>(r, S, b0, per_bin, partials);
            prof_end(tok, s, 16.0 * double(per_bin) * double(nb));
            after_launch("marginal kernel launch");
            launch_reduce_rows(partials, nb, bpb, o + b0, s);
        }
    }
}

void bloch_device(const double2 *a, size_t batch, uint32_t n, uint32_t q, double *xyz,
                  ThreadContext &ctx, cudaStream_t s) {
    for (size_t r0 = 0; r0 < batch; r0 += 16384) {
        const uint32_t rows = uint32_t(std::min<size_t>(16384, batch - r0));
        const unsigned bx = std::max(1u, blocks_for(uint64_t(1) << (n - 1)) / rows);
        double *partials = ctx_partials(ctx, size_t(rows) * 3 * bx);
        const ProfToken tok = prof_begin(PROF_OTHER, s);
        k_bloch<<<dim3(bx, rows), kAT, 0, s>>>(a + (uint64_t(r0) << n), n, q, partials);
        prof_end(tok, s, 16.0 * double(uint64_t(rows) << n));
        after_launch("Bloch vector kernel launch");
        reduce_to_host(partials, rows * 3, bx, xyz + 3 * r0, ctx, s);
    }
}

void overlap_device(const double2 *l, const double2 *r, size_t batch, uint32_t n, double *out,
                    ThreadContext &ctx, cudaStream_t s) {
    for (size_t r0 = 0; r0 < batch; r0 += 16384) {
        const uint32_t rows = uint32_t(std::min<size_t>(16384, batch - r0));
        const unsigned bx = std::max(1u, blocks_for(uint64_t(1) << n) / rows);
        double *partials = ctx_partials(ctx, size_t(rows) * 2 * bx);
        const ProfToken tok = prof_begin(PROF_OTHER, s);
        k_overlap<<<dim3(bx, rows), kAT, 0, s>>>(l + (uint64_t(r0) << n), r + (uint64_t(r0) << n),
                                                  n, partials);
        prof_end(tok, s, 32.0 * double(uint64_t(rows) << n));
        after_launch("overlap kernel launch");
        reduce_to_host(partials, rows * 2, bx, out + 2 * r0, ctx, s);
    }
}

void probability_cotangent_device(const double2 *psi, size_t batch, uint32_t n,
                                  const Selection &S, const double *g, double2 *lam,
                                  cudaStream_t s) {
    const uint64_t total = uint64_t(batch) << n;
    const ProfToken tok = prof_begin(PROF_OTHER, s);
    k_probability_cotangent<<<blocks_for(total), kAT, 0, s>>>(psi, total, n, S, g, lam);
    prof_end(tok, s, 40.0 * double(total));
    after_launch("cotangent kernel launch");
}

void scaled_copy_device(const double2 *x, size_t batch, uint32_t n, const double *alpha_host,
                        double2 *out, ThreadContext &ctx, cudaStream_t s) {
    std::vector<double2> al(batch);
    for (size_t r = 0; r < batch; ++r) al[r] = make_double2(alpha_host[2 * r], alpha_host[2 * r + 1]);
    std::vector<const std::vector<double2> *> refs{&al};
    auto p = upload_tables(refs, ctx, s);
    const uint64_t total = uint64_t(batch) << n;
    const ProfToken tok = prof_begin(PROF_OTHER, s);
    k_scaled_copy<<<blocks_for(total), kAT, 0, s>>>(x, total, n, p[0], out);
    prof_end(tok, s, 32.0 * double(total));
    after_launch("scaled copy kernel launch");
}

}  // namespace arcqml
