// sample.cu — bit-exact shot sampling from a device state (the reference's sample_counts,
// crates/arcqml-sim/src/statevector/api/measurement.rs:18-60).
//
// The reference forms p_i = re^2 + im^2 without fused multiply-add, a sequential f64 running
// sum, and per shot target = u * total with u the next f64 of StdRng::seed_from_u64(seed); the
// shot lands on the first index whose running sum exceeds target. Reproducing its counts bit for
// bit needs the running sum in exactly that order, so k_running_sum keeps one dependency chain
// (one thread adds; the other warps of the block stream amplitudes in and running sums out,
// three chunks in flight). Shots are independent: StdRng is ChaCha12 with a 64-bit block
// counter, so shot s reads keystream words 2s and 2s+1 of block s / 8 directly, and every thread
// generates one block and bisects the running sums for its 8 shots.
#include <cuda_runtime.h>

#include "launch.h"
#include "profile.h"
#include "rt_internal.h"

namespace arcqml {
namespace {

constexpr int kSumThreads = 256;
constexpr int kSumChunk = 2048;  // amplitudes per chunk; three chunks of running sums in smem

__global__ void __launch_bounds__(kSumThreads)
    k_running_sum(const double2 *__restrict__ amps, uint64_t dim, double *__restrict__ cum) {
    __shared__ double buf[3][kSumChunk];
    const uint64_t nchunks = (dim + kSumChunk - 1) / kSumChunk;
    const int warp = threadIdx.x >> 5;
    const int io_tid = threadIdx.x - 32;  // warps 1.. move data
    const int io_threads = kSumThreads - 32;
    auto load = [&](uint64_t c) {
        const uint64_t base = c * kSumChunk;
        const uint64_t len = dim - base < uint64_t(kSumChunk) ? dim - base : uint64_t(kSumChunk);
        double *b = buf[c % 3];
        for (uint64_t j = io_tid; j < len; j += io_threads) {
            const double2 a = amps[base + j];
            b[j] = __dadd_rn(__dmul_rn(a.x, a.x), __dmul_rn(a.y, a.y));
        }
    };
    auto store = [&](uint64_t c) {
        const uint64_t base = c * kSumChunk;
        const uint64_t len = dim - base < uint64_t(kSumChunk) ? dim - base : uint64_t(kSumChunk);
        const double *b = buf[c % 3];
        for (uint64_t j = io_tid; j < len; j += io_threads) cum[base + j] = b[j];
    };
    if (warp > 0) load(0);
    __syncthreads();
    double run = 0.0;
    for (uint64_t c = 0; c < nchunks; ++c) {
        if (warp == 0) {
            if (threadIdx.x == 0) {
                const uint64_t base = c * kSumChunk;
                const int len = int(dim - base < uint64_t(kSumChunk) ? dim - base : kSumChunk);
                double *b = buf[c % 3];
#pragma unroll 16
                for (int j = 0; j < len; ++j) {
                    run = __dadd_rn(run, b[j]);
                    b[j] = run;
                }
            }
        } else {
            if (c >= 1) store(c - 1);
            if (c + 1 < nchunks) load(c + 1);
        }
        __syncthreads();
    }
    if (warp > 0 && nchunks >= 1) store(nchunks - 1);
}

__device__ __forceinline__ uint32_t rotl(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

#define ARCQML_QR(a, b, c, d)                                \
    a += b; d ^= a; d = rotl(d, 16);                         \
    c += d; b ^= c; b = rotl(b, 12);                         \
    a += b; d ^= a; d = rotl(d, 8);                          \
    c += d; b ^= c; b = rotl(b, 7);

struct SampleKey {
    uint32_t k[8];
};

__global__ void __launch_bounds__(256)
    k_sample(const double *__restrict__ cum, uint64_t dim, uint64_t shots,
             const __grid_constant__ SampleKey key, uint64_t *__restrict__ out) {
    const uint64_t blk = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (blk * 8 >= shots) return;
    uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                      key.k[0], key.k[1], key.k[2], key.k[3],
                      key.k[4], key.k[5], key.k[6], key.k[7],
                      uint32_t(blk), uint32_t(blk >> 32), 0u, 0u};
    uint32_t x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = s[i];
#pragma unroll
    for (int r = 0; r < 6; ++r) {  // 12 rounds
        ARCQML_QR(x[0], x[4], x[8], x[12]);
        ARCQML_QR(x[1], x[5], x[9], x[13]);
        ARCQML_QR(x[2], x[6], x[10], x[14]);
        ARCQML_QR(x[3], x[7], x[11], x[15]);
        ARCQML_QR(x[0], x[5], x[10], x[15]);
        ARCQML_QR(x[1], x[6], x[11], x[12]);
        ARCQML_QR(x[2], x[7], x[8], x[13]);
        ARCQML_QR(x[3], x[4], x[9], x[14]);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] += s[i];
    const double total = cum[dim - 1];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
        const uint64_t shot = blk * 8 + p;
        if (shot >= shots) break;
        const uint64_t r = uint64_t(x[2 * p]) | (uint64_t(x[2 * p + 1]) << 32);
        // (r >> 11) * 2^-53 is exact; one rounded product with the total
        const double target = __dmul_rn(double(r >> 11) * 0x1.0p-53, total);
        uint64_t lo = 0, hi = dim;
        while (lo < hi) {
            const uint64_t mid = lo + (hi - lo) / 2;
            if (target < cum[mid]) hi = mid;
            else lo = mid + 1;
        }
        out[shot] = lo < dim ? lo : dim - 1;
    }
}

#undef ARCQML_QR

}  // namespace

// StdRng::seed_from_u64 key expansion (PCG32 XSH-RR outputs, rand_core's published rule).
static void stdrng_key(uint64_t seed, uint32_t key[8]) {
    uint64_t st = seed;
    for (int i = 0; i < 8; ++i) {
        st = st * 6364136223846793005ull + 11634580027462260723ull;
        const uint32_t xs = uint32_t(((st >> 18) ^ st) >> 27);
        const uint32_t rot = uint32_t(st >> 59);
        key[i] = (xs >> rot) | (xs << ((32 - rot) & 31));
    }
}

void launch_sample(const double2 *amps, uint32_t n, uint64_t shots, uint64_t seed, double *cum,
                   uint64_t *out, cudaStream_t s) {
    const uint64_t dim = uint64_t(1) << n;
    ProfToken tok = prof_begin(PROF_OTHER, s);
    k_running_sum<<<1, kSumThreads, 0, s>>>(amps, dim, cum);
    prof_end(tok, s, 24.0 * double(dim));
    check_cuda(cudaGetLastError(), "running-sum kernel launch");
    SampleKey key;
    stdrng_key(seed, key.k);
    const uint64_t blocks = (shots + 7) / 8;
    const unsigned grid = unsigned((blocks + 255) / 256);
    tok = prof_begin(PROF_OTHER, s);
    k_sample<<<grid, 256, 0, s>>>(cum, dim, shots, key, out);
    prof_end(tok, s, 8.0 * double(shots));
    check_cuda(cudaGetLastError(), "sample kernel launch");
}

}  // namespace arcqml
