// shard.cu — bit-slice packing for states sharded over ranks on their highest ("global") qubits.
//
// A global-qubit swap exchanges k global qubits with k local qubits. Rank r keeps the part of its
// shard whose local slice bits equal r's own global bits and sends the slice with value y to the
// rank whose global bits are y; that rank's slice with r's value lands in the same slots. The
// kernels here move slices between the shard and contiguous staging blocks (one per peer), in
// chunks of the remaining ("other") index bits, so the exchange itself is plain contiguous
// point-to-point traffic and the unpack writes back exactly the slots the pack emptied.
#include <cuda_runtime.h>

#include <algorithm>
#include "launch.h"
#include "profile.h"
#include "rt_internal.h"

namespace arcqml {
namespace {

constexpr int kSliceThreads = 256;

struct SliceArgs {
    uint32_t k;
    uint32_t sorted[kMaxSliceBits];  // slice positions, ascending (zero insertion order)
    uint64_t ybit[kMaxSliceBits];    // index bit set by bit i of the slice value
};

__device__ __forceinline__ uint64_t slice_index(uint64_t o, uint64_t y, const SliceArgs &A) {
    for (uint32_t i = 0; i < A.k; ++i) {
        const uint32_t p = A.sorted[i];
        o = ((o >> p) << (p + 1)) | (o & ((uint64_t(1) << p) - 1));
    }
    for (uint32_t i = 0; i < A.k; ++i)
        if ((y >> i) & 1) o |= A.ybit[i];
    return o;
}

// grid.y = staging block, grid.x strides over the chunk.
template <bool UNPACK>
__global__ void __launch_bounds__(kSliceThreads)
    k_shard_slices(double2 *__restrict__ amps, double2 *__restrict__ staging, uint64_t chunk_begin,
                   uint64_t chunk_len, uint64_t skip, const __grid_constant__ SliceArgs A) {
    const uint64_t blk = blockIdx.y;
    const uint64_t y = blk + (blk >= skip ? 1 : 0);
    double2 *st = staging + blk * chunk_len;
    for (uint64_t j = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < chunk_len;
         j += uint64_t(gridDim.x) * blockDim.x) {
        const uint64_t g = slice_index(chunk_begin + j, y, A);
        if (UNPACK) amps[g] = st[j];
        else st[j] = amps[g];
    }
}

// grid.y = slice value y; sources[y] (nullptr: skip) holds the chunk's amplitudes of value y,
// possibly in another GPU's memory (a peer mapping): plain loads over NVLink, local stores.
struct SliceSources {
    const double2 *src[1u << kMaxSliceBits];
};

__global__ void __launch_bounds__(kSliceThreads)
    k_shard_slices_from(double2 *__restrict__ amps, uint64_t chunk_begin, uint64_t chunk_len,
                        const __grid_constant__ SliceArgs A,
                        const __grid_constant__ SliceSources S) {
    const uint64_t y = blockIdx.y;
    const double2 *src = S.src[y];
    if (!src) return;
    for (uint64_t j = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < chunk_len;
         j += uint64_t(gridDim.x) * blockDim.x)
        amps[slice_index(chunk_begin + j, y, A)] = src[j];
}

int g_sms = 0;

}  // namespace

void launch_slices_from(double2 *amps, const uint32_t *positions, uint32_t k,
                        uint64_t chunk_begin, uint64_t chunk_len, const double2 *const *sources,
                        cudaStream_t s) {
    SliceArgs A{};
    A.k = k;
    for (uint32_t i = 0; i < k; ++i) {
        A.sorted[i] = positions[i];
        A.ybit[i] = uint64_t(1) << positions[i];
    }
    std::sort(A.sorted, A.sorted + k);
    SliceSources S{};
    uint32_t active = 0;
    for (uint32_t y = 0; y < (1u << k); ++y) {
        S.src[y] = reinterpret_cast<const double2 *>(sources[y]);
        active += sources[y] ? 1u : 0u;
    }
    if (!active || !chunk_len) return;
    if (g_sms == 0) {
        int dev = 0;
        check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
        check_cuda(cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev),
                   "cudaDeviceGetAttribute");
    }
    const uint64_t want = (uint64_t(g_sms) * 8 + active - 1) / active;
    const uint64_t need = (chunk_len + kSliceThreads - 1) / kSliceThreads;
    const unsigned bx = unsigned(std::max<uint64_t>(1, std::min(want, need)));
    const ProfToken tok = prof_begin(PROF_SHARD, s);
    k_shard_slices_from<<<dim3(bx, 1u << k), kSliceThreads, 0, s>>>(amps, chunk_begin, chunk_len,
                                                                      A, S);
    prof_end(tok, s, 32.0 * double(chunk_len) * double(active));
    check_cuda(cudaGetLastError(), "shard slice gather kernel launch");
}

void launch_slices(double2 *amps, uint32_t n_local, const uint32_t *positions, uint32_t k,
                   uint64_t chunk_begin, uint64_t chunk_len, uint64_t skip, double2 *staging,
                   bool unpack, cudaStream_t s) {
    SliceArgs A{};
    A.k = k;
    for (uint32_t i = 0; i < k; ++i) {
        A.sorted[i] = positions[i];
        A.ybit[i] = uint64_t(1) << positions[i];
    }
    std::sort(A.sorted, A.sorted + k);
    const uint64_t values = uint64_t(1) << k;
    const uint64_t nblocks = values - (skip < values ? 1 : 0);
    if (nblocks == 0 || chunk_len == 0) return;
    if (g_sms == 0) {
        int dev = 0;
        check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
        check_cuda(cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev),
                   "cudaDeviceGetAttribute");
    }
    // about 8 resident 256-thread blocks per SM over all staging blocks
    const uint64_t want = (uint64_t(g_sms) * 8 + nblocks - 1) / nblocks;
    const uint64_t need = (chunk_len + kSliceThreads - 1) / kSliceThreads;
    const unsigned bx = unsigned(std::max<uint64_t>(1, std::min(want, need)));
    const ProfToken tok = prof_begin(PROF_SHARD, s);
    if (unpack)
        k_shard_slices<true><<<dim3(bx, unsigned(nblocks)), kSliceThreads, 0, s>>>(
            amps, staging, chunk_begin, chunk_len, skip, A);
    else
        k_shard_slices<false><<<dim3(bx, unsigned(nblocks)), kSliceThreads, 0, s>>>(
            amps, staging, chunk_begin, chunk_len, skip, A);
    prof_end(tok, s, 32.0 * double(chunk_len) * double(nblocks));
    check_cuda(cudaGetLastError(), "shard slice kernel launch");
    (void)n_local;
}

}  // namespace arcqml
