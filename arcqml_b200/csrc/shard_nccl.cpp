// shard_nccl.cpp — a global-qubit swap of a sharded state over the caller's NCCL communicator.
//
// A state of n qubits over P = 2^g ranks keeps on rank r the 2^(n-g) amplitudes whose top g
// index bits equal r. Swapping k global qubits (rank bits global_bits[i]) with k local qubits
// (positions local_positions[i] of the shard) is an all-to-all among the 2^k ranks that differ in
// those bits: each rank packs the slices of its shard whose slice value y (bit i of y = local bit
// local_positions[i]) differs from its own value x into staging blocks (shard.cu), sends block y
// to the rank whose global bits are y and receives that rank's block x, and unpacks what it
// received into the slots the pack emptied. Chunks of the remaining index bits bound the staging
// memory. Everything runs on the caller's stream; the NCCL library is the one the process has
// loaded (the communicator's own), reached with dlopen, so the runtime links no NCCL import.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <mutex>
#include <sstream>

#include "../../include/arcqml_runtime_v2.h"
#include "launch.h"
#include "rt_internal.h"

namespace arcqml {
namespace {

// The few NCCL entry points used here, with the library's documented C types: results and data
// types are C enums (ncclSuccess = 0, ncclInt8 = 0), communicators opaque pointers.
using nccl_comm = void *;
struct Nccl {
    bool tried = false, ok = false;
    std::string why;
    int (*group_start)() = nullptr;
    int (*group_end)() = nullptr;
    int (*send)(const void *, size_t, int, int, nccl_comm, cudaStream_t) = nullptr;
    int (*recv)(void *, size_t, int, int, nccl_comm, cudaStream_t) = nullptr;
    int (*user_rank)(nccl_comm, int *) = nullptr;
    int (*count)(nccl_comm, int *) = nullptr;
    const char *(*error_string)(int) = nullptr;
};
constexpr int kNcclSuccess = 0;
constexpr int kNcclInt8 = 0;

std::mutex g_nccl_mu;
Nccl g_nccl;

template <class F>
bool sym(void *lib, const char *name, F &out) {
    out = reinterpret_cast<F>(dlsym(lib, name));
    return out != nullptr;
}

const Nccl &nccl() {
    std::lock_guard<std::mutex> lock(g_nccl_mu);
    if (g_nccl.tried) return g_nccl;
    g_nccl.tried = true;
    // prefer the NCCL already in the process (the one that made the communicator)
    void *lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW);
    if (!lib) {
        g_nccl.why = "libnccl.so.2 could not be loaded";
        return g_nccl;
    }
    g_nccl.ok = sym(lib, "ncclGroupStart", g_nccl.group_start) &&
                sym(lib, "ncclGroupEnd", g_nccl.group_end) && sym(lib, "ncclSend", g_nccl.send) &&
                sym(lib, "ncclRecv", g_nccl.recv) &&
                sym(lib, "ncclCommUserRank", g_nccl.user_rank) &&
                sym(lib, "ncclCommCount", g_nccl.count) &&
                sym(lib, "ncclGetErrorString", g_nccl.error_string);
    if (!g_nccl.ok) g_nccl.why = "libnccl.so.2 lacks a needed entry point";
    return g_nccl;
}

void check_nccl(const Nccl &N, int r, const char *what) {
    if (r == kNcclSuccess) return;
    std::ostringstream m;
    m << what << " failed: " << (N.error_string ? N.error_string(r) : "NCCL error") << " (" << r
      << ")";
    fail(m.str());
}

}  // namespace

void shard_swap_nccl(double2 *shard, uint32_t n_local, const uint32_t *global_bits,
                     const uint32_t *local_positions, uint32_t k, void *comm, double2 *staging,
                     size_t staging_len, cudaStream_t s) {
    const Nccl &N = nccl();
    if (!N.ok) fail(N.why);
    int rank = 0, world = 0;
    check_nccl(N, N.user_rank(comm, &rank), "ncclCommUserRank");
    check_nccl(N, N.count(comm, &world), "ncclCommCount");
    if (world < 1 || (world & (world - 1))) fail("the communicator's size is not a power of two");
    uint32_t g = 0;
    while ((1 << g) < world) ++g;
    for (uint32_t i = 0; i < k; ++i) {
        if (global_bits[i] >= g) {
            std::ostringstream m;
            m << "global bit " << global_bits[i] << " outside the " << g << " rank bits";
            fail(m.str());
        }
        for (uint32_t j = 0; j < i; ++j)
            if (global_bits[j] == global_bits[i]) fail("global bits repeat");
    }
    const uint64_t nblk = (uint64_t(1) << k) - 1;
    const uint64_t others = uint64_t(1) << (n_local - k);
    uint64_t chunk = others;
    while (chunk > 1 && 2 * nblk * chunk > staging_len) chunk >>= 1;
    if (2 * nblk * chunk > staging_len) fail("staging buffer too small for one chunk");
    uint64_t x = 0;
    for (uint32_t i = 0; i < k; ++i) x |= uint64_t((rank >> global_bits[i]) & 1) << i;
    double2 *send = staging;
    double2 *recv = staging + nblk * chunk;
    for (uint64_t c0 = 0; c0 < others; c0 += chunk) {
        launch_slices(shard, n_local, local_positions, k, c0, chunk, x, send, false, s);
        check_nccl(N, N.group_start(), "ncclGroupStart");
        for (uint64_t y = 0; y <= nblk; ++y) {
            if (y == x) continue;
            int peer = rank;
            for (uint32_t i = 0; i < k; ++i)
                peer = (peer & ~(1 << global_bits[i])) | int(((y >> i) & 1) << global_bits[i]);
            const uint64_t blk = y - (y > x ? 1 : 0);
            const size_t bytes = size_t(chunk) * sizeof(double2);
            check_nccl(N, N.send(send + blk * chunk, bytes, kNcclInt8, peer, comm, s), "ncclSend");
            check_nccl(N, N.recv(recv + blk * chunk, bytes, kNcclInt8, peer, comm, s), "ncclRecv");
        }
        check_nccl(N, N.group_end(), "ncclGroupEnd");
        launch_slices(shard, n_local, local_positions, k, c0, chunk, x, recv, true, s);
    }
}

}  // namespace arcqml
