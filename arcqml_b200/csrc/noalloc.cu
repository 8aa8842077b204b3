// noalloc.cu — row norms that allocate no device memory.
//
// Some callers of this runtime cannot allocate GPU memory while they run: code inside a
// region that must not touch the allocator (a caller that has handed all device memory to its
// own pool, or that runs where a cudaMalloc would synchronise the device and stall other work).
// arcqml_rt_v2_norms needs a scratch buffer for its per-block partial sums and takes it from a
// per-thread workspace it grows with cudaMalloc. This file gives those callers the same
// computation with the scratch in a fixed static device array instead.
//
// The array is a file-scope __device__ variable: every GPU that loads the library holds it
// (192 KiB) until the process exits. Host code cannot use its name as a device address; the
// address is fetched once per device with cudaGetSymbolAddress (on the first call made with that
// device current) and passed to the kernels; it is kept for the life of the process, so a
// cudaDeviceReset between calls (which would invalidate it) is not supported. All calls share the array, so calls that overlap
// on the GPU (different streams or threads at the same time) race on it.
#include <cuda_runtime.h>

#include <mutex>
#include <new>
#include <sstream>

#include "../../include/arcqml_runtime_v2.h"
#include "launch.h"
#include "rt_internal.h"

namespace arcqml {

namespace {

constexpr size_t kNoAllocMaxRows = 8192;       // batch rows per call
constexpr size_t kNoAllocPartials = 16384;     // block partial sums (rows x blocks per row)
constexpr int kNoAllocMaxDevices = 64;

// [0, kNoAllocPartials): block partials; then one sum per row.
static __device__ __align__(256) double g_norm_scratch[kNoAllocPartials + kNoAllocMaxRows];

std::mutex g_setup_mu;
double *g_scratch_by_device[kNoAllocMaxDevices] = {};

// Device address of the scratch array for the current device (set up on first use).
double *scratch_for_current_device() {
    int dev = 0;
    check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= kNoAllocMaxDevices) fail("device index outside the supported range");
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_by_device[dev]) {
        void *p = nullptr;
        check_cuda(cudaGetSymbolAddress(&p, g_norm_scratch), "cudaGetSymbolAddress");
        g_scratch_by_device[dev] = static_cast<double *>(p);
    }
    return g_scratch_by_device[dev];
}

template <class F>
int32_t guarded_noalloc(F &&f) {
    try {
        f();
        return 0;
    } catch (const Error &e) {
        set_last_error(e.msg);
        return 1;
    } catch (const std::bad_alloc &) {
        set_last_error("out of host memory");
        return 2;
    } catch (...) {
        set_last_error("runtime failure");
        return 3;
    }
}

}  // namespace

}  // namespace arcqml

using namespace arcqml;

#pragma GCC visibility push(default)
extern "C" int32_t arcqml_rt_v2_norms_noalloc(const arcqml_c128 *amplitudes, size_t batch,
                                              size_t num_qubits, double *norms, void *stream) {
    return guarded_noalloc([&] {
        if (!amplitudes) fail("amplitude buffer is null");
        if (!norms) fail("norm buffer is null");
        if (batch == 0) fail("batch size must be non-zero");
        if (num_qubits >= kMaxQubits) {
            std::ostringstream m;
            m << "state dimension overflow for " << num_qubits << " qubits";
            fail(m.str());
        }
        if (batch > kNoAllocMaxRows) {
            std::ostringstream m;
            m << "batch of " << batch << " rows exceeds the " << kNoAllocMaxRows
              << "-row limit of the allocation-free norm entry point";
            fail(m.str());
        }
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        double *scratch = scratch_for_current_device();
        double *partials = scratch;
        double *sums = scratch + kNoAllocPartials;
        // launch_norms caps the blocks per row at ceil(blocks / batch): at most
        // adjoint_max_blocks() + batch partial sums in total.
        if (size_t(adjoint_max_blocks()) + batch > kNoAllocPartials)
            fail("this GPU needs more partial sums than the allocation-free scratch holds");
        const unsigned bx = launch_norms(reinterpret_cast<const double2 *>(amplitudes), batch,
                                         uint32_t(num_qubits), partials, s);
        // every partial the reduction reads was just written: nothing needs clearing
        launch_reduce_rows(partials, uint32_t(batch), bx, sums, s);
        check_cuda(cudaMemcpyAsync(norms, sums, batch * sizeof(double), cudaMemcpyDeviceToHost, s),
                   "cudaMemcpyAsync (norms)");
        check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    });
}
#pragma GCC visibility pop
