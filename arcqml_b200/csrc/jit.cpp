// jit.cpp — per-pass fused kernels compiled at run time.
//
// The precompiled pass kernel (fused.cu) interprets the pass's op table: per op it loads the op
// descriptor, branches on its kind and register bits, and only then does the arithmetic, so the
// dependent-latency chains of consecutive gates cannot overlap. Here each pass whose ops all have
// fast paths becomes its own kernel: the same tile loop (fused_body in fused_core.cuh) with the
// pass's gates written out in order, register bits as template constants and matrix offsets as
// literals. The compiler then schedules across gates. Parameter values stay in the uploaded
// matrix table, so a kernel is reused for every parameter vector of the same circuit structure
// (kernels are cached by their source text, per device).
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

// ARCQML_JIT_ADJ_WARP=1: adjoint kernels reduce each gradient over the warp (one accumulator
// column per warp instead of per thread) and ask for two resident CTAs per SM.
bool adjoint_per_warp() {
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_JIT_ADJ_WARP");
        return e && e[0] == '1';
    }();
    return on;
}

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

// The fast path of op o on the register array `r` (U in forward passes, U^dagger in adjoint
// passes: the planner stores the daggered matrices). False for a combination without one.
bool emit_apply(std::ostringstream &c, const FOp &o, const char *r, uint32_t rb,
                const SubBlock &S, uint32_t tbits) {
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

// Gradient then U^dagger on psi and lambda, as adj_fast does it.
bool emit_adjoint(std::ostringstream &c, const FOp &o, uint32_t rb, const SubBlock &S,
                  uint32_t tbits) {
    if (o.gkind == GK_NONE) {
        if (!emit_apply(c, o, "v", rb, S, tbits)) return false;
        c << "\n        ";
        return emit_apply(c, o, "w", rb, S, tbits);
    }
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
    // 0.5 * z, times |sigma|^2 in a scaled pass
    c << "\n        " << (acc_per_warp(true, rb) ? "accumulate_warp" : "accumulate") << "(sacc, "
      << o.acc[0] << "u * kCols, ";
    if (o.sgrad) c << "M[" << o.soff << "].y * z); }";
    else c << "0.5 * z); }";
    return true;
}

// Source of the kernel `arcqml_pass` for one pass; empty when some op has no fast path.
std::string pass_source(const Step &st, bool adj, uint32_t rb) {
    std::ostringstream c;
    const uint32_t threads = 1u << (st.header.k - rb);
    const uint32_t cols = acc_per_warp(adj, rb) ? threads / 32u : threads;
    c << "struct PassOps {\n"
         "    static constexpr bool kAccPerWarp = " << (acc_per_warp(adj, rb) ? "true" : "false")
      << ";\n"
         "    template <int RB, bool ADJ>\n"
         "    __device__ static __forceinline__ void run(uint32_t sb, uint32_t, double2 *tp,\n"
         "            double2 *tl, const FOp *, const double2 *M, const SubBlock *, double *sacc,\n"
         "            uint32_t nthreads, uint64_t gbase) {\n"
         "        double2 v[1 << RB], w[1 << RB];\n"
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
            const bool ok = adj ? emit_adjoint(c, st.ops[oi], rb, S, kb)
                                : emit_apply(c, st.ops[oi], "v", rb, S, kb);
            if (!ok) return std::string();
            c << "\n";
        }
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
         "    }\n"
         "};\n";
    const int bound = (adj || rb == 4) ? 256 : 512;
    const int min_blocks = (adj && adjoint_per_warp() && rb == 3) ? 2 : 1;
    c << "extern \"C\" __global__ void __launch_bounds__(" << bound << ", " << min_blocks << ")\n"
         "arcqml_pass(double2 *__restrict__ psi, double2 *__restrict__ lam, uint32_t n,\n"
         "            uint32_t tiles_log, uint64_t total_tiles, const PassHeader *__restrict__ hdr,\n"
         "            const SubBlock *__restrict__ subs, const FOp *__restrict__ gops,\n"
         "            const double2 *__restrict__ gmats, double *__restrict__ partials,\n"
         "            uint32_t stride) {\n"
         "    fused_body<" << rb << ", " << (adj ? "true" : "false")
      << ", PassOps>(psi, lam, n, tiles_log, total_tiles, hdr, subs, gops, gmats, partials,"
         " stride);\n}\n";
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
    std::vector<std::string> srcs(sch.steps.size());
    for (size_t i = 0; i < sch.steps.size(); ++i)
        if (sch.steps[i].is_pass) {
            const std::string pass = pass_source(sch.steps[i], adj, sch.steps[i].header.rb);
            if (!pass.empty()) srcs[i] = full_source(pass);
        }
    int dev = 0;
    check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lock(g_mu);
    auto &cache = g_cache[dev];
    std::vector<size_t> todo;
    for (size_t i = 0; i < srcs.size(); ++i) {
        if (srcs[i].empty()) continue;
        auto it = cache.find(srcs[i]);
        if (it != cache.end()) {
            fns[i] = it->second;
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
                if (it != cache.end()) fns[i] = it->second;
            }
    }
    return fns;
}

bool jit_acc_per_warp(bool adjoint, uint32_t rb) { return acc_per_warp(adjoint, rb); }

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
