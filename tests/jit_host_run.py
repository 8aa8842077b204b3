"""Runs the run-time compiled pass code on the CPU (test infrastructure).

The runtime exports a plan's fused-pass schedule with the `struct PassOps` source it generates
for every pass (arcqml_rt_v2_plan_schedule_export). Here each source is built as host C++ with
fused_core.cuh (ARCQML_HOST_RUN leaves out the GPU-only parts) and small stand-ins for the CUDA
built-ins, and driven by a host tile loop that mirrors fused_body: tile T's element j is global
index tile_base(T) | scatter(j over the tile qubits S), held in the tile buffer at phys(j); each
sub-block runs thread by thread (threads never share registers within a sub-block, so running
them one after another equals running them together), and the accumulator columns are summed
at the end. The generated code itself, not a restatement of it, is what runs. Reads past the
matrix table meet NaN entries and writes past the accumulator rows hit a checked guard region.
"""
import ctypes as C
import os
import struct
import subprocess
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "arcqml_b200", "csrc")
HEADER_BYTES, SUB_BYTES, OP_BYTES = 48, 24, 64
GUARD = 256  # NaN matrix-table entries after the end

PRELUDE = r"""
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#define __host__
#define __device__
#define __forceinline__ inline
#define __global__
#define __launch_bounds__(...)
#define __restrict__
#define __grid_constant__
#define ARCQML_HOST_RUN 1
struct double2 { double x, y; };
inline double2 make_double2(double a, double b) { return double2{a, b}; }
struct HostDim { unsigned x = 0, y = 0, z = 0; };
static HostDim threadIdx, blockDim;
inline int __double2hiint(double d) { uint64_t u; std::memcpy(&u, &d, 8); return int(uint32_t(u >> 32)); }
inline int __double2loint(double d) { uint64_t u; std::memcpy(&u, &d, 8); return int(uint32_t(u)); }
inline double __hiloint2double(int hi, int lo) {
    const uint64_t u = (uint64_t(uint32_t(hi)) << 32) | uint32_t(lo);
    double d;
    std::memcpy(&d, &u, 8);
    return d;
}
using std::fma;
#include "fused.h"
namespace arcqml {
#include "fused_core.cuh"

// Returns 0, or 1 when the pass code wrote past its accumulator rows (a guard region).
template <int RB, bool ADJ, class Ops>
int drive(uint32_t n, double2 *psi, double2 *lam, const PassHeader *h, const double2 *mats,
          double *acc) {
    const uint32_t k = h->k, D = 1u << k, threads = 1u << (k - RB);
    const uint64_t tiles = uint64_t(1) << (n - k);
    std::vector<double2> tp(D), tl(D);
    // accumulator rows hold one column per Ops::kAccLanes threads, acc_row_stride apart
    const uint32_t cols = threads / uint32_t(Ops::kAccLanes);
    const uint32_t stride = acc_row_stride(cols, uint32_t(Ops::kAccLanes));
    const size_t rows = size_t(h->nacc) * stride, guard = 64;
    std::vector<double> sacc(rows + guard, 0.0);
    for (size_t i = rows; i < rows + guard; ++i) sacc[i] = 12345.0;
    blockDim.x = threads;
    for (uint64_t T = 0; T < tiles; ++T) {
        uint64_t g = T;
        for (uint32_t b = 0; b < k; ++b) {
            const uint32_t p = h->S[b];
            g = ((g >> p) << (p + 1)) | (g & ((uint64_t(1) << p) - 1));
        }
        auto gidx = [&](uint32_t j) {
            uint64_t x = g;
            for (uint32_t b = 0; b < k; ++b)
                if ((j >> b) & 1u) x |= uint64_t(1) << h->S[b];
            return x;
        };
        for (uint32_t j = 0; j < D; ++j) {
            tp[phys(j)] = psi[gidx(j)];
            if (ADJ) tl[phys(j)] = lam[gidx(j)];
        }
        for (uint32_t sb = 0; sb < h->nsub; ++sb)
            for (uint32_t t = 0; t < threads; ++t) {
                threadIdx.x = t;
                Ops::template run<RB, ADJ>(sb, k, tp.data(), tl.data(), nullptr, mats, nullptr,
                                           sacc.data(), stride, g);
            }
        for (uint32_t j = 0; j < D; ++j) {
            psi[gidx(j)] = tp[phys(j)];
            if (ADJ) lam[gidx(j)] = tl[phys(j)];
        }
    }
    for (uint32_t a = 0; a < h->nacc; ++a) {
        double s = 0.0;
        for (uint32_t t = 0; t < cols; ++t) s += sacc[size_t(a) * stride + t];
        acc[a] = s * Ops::row_factor(a, mats);
    }
    for (size_t i = rows; i < rows + guard; ++i)
        if (sacc[i] != 12345.0) return 1;
    return 0;
}
"""


class Pass:
    def __init__(self, header, subs, ops, mats, parents, alias, code):
        self.header, self.subs, self.ops, self.mats = header, subs, ops, mats
        self.parents, self.alias, self.code = parents, alias, code
        k, nsub, nops, nmat, nacc, acc_base, rb = struct.unpack_from("<7I", header, 0)
        self.k, self.nacc, self.rb = k, nacc, rb


def parse(blob: bytes):
    off = 0

    def u32():
        nonlocal off
        v = struct.unpack_from("<I", blob, off)[0]
        off += 4
        return v

    def take(nbytes):
        nonlocal off
        b = blob[off:off + nbytes]
        off += nbytes
        return b

    steps = []
    for _ in range(u32()):
        if not u32():
            steps.append(("dense", u32()))
            continue
        header = take(HEADER_BYTES)
        subs = take(u32() * SUB_BYTES)
        ops = take(u32() * OP_BYTES)
        mats = np.frombuffer(take(u32() * 16), dtype=np.complex128).copy()
        npar = u32()
        parents = list(struct.unpack(f"<{npar}Q", take(8 * npar)))
        nal = u32()
        flat = struct.unpack(f"<{2 * nal}Q", take(16 * nal))
        alias = list(zip(flat[0::2], flat[1::2]))  # (accumulator, further parent)
        code = take(u32()).decode()
        steps.append(("pass", Pass(header, subs, ops, mats, parents, alias, code)))
    assert off == len(blob)
    return steps


def build(steps, adjoint: bool, workdir: str):
    src = [PRELUDE]
    for i, (kind, p) in enumerate(steps):
        if kind != "pass":
            continue
        assert p.code, "a pass without a run-time compiled form"
        body = p.code.split('extern "C"')[0]
        src.append(f"namespace pass_{i} {{\n{body}\n}}  // namespace pass_{i}\n")
        src.append(
            f'extern "C" int run_pass_{i}(uint32_t n, double2 *psi, double2 *lam, '
            f"const PassHeader *h, const double2 *mats, double *acc) {{\n"
            f"    return drive<{p.rb}, {'true' if adjoint else 'false'}, pass_{i}::PassOps>"
            f"(n, psi, lam, h, mats, acc);\n}}\n")
    src.append("}  // namespace arcqml\n")
    cpp = os.path.join(workdir, "passes.cpp")
    so = os.path.join(workdir, "passes.so")
    with open(cpp, "w") as f:
        f.write("".join(src))
    r = subprocess.run(["g++", "-std=c++17", "-O1", "-shared", "-fPIC", "-w", "-I", CSRC, cpp,
                        "-o", so], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    return C.CDLL(so)


def run(runtime, plan, n, state, adjoint=False, lam=None, requires_grad=None):
    """Forward: the new state. Adjoint: (psi_0, lambda_0, gradients by parent)."""
    req = None if requires_grad is None else np.asarray(requires_grad, np.uint8)
    steps = parse(runtime.plan_schedule_export(plan, n, adjoint, req))
    psi = np.ascontiguousarray(state, dtype=np.complex128).copy()
    lm = None if lam is None else np.ascontiguousarray(lam, dtype=np.complex128).copy()
    grads = np.zeros(0 if req is None else len(req))
    with tempfile.TemporaryDirectory() as d:
        lib = build(steps, adjoint, d)
        for i, (kind, p) in enumerate(steps):
            assert kind == "pass", "custom gates between passes are not run here"
            hdr = C.create_string_buffer(p.header, len(p.header))
            acc = np.zeros(max(1, p.nacc))
            fn = getattr(lib, f"run_pass_{i}")
            fn.restype = C.c_int
            # the matrix table followed by NaN entries: a read past its end poisons the result
            mats = np.concatenate([p.mats, np.full(GUARD, np.nan, dtype=np.complex128)])
            status = fn(C.c_uint32(n), C.c_void_p(psi.ctypes.data),
                        C.c_void_p(lm.ctypes.data if lm is not None else 0), hdr,
                        C.c_void_p(mats.ctypes.data), C.c_void_p(acc.ctypes.data))
            assert status == 0, f"pass {i} wrote past its accumulator rows"
            for a, parent in enumerate(p.parents):
                grads[parent] += 2.0 * acc[a]
            for a, parent in p.alias:
                grads[parent] += 2.0 * acc[a]
    return psi if not adjoint else (psi, lm, grads)
