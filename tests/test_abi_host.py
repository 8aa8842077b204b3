"""C-ABI checks that need no GPU: exports, struct layouts, validation, host-only entry points."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

from arcqml_b200 import circuit as cm

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")


def declared_symbols():
    names = set()
    for f in os.listdir(INCLUDE):
        if f.endswith(".h"):
            text = open(os.path.join(INCLUDE, f)).read()
            names |= set(re.findall(r"\b(arcqml_rt_\w+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol(runtime):
    out = subprocess.run(["nm", "-D", "--defined-only", runtime.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing
    # the 14 symbols arcqml-runtime-sys binds (crates/arcqml-runtime-sys/src/lib.rs:28-103)
    assert set(runtime.V1_SYMBOLS) <= exported
    assert len(runtime.V1_SYMBOLS) == 14


def test_static_archive_holds_the_abi(runtime):
    archive = runtime.LIB_PATH[:-3] + ".a"
    out = subprocess.run(["nm", "--defined-only", archive], capture_output=True, text=True,
                         check=True).stdout
    for s in runtime.V1_SYMBOLS:
        assert re.search(rf"\bT {s}\b", out), s


LAYOUT_PROBE = r"""
#include <stdio.h>
#include <stddef.h>
#include "arcqml_runtime.h"
#define P(T, F) printf(#T "." #F " %zu\n", offsetof(T, F));
int main(void) {
  printf("GateDescriptor %zu\nOperationDescriptor %zu\nParameterBindingDescriptor %zu\n"
         "DerivativeMatrixHandle %zu\nCircuitPlanHandle %zu\narcqml_c128 %zu\n",
         sizeof(GateDescriptor), sizeof(OperationDescriptor), sizeof(ParameterBindingDescriptor),
         sizeof(DerivativeMatrixHandle), sizeof(CircuitPlanHandle), sizeof(arcqml_c128));
  P(GateDescriptor, opcode) P(GateDescriptor, arity) P(GateDescriptor, parameters)
  P(GateDescriptor, matrix) P(GateDescriptor, matrix_len) P(GateDescriptor, name)
  P(GateDescriptor, name_len) P(OperationDescriptor, qubits) P(OperationDescriptor, qubits_len)
  P(OperationDescriptor, parameters) P(OperationDescriptor, parameters_len)
  return 0;
}
"""


def test_header_layouts_match_repr_c(tmp_path, runtime):
    """repr(C) layouts of crates/arcqml-runtime-abi/src/lib.rs:13-110 on x86_64."""
    src = tmp_path / "probe.c"
    src.write_text(LAYOUT_PROBE)
    exe = tmp_path / "probe"
    subprocess.run(["/usr/bin/gcc", "-I", INCLUDE, str(src), "-o", str(exe)], check=True)
    got = dict(line.rsplit(" ", 1) for line in subprocess.run([str(exe)], capture_output=True,
                                                                text=True).stdout.splitlines())
    got = {k: int(v) for k, v in got.items()}
    expect = {"GateDescriptor": 72, "OperationDescriptor": 104, "ParameterBindingDescriptor": 16,
              "DerivativeMatrixHandle": 24, "CircuitPlanHandle": 8, "arcqml_c128": 16,
              "GateDescriptor.opcode": 4, "GateDescriptor.arity": 8,
              "GateDescriptor.parameters": 16, "GateDescriptor.matrix": 40,
              "GateDescriptor.matrix_len": 48, "GateDescriptor.name": 56,
              "GateDescriptor.name_len": 64, "OperationDescriptor.qubits": 72,
              "OperationDescriptor.qubits_len": 80, "OperationDescriptor.parameters": 88,
              "OperationDescriptor.parameters_len": 96}
    assert got == expect
    # the ctypes mirror agrees
    assert C.sizeof(runtime.GateDescriptor) == 72
    assert C.sizeof(runtime.OperationDescriptor) == 104
    assert C.sizeof(runtime.DerivativeMatrixHandle) == 24


def test_abi_version(runtime):
    assert runtime.load().arcqml_rt_abi_version() == 1
    runtime.ensure_compatible()


def test_plan_push_validation_messages(runtime):
    plan = runtime.CircuitPlan.with_capacity(4)
    with pytest.raises(runtime.RuntimeError, match="has arity 2, descriptor says 1"):
        plan.push(cm.PlanOp(16, (0,), (0, 0, 0)))
    with pytest.raises(runtime.RuntimeError, match="expects 2 qubits, got 1"):
        runtime.apply_gate(np.zeros(4, np.complex128), 2, runtime.gate_descriptor(16, 2), [0])
    with pytest.raises(runtime.RuntimeError, match="duplicate qubit"):
        plan.push(cm.PlanOp(16, (1, 1), (0, 0, 0)))
    with pytest.raises(runtime.RuntimeError, match="does not have parameter slot 1"):
        plan.push(cm.PlanOp(11, (0,), (0.1, 0, 0), None, ((1, 1),)))
    with pytest.raises(runtime.RuntimeError, match="unknown gate opcode 39"):
        plan.push(cm.PlanOp(39, (0,), (0, 0, 0)))
    with pytest.raises(runtime.RuntimeError, match="expects 16 matrix entries"):
        plan.push(cm.PlanOp(38, (0, 1), (0, 0, 0), np.eye(2, dtype=np.complex128)))
    plan.push(cm.PlanOp(11, (0,), (0.1, 0, 0), None, ((0, 1),)))
    assert len(plan) == 1


def test_descriptor_abi_version_rejected(runtime):
    keep = []
    g = runtime.gate_descriptor(1, 1, abi_version=2)
    a = np.array([1, 0], np.complex128)
    with pytest.raises(runtime.RuntimeError, match="ABI mismatch: expected 1, got 2"):
        runtime.apply_gate(a, 1, g, [0])


def test_state_length_errors_before_any_device_work(runtime):
    """kernel_tests.rs:25-68: wrong lengths and unrepresentable dimensions are errors."""
    a = np.array([1], np.complex128)
    g = runtime.gate_descriptor(1, 1)
    with pytest.raises(runtime.RuntimeError, match="expected 2, got 1"):
        runtime.apply_gate(a, 1, g, [0])
    with pytest.raises(runtime.RuntimeError, match="expected 2, got 1"):
        runtime.apply_adjoint_gate(a, 1, g, [0])
    with pytest.raises(runtime.RuntimeError, match="overflow"):
        runtime.apply_gate(a, 64, g, [0])
    with pytest.raises(runtime.RuntimeError, match="out of range"):
        runtime.apply_gate(np.zeros(2, np.complex128), 1, g, [3])


def test_last_error_protocol(runtime):
    L = runtime.load()
    plan = runtime.CircuitPlan.with_capacity(1)
    with pytest.raises(runtime.RuntimeError):
        plan.push(cm.PlanOp(16, (0,), (0, 0, 0)))
    n = L.arcqml_rt_last_error(None, 0)
    assert n > 0
    buf = (C.c_uint8 * 4)()
    assert L.arcqml_rt_last_error(buf, 4) == n  # truncated copy, full length returned


def test_last_error_is_per_thread(runtime):
    """The status message is thread-local (callers fail concurrently from worker threads,
    row_major.rs:116-130): each thread fails, waits until every thread has failed, then reads
    its own message."""
    import threading
    L = runtime.load()
    g = runtime.gate_descriptor(1, 1)
    nthreads = 8
    barrier = threading.Barrier(nthreads, timeout=60)
    got = [None] * nthreads

    def read():
        n = L.arcqml_rt_last_error(None, 0)
        buf = (C.c_uint8 * (n + 1))()
        L.arcqml_rt_last_error(buf, n + 1)
        return bytes(buf[:n]).decode()

    def body(t):
        a = np.zeros(t + 3, np.complex128)  # length t + 3 is never 2^1
        q = (C.c_size_t * 1)(0)
        for _ in range(50):
            assert L.arcqml_rt_v1_apply_gate(a.ctypes.data, a.size, 1, C.byref(g), q, 1) != 0
            barrier.wait()
            msg = read()
            if got[t] is None or f"got {t + 3}" in got[t]:
                got[t] = msg  # keeps the first wrong message
            barrier.wait()

    threads = [threading.Thread(target=body, args=(t,)) for t in range(nthreads)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    for t in range(nthreads):
        assert f"expected 2, got {t + 3}" in got[t], got


def test_destroy_is_idempotent(runtime):
    L = runtime.load()
    h = runtime.CircuitPlanHandle()
    L.arcqml_rt_v1_circuit_plan_destroy(C.byref(h))
    L.arcqml_rt_v1_circuit_plan_destroy(None)
    m = runtime.DerivativeMatrixHandle()
    L.arcqml_rt_v1_derivative_matrix_destroy(C.byref(m))
    L.arcqml_rt_v1_derivative_matrix_destroy(None)


PARAM_OPS = [(11, 1), (12, 1), (13, 1), (14, 1), (15, 1), (22, 2), (23, 2), (24, 2), (25, 2),
             (30, 2), (31, 2), (32, 2), (33, 2), (34, 2)]


@pytest.mark.parametrize("opcode,arity", PARAM_OPS)
def test_derivative_matrix_create_matches_oracle(runtime, oracle, opcode, arity):
    """Host-built dU/dp (DerivativeMatrix::create) equals the oracle's for every slot."""
    params = (0.37, -1.1, 0.52)
    for slot in range(cm.slot_count(opcode)):
        m = runtime.DerivativeMatrix.create(runtime.gate_descriptor(opcode, arity, params), slot).matrix()
        ref = oracle.derivative_matrix(opcode, arity, params, slot)
        assert np.max(np.abs(m - ref)) < 1e-14, (opcode, slot)


def test_derivative_matrix_rejects_invalid_slot(runtime):
    with pytest.raises(runtime.RuntimeError, match="does not have parameter slot"):
        runtime.DerivativeMatrix.create(runtime.gate_descriptor(4, 1), 0)
    with pytest.raises(runtime.RuntimeError, match="does not have parameter slot 3"):
        runtime.DerivativeMatrix.create(runtime.gate_descriptor(15, 1, (0.1, 0.2, 0.3)), 3)


def test_plan_parameters_update(runtime):
    plan = runtime.CircuitPlan.compile([cm.PlanOp(11, (0,), (0.1, 0, 0), None, ((0, 1),))])
    plan.set_parameters(np.array([0.0, 0.5]))
    with pytest.raises(runtime.RuntimeError, match="out of range"):
        plan.set_parameters(np.array([0.0]))


def header_declarations():
    """{name: (result, [parameter types])} of every arcqml_rt_* function in include/*.h."""
    decls = {}
    for f in sorted(os.listdir(INCLUDE)):
        if not f.endswith(".h"):
            continue
        text = re.sub(r"/\*.*?\*/|//[^\n]*", " ", open(os.path.join(INCLUDE, f)).read(),
                      flags=re.S)
        for m in re.finditer(r"([A-Za-z_][\w \*]*?)\b(arcqml_rt_\w+)\s*\(([^)]*)\)\s*;", text):
            params = [p.strip() for p in m.group(3).split(",") if p.strip() not in ("", "void")]
            decls[m.group(2)] = (m.group(1).strip(), params)
    return decls


C_KINDS = {"size_t": "u64", "uint64_t": "u64", "int32_t": "i32", "uint32_t": "u32",
           "double": "f64"}


def c_kind(decl: str) -> str:
    """Argument class of a C declaration: a pointer, or the width and kind of a scalar."""
    if "*" in decl or "[" in decl:
        return "ptr"
    for t, k in C_KINDS.items():
        if re.search(rf"\b{t}\b", decl):
            return k
    raise AssertionError(f"unclassified C type: {decl}")


def test_binding_signatures_match_the_headers(runtime):
    """The ctypes argument and result types of every bound entry point agree with the C
    declarations in include/*.h (count, pointer or integer width, double)."""
    import ctypes as C
    kinds = {C.c_void_p: "ptr", C.c_size_t: "u64", C.c_uint64: "u64", C.c_int32: "i32",
             C.c_uint32: "u32", C.c_double: "f64", None: "void"}
    assert C.sizeof(C.c_size_t) == 8
    decls = header_declarations()
    assert set(runtime.SIGNATURES) <= set(decls), set(runtime.SIGNATURES) - set(decls)
    for name, (res, args) in runtime.SIGNATURES.items():
        cres, cparams = decls[name]
        want = [c_kind(p) for p in cparams]
        got = [kinds[a] for a in args]
        assert got == want, (name, got, want)
        assert kinds[res] == ("void" if cres == "void" else c_kind(cres)), (name, res, cres)


def test_shard_swap_nccl_argument_checks(runtime):
    """arcqml_rt_v2_shard_swap_nccl rejects a missing communicator, staging buffer or bit list
    and bad slice positions before it touches NCCL or the device."""
    L = runtime.load()
    gb = (C.c_uint32 * 1)(0)
    lp = (C.c_uint32 * 1)(3)
    fake = C.c_void_p(0x1000)  # never dereferenced: the checks fail first
    cases = [
        ((fake, 10, gb, lp, 1, None, fake, 64, None), "communicator is null"),
        ((fake, 10, None, lp, 1, fake, fake, 64, None), "global bit list is null"),
        ((fake, 10, gb, lp, 1, fake, None, 64, None), "staging buffer is null"),
        ((fake, 2, gb, lp, 1, fake, fake, 64, None), "outside the 2-qubit shard"),
        ((fake, 10, gb, lp, 0, fake, fake, 64, None), "between 1 and 8 positions"),
    ]
    for args, msg in cases:
        assert L.arcqml_rt_v2_shard_swap_nccl(*args) != 0
        assert msg in runtime.last_error()
