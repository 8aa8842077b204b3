"""The static archive linked into an executable the way arcqml-runtime-sys links it.

crates/arcqml-runtime-sys/build.rs:10-21 links the static library arcqml_runtime_private from
ARCQML_RUNTIME_LIB_DIR; the archive holds CUDA objects, so the final link adds the CUDA runtime
and the C++ library (the link line of INTEGRATION.md: cudart_static, stdc++, rt, dl; pthread
and m come with every Rust std link). tests/link_consumer.c is compiled against
include/arcqml_runtime.h and linked against libarcqml_runtime_private.a with that line; a
missing object or library shows up as a link failure here. On CPU the program checks the ABI
version, plan building and the last-error protocol; on a B200 it runs
arcqml_rt_v1_circuit_plan_apply and arcqml_rt_v1_adjoint_backward on a 10-qubit random plan,
compared with the oracle at 1e-10.
"""
import os
import struct
import subprocess

import numpy as np
import pytest

from plans import random_plan, random_state

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CUDA_LIB = "/usr/local/cuda/lib64"
LINK_LINE = ["-L" + CUDA_LIB, "-lcudart_static", "-lstdc++", "-lrt", "-ldl", "-lpthread", "-lm"]


@pytest.fixture(scope="module")
def consumer(runtime, tmp_path_factory):
    out = tmp_path_factory.mktemp("link")
    obj, exe = str(out / "link_consumer.o"), str(out / "link_consumer")
    subprocess.run(["gcc", "-std=c11", "-O2", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    "-c", os.path.join(HERE, "link_consumer.c"), "-o", obj], check=True)
    archive = os.path.join(ROOT, "arcqml_b200", "libarcqml_runtime_private.a")
    r = subprocess.run(["gcc", "-o", exe, obj, archive] + LINK_LINE, capture_output=True,
                       text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_static_archive_links_and_runs_host_calls(consumer):
    r = subprocess.run([consumer, "check"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, (r.returncode, r.stderr)
    assert "abi 1" in r.stdout
    assert "expects 1 qubits, got 2" in r.stdout


def write_input(path, n, ops, req, upstream, init, lam):
    with open(path, "wb") as f:
        f.write(struct.pack("<II", n, len(ops)))
        for o in ops:
            p = list(o.params) + [0.0] * (3 - len(o.params))
            f.write(struct.pack("<II3d", o.opcode, len(o.qubits), *p[:3]))
            f.write(struct.pack(f"<{len(o.qubits)}Q", *o.qubits))
            f.write(struct.pack("<I", len(o.bindings)))
            for s, par in o.bindings:
                f.write(struct.pack("<QQ", s, par))
        f.write(struct.pack("<Q", len(req)))
        f.write(np.asarray(req, np.uint8).tobytes())
        f.write(struct.pack("<d", upstream))
        f.write(np.ascontiguousarray(init, np.complex128).tobytes())
        f.write(np.ascontiguousarray(lam, np.complex128).tobytes())


@pytest.mark.gpu
def test_static_archive_plan_apply_and_adjoint_match_oracle(consumer, oracle, tmp_path):
    g = np.random.Generator(np.random.PCG64(2718))
    n, num_params = 10, 24
    ops = random_plan(g, n, 160, num_params)
    init = random_state(g, n)
    lam_in = random_state(g, n)
    req = np.ones(num_params + 1, np.uint8)
    req[0] = 0
    req[5] = 0
    upstream = 0.75
    inp, outp = str(tmp_path / "in.bin"), str(tmp_path / "out.bin")
    write_input(inp, n, ops, req, upstream, init, lam_in)
    r = subprocess.run([consumer, "run", inp, outp], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, (r.returncode, r.stderr)
    raw = open(outp, "rb").read()
    dim = 1 << n
    c = np.frombuffer(raw[:3 * dim * 16], np.complex128)
    final, psi0, lam0 = c[:dim], c[dim:2 * dim], c[2 * dim:]
    grads = np.frombuffer(raw[3 * dim * 16:], np.float64)

    want_final = oracle.plan_apply(ops, init, n)
    w_psi0, w_lam0, w_grads = oracle.adjoint_backward(ops, want_final, lam_in, n, upstream, req,
                                                      len(req))
    tol = 1e-10
    assert np.max(np.abs(final - want_final)) <= tol
    assert np.max(np.abs(psi0 - w_psi0)) <= tol
    assert np.max(np.abs(lam0 - w_lam0)) <= tol * max(1.0, float(np.max(np.abs(w_lam0))))
    scale = max(1.0, float(np.max(np.abs(w_grads))))
    np.testing.assert_allclose(grads, w_grads, rtol=0, atol=tol * scale)
