"""The run-time compiled pass code, built as host code and run on the CPU (jit_host_run.py),
against the oracle: the generated sources and the fused_core.cuh helpers they call, for the
default configuration and for ARCQML_SUBBLOCK_REORDER=1 / ARCQML_FAST_CNOT=1 (subprocesses)."""
import math
import os
import shutil
import subprocess
import sys

import numpy as np
import pytest

import jit_host_run as J
from arcqml_b200 import circuit as cm
from arcqml_b200 import workloads
from plans import random_state, random_terms

pytestmark = pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")


def check(runtime, oracle, c, n, seed, terms=12):
    g = np.random.Generator(np.random.PCG64(seed))
    ops = c.compile_plan(1)
    plan = runtime.CircuitPlan.create(ops)
    init = random_state(g, n)
    psi = J.run(runtime, plan, n, init)
    ref = oracle.plan_apply(ops, init, n)
    assert float(np.max(np.abs(psi - ref))) < 1e-12
    _, lam = oracle.expectation_and_apply(random_terms(g, n, terms), ref, n)
    req = list(c.requires_grad_mask(True))
    p0, l0, gr = J.run(runtime, plan, n, psi, adjoint=True, lam=-0.6 * lam, requires_grad=req)
    _, rl0, rg = oracle.adjoint_backward(ops, ref, lam, n, -0.6, req, len(req))
    assert float(np.max(np.abs(p0 - init))) < 1e-10
    assert float(np.max(np.abs(l0 - rl0))) <= 1e-10 * max(1.0, float(np.max(np.abs(rl0))))
    assert float(np.max(np.abs(gr - rg))) <= 1e-10 * max(1.0, float(np.max(np.abs(rg))))


def brickwork_edges(n, seed):
    c = workloads.brickwork(n, 4, seed=seed)
    for q in range(n):  # scaled forms refused at pi, growth caps, fixed phases
        c.rot("ry", math.pi * (1 - 1e-9), q)
        c.rot("rx", math.pi, q)
        c.append("phase", (q,), 3 * math.pi)
    for _ in range(25):
        c.rot("rz", math.pi * (1 - 1e-9), 2)
    return c


def fast_shapes(n, seed):
    """Every fast gate shape: rotations (trained), H / SX / S / T / Z, U3 as a dense 2x2,
    RXX / RYY as dense 4x4s, fixed phases, CZ between any qubits."""
    g = np.random.Generator(np.random.PCG64(seed))
    c = cm.Circuit(n)
    for _ in range(3):
        for q in range(n):
            r = g.uniform()
            if r < 0.5:
                c.rot(("rx", "ry", "rz")[int(g.integers(0, 3))], float(g.uniform(-3, 3)), q)
            elif r < 0.65:
                c.append(("h", "sx", "s", "t", "z")[int(g.integers(0, 5))], (q,))
            elif r < 0.8:
                c.append("u3", (q,), *(float(x) for x in g.uniform(-3, 3, 3)))
            else:
                c.append("phase", (q,), float(g.uniform(-3, 3)))
        for _ in range(n // 2):
            a, b = (int(x) for x in g.choice(n, size=2, replace=False))
            c.append("cz", (a, b))
            if abs(a - b) == 1 and g.uniform() < 0.5:
                c.append(("rxx", "ryy")[int(g.integers(0, 2))], (a, b), float(g.uniform(-3, 3)))
    return c


@pytest.mark.parametrize("n", [10, 13])
def test_compiled_brickwork_passes_run_on_host(runtime, oracle, n):
    check(runtime, oracle, brickwork_edges(n, n), n, seed=n)


@pytest.mark.parametrize("n,seed", [(9, 1), (12, 2)])
def test_compiled_fast_shape_passes_run_on_host(runtime, oracle, n, seed):
    check(runtime, oracle, fast_shapes(n, seed), n, seed=seed)


def cnot_ring(n, seed):
    g = np.random.Generator(np.random.PCG64(seed))
    c = cm.Circuit(n)
    for _ in range(3):
        for q in range(n):
            c.rot("ry", float(g.uniform(-3, 3)), q)
            c.rot("rz", float(g.uniform(-3, 3)), q)
        for q in range(n):
            c.append("cnot", (q, (q + 1) % n))
        c.append("x", (int(g.integers(0, n)),))
    return c


@pytest.mark.parametrize("env", ["ARCQML_SUBBLOCK_REORDER", "ARCQML_FAST_CNOT"])
def test_switches_run_their_compiled_code_on_host(env):
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    code = ("import sys; sys.path[:0] = [%r, %r, %r]\n"
            "import oracle, test_jit_host_run as T\n"
            "from arcqml_b200 import runtime\n"
            "T.check(runtime, oracle, T.brickwork_edges(10, 3), 10, seed=3)\n"
            "T.check(runtime, oracle, T.fast_shapes(12, 4), 12, seed=4)\n"
            "if %r == 'ARCQML_FAST_CNOT':\n"
            "    for n in (10, 13):\n"
            "        T.check(runtime, oracle, T.cnot_ring(n, n), n, seed=n)\n"
            "print('host-run-ok')\n") % (root, here, os.path.join(root, "oracle"), env)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       env=dict(os.environ, **{env: "1"}), timeout=900)
    assert r.returncode == 0 and "host-run-ok" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
