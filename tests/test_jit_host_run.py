"""The run-time compiled pass code, built as host code and run on the CPU (jit_host_run.py),
against the oracle: the generated sources and the fused_core.cuh helpers they call, for the
default configuration and with ARCQML_SUBBLOCK_REORDER=0 / ARCQML_FAST_CNOT=0 /
ARCQML_FAST_DIAG=0 (subprocesses)."""
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


def general_shapes(n, seed):
    """Gates that only the FAST_DIAG paths (on unless ARCQML_FAST_DIAG=0) compile: diagonals with controls (CPHASE, CRZ, CS,
    CT), two-qubit diagonals (RZZ), controlled one-target gates (CRX, CRY, CH, CY, Toffoli,
    3-control X), trained PHASE / U3 / RXX / RYY / RZX / fSim (generic slot gradients), with
    qubits in registers, thread bits and outside the tile, and parameters shared across gates;
    Pauli rotations keep the scaled passes mixed."""
    g = np.random.Generator(np.random.PCG64(seed))
    c = cm.Circuit(n)
    shared = c.add_parameter(float(g.uniform(-3, 3)))

    def angle():
        if g.uniform() < 0.2:
            return shared
        return c.add_parameter(float(g.uniform(-3, 3))) if g.uniform() < 0.8 else float(g.uniform(-3, 3))

    def qubits(k):
        return [int(x) for x in g.choice(n, size=k, replace=False)]
    for _ in range(4):
        for q in range(n):
            if g.uniform() < 0.5:
                c.rot(("rx", "ry", "rz")[int(g.integers(0, 3))], float(g.uniform(-3, 3)), q)
        for _ in range(n):
            r = int(g.integers(0, 16))
            if r == 0:
                c.append("phase", qubits(1), angle())
            elif r == 1:
                c.append("u3", qubits(1), angle(), angle(), angle())
            elif r in (2, 3, 4, 5, 6):
                c.append(("cphase", "crz", "crx", "cry", "rzz")[r - 2], qubits(2), angle())
            elif r in (7, 8, 9):
                a, b = qubits(2)
                if g.uniform() < 0.6:  # neighbours: both targets in the tile more often
                    a, b = a, (a + 1) % n
                c.append(("rxx", "ryy", "rzx")[r - 7], (a, b), angle())
            elif r == 10:
                c.append("fsim", qubits(2), angle(), angle())
            elif r in (11, 12, 13, 14):
                c.append(("cs", "ct", "ch", "cy")[r - 11], qubits(2))
            else:
                qs = qubits(4)
                if g.uniform() < 0.5:
                    c.append("toffoli", qs[:3])
                else:
                    c.mcx(qs[:3], qs[3])
    return c


SWITCHES = ("ARCQML_SUBBLOCK_REORDER", "ARCQML_FAST_CNOT", "ARCQML_FAST_DIAG", "ARCQML_LOOKAHEAD")


@pytest.mark.parametrize("env", SWITCHES + ("all",))
def test_switches_off_run_their_compiled_code_on_host(env):
    """Each switch turned off alone, and all of them off (subprocesses): the brickwork and
    fast-path circuits, and the CNOT rings while one of FAST_CNOT / FAST_DIAG still gives them
    compiled code."""
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    rings = env != "all"
    code = ("import sys; sys.path[:0] = [%r, %r, %r]\n"
            "import oracle, test_jit_host_run as T\n"
            "from arcqml_b200 import runtime\n"
            "T.check(runtime, oracle, T.brickwork_edges(10, 3), 10, seed=3)\n"
            "T.check(runtime, oracle, T.fast_shapes(12, 4), 12, seed=4)\n"
            "for n in ((10, 13) if %r else ()):\n"
            "    T.check(runtime, oracle, T.cnot_ring(n, n), n, seed=n)\n"
            "print('host-run-ok')\n") % (root, here, os.path.join(root, "oracle"), rings)
    off = SWITCHES if env == "all" else (env,)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       env=dict(os.environ, **{k: "0" for k in off}), timeout=900)
    assert r.returncode == 0 and "host-run-ok" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_general_bit_positions_run_their_compiled_code_on_host():
    """Default configuration (subprocess, FAST_DIAG on): controlled diagonals, two-qubit
    diagonals, controlled one-target gates and generic slot gradients as compiled pass code, run
    on the CPU against the oracle; every pass of these circuits has a compiled form, and it
    compiles for sm_100a."""
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    code = ("import sys; sys.path[:0] = [%r, %r, %r]\n"
            "import oracle, test_jit_host_run as T\n"
            "from arcqml_b200 import runtime\n"
            "for n, seed in ((9, 1), (12, 2), (13, 3)):\n"
            "    T.check(runtime, oracle, T.general_shapes(n, seed), n, seed=seed, terms=20)\n"
            "T.check(runtime, oracle, T.brickwork_edges(10, 3), 10, seed=3)\n"
            "T.check(runtime, oracle, T.fast_shapes(12, 4), 12, seed=4)\n"
            "p = runtime.CircuitPlan.create(T.general_shapes(13, 5).compile_plan(1))\n"
            "for adj in (False, True):\n"
            "    r = p.jit_check(13, adj)\n"
            "    assert r['eligible'] >= 1 and r['compiled'] == r['eligible'], r\n"
            "print('general-ok')\n") % (root, here, os.path.join(root, "oracle"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       env={k: v for k, v in os.environ.items() if not k.startswith("ARCQML_")},
                       timeout=1200)
    assert r.returncode == 0 and "general-ok" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_all_switches_together_run_their_compiled_code_on_host():
    """The default configuration (all three switches on; subprocess with none set): reordered
    sub-blocks holding CNOT exchanges, controlled gates and generic gradients, run on the CPU
    against the oracle."""
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    code = ("import sys; sys.path[:0] = [%r, %r, %r]\n"
            "import oracle, test_jit_host_run as T\n"
            "from arcqml_b200 import runtime\n"
            "for n, seed in ((10, 21), (13, 22)):\n"
            "    c = T.general_shapes(n, seed)\n"
            "    for q in range(n):\n"
            "        c.append('cnot', (q, (q + 3) %% n))\n"
            "    T.check(runtime, oracle, c, n, seed=seed, terms=15)\n"
            "    T.check(runtime, oracle, T.cnot_ring(n, seed), n, seed=seed)\n"
            "T.check(runtime, oracle, T.brickwork_edges(12, 5), 12, seed=5)\n"
            "print('all-ok')\n") % (root, here, os.path.join(root, "oracle"))
    env = {k: v for k, v in os.environ.items() if not k.startswith("ARCQML_")}
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env,
                       timeout=1200)
    assert r.returncode == 0 and "all-ok" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_one_cta_adjoint_code_runs_on_host():
    """ARCQML_ADJ_2CTA=0 (subprocess): adjoint kernels with one gradient column per thread (the
    default has one per four lanes, accumulate_quad) run on the CPU against the oracle."""
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    code = ("import sys; sys.path[:0] = [%r, %r, %r]\n"
            "import oracle, test_jit_host_run as T\n"
            "from arcqml_b200 import runtime\n"
            "T.check(runtime, oracle, T.brickwork_edges(10, 3), 10, seed=3)\n"
            "T.check(runtime, oracle, T.cnot_ring(13, 13), 13, seed=13)\n"
            "T.check(runtime, oracle, T.general_shapes(12, 2), 12, seed=2, terms=20)\n"
            "print('column-ok')\n") % (root, here, os.path.join(root, "oracle"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       env=dict(os.environ, ARCQML_ADJ_2CTA="0"), timeout=900)
    assert r.returncode == 0 and "column-ok" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.parametrize("n", [10, 13])
def test_merged_adjoint_rotations_run_on_host(runtime, oracle, n):
    """Rotation runs the adjoint passes merge (test_planner_emulation.merge_runs): the compiled
    code of the merged ops and the rows shared by several parameters."""
    from test_planner_emulation import merge_runs
    check(runtime, oracle, merge_runs(n, 40 + n), n, seed=n)


def test_cancelling_rotation_runs_run_on_host(runtime, oracle):
    """Merged runs whose angles cancel (test_planner_emulation.cancel_runs): the compiled code
    of the identity-valued merged rotations."""
    from test_planner_emulation import cancel_runs
    check(runtime, oracle, cancel_runs(10, 62), 10, seed=62)
