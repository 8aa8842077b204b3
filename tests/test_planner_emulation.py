"""The engine's fused-pass schedules run on the CPU (arcqml_rt_v2_plan_emulate) against the
oracle: pass partitioning, tile mapping, op encoding, forward merges, scaled rotation forms and
gradient bookkeeping, checked without a GPU (forward 1e-12, gradients 1e-10)."""
import math

import numpy as np
import pytest

from arcqml_b200 import circuit as cm
from arcqml_b200 import workloads
from plans import random_plan, random_state, random_terms


def check(runtime, oracle, ops, n, terms, init, req, up):
    plan = runtime.CircuitPlan.create(ops)
    psi = runtime.plan_emulate(plan, init, n)
    ref = oracle.plan_apply(ops, init, n)
    assert float(np.max(np.abs(psi - ref))) < 1e-12
    _, lam = oracle.expectation_and_apply(terms, ref, n)
    p0, l0, g = runtime.plan_emulate(plan, psi, n, adjoint=True, lam=up * lam,
                                     requires_grad=req, num_gradients=len(req))
    rp0, rl0, rg = oracle.adjoint_backward(ops, ref, lam, n, up, req, len(req))
    assert float(np.max(np.abs(p0 - init))) < 1e-10
    assert float(np.max(np.abs(l0 - rl0))) <= 1e-10 * max(1.0, float(np.max(np.abs(rl0))))
    assert float(np.max(np.abs(g - rg))) <= 1e-10 * max(1.0, float(np.max(np.abs(rg))))


@pytest.mark.parametrize("n,num_ops", [(8, 150), (10, 200), (13, 160)])
def test_random_plans_over_every_opcode(runtime, oracle, n, num_ops):
    g = np.random.Generator(np.random.PCG64(1000 + n))
    npar = 10
    ops = random_plan(g, n, num_ops, npar)
    req = [0] + [int(x) for x in (g.uniform(size=npar) < 0.8)]
    check(runtime, oracle, ops, n, random_terms(g, n, 20), random_state(g, n), req,
          float(g.normal()))


@pytest.mark.parametrize("n", [9, 12])
def test_brickwork_and_edge_angles(runtime, oracle, n):
    g = np.random.Generator(np.random.PCG64(n))
    c = workloads.brickwork(n, 5, seed=n)
    for q in range(n):  # rotations at and near pi: forms refused or growth capped
        c.rot("ry", math.pi * (1 - 1e-9), q)
        c.rot("rx", math.pi, q)
        c.append("phase", (q,), 3 * math.pi)
    for _ in range(30):
        c.rot("rz", math.pi * (1 - 1e-9), 1)
    ops = c.compile_plan(1)
    req = list(c.requires_grad_mask(True))
    check(runtime, oracle, ops, n, workloads.random_pauli_sum(n, 25, seed=n).compiled_terms(),
          random_state(g, n), req, -0.7)


def test_emulator_rejects_small_states_and_bad_buffers(runtime):
    plan = runtime.CircuitPlan.create(cm.Circuit(4).append("h", (0,)).compile_plan(1))
    with pytest.raises(runtime.RuntimeError, match="below 8 qubits"):
        runtime.plan_emulate(plan, np.zeros(16, np.complex128), 4)


def test_plain_form_schedules_with_scaling_off():
    """ARCQML_SCALED=0 (subprocess): the plain rotation forms and their forward merges into
    dense 2x2s, emulated against the oracle."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    code = ("import sys; sys.path[:0] = [%r, %r, %r]\n"
            "import oracle, test_planner_emulation as T\n"
            "from arcqml_b200 import runtime\n"
            "T.test_brickwork_and_edge_angles(runtime, oracle, 10)\n"
            "print('plain-ok')\n") % (root, here, os.path.join(root, "oracle"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       env=dict(os.environ, ARCQML_SCALED="0"), timeout=600)
    assert r.returncode == 0 and "plain-ok" in r.stdout, r.stdout + r.stderr


def test_reordered_subblocks_emulate_correctly_and_pack_tighter():
    """ARCQML_SUBBLOCK_REORDER=1 (subprocess): commuting gates packed into fewer register
    sub-blocks; the emulated schedules still match the oracle, and the 32-qubit benchmark
    circuit needs fewer sub-blocks than in circuit order."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    code = ("import sys; sys.path[:0] = [%r, %r, %r]\n"
            "import oracle, test_planner_emulation as T\n"
            "from arcqml_b200 import runtime, workloads\n"
            "for n, m in ((8, 150), (10, 200), (13, 160)):\n"
            "    T.test_random_plans_over_every_opcode(runtime, oracle, n, m)\n"
            "for n in (9, 12):\n"
            "    T.test_brickwork_and_edge_angles(runtime, oracle, n)\n"
            "c = workloads.brickwork(32, 20, seed=1234)\n"
            "p = runtime.CircuitPlan.create(c.compile_plan(1))\n"
            "print('blocks', p.schedule_stats(32, False)['sub_blocks'],"
            " p.schedule_stats(32, True)['sub_blocks'])\n") % (
        root, here, os.path.join(root, "oracle"))
    counts = {}
    for on in ("0", "1"):
        env = dict(os.environ, ARCQML_SUBBLOCK_REORDER=on)
        r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                           env=env, timeout=600)
        assert r.returncode == 0, r.stdout + r.stderr
        counts[on] = [int(x) for x in r.stdout.split("blocks")[1].split()]
    assert counts["1"][0] < counts["0"][0] and counts["1"][1] < counts["0"][1], counts


def qnn_like(n, seed):
    """RY / RZ layers, a CNOT ring (controls in registers, thread bits and outside the tile)
    and X gates."""
    g = np.random.Generator(np.random.PCG64(seed))
    c = cm.Circuit(n)
    for _ in range(4):
        for q in range(n):
            c.rot("ry", float(g.uniform(-3, 3)), q)
            c.rot("rz", float(g.uniform(-3, 3)), q)
        for q in range(n):
            c.append("cnot", (q, (q + 1) % n))
        c.append("x", (int(g.integers(0, n)),))
    return c


def check_qnn_like(runtime, oracle):
    for n in (10, 14):
        c = qnn_like(n, n)
        g = np.random.Generator(np.random.PCG64(n + 1))
        check(runtime, oracle, c.compile_plan(1), n, random_terms(g, n, 10),
              random_state(g, n), list(c.requires_grad_mask(True)), 0.9)


def test_fast_cnot_paths_emulate_correctly_and_compile():
    """ARCQML_FAST_CNOT=0 (subprocess; on by default, so the default configuration covers
    X and CNOT as register exchanges): random plans and CNOT-ring circuits match the oracle
    through the emulator, and the 10-qubit CNOT-ring circuit's passes still all have compiled
    forms (through the controlled one-target code) that compile."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    code = ("import sys; sys.path[:0] = [%r, %r, %r]\n"
            "import oracle, test_planner_emulation as T\n"
            "from arcqml_b200 import runtime\n"
            "for n, m in ((8, 150), (10, 200), (13, 160)):\n"
            "    T.test_random_plans_over_every_opcode(runtime, oracle, n, m)\n"
            "T.check_qnn_like(runtime, oracle)\n"
            "p = runtime.CircuitPlan.create(T.qnn_like(10, 3).compile_plan(1))\n"
            "for adj in (False, True):\n"
            "    r = p.jit_check(10, adj)\n"
            "    assert r['eligible'] >= 1 and r['compiled'] == r['eligible'], r\n"
            "print('cnot-ok')\n") % (root, here, os.path.join(root, "oracle"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       env=dict(os.environ, ARCQML_FAST_CNOT="0"), timeout=600)
    assert r.returncode == 0 and "cnot-ok" in r.stdout, r.stdout + r.stderr


def test_cnot_ring_circuits_in_the_default_configuration(runtime, oracle):
    check_qnn_like(runtime, oracle)


@pytest.mark.parametrize("seed", range(6))
def test_random_plan_sweep(runtime, oracle, seed):
    """Random plans over every opcode on 8-16 qubits (every tile size the fused path uses,
    3 and 4 forward register bits), forward and adjoint through the emulated schedules."""
    g = np.random.Generator(np.random.PCG64(9000 + seed))
    n = (8, 9, 11, 12, 14, 16)[seed]
    npar = int(g.integers(3, 12))
    ops = random_plan(g, n, int(g.integers(80, 260)), npar)
    req = [int(g.uniform() < 0.3)] + [int(x) for x in (g.uniform(size=npar) < 0.8)]
    check(runtime, oracle, ops, n, random_terms(g, n, int(g.integers(5, 30))),
          random_state(g, n), req, float(g.normal()))


def test_general_bit_position_schedules_emulate_correctly():
    """ARCQML_FAST_DIAG=0 (subprocess; on by default, where controlled diagonals, two-qubit
    diagonals and controlled one-target gates get their compiled-kernel codes and
    generic-gradient ops keep their plain forms in scaled passes): random plans over every
    opcode and the general-shape circuits match the oracle through the emulated schedules."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    code = ("import sys; sys.path[:0] = [%r, %r, %r]\n"
            "import numpy as np, oracle, test_planner_emulation as T, test_jit_host_run as H\n"
            "from plans import random_state, random_terms\n"
            "from arcqml_b200 import runtime\n"
            "for n, m in ((8, 150), (10, 200), (13, 160)):\n"
            "    T.test_random_plans_over_every_opcode(runtime, oracle, n, m)\n"
            "for n, seed in ((9, 11), (13, 12), (16, 13)):\n"
            "    c = H.general_shapes(n, seed)\n"
            "    g = np.random.Generator(np.random.PCG64(seed))\n"
            "    T.check(runtime, oracle, c.compile_plan(1), n, random_terms(g, n, 15),\n"
            "            random_state(g, n), list(c.requires_grad_mask(True)), -1.3)\n"
            "print('general-ok')\n") % (root, here, os.path.join(root, "oracle"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       env=dict(os.environ, ARCQML_FAST_DIAG="0"), timeout=900)
    assert r.returncode == 0 and "general-ok" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_one_plan_from_many_threads(runtime, oracle):
    """A plan is read-only after it is built (CircuitPlan is Send + Sync in
    crates/arcqml-runtime-sys/src/lib.rs:199-200): eight threads emulate its forward and adjoint
    schedules at the same time, each on its own state, and every result matches the oracle."""
    import threading
    n = 11
    g = np.random.Generator(np.random.PCG64(4242))
    npar = 8
    ops = random_plan(g, n, 180, npar)
    req = [0] + [1] * npar
    plan = runtime.CircuitPlan.create(ops)
    inits = [random_state(g, n) for _ in range(8)]
    terms = random_terms(g, n, 12)
    out = [None] * 8

    def body(t):
        psi = runtime.plan_emulate(plan, inits[t], n)
        _, lam = oracle.expectation_and_apply(terms, psi, n)
        out[t] = (psi, runtime.plan_emulate(plan, psi, n, adjoint=True, lam=lam,
                                            requires_grad=req, num_gradients=len(req)))

    threads = [threading.Thread(target=body, args=(t,)) for t in range(8)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    for t in range(8):
        ref = oracle.plan_apply(ops, inits[t], n)
        psi, (p0, l0, gr) = out[t]
        assert float(np.max(np.abs(psi - ref))) < 1e-12
        _, lam = oracle.expectation_and_apply(terms, ref, n)
        _, rl0, rg = oracle.adjoint_backward(ops, ref, lam, n, 1.0, req, len(req))
        assert float(np.max(np.abs(p0 - inits[t]))) < 1e-10
        assert float(np.max(np.abs(gr - rg))) <= 1e-10 * max(1.0, float(np.max(np.abs(rg))))


def test_custom_unitaries_through_the_circuit_api(runtime, oracle):
    """Circuit.custom_unitary on 1, 2 and 3 qubits (the last runs between fused passes as a
    dense step) inside a trained circuit, through the emulated schedules against the oracle;
    a non-unitary or mis-sized matrix is rejected when appended."""
    from plans import random_unitary
    n = 10
    g = np.random.Generator(np.random.PCG64(515))
    c = cm.Circuit(n)
    for layer in range(3):
        for q in range(n):
            c.rot(("rx", "ry", "rz")[(q + layer) % 3], float(g.uniform(-3, 3)), q)
        c.custom_unitary("u1", random_unitary(g, 1), [int(g.integers(0, n))])
        a, b = (int(x) for x in g.choice(n, size=2, replace=False))
        c.custom_unitary("u2", random_unitary(g, 2), [a, b])
        c.custom_unitary("u3", random_unitary(g, 3), [int(x) for x in g.choice(n, 3, False)])
        c.append("cz", (layer, layer + 1))
    check(runtime, oracle, c.compile_plan(1), n, random_terms(g, n, 10), random_state(g, n),
          list(c.requires_grad_mask(True)), 0.8)
    with pytest.raises(cm.CircuitError, match="not unitary"):
        c.custom_unitary("bad", np.eye(2) * 1.1, [0])
    with pytest.raises(cm.CircuitError, match="expected 16 entries"):
        c.custom_unitary("bad", np.eye(2), [0, 1])


def merge_runs(n, seed):
    """Runs of rotations the adjoint sweep merges, and neighbours that must stop a merge: RX/RY
    pairs on one qubit, RZ runs across CZ and a CNOT control (merged) and across a CNOT target
    or H (not), shared parameters within one run, parameters without gradients, and brickwork
    layers around them."""
    g = np.random.Generator(np.random.PCG64(seed))
    c = workloads.brickwork(n, 2, seed=seed)
    shared = c.add_parameter(0.37)
    frozen = c.add_parameter(-1.1, requires_grad=False)

    def ang():
        return float(g.uniform(-math.pi, math.pi))

    for q in range(n):
        r = (q + 1) % n
        c.rot("rx", ang(), q)
        c.rot("rx", ang(), q)
        c.append("rx", (q,), frozen)
        c.rot("ry", ang(), r)
        c.append("ry", (r,), shared)
        c.append("ry", (r,), shared)
        c.rot("rz", ang(), q)
        c.append("cz", (q, r))
        c.rot("rz", ang(), q)
        c.append("cnot", (q, r))      # q is a control: the RZ run goes on
        c.append("rz", (q,), frozen)
        c.rot("rz", ang(), q)
        c.append("cnot", (r, q))      # q is the target: the RZ run ends
        c.rot("rz", ang(), q)
        c.rot("rx", ang(), r)
        c.append("cz", (r, q))        # touches r: the RX run ends
        c.rot("rx", ang(), r)
        c.append("h", (q,))
        c.rot("rz", ang(), q)
    return c


def adjoint_schedule(runtime, c, n):
    import jit_host_run as J
    plan = runtime.CircuitPlan.create(c.compile_plan(1))
    req = np.asarray(c.requires_grad_mask(True), np.uint8)
    steps = J.parse(runtime.plan_schedule_export(plan, n, True, req))
    return [p for kind, p in steps if kind == "pass"]


@pytest.mark.parametrize("n", [9, 12])
def test_adjoint_rotation_merges_match_oracle(runtime, oracle, n):
    """Adjoint passes merge each rotation into the previous one about the same axis on its
    qubit (one rotation on psi and lambda, one gradient row for both parameters); the sweep
    still returns every gradient, and merged rows reach every parameter they stand for."""
    g = np.random.Generator(np.random.PCG64(70 + n))
    c = merge_runs(n, 70 + n)
    ops = c.compile_plan(1)
    req = list(c.requires_grad_mask(True))
    check(runtime, oracle, ops, n, random_terms(g, n, 20), random_state(g, n), req, 0.9)
    passes = adjoint_schedule(runtime, c, n)
    nops = sum(len(p.ops) // 64 for p in passes)
    assert nops < len(ops) - 3 * n  # every qubit has at least three merges
    assert sum(len(p.alias) for p in passes) >= n
    plan = runtime.CircuitPlan.create(ops)
    fwd = runtime.plan_schedule_summary(plan, n, False)  # forward passes merge the same runs
    assert fwd["ops"] < len(ops) - 3 * n and fwd["aliases"] == 0


def test_rotation_merges_off_emulate_correctly():
    """ARCQML_ROT_MERGE=0 (subprocess): every adjoint rotation keeps its own op and gradient row
    (forward passes still merge one-qubit gates within a register sub-block)."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    code = ("import sys; sys.path[:0] = [%r, %r, %r]\n"
            "import numpy as np, oracle, test_planner_emulation as T\n"
            "from arcqml_b200 import runtime\n"
            "n = 10; c = T.merge_runs(n, 5); g = np.random.Generator(np.random.PCG64(5))\n"
            "T.check(runtime, oracle, c.compile_plan(1), n, T.random_terms(g, n, 20),\n"
            "        T.random_state(g, n), list(c.requires_grad_mask(True)), -0.4)\n"
            "ps = T.adjoint_schedule(runtime, c, n)\n"
            "assert sum(len(p.alias) for p in ps) == 0\n"
            "assert sum(len(p.ops) // 64 for p in ps) == len(c.compile_plan(1))\n"
            "print('merge-off-ok')\n") % (root, here, os.path.join(root, "oracle"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       env=dict(os.environ, ARCQML_ROT_MERGE="0"), timeout=600)
    assert r.returncode == 0 and "merge-off-ok" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_lookahead_tiles_take_fewer_passes(runtime):
    """By default each pass keeps the better of two tile choices, targets in gate order or
    lookahead (each qubit the one whose tile holds the most remaining gates); with
    ARCQML_LOOKAHEAD=0 (subprocess) only the first. The 32-qubit benchmark's schedules take fewer
    passes by default, and the first-come schedules still emulate correctly."""
    import json
    import os
    import subprocess
    import sys
    c = workloads.brickwork(32, 20, seed=1234)
    plan = runtime.CircuitPlan.create(c.compile_plan(1))
    default = [plan.schedule_stats(32, adj)["passes"] for adj in (False, True)]
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    code = ("import sys, json; sys.path[:0] = [%r, %r, %r]\n"
            "import numpy as np, oracle, test_planner_emulation as T\n"
            "from arcqml_b200 import runtime, workloads as W\n"
            "c = W.brickwork(32, 20, seed=1234); p = runtime.CircuitPlan.create(c.compile_plan(1))\n"
            "counts = [p.schedule_stats(32, a)['passes'] for a in (False, True)]\n"
            "T.test_brickwork_and_edge_angles(runtime, oracle, 12)\n"
            "print(json.dumps(counts))\n") % (root, here, os.path.join(root, "oracle"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       env=dict(os.environ, ARCQML_LOOKAHEAD="0"), timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    first_come = json.loads(r.stdout.strip().splitlines()[-1])
    assert default[0] < first_come[0] and default[1] < first_come[1], (default, first_come)


def test_identity_angle_rotations_beside_merged_runs(runtime, oracle):
    """RX / RY at angle 0 are the identity and are emitted as diagonals, so they must not head a
    run that later rotations about the same axis merge into: each qubit gets a CZ, then RX(0) or
    RY(0) as its first one-qubit gate, then rotations about the same axis; forward and adjoint
    against the oracle, with and without gradients on the zero-angle rotations."""
    n = 10
    g = np.random.Generator(np.random.PCG64(37))
    c = cm.Circuit(n)
    for layer in range(4):
        for a in range(layer % 2, n - 1, 2):
            c.append("cz", (a, a + 1))
        for q in range(n):
            axis = ("rx", "ry")[(q + layer) % 2]
            if (q + layer) % 3 == 0:
                c.append(axis, (q,), 0.0)  # a constant identity
            else:
                c.rot(axis, 0.0, q)
            for _ in range(2):
                c.rot(axis, float(g.uniform(-math.pi, math.pi)), q)
            c.rot("rz", float(g.uniform(-math.pi, math.pi)), q)
    ops = c.compile_plan(1)
    check(runtime, oracle, ops, n, random_terms(g, n, 20), random_state(g, n),
          list(c.requires_grad_mask(True)), 0.6)


def test_cached_tile_choices_follow_the_gate_structure(runtime, oracle):
    """A plan keeps the tile qubits its schedules took, keyed by the gates' structure: the same
    schedule again is identical, and new values that change the structure (rotations set to 0
    become diagonals) are planned afresh; forward and adjoint of the changed plan against the
    oracle."""
    n = 12
    g = np.random.Generator(np.random.PCG64(55))
    c = workloads.brickwork(n, 5, seed=55)
    ops = c.compile_plan(1)
    req = list(c.requires_grad_mask(True))
    plan = runtime.CircuitPlan.create(ops)
    for adjoint in (False, True):
        a = runtime.plan_schedule_export(plan, n, adjoint, req if adjoint else None)
        b = runtime.plan_schedule_export(plan, n, adjoint, req if adjoint else None)
        assert a == b
    vals = np.array([p.f64() for p in c.parameters])
    vals[::3] = 0.0
    c.set_parameter_values(vals)
    plan.set_parameters(np.concatenate([[0.0], vals]))
    ops2 = c.compile_plan(1)
    init = random_state(g, n)
    psi = runtime.plan_emulate(plan, init, n)
    ref = oracle.plan_apply(ops2, init, n)
    assert float(np.max(np.abs(psi - ref))) < 1e-12
    _, lam = oracle.expectation_and_apply(random_terms(g, n, 15), ref, n)
    p0, l0, grads = runtime.plan_emulate(plan, psi, n, adjoint=True, lam=lam,
                                         requires_grad=req, num_gradients=len(req))
    _, rl0, rg = oracle.adjoint_backward(ops2, ref, lam, n, 1.0, req, len(req))
    assert float(np.max(np.abs(p0 - init))) < 1e-10
    assert float(np.max(np.abs(grads - rg))) <= 1e-10 * max(1.0, float(np.max(np.abs(rg))))


def cancel_runs(n, seed):
    """Same-axis runs whose angles cancel (RY(a) RY(-a), RX(a) RX(-a)) after a CZ layer, then a
    further rotation about that axis and an RZ, on every qubit."""
    g = np.random.Generator(np.random.PCG64(seed))
    c = cm.Circuit(n)
    for layer in range(4):
        for a in range(layer % 2, n - 1, 2):
            c.append("cz", (a, a + 1))
        for q in range(n):
            axis = ("rx", "ry")[(q + layer) % 2]
            t = float(g.uniform(-math.pi, math.pi))
            c.rot(axis, t, q)
            c.rot(axis, -t, q)
            c.rot(axis, float(g.uniform(-math.pi, math.pi)), q)
            c.rot("rz", float(g.uniform(-math.pi, math.pi)), q)
    return c


def test_rotation_runs_that_cancel(runtime, oracle):
    """Runs whose angles cancel merge into the identity, which is still a rotation of the run's
    axis for the rotations merged after it; forward and adjoint against the oracle."""
    n = 9
    g = np.random.Generator(np.random.PCG64(61))
    c = cancel_runs(n, 61)
    check(runtime, oracle, c.compile_plan(1), n, random_terms(g, n, 15), random_state(g, n),
          list(c.requires_grad_mask(True)), -0.8)


def edge_family(n, seed):
    """Random layers of rotations about random axes, 40 % of them at edge angles (0, pi, -pi,
    pi (1 - 1e-9), 1e-300, 2 pi), some with constant angles, phase and X-type gates, then CZ or
    CNOT between neighbours: the circuits in which the merge and form edge cases turned up."""
    g = np.random.Generator(np.random.PCG64(seed))
    c = cm.Circuit(n)
    angles = (0.0, math.pi, -math.pi, math.pi * (1 - 1e-9), 1e-300, 2 * math.pi)
    for layer in range(int(g.integers(3, 8))):
        for q in range(n):
            for _ in range(int(g.integers(1, 4))):
                axis = ("rx", "ry", "rz")[int(g.integers(0, 3))]
                a = angles[int(g.integers(0, len(angles)))] if g.uniform() < 0.4 \
                    else float(g.uniform(-3, 3))
                if g.uniform() < 0.2:
                    c.append(axis, (q,), a)
                else:
                    c.rot(axis, a, q)
            if g.uniform() < 0.2:
                c.append(("s", "t", "h", "x", "sdg")[int(g.integers(0, 5))], (q,))
        for a in range(layer % 2, n - 1, 2):
            r = g.uniform()
            c.append("cz" if r < 0.6 else "cnot", (a, a + 1) if r < 0.8 else (a + 1, a))
    return c


@pytest.mark.parametrize("seed", [5, 6, 17, 33, 64, 72, 73, 98])
def test_edge_family_sweep(runtime, oracle, seed):
    """Seeded circuits of the edge family, forward and adjoint against the oracle (in all but
    seed 6 a merged run of rotations that cancel made the planner fail before it tested the
    run's own axis form)."""
    g = np.random.Generator(np.random.PCG64(1000 + seed))
    n = int(g.integers(9, 14))
    c = edge_family(n, seed)
    check(runtime, oracle, c.compile_plan(1), n, random_terms(g, n, 15), random_state(g, n),
          list(c.requires_grad_mask(True)), float(g.normal()))
