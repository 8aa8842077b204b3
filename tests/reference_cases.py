"""The reference's own known-answer tests for the statevector path, restated once.

Each ``case_*`` function takes a backend (``backends.OracleBackend`` or
``backends.RuntimeBackend``) and asserts the reference test's expectation with the reference's
tolerance. Sources (paths inside the ArcQML project) are cited per case.
"""
from __future__ import annotations

import json
import math
import os

import numpy as np

from backends import op

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

X, H, S, RX, RY, RZ, CNOT, CRY, SWAP = 1, 4, 5, 11, 12, 13, 16, 24, 26


def close(a, b, tol):
    assert np.max(np.abs(np.asarray(a) - np.asarray(b))) < tol, (a, b)


def case_x_gate_in_place(be):
    """crates/arcqml-kernel/tests/kernel_tests.rs:15-22"""
    a = be.apply_gate(np.array([1, 0], np.complex128), 1, op(X, [0]))
    close(a, [0, 1], 1e-12)


def case_adjoint_reverses_phase_gate(be):
    """kernel_tests.rs:92-100"""
    a = be.apply_gate(np.array([0, 1], np.complex128), 1, op(S, [0]))
    a = be.apply_gate(a, 1, op(S, [0]), adjoint=True)
    close(a, [0, 1], 1e-12)


def case_rotation_derivative_central_difference(be):
    """kernel_tests.rs:115-168: d/dtheta of RX/RY/RZ on every wire of 3 qubits."""
    k = json.load(open(os.path.join(GOLDEN, "kernel_kats.json")))["rotation_derivative"]
    inp = np.array([complex(a, b) for a, b in k["input"]])
    theta, eps = k["theta"], k["epsilon"]
    for code in (RX, RY, RZ):
        for wire in range(3):
            actual = be.parameter_derivative(inp, 3, op(code, [wire], [theta]), 0)
            plus = be.apply_gate(inp, 3, op(code, [wire], [theta + eps]))
            minus = be.apply_gate(inp, 3, op(code, [wire], [theta - eps]))
            close(actual, (plus - minus) / (2 * eps), k["tolerance"])


def case_batch_ry_rows(be):
    """kernel_tests.rs:171-191 (each row of a [2, 2] batch)."""
    rows = [np.array([1, 0], np.complex128), np.array([0, 1], np.complex128)]
    expect = [[0, 1], [-1, 0]]
    for r, e in zip(rows, expect):
        a = be.apply_gate(r, 1, op(RY, [0], [math.pi]))
        close(a, e, 1e-12)
        close(be.apply_gate(a, 1, op(RY, [0], [math.pi]), adjoint=True), r, 1e-12)


def case_batch_cnot_little_endian(be):
    """kernel_tests.rs:194-219: CNOT(0 -> 1); row |01> -> |11>, row |10> unchanged."""
    r0 = np.zeros(4, np.complex128); r0[1] = 1
    r1 = np.zeros(4, np.complex128); r1[2] = 1
    close(be.apply_gate(r0, 2, op(CNOT, [0, 1]))[3], 1, 1e-12)
    close(be.apply_gate(r1, 2, op(CNOT, [0, 1]))[2], 1, 1e-12)


def case_mixed_pauli_observable(be):
    """crates/arcqml-observable/tests/compiled_hamiltonian_tests.rs:13-41"""
    s = 1 / math.sqrt(2)
    state = np.array([s, 1j * s])
    terms = [(0.5, 0, 0, 0), (2.0, 1, 0, 0), (-3.0, 1, 1, 1), (4.0, 0, 1, 0)]
    v, hpsi = be.expectation_and_apply(terms, state, 1)
    close(v, -2.5, 1e-12)
    close(hpsi, [complex(1.5 * s, 2.0 * s), complex(2.0 * s, -6.5 * s)], 1e-12)


def _run(be, ops, init, n, terms, upstream, req, ng):
    psi = be.plan_apply(ops, init, n)
    v, lam = be.expectation_and_apply(terms, psi, n)
    psi0, lam0, g = be.adjoint_backward(ops, psi, lam, n, upstream, req, ng)
    return v, g, 2.0 * lam0, psi0


def case_single_run_shared_parameter(be):
    """crates/arcqml-sim/tests/run_tests.rs:55-100: RY(t) RY(t) on [cos a, sin a], <Z>."""
    a, t = 0.31, -0.27
    z = [(1.0, 0, 1, 0)]

    def single(angle, theta):
        init = np.array([math.cos(angle), math.sin(angle)], np.complex128)
        return be.expectation_and_apply(z, be.plan_apply([op(RY, [0], [theta])], init, 1), 1)[0]

    ops = [op(RY, [0], [t], bindings=[(0, 1)]), op(RY, [0], [t], bindings=[(0, 1)])]
    init = np.array([math.cos(a), math.sin(a)], np.complex128)
    v, g, init_grad, psi0 = _run(be, ops, init, 1, z, 1.0, [1, 1], 2)
    close(v, math.cos(2 * a + 2 * t), 1e-6)
    close(g[1], -2 * math.sin(2 * a + 2 * t), 1e-6)
    close(psi0, init, 1e-10)  # the sweep restores psi_0
    direction = np.array([-math.sin(a), math.cos(a)])
    analytic = float(np.sum((np.conj(init_grad) * direction).real))
    eps = 1e-6
    numeric = (single(a + eps, 2 * t) - single(a - eps, 2 * t)) / (2 * eps)
    close(analytic, numeric, 1e-6)


def _generic_circuit(theta, phi, bind=True):
    b = (lambda s, p: [(s, p)]) if bind else (lambda s, p: [])
    return [op(H, [0]), op(RY, [0], [theta], bindings=b(0, 1)),
            op(CRY, [0, 1], [phi], bindings=b(0, 2)), op(SWAP, [0, 1]),
            op(RY, [1], [theta], bindings=b(0, 1))]


X1 = [(1.0, 2, 0, 0)]


def case_batch_run_generic_gates(be):
    """run_tests.rs:147-238: H, RY(t), CRY(p), SWAP, RY(t); <X1>; loss 0.43 v0 - 0.29 v1."""
    angles, t, p = [0.19, -0.34], 0.23, -0.41
    w = [0.43, -0.29]

    def rows(ang):
        return [np.array([math.cos(x), math.sin(x), 0, 0], np.complex128) for x in ang]

    def loss(ang, tt, pp):
        return sum(wi * be.expectation_and_apply(X1, be.plan_apply(_generic_circuit(tt, pp, False), r, 2), 2)[0]
                   for wi, r in zip(w, rows(ang)))

    g = np.zeros(3)
    init_grads = []
    for wi, r in zip(w, rows(angles)):
        _, gr, ig, _ = _run(be, _generic_circuit(t, p), r, 2, X1, wi, [1, 1, 1], 3)
        g += gr
        init_grads.append(ig)
    eps = 1e-6
    close(g[1], (loss(angles, t + eps, p) - loss(angles, t - eps, p)) / (2 * eps), 1e-6)
    close(g[2], (loss(angles, t, p + eps) - loss(angles, t, p - eps)) / (2 * eps), 1e-6)
    analytic = 0.0
    for x, ig in zip(angles, init_grads):
        d = np.array([-math.sin(x), math.cos(x), 0, 0])
        analytic += float(np.sum((np.conj(ig) * d).real))
    numeric = (loss([x + eps for x in angles], t, p) - loss([x - eps for x in angles], t, p)) / (2 * eps)
    close(analytic, numeric, 1e-6)


def case_batch_adjoint_matches_gatewise(be):
    """crates/arcqml-sim/tests/row_major_batch_tests.rs:73-149, tolerance 1e-10.

    The gatewise side keeps every intermediate state and back-propagates through per-gate
    nodes (crates/arcqml-sim/src/statevector/execution/gatewise/single.rs:89-190): the
    expectation node sends 2 g H psi, each gate node sends U^dag grad and adds
    Re<grad|dU psi_in> to its parameter.
    """
    rows = [np.array([1, 0, 0, 0], np.complex128), np.array([0, 0, 0, 1], np.complex128),
            np.array([0.8, 0.6j, 0, 0], np.complex128)]
    w = [0.43, -0.29, 0.17]
    t, p = 0.23, -0.41
    ops = _generic_circuit(t, p)
    g_adj = np.zeros(3)
    g_gw = np.zeros(3)
    for wi, r in zip(w, rows):
        v, gr, ig, _ = _run(be, ops, r, 2, X1, wi, [1, 1, 1], 3)
        g_adj += gr
        # gatewise
        states = [r]
        for o in ops:
            states.append(be.apply_gate(states[-1], 2, o))
        v_gw, hpsi = be.expectation_and_apply(X1, states[-1], 2)
        close(v, v_gw, 1e-10)
        grad = 2.0 * wi * hpsi
        for k in range(len(ops) - 1, -1, -1):
            o = ops[k]
            for slot, parent in o.bindings:
                d = be.parameter_derivative(states[k], 2, o, slot)
                g_gw[parent] += float(np.sum((np.conj(grad) * d).real))
            grad = be.apply_gate(grad, 2, o, adjoint=True)
        close(ig, grad, 1e-10)
    close(g_adj[1:], g_gw[1:], 1e-10)


def case_python_single_training_step(be):
    """python/tests/test_single.py:12-31: RY(pi/3) on |0>, <Z> = 0.5, mse vs 0 = 0.125,
    d loss / d theta = -sqrt(3)/4 (12 decimal places)."""
    ops = [op(RY, [0], [math.pi / 3], bindings=[(0, 1)])]
    init = np.array([1, 0], np.complex128)
    psi = be.plan_apply(ops, init, 1)
    v, lam = be.expectation_and_apply([(1.0, 0, 1, 0)], psi, 1)
    loss = 0.5 * v * v
    _, _, g = be.adjoint_backward(ops, psi, lam, 1, v, [0, 1], 2)
    close(v, 0.5, 1e-12)
    close(loss, 0.125, 1e-12)
    close(g[1], -math.sqrt(3) / 4, 1e-12)


def h2_problem():
    d = json.load(open(os.path.join(GOLDEN, "h2_vqe.json")))
    from arcqml_b200.observable import SparsePauliOp

    ham = SparsePauliOp.from_json(json.dumps(d["hamiltonian"]))
    return d, ham.compiled_terms()


def h2_ops(d, values):
    a = d["ansatz"]
    n = a["num_qubits"]
    ops = [op(X, [q]) for q in range(a["active_electrons"])]
    k = 0
    for _ in range(a["layers"]):
        for q in range(n):
            ops.append(op(RY, [q], [values[k]], bindings=[(0, k + 1)]))
            ops.append(op(RZ, [q], [values[k + 1]], bindings=[(0, k + 2)]))
            k += 2
        for q in range(n):
            ops.append(op(CNOT, [q, (q + 1) % n]))
    return ops


def case_h2_vqe_trajectory(be, oracle_adam):
    """examples/rust/h2_vqe.rs:14-92 with the energies of docs/tutorial/h2_vqe.md:499-501."""
    d, terms = h2_problem()
    a = d["ansatz"]
    n = a["num_qubits"]
    npar = 2 * n * a["layers"]
    amp, freq = a["initial_angle"]["amplitude"], a["initial_angle"]["frequency"]
    values = np.array([amp * math.sin(freq * (k + 1)) for k in range(npar)])
    adam = d["adam"]
    state = {}
    init = np.zeros(1 << n, np.complex128); init[0] = 1
    energies = {}
    for step in range(1, a["steps"] + 1):
        ops = h2_ops(d, values)
        psi = be.plan_apply(ops, init, n)
        _, lam = be.expectation_and_apply(terms, psi, n)
        _, _, g = be.adjoint_backward(ops, psi, lam, n, 1.0, [0] + [1] * npar, npar + 1)
        values = oracle_adam(values, g[1:], state, lr=adam["lr"], beta1=adam["beta1"],
                             beta2=adam["beta2"], eps=adam["eps"], weight_decay=adam["weight_decay"])
        if str(step) in d["energy_after_step"]:
            psi = be.plan_apply(h2_ops(d, values), init, n)
            energies[str(step)] = be.expectation_and_apply(terms, psi, n)[0]
    for step, kat in d["energy_after_step"].items():
        # printed with 12 decimals: the true value lies within 5e-13 of the printed one
        close(energies[step], kat["energy"], 1e-12)


ALL_CASES = [
    case_x_gate_in_place, case_adjoint_reverses_phase_gate,
    case_rotation_derivative_central_difference, case_batch_ry_rows,
    case_batch_cnot_little_endian, case_mixed_pauli_observable,
    case_single_run_shared_parameter, case_batch_run_generic_gates,
    case_batch_adjoint_matches_gatewise, case_python_single_training_step,
]
