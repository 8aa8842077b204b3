"""The oracle's analysis restatement (crates/arcqml-analysis/src/statevector) and the adjoint
cotangents of each analysis output, pinned by the reference's own tests
(crates/arcqml-analysis/tests/statevector_analysis.rs, tolerance 1e-12 as there).

Cotangents (lambda for grads += 2 Re<lambda| dU |psi> of the adjoint sweep):
* probabilities with upstream g[i]:            lambda_i = g[i] psi_i
* marginal probabilities with upstream g[m]:   lambda_i = g[m(i)] psi_i
* complex upstream g on the amplitudes:        lambda = g / 2
* fidelity |<a|psi>|^2 (psi differentiated):   lambda = <a|psi> a
"""
import math

import numpy as np
import pytest

from arcqml_b200 import circuit as cm

TOL = 1e-12
S = 1.0 / math.sqrt(2.0)
BELL = np.array([S, 0, 0, S], np.complex128)


def test_probabilities_and_marginals_like_reference(oracle):
    # statevector_analysis.rs:76-89
    assert np.allclose(oracle.probabilities(BELL, 2), [0.5, 0, 0, 0.5], atol=TOL, rtol=0)
    assert np.allclose(oracle.marginal_probabilities(BELL, 2, [0]), [0.5, 0.5], atol=TOL, rtol=0)
    assert np.allclose(oracle.marginal_probabilities(BELL, 2, [0, 1]), [0.5, 0, 0, 0.5],
                       atol=TOL, rtol=0)


def test_marginal_output_order_is_descending_qubits():
    # marginal.rs:9-11: selecting [0, 2] lists q2q0 = 00, 01, 10, 11
    import oracle as O
    for idx in range(8):
        a = np.zeros(8, np.complex128)
        a[idx] = 1.0
        m = O.marginal_probabilities(a, 3, [0, 2])
        want = ((idx >> 2) & 1) << 1 | (idx & 1)
        assert np.array_equal(m, np.eye(4)[want])
        assert np.array_equal(O.marginal_probabilities(a, 3, [2, 0]), m)


def test_fidelity_and_bloch_like_reference(oracle):
    # statevector_analysis.rs:92-107
    zero = np.array([1, 0, 0, 0], np.complex128)
    assert abs(oracle.overlap_fidelity(BELL, BELL, 2)[1] - 1.0) < TOL
    assert abs(oracle.overlap_fidelity(BELL, zero, 2)[1] - 0.5) < TOL
    assert np.allclose(oracle.bloch_vector(np.array([S, S], np.complex128), 1, 0), [1, 0, 0],
                       atol=TOL, rtol=0)


def test_marginal_selection_errors(oracle):
    # statevector_analysis.rs:183-199 (empty, duplicate, out of range)
    for sel in ([], [0, 0], [2]):
        with pytest.raises(ValueError):
            oracle.marginal_probabilities(BELL, 2, sel)
    with pytest.raises(ValueError):
        oracle.bloch_vector(BELL, 2, 2)


def bloch_reference(a, n, q):
    """<X_q>, <Y_q>, <Z_q> from dense Pauli matrices."""
    X = np.array([[0, 1], [1, 0]]); Y = np.array([[0, -1j], [1j, 0]]); Z = np.diag([1, -1])
    out = []
    for P in (X, Y, Z):
        op = np.array([[1.0]])
        for k in reversed(range(n)):
            op = np.kron(op, P if k == q else np.eye(2))
        out.append(float(np.vdot(a, op @ a).real))
    return out


def test_bloch_and_overlap_on_random_states(oracle):
    g = np.random.Generator(np.random.PCG64(3))
    n = 4
    a = g.normal(size=16) + 1j * g.normal(size=16)
    a /= np.linalg.norm(a)
    b = g.normal(size=16) + 1j * g.normal(size=16)
    b /= np.linalg.norm(b)
    for q in range(n):
        assert np.allclose(oracle.bloch_vector(a, n, q), bloch_reference(a, n, q), atol=TOL)
    s, f = oracle.overlap_fidelity(a, b, n)
    assert abs(s - np.vdot(a, b)) < TOL and abs(f - abs(np.vdot(a, b)) ** 2) < TOL


def run_grad(oracle, c, lam_of_psi):
    ops = c.compile_plan(1)
    n = c.num_qubits
    init = np.zeros(1 << n, np.complex128)
    init[0] = 1.0
    psi = oracle.plan_apply(ops, init, n)
    req = c.requires_grad_mask(True)
    _, _, g = oracle.adjoint_backward(ops, psi, lam_of_psi(psi), n, 1.0, req, len(req))
    return g[1]


def ry_circuit(theta, entangle=False):
    c = cm.Circuit(2 if entangle else 1)
    c.rot("ry", theta, 0)
    if entangle:
        c.append("cnot", (0, 1))
    return c


def test_cotangents_reproduce_reference_gradients(oracle):
    t = 0.4
    # amplitudes with complex upstream (0, 1): 0.5 cos(t / 2)   (statevector_analysis.rs:111-129)
    up = np.array([0, 1], np.complex128)
    assert abs(run_grad(oracle, ry_circuit(t), lambda p: up / 2) - 0.5 * math.cos(t / 2)) < TOL
    # probabilities with upstream (0, 1): 0.5 sin(t)   (:133-142)
    g = np.array([0.0, 1.0])
    assert abs(run_grad(oracle, ry_circuit(t), lambda p: g * p) - 0.5 * math.sin(t)) < TOL

    # marginal of qubit 1 after RY(t) q0, CNOT 0->1, upstream (0, 1): 0.5 sin(t)   (:144-148)
    def marg(p):
        m = np.array([(i >> 1) & 1 for i in range(4)])
        return g[m] * p
    assert abs(run_grad(oracle, ry_circuit(t, True), marg) - 0.5 * math.sin(t)) < TOL
    # fidelity with the target RY(0.8)|0>: value cos^2((t - 0.8) / 2), gradient -0.5 sin(t - 0.8)
    t, phi = 0.2, 0.8   # (:151-180)
    target = np.array([math.cos(phi / 2), math.sin(phi / 2)], np.complex128)
    ops = ry_circuit(t).compile_plan(1)
    psi = oracle.plan_apply(ops, np.array([1, 0], np.complex128), 1)
    assert abs(oracle.overlap_fidelity(psi, target, 1)[1] - math.cos((t - phi) / 2) ** 2) < TOL

    def fid(p):
        s, _ = oracle.overlap_fidelity(target, p, 1)   # <a|psi>
        return s * target
    assert abs(run_grad(oracle, ry_circuit(t), fid) + 0.5 * math.sin(t - phi)) < TOL
