"""arcqml_b200.unitary on CPU through the oracle backend, pinned by the reference's own tests
(crates/arcqml-unitary/tests/fit_tests.rs and dense_tests.rs; tolerances as there: 1e-8 for the
fit, 1e-12 for matrices)."""
import math

import numpy as np
import pytest

from arcqml_b200 import circuit as cm
from arcqml_b200 import unitary as U
from unitary_support import OracleUnitaryBackend


@pytest.fixture
def be(oracle):
    return OracleUnitaryBackend(oracle)


def fixed(name, theta, q=0, n=1):
    c = cm.Circuit(n)
    c.append(name, (q,), float(theta))
    return c


def ry_target(theta, be):
    return U.unitary_from_circuit(fixed("ry", theta), be)


def two_gate_target(ry, rz, be):
    c = fixed("ry", ry)
    c.append("rz", (0,), float(rz))
    return U.unitary_from_circuit(c, be)


def test_loss_ignores_global_phase(be):
    # fit_tests.rs:29-47
    phase = complex(math.cos(0.37), math.sin(0.37))
    target = U.DenseUnitary.from_row_major([phase, 0, 0, phase], 2)
    c = cm.Circuit(1)
    assert abs(U.unitary_fidelity(target, c, be) - 1.0) < 1e-8
    assert abs(U.unitary_loss_value(target, c, be)) < 1e-8


def central_difference(target, c, index, value, be, eps=1e-6):
    vals = c.parameter_values().copy()
    vals[index] = value + eps
    c.set_parameter_values(vals)
    plus = U.unitary_loss_value(target, c, be)
    vals[index] = value - eps
    c.set_parameter_values(vals)
    minus = U.unitary_loss_value(target, c, be)
    vals[index] = value
    c.set_parameter_values(vals)
    return (plus - minus) / (2 * eps)


def test_analytic_gradient_matches_central_difference(be):
    # fit_tests.rs:49-79
    target = ry_target(0.8, be)
    c = cm.Circuit(1)
    c.rot("ry", 0.2, 0)
    loss = U.unitary_loss(target, c, be)
    loss.backward()
    assert abs(c.parameters[0].grad - central_difference(target, c, 0, 0.2, be)) < 1e-8


def test_gradients_of_several_gates(be):
    # fit_tests.rs:81-117
    target = two_gate_target(0.8, -0.3, be)
    c = cm.Circuit(1)
    c.rot("ry", 0.2, 0)
    c.rot("rz", 0.1, 0)
    grads = U.unitary_loss(target, c, be).backward()
    for i, v in enumerate([0.2, 0.1]):
        assert abs(grads[i] - central_difference(target, c, i, v, be)) < 1e-8


def test_rejects_mismatched_qubit_counts(be):
    # fit_tests.rs:119-131
    with pytest.raises(U.UnitaryError, match="target has 1 qubits but circuit has 2 qubits"):
        U.unitary_loss(ry_target(0.0, be), cm.Circuit(2), be)


def test_loss_value_and_upstream_scaling(be):
    # fit_tests.rs:133-190
    target = ry_target(0.8, be)
    c = cm.Circuit(1)
    c.rot("ry", 0.2, 0)
    loss = U.unitary_loss(target, c, be)
    assert abs(loss.value - U.unitary_loss_value(target, c, be)) < 1e-8
    g1 = loss.backward()[0]
    c.parameters[0].grad = None
    g2 = U.unitary_loss(target, c, be).backward(2.5)[0]
    assert abs(g2 - 2.5 * g1) < 1e-8
    with pytest.raises(U.UnitaryError, match="already run"):
        loss.backward()


def test_hadamard_and_little_endian_cnot_matrices(be):
    # dense_tests.rs:13-49
    s = 1 / math.sqrt(2)
    h = U.unitary_from_circuit(cm.Circuit(1).append("h", (0,)), be)
    assert h.dimension == 2
    assert np.max(np.abs(h.as_row_major() - np.array([s, s, s, -s]))) < 1e-12
    cx = U.unitary_from_circuit(cm.Circuit(2).append("cnot", (0, 1)), be)
    want = [1, 0, 0, 0, 0, 0, 0, 1, 0, 0, 1, 0, 0, 1, 0, 0]
    assert np.max(np.abs(cx.as_row_major() - np.array(want))) < 1e-12


def test_dense_unitary_construction_and_validation():
    # dense_tests.rs:51-123 and the checks of dense/unitary.rs, dense/validate.rs
    s = 1 / math.sqrt(2)
    h = U.unitary_from_matrix([[s, s], [s, -s]])
    assert h.num_qubits == 1 and h == U.DenseUnitary.from_row_major([s, s, s, -s], 2)
    with pytest.raises(U.UnitaryError, match="matrix is not unitary"):
        U.unitary_from_matrix([[1, 1], [0, 1]])
    with pytest.raises(U.UnitaryError, match="nonzero power of two, got 3"):
        U.DenseUnitary.from_row_major([1] * 9, 3)
    with pytest.raises(U.UnitaryError, match="length mismatch: expected 4, got 3"):
        U.DenseUnitary.from_row_major([1, 0, 0], 2)
    with pytest.raises(U.UnitaryError, match="non-finite"):
        U.DenseUnitary.from_row_major([1, 0, 0, float("nan")], 2)
    with pytest.raises(U.UnitaryError, match="square rank-2"):
        U.unitary_from_matrix(np.zeros((2, 4)))
    with pytest.raises(U.UnitaryError, match="tolerance must be finite"):
        h.validate(-1.0)


def test_random_circuit_gradients_match_central_differences(be):
    g = np.random.Generator(np.random.PCG64(11))
    n = 3
    c = cm.Circuit(n)
    for layer in range(2):
        for q in range(n):
            c.rot(("rx", "ry", "rz")[int(g.integers(0, 3))], float(g.uniform(-3, 3)), q)
        c.append("cz", (layer % 2, layer % 2 + 1))
        c.append("crx", (2, 0), c.add_parameter(float(g.uniform(-3, 3))))
    t = cm.Circuit(n)
    for q in range(n):
        t.append("ry", (q,), float(g.uniform(-3, 3)))
    t.append("cnot", (0, 2))
    target = U.unitary_from_circuit(t, be)
    grads = U.unitary_loss(target, c, be).backward()
    vals = c.parameter_values()
    for i in range(len(vals)):
        assert abs(grads[i] - central_difference(target, c, i, vals[i], be)) < 1e-8
