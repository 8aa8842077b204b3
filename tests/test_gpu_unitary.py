"""Whole-circuit unitaries and unitary fitting on the device against the oracle backend (needs
a B200): the [D, D] basis batch through plan_apply, the trace overlap from per-row overlaps, the
fit gradient through scaled_copy and the batched adjoint sweep; per-gate (3 and 5 qubits) and
fused (9 qubits) paths."""
import math

import numpy as np
import pytest

from arcqml_b200 import circuit as cm
from arcqml_b200 import unitary as U
from unitary_support import OracleUnitaryBackend

pytestmark = pytest.mark.gpu


def random_circuit(g, n, layers, trained=True):
    c = cm.Circuit(n)
    for layer in range(layers):
        for q in range(n):
            name = ("rx", "ry", "rz")[int(g.integers(0, 3))]
            v = float(g.uniform(-math.pi, math.pi))
            if trained:
                c.rot(name, v, q)
            else:
                c.append(name, (q,), v)
        for a in range(layer % 2, n - 1, 2):
            c.append("cz", (a, a + 1))
        if n > 2:
            c.append("cry", (n - 1, 0), c.add_parameter(float(g.uniform(-3, 3))) if trained
                     else float(g.uniform(-3, 3)))
    return c


@pytest.mark.parametrize("n", [3, 5, 9])
def test_unitary_fit_on_device_matches_oracle(runtime, oracle, n):
    g = np.random.Generator(np.random.PCG64(50 + n))
    ob = OracleUnitaryBackend(oracle)
    target_circuit = random_circuit(g, n, 2, trained=False)
    c = random_circuit(g, n, 3)
    t_dev = U.unitary_from_circuit(target_circuit)
    t_ref = U.unitary_from_circuit(target_circuit, ob)
    assert float(np.max(np.abs(t_dev.as_row_major() - t_ref.as_row_major()))) < 1e-12
    loss = U.unitary_loss(t_ref, c)
    ref = U.unitary_loss(t_ref, c, ob)
    assert abs(loss.value - ref.value) <= 1e-10
    assert abs(loss.overlap - ref.overlap) <= 1e-10 * max(1.0, abs(ref.overlap))
    g_dev = loss.backward(0.75)
    for p in c.parameters:
        p.grad = None
    g_ref = ref.backward(0.75)
    assert float(np.max(np.abs(g_dev - g_ref))) <= 1e-10 * max(1.0, float(np.max(np.abs(g_ref))))


def test_reference_fit_cases_on_device(runtime):
    # crates/arcqml-unitary/tests/fit_tests.rs:29-79 and dense_tests.rs:13-49
    phase = complex(math.cos(0.37), math.sin(0.37))
    target = U.DenseUnitary.from_row_major([phase, 0, 0, phase], 2)
    assert abs(U.unitary_fidelity(target, cm.Circuit(1)) - 1.0) < 1e-8
    ry = cm.Circuit(1)
    ry.append("ry", (0,), 0.8)
    target = U.unitary_from_circuit(ry)
    c = cm.Circuit(1)
    c.rot("ry", 0.2, 0)
    grad = U.unitary_loss(target, c).backward()[0]
    eps = 1e-6
    c.set_parameter_values([0.2 + eps])
    plus = U.unitary_loss_value(target, c)
    c.set_parameter_values([0.2 - eps])
    minus = U.unitary_loss_value(target, c)
    assert abs(grad - (plus - minus) / (2 * eps)) < 1e-8
    cx = U.unitary_from_circuit(cm.Circuit(2).append("cnot", (0, 1)))
    want = [1, 0, 0, 0, 0, 0, 0, 1, 0, 0, 1, 0, 0, 1, 0, 0]
    assert float(np.max(np.abs(cx.as_row_major() - np.array(want)))) < 1e-12
