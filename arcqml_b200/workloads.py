"""Seeded synthetic workloads with the shapes of the benchmark configurations.

No public dataset or benchmark suite is involved: every circuit, observable and input state is
drawn here from numpy ``Generator(PCG64(seed))``.

* ``vqe4``      — 4-qubit VQE: 2 x [RY on every qubit, CNOT chain 0->1->2->3], 8 angles
                  U[-pi, pi]; 15-term observable with the term shapes of the reference's H2
                  fixture (I, Z_i, Z_iZ_j, four XXYY-type strings), coefficients N(0, 0.5).
* ``qnn``       — batched QNN: rows (x) RY(pi x_q)|0>, x ~ U[0,1]^n; L x [RY, RZ per qubit,
                  CNOT ring]; observable Z0; labels in {-1, +1} with P(+1) = 0.3.
* ``brickwork`` — L layers; layer l: two rotations per qubit with axes uniform in {X, Y, Z} and
                  angles U[-pi, pi], then CZ on pairs (2j + l%2, 2j + 1 + l%2).
* ``random_pauli_sum`` — T terms of weight U{1..4} on distinct random qubits, Paulis uniform in
                  {X, Y, Z}, coefficients N(0, 1).
"""
from __future__ import annotations

import math

import numpy as np

from .circuit import Circuit
from .observable import SparsePauliOp


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def brickwork(num_qubits: int, layers: int, seed: int = 1234) -> Circuit:
    g = rng(seed)
    c = Circuit(num_qubits)
    axes = ("rx", "ry", "rz")
    for layer in range(layers):
        for q in range(num_qubits):
            for _ in range(2):
                axis = axes[int(g.integers(0, 3))]
                c.rot(axis, float(g.uniform(-math.pi, math.pi)), q)
        off = layer % 2
        for a in range(off, num_qubits - 1, 2):
            c.append("cz", (a, a + 1))
    return c


def random_pauli_sum(num_qubits: int, num_terms: int, seed: int = 4321) -> SparsePauliOp:
    g = rng(seed)
    op = SparsePauliOp(num_qubits)
    for _ in range(num_terms):
        w = int(g.integers(1, min(4, num_qubits) + 1))
        qubits = g.choice(num_qubits, size=w, replace=False)
        paulis = [("X", "Y", "Z")[int(g.integers(0, 3))] for _ in range(w)]
        op.add_term(float(g.normal(0.0, 1.0)), list(zip([int(q) for q in qubits], paulis)))
    return op


def vqe4(seed: int = 1):
    g = rng(seed)
    c = Circuit(4)
    for _ in range(2):
        for q in range(4):
            c.rot("ry", float(g.uniform(-math.pi, math.pi)), q)
        for q in range(3):
            c.append("cnot", (q, q + 1))
    op = SparsePauliOp(4)
    coef = lambda: float(g.normal(0.0, 0.5))  # noqa: E731
    op.add_term(coef(), [])
    for q in range(4):
        op.add_term(coef(), [(q, "Z")])
    for a in range(4):
        for b in range(a + 1, 4):
            op.add_term(coef(), [(a, "Z"), (b, "Z")])
    for s in ("XXYY", "XYYX", "YXXY", "YYXX"):
        op.add_term(coef(), [(q, p) for q, p in enumerate(s)])
    return c, op


def qnn(num_qubits: int = 10, batch: int = 1024, layers: int = 4, seed: int = 7):
    """Returns (circuit, observable, initial states [batch, 2^n], labels [batch])."""
    g = rng(seed)
    x = g.uniform(0.0, 1.0, size=(batch, num_qubits))
    c = Circuit(num_qubits)
    for _ in range(layers):
        for q in range(num_qubits):
            c.rot("ry", float(g.uniform(-math.pi, math.pi)), q)
            c.rot("rz", float(g.uniform(-math.pi, math.pi)), q)
        for q in range(num_qubits):
            c.append("cnot", (q, (q + 1) % num_qubits))
    labels = np.where(g.uniform(size=batch) < 0.3, 1.0, -1.0)
    states = product_states(x)
    return c, SparsePauliOp.single(num_qubits, 0, "Z", 1.0), states, labels


def product_states(x: np.ndarray) -> np.ndarray:
    """Rows (x) RY(pi x_q)|0> with qubit 0 the least significant index bit."""
    b, n = x.shape
    out = np.ones((b, 1), dtype=np.complex128)
    for q in range(n - 1, -1, -1):
        c = np.cos(0.5 * math.pi * x[:, q])[:, None]
        s = np.sin(0.5 * math.pi * x[:, q])[:, None]
        # index = ... q_{n-1} ... q_0: build from the most significant qubit down
        out = np.concatenate([out[:, :, None] * c[:, :, None], out[:, :, None] * s[:, :, None]], axis=2)
        out = out.reshape(b, -1)
    return np.ascontiguousarray(out)


def half_mse_upstream(values: np.ndarray, labels: np.ndarray):
    """loss = 0.5 mean((f - y)^2) (crates/arcqml-loss/src/mse.rs:16-26); g_b = (f_b - y_b) / B."""
    d = values - labels
    return 0.5 * float(np.mean(d * d)), d / len(values)
