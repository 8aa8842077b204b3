"""Whole-circuit unitaries and unitary fitting on the device, mirroring ``arcqml-unitary``
(``crates/arcqml-unitary/src``).

A circuit's unitary is the circuit applied to the batch of all ``D = 2^n`` basis states: row
``i`` of the device batch is ``U|i>``, column ``i`` of ``U`` (``evolve/circuit.rs``). Fitting
compares it with a target ``T`` through the trace overlap ``s = Tr(T^dagger U) = sum_i
<T|i>, U|i>>`` (``fit/loss.rs:5-19``), the fidelity ``|s|^2 / D^2`` clamped to [0, 1] and the
loss ``1 - fidelity`` (``:21-26``). The analytic gradient of ``fit/adjoint.rs:8-68``,
``-2 Re(conj(s) <T|i>| dG |psi_i>) / D^2`` summed over the rows, is the batched adjoint sweep of
the runtime with ``lambda_i = -(g s / D^2) T|i>`` for an upstream factor ``g``.

Every step is an existing device entry point: ``plan_apply`` on the ``[D, D]`` batch,
``overlap`` per row, ``scaled_copy`` for lambda and ``adjoint_backward``. The arithmetic goes
through a backend object (``DeviceBackend`` by default), so the same code also runs against a
CPU implementation in the tests.
"""
from __future__ import annotations

import math

import numpy as np

from .circuit import Circuit

DEFAULT_UNITARY_TOLERANCE = 1e-10  # lib.rs:37-38


class UnitaryError(ValueError):
    """Errors with the messages of ``UnitaryError`` (``error.rs``)."""


def _qubits_from_dimension(dimension: int) -> int:
    if dimension <= 0 or dimension & (dimension - 1):
        raise UnitaryError(f"unitary dimension must be a nonzero power of two, got {dimension}")
    return dimension.bit_length() - 1


class DenseUnitary:
    """Row-major ``U[output, input]`` of ``num_qubits`` qubits (``dense/unitary.rs``)."""

    def __init__(self, data: np.ndarray, dimension: int):
        self.num_qubits = _qubits_from_dimension(dimension)
        self.dimension = dimension
        self._data = data

    @classmethod
    def from_row_major(cls, values, dimension: int) -> "DenseUnitary":
        """Copies the values after the checks of ``from_row_major`` (power-of-two dimension,
        length, finite values); unitarity is ``validate``'s job."""
        _qubits_from_dimension(dimension)
        a = np.array(values, dtype=np.complex128).reshape(-1)
        if a.size != dimension * dimension:
            raise UnitaryError("unitary matrix length mismatch: "
                               f"expected {dimension * dimension}, got {a.size}")
        if not np.all(np.isfinite(a.real)) or not np.all(np.isfinite(a.imag)):
            raise UnitaryError("unitary matrix contains non-finite values")
        return cls(a, dimension)

    @classmethod
    def from_matrix(cls, matrix, tolerance: float = DEFAULT_UNITARY_TOLERANCE) -> "DenseUnitary":
        """A square complex matrix, checked for unitarity (``unitary_from_tensor``)."""
        m = np.asarray(matrix)
        if m.ndim != 2 or m.shape[0] != m.shape[1]:
            raise UnitaryError(f"unitary matrix must be a square rank-2 tensor, got shape "
                               f"{list(m.shape)}")
        u = cls.from_row_major(m.astype(np.complex128), m.shape[0])
        u.validate(tolerance)
        return u

    def as_row_major(self) -> np.ndarray:
        return self._data

    def matrix(self) -> np.ndarray:
        return self._data.reshape(self.dimension, self.dimension)

    def validate(self, tolerance: float = DEFAULT_UNITARY_TOLERANCE) -> None:
        """Largest |(U^dagger U - I)_ij| against the tolerance (``dense/validate.rs``)."""
        if not math.isfinite(tolerance) or tolerance < 0.0:
            raise UnitaryError(f"tolerance must be finite and nonnegative, got {tolerance}")
        m = self.matrix()
        dev = float(np.max(np.abs(m.conj().T @ m - np.eye(self.dimension))))
        if dev > tolerance:
            raise UnitaryError(f"matrix is not unitary: maximum deviation {dev} exceeds "
                               f"tolerance {tolerance}")

    def __eq__(self, other) -> bool:
        return (isinstance(other, DenseUnitary) and self.dimension == other.dimension
                and np.array_equal(self._data, other._data))


class DeviceBackend:
    """The runtime's device entry points on ``[D, D]`` complex128 CUDA batches."""

    def basis_batch(self, n: int):
        import torch
        return torch.eye(1 << n, dtype=torch.complex128,
                         device=torch.device("cuda", torch.cuda.current_device()))

    def apply(self, plan_ops, batch, n: int) -> None:
        from . import runtime as rt
        rt.plan_apply_device(rt.CircuitPlan.create(plan_ops), batch, n)

    def rows_of(self, target: DenseUnitary):
        import torch
        rows = np.ascontiguousarray(target.matrix().T)  # row i = T|i>
        return torch.from_numpy(rows).to(torch.device("cuda", torch.cuda.current_device()))

    def trace_overlap(self, target_rows, batch, n: int) -> complex:
        from . import runtime as rt
        per_row = rt.overlap_device(target_rows, batch, n)
        return complex(np.sum(per_row))  # rows in order

    def scaled(self, rows, factor: complex, n: int):
        from . import runtime as rt
        return rt.scaled_copy_device(rows, n, np.full(rows.shape[0], factor))

    def adjoint(self, plan_ops, batch, lam, n: int, requires_grad) -> np.ndarray:
        from . import runtime as rt
        req = np.ascontiguousarray(requires_grad, dtype=np.uint8)
        ones = np.ones(batch.shape[0], dtype=np.float64)
        return rt.adjoint_backward_device(rt.CircuitPlan.create(plan_ops), batch, lam, n, ones,
                                          req, len(req))

    def to_host(self, batch) -> np.ndarray:
        return batch.cpu().numpy()


def _check(target: DenseUnitary, circuit: Circuit) -> None:
    if target.num_qubits != circuit.num_qubits:
        raise UnitaryError(f"target has {target.num_qubits} qubits but circuit has "
                           f"{circuit.num_qubits} qubits")


def _forward(circuit: Circuit, backend):
    n = circuit.num_qubits
    ops = circuit.compile_plan(1)
    batch = backend.basis_batch(n)
    backend.apply(ops, batch, n)
    return ops, batch


def unitary_from_circuit(circuit: Circuit, backend=None) -> DenseUnitary:
    """``U[output, input]`` of the circuit (``lib.rs:40-51``)."""
    backend = backend or DeviceBackend()
    _, batch = _forward(circuit, backend)
    rows = backend.to_host(batch)  # row i = U|i> = column i
    d = 1 << circuit.num_qubits
    return DenseUnitary(np.ascontiguousarray(rows.T).reshape(-1), d)


def _fidelity_and_loss(overlap: complex, dimension: int):
    f = (overlap.real * overlap.real + overlap.imag * overlap.imag) / float(dimension) ** 2
    f = min(max(f, 0.0), 1.0)
    return f, 1.0 - f


def _values(target: DenseUnitary, circuit: Circuit, backend):
    _check(target, circuit)
    ops, batch = _forward(circuit, backend)
    rows = backend.rows_of(target)
    s = backend.trace_overlap(rows, batch, circuit.num_qubits)
    return ops, batch, rows, s


def unitary_fidelity(target: DenseUnitary, circuit: Circuit, backend=None) -> float:
    """``|Tr(T^dagger U)|^2 / D^2`` clamped to [0, 1]: blind to a global phase."""
    _, _, _, s = _values(target, circuit, backend or DeviceBackend())
    return _fidelity_and_loss(s, target.dimension)[0]


def unitary_loss_value(target: DenseUnitary, circuit: Circuit, backend=None) -> float:
    """``1 - unitary_fidelity`` without keeping anything for a backward pass."""
    _, _, _, s = _values(target, circuit, backend or DeviceBackend())
    return _fidelity_and_loss(s, target.dimension)[1]


class UnitaryLoss:
    """Result of ``unitary_loss``: ``value`` and ``backward(upstream)``, which runs the adjoint
    sweep and accumulates the gradients into the circuit's parameters (``fit/api.rs:42-118``)."""

    def __init__(self, target, circuit, backend, ops, batch, rows, overlap):
        self.target, self.circuit, self._backend = target, circuit, backend
        self._ops, self._batch, self._rows, self.overlap = ops, batch, rows, overlap
        self.fidelity, self.value = _fidelity_and_loss(overlap, target.dimension)

    def backward(self, upstream: float = 1.0) -> np.ndarray:
        if self._batch is None:
            raise UnitaryError("unitary_loss backward was already run")
        n, d = self.circuit.num_qubits, self.target.dimension
        factor = -float(upstream) * self.overlap / float(d) ** 2
        lam = self._backend.scaled(self._rows, factor, n)
        req = self.circuit.requires_grad_mask(True, False)
        grads = self._backend.adjoint(self._ops, self._batch, lam, n, req)[1:].copy()
        for p, g in zip(self.circuit.parameters, grads):
            if p.requires_grad:
                g = float(np.float32(g)) if p.dtype == "f32" else float(g)
                p.grad = g if getattr(p, "grad", None) is None else p.grad + g
        self._batch = None  # the sweep ran the batch back to the basis states
        return grads


def unitary_loss(target: DenseUnitary, circuit: Circuit, backend=None) -> UnitaryLoss:
    """Differentiable ``1 - fidelity``: ``.value``, then ``.backward(upstream)``."""
    backend = backend or DeviceBackend()
    ops, batch, rows, s = _values(target, circuit, backend)
    return UnitaryLoss(target, circuit, backend, ops, batch, rows, s)


def unitary_from_matrix(matrix, tolerance: float = DEFAULT_UNITARY_TOLERANCE) -> DenseUnitary:
    """``unitary_from_tensor`` (``lib.rs:53-63``): a square complex matrix checked to the
    tolerance."""
    return DenseUnitary.from_matrix(matrix, tolerance)


__all__ = ["DenseUnitary", "DeviceBackend", "UnitaryError", "UnitaryLoss",
           "DEFAULT_UNITARY_TOLERANCE", "unitary_fidelity", "unitary_from_circuit",
           "unitary_from_matrix", "unitary_loss", "unitary_loss_value"]
