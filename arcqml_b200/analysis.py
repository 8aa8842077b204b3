"""Analysis of simulator states on the device, mirroring ``arcqml-analysis``
(``crates/arcqml-analysis/src/statevector``): ``probabilities``, ``marginal_probabilities``,
``bloch_vector`` and ``fidelity``, plus the adjoint cotangents that make losses built on them
trainable through ``StateVectorSimulator.gradient`` (the reference differentiates these outputs
with its autograd core; here each becomes the lambda of the reverse sweep).

Errors carry the reference's ``AnalysisError`` messages (``error.rs``).
"""
from __future__ import annotations

import math
from typing import NamedTuple, Optional, Sequence

import numpy as np

from . import runtime as rt


class AnalysisError(ValueError):
    pass


class BlochVector(NamedTuple):
    """(<X>, <Y>, <Z>) of one qubit's reduced state (bloch.rs:4-13)."""
    x: float
    y: float
    z: float


def _run(fn):
    try:
        return fn()
    except rt.RuntimeError as e:
        raise AnalysisError(str(e)) from None


def probabilities(simulator) -> np.ndarray:
    """Basis probabilities |psi_i|^2, q0 the least significant index bit (probabilities.rs)."""
    return rt.probabilities_device(simulator.state, simulator.num_qubits).cpu().numpy()


def marginal_probabilities(simulator, qubits: Sequence[int]) -> np.ndarray:
    """Probabilities of the selected qubits, listed with the highest selected qubit as the most
    significant output bit (marginal.rs:9-32): selecting [0, 2] gives q2q0 = 00, 01, 10, 11."""
    out = _run(lambda: rt.marginal_probabilities_device(simulator.state, simulator.num_qubits,
                                                        list(qubits)))
    return out.cpu().numpy()


def bloch_vector(simulator, qubit: int) -> BlochVector:
    """Bloch vector of one qubit (bloch.rs:23-56); reads the state, changes nothing."""
    v = _run(lambda: rt.bloch_vector_device(simulator.state, simulator.num_qubits, qubit))
    return BlochVector(float(v[0]), float(v[1]), float(v[2]))


def overlap(lhs, rhs) -> complex:
    """<lhs|rhs> of two simulators' states."""
    _same_size(lhs, rhs)
    return rt.overlap_device(lhs.state, rhs.state, lhs.num_qubits)


def fidelity(lhs, rhs) -> float:
    """|<lhs|rhs>|^2, not clipped to [0, 1] (fidelity.rs:6-30)."""
    s = overlap(lhs, rhs)
    h = math.hypot(s.real, s.imag)
    return h * h


def _same_size(lhs, rhs):
    if lhs.num_qubits != rhs.num_qubits:
        raise AnalysisError("cannot compare states with different qubit counts: "
                            f"{lhs.num_qubits} and {rhs.num_qubits}")


# ---------------------------------------------------------------- cotangents
# lambda for StateVectorSimulator.gradient, whose sweep adds 2 Re<lambda| dU |psi> per slot


def probabilities_cotangent(simulator, upstream, qubits: Optional[Sequence[int]] = None):
    """lambda for an upstream gradient of ``probabilities`` (qubits=None) or of
    ``marginal_probabilities(qubits)``: lambda_i = upstream[bin(i)] psi_i."""
    import torch
    g = torch.as_tensor(np.ascontiguousarray(upstream, dtype=np.float64)).to(simulator.state.device)
    return _run(lambda: rt.probability_cotangent_device(simulator.state, simulator.num_qubits, g,
                                                        None if qubits is None else list(qubits)))


def amplitudes_cotangent(simulator, upstream):
    """lambda for a complex upstream gradient of the amplitudes (the reference's
    ``amplitudes().backward_with_grad``): upstream / 2."""
    import torch
    g = torch.as_tensor(np.ascontiguousarray(upstream, dtype=np.complex128)).to(simulator.state.device)
    return rt.scaled_copy_device(g, simulator.num_qubits, 0.5)


def fidelity_cotangent(simulator, target) -> object:
    """lambda for d|<target|psi>|^2 with psi the simulator's state: <target|psi> target."""
    _same_size(simulator, target)
    s = rt.overlap_device(target.state, simulator.state, simulator.num_qubits)
    return rt.scaled_copy_device(target.state, simulator.num_qubits, s)
