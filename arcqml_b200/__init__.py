"""ArcQML statevector engine for NVIDIA B200 (sm_100a).

The product is the C-ABI library ``libarcqml_runtime_private.so`` (built from ``csrc/`` by
``arcqml_b200.build``), a drop-in for ArcQML's closed runtime behind ``arcqml-runtime-sys``.
This package is its Python host layer: the circuit/observable data model, the ctypes binding
of the C ABI (``runtime``), device-resident simulators (``simulator``) and the seeded
benchmark workloads (``workloads``).
"""
from .circuit import Circuit, ParameterId, PlanOp, basis_state  # noqa: F401
from .observable import Hamiltonian, PauliSum, SparsePauliOp  # noqa: F401

__all__ = ["Circuit", "ParameterId", "PlanOp", "basis_state", "SparsePauliOp", "PauliSum",
           "Hamiltonian"]
