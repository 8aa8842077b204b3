"""Circuit data model and plan compilation for the statevector path.

Mirrors the parts of ArcQML's ``arcqml-circuit`` and ``arcqml-kernel`` that feed the runtime
C ABI:

* gate names, opcodes, arity and parameter slots — ``crates/arcqml-circuit/src/gate.rs:12-109``,
  ``gate_metadata.rs:7-93``, opcodes ``crates/arcqml-runtime-abi/src/lib.rs:113-153``;
* circuit parameters (scalar F32/F64 values, F32 cast to f64 when bound) —
  ``crates/arcqml-circuit/src/circuit_parameters.rs:10-27``;
* ``RuntimeCircuitPlan::compile`` — per operation a bound descriptor plus up to three
  ``(parameter_slot, parent_index = ParameterId + offset)`` bindings, custom unitaries pushed
  without bindings — ``crates/arcqml-kernel/src/runtime.rs:16-68``,
  ``crates/arcqml-kernel/src/circuit/binding.rs:28-138``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional, Sequence, Tuple, Union

import numpy as np

# name -> (opcode, arity, number of parameter slots)
GATES = {
    "i": (0, 1, 0), "x": (1, 1, 0), "y": (2, 1, 0), "z": (3, 1, 0), "h": (4, 1, 0),
    "s": (5, 1, 0), "sdg": (6, 1, 0), "t": (7, 1, 0), "tdg": (8, 1, 0),
    "sx": (9, 1, 0), "sxdg": (10, 1, 0),
    "rx": (11, 1, 1), "ry": (12, 1, 1), "rz": (13, 1, 1), "phase": (14, 1, 1),
    "u3": (15, 1, 3),
    "cnot": (16, 2, 0), "cy": (17, 2, 0), "cz": (18, 2, 0), "ch": (19, 2, 0),
    "cs": (20, 2, 0), "ct": (21, 2, 0), "cphase": (22, 2, 1),
    "crx": (23, 2, 1), "cry": (24, 2, 1), "crz": (25, 2, 1),
    "swap": (26, 2, 0), "iswap": (27, 2, 0), "dcx": (28, 2, 0), "ecr": (29, 2, 0),
    "rxx": (30, 2, 1), "ryy": (31, 2, 1), "rzz": (32, 2, 1), "rzx": (33, 2, 1),
    "fsim": (34, 2, 2),
    "toffoli": (35, 3, 0), "cswap": (36, 3, 0),
}
OPCODE_NAMES = {v[0]: k for k, v in GATES.items()}
OPCODE_NAMES[37] = "mcx"
OPCODE_NAMES[38] = "custom"
MCX = 37
CUSTOM_UNITARY = 38


def slot_count(opcode: int) -> int:
    """Differentiable slots per opcode, crates/arcqml-kernel/src/statevector/single.rs:169-197."""
    for _, (op, _, slots) in GATES.items():
        if op == opcode:
            return slots
    return 0


@dataclass(frozen=True)
class ParameterId:
    index: int


Gateparam = Union[float, ParameterId]


@dataclass
class Operation:
    """A gate on qubits with fixed values or parameter references per slot."""

    opcode: int
    qubits: Tuple[int, ...]
    gateparams: Tuple[Gateparam, ...] = ()
    matrix: Optional[np.ndarray] = None
    name: str = ""


@dataclass
class PlanOp:
    """One bound plan entry: the OperationDescriptor the runtime receives."""

    opcode: int
    qubits: Tuple[int, ...]
    params: Tuple[float, float, float]
    matrix: Optional[np.ndarray] = None
    bindings: Tuple[Tuple[int, int], ...] = ()
    name: str = ""


@dataclass
class Parameter:
    value: float
    dtype: str = "f64"  # "f32" or "f64"
    requires_grad: bool = True
    name: str = ""

    def f64(self) -> float:
        if self.dtype == "f32":
            return float(np.float32(self.value))
        return float(self.value)


class CircuitError(ValueError):
    pass


@dataclass
class Circuit:
    """n-qubit circuit with a parameter table (crates/arcqml-circuit/src/circuit.rs:7-214)."""

    num_qubits: int
    operations: list = field(default_factory=list)
    parameters: list = field(default_factory=list)

    # -- parameters -------------------------------------------------------
    def add_parameter(self, value: float, dtype: str = "f64", requires_grad: bool = True,
                      name: str = "") -> ParameterId:
        if dtype not in ("f32", "f64"):
            raise CircuitError(f"unsupported parameter dtype {dtype}")
        pid = ParameterId(len(self.parameters))
        self.parameters.append(Parameter(float(value), dtype, requires_grad,
                                         name or f"parameter_{pid.index}"))
        return pid

    def parameter_values(self) -> np.ndarray:
        return np.array([p.f64() for p in self.parameters], dtype=np.float64)

    def set_parameter_values(self, values: Sequence[float]) -> None:
        if len(values) != len(self.parameters):
            raise CircuitError("parameter count mismatch")
        for p, v in zip(self.parameters, values):
            p.value = float(np.float32(v)) if p.dtype == "f32" else float(v)

    # -- gates ------------------------------------------------------------
    def append(self, name: str, qubits: Sequence[int], *gateparams: Gateparam) -> "Circuit":
        name = name.lower()
        if name not in GATES:
            raise CircuitError(f"unknown gate {name}")
        opcode, arity, slots = GATES[name]
        qubits = tuple(int(q) for q in qubits)
        self._validate_qubits(qubits, arity, name)
        if len(gateparams) != slots:
            raise CircuitError(f"gate {name} takes {slots} parameters, got {len(gateparams)}")
        for g in gateparams:
            if isinstance(g, ParameterId) and not 0 <= g.index < len(self.parameters):
                raise CircuitError(f"invalid parameter id {g.index}")
        self.operations.append(Operation(opcode, qubits, tuple(gateparams), name=name))
        return self

    def mcx(self, controls: Sequence[int], target: int) -> "Circuit":
        qubits = tuple(int(q) for q in controls) + (int(target),)
        self._validate_qubits(qubits, len(qubits), "mcx")
        self.operations.append(Operation(MCX, qubits, (), name="MCX"))
        return self

    def custom_unitary(self, name: str, matrix, qubits: Sequence[int]) -> "Circuit":
        qubits = tuple(int(q) for q in qubits)
        k = len(qubits)
        m = np.ascontiguousarray(np.asarray(matrix, dtype=np.complex128)).reshape(-1)
        dim = 1 << k
        if m.size != dim * dim:
            raise CircuitError(f"custom unitary {name}: expected {dim * dim} entries, got {m.size}")
        u = m.reshape(dim, dim)
        if not np.all(np.isfinite(u)) or np.max(np.abs(u.conj().T @ u - np.eye(dim))) > 1e-12:
            raise CircuitError(f"custom unitary {name} is not unitary")
        self._validate_qubits(qubits, k, name)
        self.operations.append(Operation(CUSTOM_UNITARY, qubits, (), m.copy(), name=name))
        return self

    def _validate_qubits(self, qubits, arity, name):
        if len(qubits) != arity or arity == 0:
            raise CircuitError(f"gate {name} expects {arity} qubits, got {len(qubits)}")
        if len(set(qubits)) != len(qubits):
            raise CircuitError(f"gate {name} has duplicate qubits")
        for q in qubits:
            if not 0 <= q < self.num_qubits:
                raise CircuitError(f"qubit {q} out of range for {self.num_qubits} qubits")

    # -- parameterised builders (new F64 parameter per call) ----------------
    def rot(self, name: str, value: float, qubit: int) -> ParameterId:
        pid = self.add_parameter(value, name=f"{name}_q{qubit}_theta_{len(self.parameters)}")
        self.append(name, (qubit,), pid)
        return pid

    def num_parameters(self) -> int:
        return len(self.parameters)

    # -- plan compile -------------------------------------------------------
    def compile_plan(self, parameter_parent_offset: int = 1):
        """RuntimeCircuitPlan::compile (crates/arcqml-kernel/src/runtime.rs:16-68)."""
        plan = []
        for op in self.operations:
            if op.opcode == CUSTOM_UNITARY:
                plan.append(PlanOp(op.opcode, op.qubits, (0.0, 0.0, 0.0), op.matrix, (), op.name))
                continue
            values = [0.0, 0.0, 0.0]
            bindings = []
            for slot, g in enumerate(op.gateparams):
                if isinstance(g, ParameterId):
                    values[slot] = self.parameters[g.index].f64()
                    bindings.append((slot, g.index + parameter_parent_offset))
                else:
                    values[slot] = float(g)
            plan.append(PlanOp(op.opcode, op.qubits, tuple(values), None, tuple(bindings), op.name))
        return plan

    def requires_grad_mask(self, with_initial_state: bool, initial_requires_grad: bool = False):
        mask = [1 if initial_requires_grad else 0] if with_initial_state else []
        mask += [1 if p.requires_grad else 0 for p in self.parameters]
        return np.array(mask, dtype=np.uint8)


def basis_state(num_qubits: int, index: int = 0, batch: int = 1) -> np.ndarray:
    a = np.zeros((batch, 1 << num_qubits), dtype=np.complex128)
    a[:, index] = 1.0
    return a[0] if batch == 1 else a
