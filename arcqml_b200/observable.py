"""Sparse Pauli observables compiled to XOR masks.

Mirrors ``SparsePauliOp`` (``crates/arcqml-observable/src/sparse_pauli_op.rs``) and its internal
``CompiledHamiltonian`` term form (``crates/arcqml-observable/src/compiled_hamiltonian.rs:30-78``):
each term becomes ``(coefficient, flip_mask, phase_mask, y_count_mod_four)`` with
flip = X|Y bits, phase = Y|Z bits. Terms keep insertion order. The JSON layout is the reference's
``{"num_qubits": n, "terms": [{"coefficient": c, "paulis": [{"qubit": q, "pauli": "X"}]}]}``
(``sparse_pauli_op.rs:187-240``).
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from typing import List, Sequence, Tuple

import numpy as np


class ObservableError(ValueError):
    pass


@dataclass
class SparsePauliOp:
    num_qubits: int
    terms: List[Tuple[float, Tuple[Tuple[int, str], ...]]] = field(default_factory=list)

    def __post_init__(self):
        if int(self.num_qubits) <= 0:  # EmptyQubitError (sparse_pauli_op.rs:107-110)
            raise ObservableError("a Pauli operator acts on at least one qubit")

    @classmethod
    def constant(cls, num_qubits: int, value: float) -> "SparsePauliOp":
        return cls(num_qubits, [(float(value), ())])

    @classmethod
    def single(cls, num_qubits: int, qubit: int, pauli: str, coefficient: float = 1.0):
        op = cls(num_qubits)
        op.add_term(coefficient, [(qubit, pauli)])
        return op

    @classmethod
    def from_json(cls, text: str) -> "SparsePauliOp":
        """The reference's JSON form (``sparse_pauli_op.rs:180-240``): Pauli names X, Y or Z
        only (an identity factor is left out, not written as "I")."""
        try:
            d = json.loads(text)
            n = int(d["num_qubits"])
            terms = [(float(t["coefficient"]), [(int(p["qubit"]), p["pauli"]) for p in t["paulis"]])
                     for t in d["terms"]]
        except (ValueError, KeyError, TypeError) as e:
            raise ObservableError(f"invalid observable JSON: {e}") from None
        op = cls(n)
        for i, (c, ps) in enumerate(terms):
            for j, (_, name) in enumerate(ps):
                if name not in ("X", "Y", "Z"):
                    raise ObservableError(f"terms[{i}].paulis[{j}].pauli must be X, Y or Z, "
                                          f"got {name}")
            op.add_term(c, ps)
        return op

    def to_json(self) -> str:
        return json.dumps({"num_qubits": self.num_qubits, "terms": [
            {"coefficient": c, "paulis": [{"qubit": q, "pauli": p} for q, p in ps]}
            for c, ps in self.terms]})

    def add_term(self, coefficient: float, paulis: Sequence[Tuple[int, str]]) -> "SparsePauliOp":
        seen = set()
        clean = []
        for q, p in paulis:
            p = p.upper()
            if p not in ("I", "X", "Y", "Z"):
                raise ObservableError(f"unknown Pauli {p}")
            if not 0 <= q < self.num_qubits:
                raise ObservableError(f"qubit {q} out of range for {self.num_qubits} qubits")
            if q in seen:
                raise ObservableError(f"duplicate qubit {q} in Pauli string")
            seen.add(q)
            clean.append((int(q), p))
        if not np.isfinite(coefficient):
            raise ObservableError("coefficient must be finite")
        self.terms.append((float(coefficient), tuple(clean)))
        return self

    def __len__(self) -> int:
        return len(self.terms)

    def scale(self, factor: float) -> "SparsePauliOp":
        """Every coefficient times factor (``sparse_pauli_op.rs:339-356``)."""
        if not np.isfinite(factor):
            raise ObservableError("coefficient must be finite")
        return SparsePauliOp(self.num_qubits, [(c * float(factor), ps) for c, ps in self.terms])

    def simplify(self, tolerance: float = 1e-12) -> "SparsePauliOp":
        """Equal Pauli strings merged (coefficients summed in term order), terms with
        |coefficient| <= tolerance dropped, strings in canonical order
        (``sparse_pauli_op.rs:358-387``)."""
        if not (np.isfinite(tolerance) and tolerance >= 0.0):
            raise ObservableError(f"invalid simplify tolerance {tolerance}")
        sums = {}
        for c, ps in self.terms:
            key = tuple(sorted((q, p) for q, p in ps if p != "I"))
            sums[key] = sums.get(key, 0.0) + c
        return SparsePauliOp(self.num_qubits,
                             [(c, k) for k, c in sorted(sums.items()) if abs(c) > tolerance])

    def compiled_terms(self):
        """[(coefficient, flip_mask, phase_mask, y_count_mod_four)] in insertion order."""
        out = []
        for c, ps in self.terms:
            flip = phase = 0
            y = 0
            for q, p in ps:
                m = 1 << q
                if p == "X":
                    flip |= m
                elif p == "Y":
                    flip |= m
                    phase |= m
                    y = (y + 1) % 4
                elif p == "Z":
                    phase |= m
            out.append((c, flip, phase, y))
        return out

    def masks(self):
        """Arrays (coefficients f64, flip u64, phase u64) for the runtime's observable API."""
        t = self.compiled_terms()
        return (np.array([x[0] for x in t], dtype=np.float64),
                np.array([x[1] for x in t], dtype=np.uint64),
                np.array([x[2] for x in t], dtype=np.uint64))


PauliSum = SparsePauliOp
Hamiltonian = SparsePauliOp
