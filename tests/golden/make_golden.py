"""Regenerates the golden fixtures in this folder from the ArcQML reference checkout.

Run in a container that has the reference checkout, naming its root as the argument or in
``ARCQML_REFERENCE_ROOT``:

    python tests/golden/make_golden.py <reference_root>

It reads, as text, the reference's own fixtures and known-answer values for the statevector
path and writes them to JSON, with the source file and line of each value:

* ``h2_vqe.json`` — the 15-term H2 Hamiltonian (examples/data/h2_hamiltonian.json), the ansatz
  constants of examples/rust/h2_vqe.rs:6-37 and the energies printed after Adam steps 1 and 100
  in docs/tutorial/h2_vqe.md:499-501;
* ``kernel_kats.json`` — the 3-qubit input state and angle of the rotation-derivative test
  (crates/arcqml-kernel/tests/kernel_tests.rs:115-127) and the mixed-Pauli observable case of
  crates/arcqml-observable/tests/compiled_hamiltonian_tests.rs:13-41.

The tests never read the reference; they read only these JSON files.
"""
from __future__ import annotations

import json
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def _line_of(text: str, needle: str) -> int:
    for i, line in enumerate(text.splitlines(), 1):
        if needle in line:
            return i
    raise ValueError(f"{needle!r} not found")


def h2(root: str) -> dict:
    ham_path = "examples/data/h2_hamiltonian.json"
    ham = json.load(open(os.path.join(root, ham_path)))
    src_path = "examples/rust/h2_vqe.rs"
    src = open(os.path.join(root, src_path), encoding="utf-8").read()
    consts = {}
    for name in ("NUM_QUBITS", "ACTIVE_ELECTRONS", "LAYERS", "STEPS"):
        m = re.search(rf"const {name}: usize = (\d+);", src)
        consts[name.lower()] = int(m.group(1))
    m = re.search(r"let ry = ([0-9.]+) \* \(([0-9.]+) \* \(parameter_index \+ 1\) as f64\)\.sin\(\);", src)
    amp, freq = float(m.group(1)), float(m.group(2))
    m = re.search(r"Adam::new\(([0-9.e-]+), ([0-9.e-]+), ([0-9.e-]+), ([0-9.e-]+), ([0-9.e-]+)\)", src)
    adam = [float(x) for x in m.groups()]
    doc_path = "docs/tutorial/h2_vqe.md"
    doc = open(os.path.join(root, doc_path), encoding="utf-8").read()
    energies = {}
    for step in (1, 100):
        m = re.search(rf"step\s+{step}: energy = (-?[0-9.]+) Ha", doc)
        energies[str(step)] = {"energy": float(m.group(1)), "digits": len(m.group(1).split(".")[1]),
                               "source": f"{doc_path}:{_line_of(doc, m.group(0))}"}
    return {
        "hamiltonian": ham,
        "hamiltonian_source": ham_path,
        "ansatz": {"source": f"{src_path}:14-37", **consts,
                   "initial_angle": {"amplitude": amp, "frequency": freq,
                                     "rule": "amplitude * sin(frequency * (index + 1))"},
                   "per_layer": "RY(p), RZ(p) on each qubit, then CNOT(q, (q+1) % n) for q = 0..n-1",
                   "prefix": "X on qubits 0..active_electrons-1"},
        "adam": {"lr": adam[0], "beta1": adam[1], "beta2": adam[2], "eps": adam[3],
                 "weight_decay": adam[4], "source": f"{src_path}:{_line_of(src, 'Adam::new')}"},
        "energy_after_step": energies,
    }


def kernel_kats(root: str) -> dict:
    path = "crates/arcqml-kernel/tests/kernel_tests.rs"
    src = open(os.path.join(root, path), encoding="utf-8").read()
    start = src.index("fn rotation_derivative_into_matches_central_difference_on_every_qubit")
    block = src[start:start + 800]
    vals = re.findall(r"Complex64::new\((-?[0-9.]+), (-?[0-9.]+)\)", block)
    theta = float(re.search(r"let theta = ([0-9.]+);", block).group(1))
    eps = float(re.search(r"let epsilon = ([0-9.e-]+);", block).group(1))
    obs_path = "crates/arcqml-observable/tests/compiled_hamiltonian_tests.rs"
    obs = open(os.path.join(root, obs_path), encoding="utf-8").read()
    return {
        "rotation_derivative": {
            "source": f"{path}:{_line_of(src, 'fn rotation_derivative_into')}",
            "input": [[float(a), float(b)] for a, b in vals[:8]],
            "theta": theta, "epsilon": eps, "tolerance": 1e-8,
        },
        "mixed_pauli": {
            "source": f"{obs_path}:{_line_of(obs, 'fn compiled_hamiltonian_should_apply_mixed_pauli_terms')}",
            "state": "[1/sqrt(2), i/sqrt(2)]",
            "terms": [[0.5, "I"], [2.0, "X"], [-3.0, "Y"], [4.0, "Z"]],
            "expectation": -2.5,
            "h_psi_over_scale": [[1.5, 2.0], [2.0, -6.5]],
            "tolerance": 1e-12,
        },
    }


def main(root: str) -> None:
    with open(os.path.join(HERE, "h2_vqe.json"), "w") as f:
        json.dump(h2(root), f, indent=1)
    with open(os.path.join(HERE, "kernel_kats.json"), "w") as f:
        json.dump(kernel_kats(root), f, indent=1)


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ARCQML_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py <reference_root> (or set ARCQML_REFERENCE_ROOT)")
    main(root)
