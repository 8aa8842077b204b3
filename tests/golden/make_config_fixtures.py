"""Oracle outputs for the two large single-state configurations at their stated sizes.

Runs the CPU oracle (oracle/liboracle.so, OpenMP over all host threads) on the seeded workloads
that ``bench.py`` and the GPU tests build, and keeps a sample of its outputs small enough to
commit:

* ``config_28q_brickwork20.npz`` — 28 qubits, 20 brickwork layers (brickwork seed 1234), the
  200-term random Pauli sum (seed 1235), forward + expectation from |0...0>;
* ``config_30q_brickwork10.npz`` — the 35-qubit configuration's generator at 30 qubits: 10
  brickwork layers (seed 1234), 50-term Pauli sum (seed 1235), forward + expectation.

Each file holds the expectation ``value``, the squared ``norm`` of the final state, the sorted
``indices`` (4096 seeded uniform indices plus the first and last) and the final state ``psi`` and
``hpsi`` = H|psi> at those indices. The GPU tests (tests/test_gpu_configs.py) run the same
workloads on the device and compare against these arrays.

Usage (the 28-qubit case takes about 20 minutes on 8 host threads and 13 GB of memory, the
30-qubit one about 40 minutes and 45 GB):

    python tests/golden/make_config_fixtures.py [28] [30]
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

# (qubits, layers, terms); circuit seed 1234 and observable seed 1235 as in bench.py
CASES = {28: (28, 20, 200), 30: (30, 10, 50)}
SAMPLES = 4096
INDEX_SEED = 2024


def fixture_name(n: int) -> str:
    _, layers, _ = CASES[n]
    return f"config_{n}q_brickwork{layers}.npz"


def sample_indices(n: int) -> np.ndarray:
    g = np.random.Generator(np.random.PCG64(INDEX_SEED + n))
    idx = g.integers(0, 1 << n, size=SAMPLES, dtype=np.int64)
    return np.unique(np.concatenate([idx, [0, (1 << n) - 1]])).astype(np.int64)


def make(n: int) -> str:
    import oracle as O
    from arcqml_b200 import workloads

    O.build()
    _, layers, terms = CASES[n]
    c = workloads.brickwork(n, layers, seed=1234)
    obs = workloads.random_pauli_sum(n, terms, seed=1235)
    ops = c.compile_plan(1)
    t0 = time.time()
    init = np.zeros(1 << n, np.complex128)
    init[0] = 1.0
    psi = O.plan_apply(ops, init, n)
    del init
    t1 = time.time()
    value, hpsi = O.expectation_and_apply(obs.compiled_terms(), psi, n)
    t2 = time.time()
    idx = sample_indices(n)
    norm = float(np.vdot(psi, psi).real)
    path = os.path.join(HERE, fixture_name(n))
    np.savez(path, value=np.float64(value), norm=np.float64(norm), indices=idx,
             psi=psi[idx], hpsi=hpsi[idx], qubits=np.int64(n), layers=np.int64(layers),
             terms=np.int64(terms))
    print(f"{n} qubits: {len(ops)} gates in {t1 - t0:.0f} s, <H> in {t2 - t1:.0f} s on "
          f"{O.num_threads()} threads; value {value!r}, norm {norm!r} -> {path}", flush=True)
    return path


if __name__ == "__main__":
    for arg in sys.argv[1:] or ["28", "30"]:
        make(int(arg))
