"""The tile cover of the observable passes (pauli_tile.cu, host code: no GPU needed).

States of 20 qubits and more evaluate a Pauli sum as passes over 12-qubit tiles (qubits 0-3 and
eight more) that together hold every term's flip mask (crates/arcqml-observable/src/
compiled_hamiltonian.rs:104-132 pairs amplitudes t and t ^ flip). The cover is the fewest passes
of a greedy by qubits and a greedy by masks; the device tests (test_gpu_observable_tiles.py)
check the values the passes produce.
"""
import numpy as np

from arcqml_b200.observable import SparsePauliOp
from arcqml_b200.workloads import random_pauli_sum


def passes(runtime, op, n):
    return runtime.Observable.from_sparse_pauli_op(op).tile_passes(n)


def test_benchmark_sums_take_few_passes(runtime):
    # the 32-qubit 200-term sum has 113 distinct flip masks above qubit 3
    assert passes(runtime, random_pauli_sum(32, 200, seed=1235), 32) == 12
    assert passes(runtime, random_pauli_sum(30, 200, seed=1235), 30) == 11
    assert passes(runtime, random_pauli_sum(35, 50, seed=1235), 35) == 6


def test_at_most_one_pass_per_distinct_mask(runtime):
    g = np.random.Generator(np.random.PCG64(3))
    for n in (20, 24, 33):
        op = random_pauli_sum(n, int(g.integers(5, 120)), seed=int(g.integers(1, 1000)))
        highs = {f & ~0xF for _, f, _, _ in op.compiled_terms() if f}
        assert 1 <= passes(runtime, op, n) <= max(1, len(highs))


def test_masks_within_one_tile_take_one_pass(runtime):
    n = 24
    op = SparsePauliOp(n)
    for q in range(4, 12):  # flips on qubits 0-11 only
        op.add_term(0.3, [(q, "X"), (q - 4, "Y")])
    op.add_term(-0.2, [(2, "X"), (11, "X"), (20, "Z")])
    assert passes(runtime, op, n) == 1


def test_no_cover_cases(runtime):
    n = 22
    empty = SparsePauliOp(n)
    assert passes(runtime, empty, n) == 0
    diag = SparsePauliOp(n)
    diag.add_term(0.5, [(3, "Z"), (21, "Z")])
    assert passes(runtime, diag, n) == 1
    wide = random_pauli_sum(n, 10, seed=9)
    wide.add_term(0.6, [(q, "X") for q in range(5, 15)])  # ten flipped qubits above qubit 3
    assert passes(runtime, wide, n) == 0
    assert passes(runtime, random_pauli_sum(19, 10, seed=2), 19) == 0  # below 20 qubits
