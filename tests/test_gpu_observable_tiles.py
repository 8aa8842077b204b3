"""The tiled observable passes (pauli_tile.cu) against the oracle (needs a B200).

States of 20 qubits and more evaluate <psi|H|psi> and H|psi> (crates/arcqml-observable/src/
compiled_hamiltonian.rs:81-132) as passes over 12-qubit tiles that cover the observable's flip
masks. Checked here: random Pauli sums of weight 1-4, groups of several terms sharing one flip
mask with different phase masks, the identity and Z-only terms, Y-heavy strings, flips on the
highest qubits, the expectation alone, the accumulate mode, batch rows, and a flip mask that
fits no tile (the gather kernel then evaluates the observable).
"""
import numpy as np
import pytest

from arcqml_b200.observable import SparsePauliOp
from arcqml_b200.workloads import random_pauli_sum
from plans import random_state

pytestmark = pytest.mark.gpu


def mixed_observable(n, seed):
    g = np.random.Generator(np.random.PCG64(seed))
    op = random_pauli_sum(n, 40, seed=seed)
    op.add_term(0.75, [])
    op.add_term(-0.3, [(0, "Z"), (n - 1, "Z")])
    for _ in range(6):  # one flip mask, several phase masks: X and Y on the same qubits
        qs = [int(x) for x in g.choice(n, size=3, replace=False)]
        for paulis in (("X", "X", "Y"), ("Y", "X", "X"), ("Y", "Y", "Y")):
            op.add_term(float(g.normal()), list(zip(qs, paulis)))
        zq = int(g.choice([q for q in range(n) if q not in qs]))
        op.add_term(float(g.normal()), list(zip(qs, ("X", "Y", "X"))) + [(zq, "Z")])
    op.add_term(1.1, [(n - 1, "X"), (n - 2, "Y"), (n - 3, "X"), (n - 4, "Y")])
    return op


def check(runtime, oracle, n, op, batch=1, seed=0):
    import torch
    g = np.random.Generator(np.random.PCG64(seed + n))
    psi = random_state(g, n, batch if batch > 1 else None)
    rows = psi.reshape(batch, -1)
    terms = op.compiled_terms()
    ref = [oracle.expectation_and_apply(terms, r, n) for r in rows]
    ob = runtime.Observable.from_sparse_pauli_op(op)
    dev = torch.from_numpy(psi).cuda()
    out = torch.empty_like(dev)
    vals = ob.expectation_and_apply(dev, out, n)
    got = out.cpu().numpy().reshape(batch, -1)
    for b in range(batch):
        v_ref, h_ref = ref[b]
        assert abs(vals[b] - v_ref) <= 1e-10 * max(1.0, abs(v_ref)), (vals[b], v_ref)
        scale = max(1.0, float(np.abs(h_ref).max()))
        assert float(np.max(np.abs(got[b] - h_ref))) <= 1e-12 * scale
    only = ob.expectation(dev, n)
    for b in range(batch):
        assert abs(only[b] - ref[b][0]) <= 1e-10 * max(1.0, abs(ref[b][0]))
    prior = torch.from_numpy(g.normal(size=psi.shape) + 1j * g.normal(size=psi.shape)).cuda()
    acc = prior.clone()
    vals2 = ob.expectation_and_accumulate(dev, acc, n)
    diff = (acc - prior).cpu().numpy().reshape(batch, -1)
    for b in range(batch):
        v_ref, h_ref = ref[b]
        assert abs(vals2[b] - v_ref) <= 1e-10 * max(1.0, abs(v_ref))
        assert float(np.max(np.abs(diff[b] - h_ref))) <= 1e-11 * max(1.0, float(np.abs(h_ref).max()))
    return ob


@pytest.mark.parametrize("n", [20, 22])
def test_tiled_observable_matches_oracle(runtime, oracle, n):
    ob = check(runtime, oracle, n, mixed_observable(n, 50 + n))
    assert ob.tile_passes(n) >= 2


def test_tiled_observable_batch_rows(runtime, oracle):
    n = 20
    ob = check(runtime, oracle, n, random_pauli_sum(n, 30, seed=5), batch=2, seed=3)
    assert ob.tile_passes(n) >= 1


def test_diagonal_only_observable_takes_one_pass(runtime, oracle):
    n = 20
    op = SparsePauliOp(n)
    op.add_term(0.5, [])
    op.add_term(-1.25, [(3, "Z"), (17, "Z")])
    op.add_term(0.8, [(19, "Z")])
    ob = check(runtime, oracle, n, op, seed=7)
    assert ob.tile_passes(n) == 1


def test_flip_mask_wider_than_a_tile_uses_the_gather_kernel(runtime, oracle):
    n = 21
    op = random_pauli_sum(n, 10, seed=9)
    op.add_term(0.6, [(q, "X") for q in range(5, 15)])  # ten flipped qubits above qubit 3
    ob = check(runtime, oracle, n, op, seed=11)
    assert ob.tile_passes(n) == 0
