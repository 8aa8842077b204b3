"""Analysis of a sharded state (marginals, Bloch vectors, overlaps) on CPU: ranks as threads
over the oracle shard backend, after a random plan has permuted the qubit layout, against the
oracle on the full state (tolerance 1e-12)."""
import numpy as np
import pytest

import oracle as O
from arcqml_b200.sharded import ShardedStateVectorSimulator, ShardError
from plans import random_plan, random_state
from shard_support import OracleShardBackend, run_threads

TOL = 1e-12


def close(a, b, tol=TOL):
    a, b = np.asarray(a), np.asarray(b)
    assert float(np.max(np.abs(a - b))) <= tol * max(1.0, float(np.max(np.abs(b)))), (a, b)


def sim_for(n, comm):
    return ShardedStateVectorSimulator(n, comm=comm, backend=OracleShardBackend(O),
                                       chunk_amplitudes=1 << 3, transport="p2p")


def analysis_world(size, n, sim_for, tol=TOL):
    """Marginals, Bloch vectors, overlaps and fidelities of sharded states after a random plan,
    on `size` thread ranks with simulators from sim_for(n, comm), against the oracle."""
    g = np.random.Generator(np.random.PCG64(size))
    a, b = random_state(g, n), random_state(g, n)
    ops = random_plan(g, n, 60, 4)
    want = O.plan_apply(ops, a, n)
    want_b = O.plan_apply(ops, b, n)
    selections = [[0], [n - 1], [n - 1, 0], [2, 5, 6], list(range(n))]

    def body(rank, comm):
        s = sim_for(n, comm)
        s.load(a)
        s.forward(ops)
        moved = s.layout.pos != list(range(n))
        marg = [s.marginal_probabilities(q) for q in selections]
        bloch = [s.bloch_vector(q) for q in range(n)]
        s2 = sim_for(n, comm)
        s2.load(b)
        s2.forward(ops)
        for q in range(n):  # the same Bloch swaps bring s2 to s's layout
            s2.bloch_vector(q)
        same = s2.layout.pos == s.layout.pos
        ov = s.overlap(s2) if same else None
        fresh = sim_for(n, comm)
        fresh.load(b)
        err = None
        if fresh.layout.pos != s.layout.pos:
            try:
                s.overlap(fresh)
            except ShardError as e:
                err = str(e)
        return moved, marg, bloch, same, ov, err, s.fidelity(s) if same else None

    res = run_threads(size, body)
    check_analysis(res, n, selections, want, want_b, tol)


def check_analysis(res, n, selections, want, want_b, tol):
    assert any(r[0] for r in res)  # the plan's swaps permuted the layout
    assert all(r[3] for r in res) and any(r[5] is not None for r in res)
    for moved, marg, bloch, same, ov, err, fid in res:
        for m, q in zip(marg, selections):
            close(m, O.marginal_probabilities(want, n, q), tol)
        for q in range(n):
            close(bloch[q], O.bloch_vector(want, n, q), tol)
        if same:
            rs, _ = O.overlap_fidelity(want, want_b, n)
            close([ov.real, ov.imag], [rs.real, rs.imag], tol)
            assert abs(fid - 1.0) < 1e-10
        if err is not None:
            assert "same qubit layout" in err


@pytest.mark.parametrize("size", [2, 4, 8])
def test_marginals_bloch_and_overlap_of_sharded_states(size):
    analysis_world(size, 7, sim_for)


def test_sharded_selection_errors():
    def body(rank, comm):
        s = sim_for(4, comm)
        s.reset()
        out = []
        for sel in ([], [1, 1], [4]):
            try:
                s.marginal_probabilities(sel)
            except ShardError as e:
                out.append(str(e))
        try:
            s.bloch_vector(-1)
        except ShardError as e:
            out.append(str(e))
        return out

    for msgs in run_threads(2, body):
        assert msgs == ["at least one qubit must be selected", "duplicate qubit in selection: 1",
                        "qubit index out of range: simulator has 4 qubits, got 4",
                        "qubit index out of range: simulator has 4 qubits, got -1"]


def test_marginal_of_global_qubits_only_and_basis_state():
    def body(rank, comm):
        s = sim_for(5, comm)
        s.reset()  # |00000>: all weight in bin 0
        return s.marginal_probabilities([4, 3]), s.bloch_vector(4)

    for marg, bloch in run_threads(4, body):
        close(marg, [1, 0, 0, 0])
        close(bloch, [0, 0, 1])
