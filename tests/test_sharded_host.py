"""Sharded statevector host logic on CPU: the layout planner, the slice packing rule, and whole
runs over world sizes 2 and 4 on gloo with the oracle computing each rank's shard, compared with
the unsharded oracle (value, psi, H psi, gradients, psi_0, lambda_0 at 1e-10)."""
import multiprocessing as mp
import socket

import numpy as np
import pytest

from arcqml_b200.circuit import PlanOp
from arcqml_b200.sharded import (Layout, PartnerStep, ShardError, SwapStep, TermsStep,
                                 flip_groups, local_terms, schedule_ops, schedule_terms)
from arcqml_b200.workloads import brickwork, random_pauli_sum
from plans import random_plan, random_state, random_terms
from shard_support import gloo_worker, slice_index, slices_numpy

RTOL = 1e-10


def close(a, b, tol=RTOL):
    a, b = np.asarray(a), np.asarray(b)
    scale = max(1.0, float(np.max(np.abs(b))) if b.size else 1.0)
    assert float(np.max(np.abs(a - b))) <= tol * scale


# ---------------------------------------------------------------------------- planner


def check_ops_schedule(ops, n, g):
    """Every op exactly once, all its qubits local when it runs, per-qubit order kept."""
    L = Layout(n, g)
    steps, final = schedule_ops(ops, L)
    seen = []
    for st in steps:
        if isinstance(st, SwapStep):
            for pg, pl in st.pairs:
                assert pg >= L.n_local > pl
            L.apply_swap(st.pairs)
        else:
            for o, i in zip(st.ops, st.indices):
                assert all(L.is_local(q) for q in ops[i].qubits)
                assert o.qubits == tuple(L.pos[q] for q in ops[i].qubits)
                assert o.bindings == ops[i].bindings
                seen.append(i)
    assert sorted(seen) == list(range(len(ops)))
    for q in range(n):
        order = [i for i in seen if q in ops[i].qubits]
        assert order == sorted(order)
    assert final.pos == L.pos
    return steps


@pytest.mark.parametrize("n,g", [(6, 1), (8, 2), (10, 3), (12, 3)])
def test_schedule_ops_random_plans(n, g):
    rng = np.random.Generator(np.random.PCG64(50 + n))
    ops = random_plan(rng, n, 150, 10)
    check_ops_schedule(ops, n, g)


def test_schedule_ops_brickwork_swaps_once_per_layer():
    n, g, layers = 16, 3, 10
    ops = brickwork(n, layers, seed=5).compile_plan(1)
    steps = check_ops_schedule(ops, n, g)
    swaps = sum(isinstance(s, SwapStep) for s in steps)
    assert swaps <= 2 * layers


def test_schedule_ops_rejects_ops_wider_than_a_shard():
    ops = [PlanOp(35, (0, 1, 2), (0.0, 0.0, 0.0))]
    with pytest.raises(ShardError, match="local qubits"):
        schedule_ops(ops, Layout(4, 2))


@pytest.mark.parametrize("n,g", [(8, 2), (12, 3)])
def test_schedule_terms_covers_every_group_without_global_flips(n, g):
    terms = random_pauli_sum(n, 80, seed=n).compiled_terms()
    flips, members = flip_groups(terms)
    L = Layout(n, g)
    steps, _ = schedule_terms(flips, L)
    seen = []
    for st in steps:
        if isinstance(st, SwapStep):
            L.apply_swap(st.pairs)
        else:
            assert isinstance(st, TermsStep)
            for gi in st.groups:
                assert all(L.is_local(q) for q in range(n) if (flips[gi] >> q) & 1)
                seen.append(gi)
            for r in range(1 << g):
                coef, flip, phase = local_terms(terms, [members[i] for i in st.groups], L, r)
                assert int(np.max(flip, initial=0)) < (1 << L.n_local)
                assert int(np.max(phase, initial=0)) < (1 << L.n_local)
    assert sorted(seen) == list(range(len(flips)))


def test_schedule_terms_sends_groups_that_flip_every_layout_to_the_partner():
    terms = [(1.0, 0b1111, 0, 0), (0.5, 0b0001, 0, 0), (2.0, 0b0111, 0b1000, 0)]
    flips, _ = flip_groups(terms)
    steps, _ = schedule_terms(flips, Layout(4, 2))
    partner = sorted(st.group for st in steps if isinstance(st, PartnerStep))
    assert partner == [0, 2]  # 4 and 3 flipped qubits: fewer than 2 left for the rank bits
    local = [gi for st in steps if isinstance(st, TermsStep) for gi in st.groups]
    assert local == [1]


def partner_terms(n, rng, count):
    """Pauli terms (coefficient, flip, phase, Y count mod 4) that flip most qubits: X, Y and Z
    on every qubit or all but one, so that every power of i occurs on the rank bits."""
    full = (1 << n) - 1
    out = []
    for _ in range(count):
        flip = full if rng.uniform() < 0.5 else full & ~(1 << int(rng.integers(0, n)))
        y = int(rng.integers(0, 1 << n)) & flip  # Y where flip and phase meet
        z = int(rng.integers(0, 1 << n)) & ~flip
        phase = y | z
        out.append((float(rng.normal()), flip, phase, bin(flip & phase).count("1") % 4))
    return out


@pytest.mark.parametrize("size,n,chunk", [(2, 6, 4), (4, 6, 2), (8, 7, 4), (4, 8, 1 << 10)])
def test_thread_world_partner_terms_match_oracle(oracle, size, n, chunk):
    """Terms flipping more qubits than a shard holds, mixed with ordinary ones, over thread
    ranks: value, H psi and the adjoint sweep's gradients against the oracle."""
    from arcqml_b200.sharded import ShardedStateVectorSimulator
    from shard_support import OracleShardBackend, run_threads, sharded_case
    rng = np.random.Generator(np.random.PCG64(300 + size + n))
    npar = 6
    terms = partner_terms(n, rng, 12) + random_terms(rng, n, 10)
    terms.append(terms[0][:1] + terms[0][1:])  # a repeated flip mask: one group, two terms
    case = dict(n=n, ops=random_plan(rng, n, 60, npar), terms=terms, init=random_state(rng, n),
                upstream=float(rng.normal()),
                req=[1] + [int(x) for x in (rng.uniform(size=npar) < 0.8)])

    def body(rank, comm):
        sim = ShardedStateVectorSimulator(n, comm=comm, backend=OracleShardBackend(oracle),
                                          chunk_amplitudes=chunk, transport="p2p")
        return sharded_case(sim, case["ops"], case["terms"], case["init"], case["upstream"],
                            case["req"])

    res = dict(enumerate(run_threads(size, body)))
    check_world(res, expected(oracle, case), size)


def test_gloo_world_partner_terms_match_oracle(oracle):
    n, size = 6, 4
    rng = np.random.Generator(np.random.PCG64(77))
    case = dict(n=n, ops=random_plan(rng, n, 50, 5),
                terms=partner_terms(n, rng, 8) + random_terms(rng, n, 8),
                init=random_state(rng, n), upstream=-0.4, req=[0] + [1] * 5, chunk=4)
    res = run_world(size, case)
    check_world(res, expected(oracle, case), size)


# ---------------------------------------------------------------------------- slice packing


@pytest.mark.parametrize("positions", [[5], [0, 3], [6, 1, 4], [2, 7, 0]])
def test_slices_pack_unpack_round_trip(positions):
    n_local = 8
    rng = np.random.Generator(np.random.PCG64(len(positions)))
    shard = rng.normal(size=1 << n_local) + 1j * rng.normal(size=1 << n_local)
    k = len(positions)
    others = 1 << (n_local - k)
    skip = 1
    chunk = others // 2
    staging = np.zeros(((1 << k) - 1) * chunk, dtype=np.complex128)
    slices_numpy(shard, positions, chunk, chunk, skip, staging, False)
    blk = 0
    for y in range(1 << k):
        if y == skip:
            continue
        for j in range(chunk):
            idx = int(slice_index(np.array([chunk + j]), y, positions)[0])
            assert all(((idx >> p) & 1) == ((y >> i) & 1) for i, p in enumerate(positions))
            assert staging[blk * chunk + j] == shard[idx]
        blk += 1
    back = shard.copy()
    back[:] = 0
    slices_numpy(back, positions, chunk, chunk, skip, staging, True)
    moved = back != 0
    assert np.array_equal(back[moved], shard[moved])
    assert moved.sum() == ((1 << k) - 1) * chunk


# ---------------------------------------------------------------------------- gloo worlds


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_world(size, case):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=gloo_worker, args=(r, size, port, case, q)) for r in range(size)]
    for p in ps:
        p.start()
    out = {}
    try:
        for _ in range(size):
            r, res = q.get(timeout=300)
            out[r] = res
    finally:
        for p in ps:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(size):
        assert not isinstance(out[r], str), out[r]
    return out


def expected(oracle, case):
    n = case["n"]
    psi_m = oracle.plan_apply(case["ops"], case["init"], n)
    value, hpsi = oracle.expectation_and_apply(case["terms"], psi_m, n)
    psi0, lam0, grads = oracle.adjoint_backward(case["ops"], psi_m, hpsi, n, case["upstream"],
                                                case["req"], len(case["req"]))
    return dict(value=value, psi_m=psi_m, hpsi=hpsi, grads=grads, psi0=psi0, lam0=lam0)


def check_world(res, exp, size):
    for r in range(size):
        got = res[r]
        close(got["value"], exp["value"])
        close(got["psi_m"], exp["psi_m"])
        close(got["hpsi"], exp["hpsi"])
        close(got["grads"], exp["grads"])
        close(got["psi0"], exp["psi0"])
        close(got["lam0"], exp["lam0"])


@pytest.mark.parametrize("size,n", [(2, 6), (4, 7)])
def test_gloo_world_random_plan_matches_oracle(oracle, size, n):
    rng = np.random.Generator(np.random.PCG64(700 + size))
    npar = 9
    case = dict(n=n, ops=random_plan(rng, n, 90, npar), terms=random_terms(rng, n, 30),
                init=random_state(rng, n), upstream=float(rng.normal()),
                req=[1] + [int(x) for x in (rng.uniform(size=npar) < 0.8)], chunk=8)
    res = run_world(size, case)
    assert res[0]["swaps"] > 0
    check_world(res, expected(oracle, case), size)


def test_gloo_world_brickwork_matches_oracle(oracle):
    n, size = 8, 4
    c = brickwork(n, 4, seed=11)
    rng = np.random.Generator(np.random.PCG64(9))
    case = dict(n=n, ops=c.compile_plan(1), terms=random_pauli_sum(n, 40, seed=3).compiled_terms(),
                init=random_state(rng, n), upstream=0.75,
                req=c.requires_grad_mask(True, False))
    res = run_world(size, case)
    check_world(res, expected(oracle, case), size)


def test_gloo_world_row_sharded_batch_matches_oracle(oracle):
    """Batch rows split over 4 ranks: values of all rows and gradients summed over all rows
    equal the oracle's batch path (crates/arcqml-sim/src/statevector/execution/adjoint/
    row_major.rs:108-162 semantics: per-row upstream, row gradients summed)."""
    from arcqml_b200.workloads import half_mse_upstream, qnn
    from shard_support import gloo_batch_worker
    case = dict(n=6, batch=14, layers=2, seed=3)
    size = 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=gloo_batch_worker, args=(r, size, port, case, q))
          for r in range(size)]
    for p in ps:
        p.start()
    out = {}
    try:
        for _ in range(size):
            r, res = q.get(timeout=300)
            out[r] = res
    finally:
        for p in ps:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    c, obs, init, labels = qnn(case["n"], case["batch"], case["layers"], case["seed"])
    n, b = case["n"], case["batch"]
    ops = c.compile_plan(1)
    psi = oracle.plan_apply(ops, init.reshape(-1), n, b).reshape(b, -1)
    terms = obs.compiled_terms()
    vals = np.array([oracle.expectation(terms, psi[i], n) for i in range(b)])
    lam = np.stack([oracle.expectation_and_apply(terms, psi[i], n)[1] for i in range(b)])
    _, up = half_mse_upstream(vals, labels)
    req = c.requires_grad_mask(True, False)
    _, _, g = oracle.adjoint_backward(ops, psi.reshape(-1), lam.reshape(-1), n, up, req, len(req), b)
    for r in range(size):
        assert not isinstance(out[r], str), out[r]
        close(out[r]["values"], vals)
        close(out[r]["grads"], g[1:])


def test_gloo_world_falls_back_when_a_rank_cannot_share_its_buffer(oracle):
    """Peer-transport setup is collective: one rank failing makes every rank use the
    point-to-point transport, and the run still matches the oracle."""
    from shard_support import gloo_fallback_worker
    n, size = 6, 2
    rng = np.random.Generator(np.random.PCG64(31))
    case = dict(n=n, ops=random_plan(rng, n, 60, 6), terms=random_terms(rng, n, 20),
                init=random_state(rng, n), upstream=0.5,
                req=[1] + [1] * 6)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=gloo_fallback_worker, args=(r, size, port, case, q))
          for r in range(size)]
    for p in ps:
        p.start()
    out = {}
    try:
        for _ in range(size):
            r, res = q.get(timeout=300)
            out[r] = res
    finally:
        for p in ps:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(size):
        assert not isinstance(out[r], str), out[r]
        assert out[r]["transport"] == "p2p"
    check_world(out, expected(oracle, case), size)


@pytest.mark.parametrize("size,n", [(2, 7), (4, 9), (8, 10)])
def test_thread_world_amplitudes_at_match_oracle(oracle, size, n):
    """amplitudes_at after a forward sweep whose swaps permuted the layout: the amplitudes at
    seeded logical indices, on every rank, equal the oracle's state there."""
    from arcqml_b200.sharded import ShardError, ShardedStateVectorSimulator
    from shard_support import OracleShardBackend, run_threads
    rng = np.random.Generator(np.random.PCG64(700 + n))
    ops = random_plan(rng, n, 80, 5)
    init = random_state(rng, n)
    idx = rng.integers(0, 1 << n, size=57)
    want = oracle.plan_apply(ops, init, n)[idx]

    def body(rank, comm):
        sim = ShardedStateVectorSimulator(n, comm=comm, backend=OracleShardBackend(oracle),
                                          transport="p2p")
        sim.load(init)
        sim.forward(ops)
        got = sim.amplitudes_at(idx)
        try:
            sim.amplitudes_at([1 << n])
        except ShardError:
            pass
        else:
            raise AssertionError("an index outside the state was accepted")
        return got, sim.stats.swaps

    for got, swaps in run_threads(size, body):
        np.testing.assert_allclose(got, want, rtol=0, atol=1e-12)
