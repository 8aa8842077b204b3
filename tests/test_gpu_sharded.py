"""Sharded statevector on the GPU runtime (needs a B200).

* the slice packing kernel against the numpy rule;
* a whole sharded run with 4 and 8 ranks emulated as threads on one GPU (exchanges are device
  copies), compared with the oracle at 1e-10 — this exercises every kernel of the sharded path;
* with two or more GPUs, the same run over NCCL with one process per GPU (torchrun).
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from arcqml_b200.workloads import brickwork, random_pauli_sum
from plans import random_plan, random_state, random_terms
from shard_support import run_threads, sharded_case, slices_numpy
from test_sharded_host import check_world, expected

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("positions,chunk_begin,chunk_len,skip", [
    ([13], 0, 1 << 12, 0), ([0, 9], 256, 1 << 10, 2), ([11, 2, 7], 0, 1 << 11, 5),
    ([3, 12, 8, 1], 64, 200, 16)])
def test_shard_slices_kernel_matches_numpy(runtime, positions, chunk_begin, chunk_len, skip):
    import torch
    n_local = 14
    rng = np.random.Generator(np.random.PCG64(sum(positions)))
    host = rng.normal(size=1 << n_local) + 1j * rng.normal(size=1 << n_local)
    k = len(positions)
    nblk = (1 << k) - (1 if skip < (1 << k) else 0)
    dev = torch.from_numpy(host).cuda()
    staging = torch.zeros(nblk * chunk_len, dtype=torch.complex128, device="cuda")
    runtime.shard_slices(dev, n_local, positions, chunk_begin, chunk_len, skip, staging, False)
    ref = np.zeros(nblk * chunk_len, dtype=np.complex128)
    slices_numpy(host, positions, chunk_begin, chunk_len, skip, ref, False)
    assert np.array_equal(staging.cpu().numpy(), ref)
    back = torch.zeros_like(dev)
    runtime.shard_slices(back, n_local, positions, chunk_begin, chunk_len, skip, staging, True)
    hb = np.zeros_like(host)
    slices_numpy(hb, positions, chunk_begin, chunk_len, skip, ref, True)
    assert np.array_equal(back.cpu().numpy(), hb)


def test_shard_slices_rejects_bad_arguments(runtime):
    import torch
    dev = torch.zeros(1 << 6, dtype=torch.complex128, device="cuda")
    st = torch.zeros(1 << 6, dtype=torch.complex128, device="cuda")
    with pytest.raises(runtime.RuntimeError, match="outside the 6-qubit shard"):
        runtime.shard_slices(dev, 6, [6], 0, 4, 0, st, False)
    with pytest.raises(runtime.RuntimeError, match="repeat"):
        runtime.shard_slices(dev, 6, [1, 1], 0, 4, 0, st, False)
    with pytest.raises(runtime.RuntimeError, match="exceeds the shard"):
        runtime.shard_slices(dev, 6, [1], 16, 32, 0, st, False)


def thread_world(size, case, transport="p2p"):
    from arcqml_b200.sharded import RuntimeBackend, ShardedStateVectorSimulator

    def body(rank, comm):
        sim = ShardedStateVectorSimulator(case["n"], comm=comm, backend=RuntimeBackend(),
                                          chunk_amplitudes=case.get("chunk", 1 << 20),
                                          transport=transport,
                                          peer_bytes=case.get("peer_bytes", 1 << 20))
        try:
            return sharded_case(sim, case["ops"], case["terms"], case["init"], case["upstream"],
                                case["req"])
        finally:
            sim.close()

    return dict(enumerate(run_threads(size, body)))


@pytest.mark.parametrize("size,n,transport", [(4, 12, "p2p"), (8, 13, "p2p"), (4, 12, "peer"),
                                              (8, 13, "peer")])
def test_emulated_ranks_random_plan_match_oracle(runtime, oracle, size, n, transport):
    rng = np.random.Generator(np.random.PCG64(900 + n))
    npar = 12
    case = dict(n=n, ops=random_plan(rng, n, 160, npar), terms=random_terms(rng, n, 40),
                init=random_state(rng, n), upstream=float(rng.normal()),
                req=[1] + [int(x) for x in (rng.uniform(size=npar) < 0.8)], chunk=1 << 9,
                peer_bytes=1 << 16)
    res = thread_world(size, case, transport)
    assert res[0]["swaps"] > 0
    check_world(res, expected(oracle, case), size)


def test_emulated_ranks_brickwork_match_oracle(runtime, oracle):
    n, size = 16, 8
    c = brickwork(n, 6, seed=21)
    rng = np.random.Generator(np.random.PCG64(17))
    case = dict(n=n, ops=c.compile_plan(1), terms=random_pauli_sum(n, 60, seed=8).compiled_terms(),
                init=random_state(rng, n), upstream=-0.5, req=c.requires_grad_mask(True, False))
    res = thread_world(size, case)
    check_world(res, expected(oracle, case), size)


@pytest.mark.skipif("not __import__('torch').cuda.is_available() or "
                    "__import__('torch').cuda.device_count() < 2", reason="needs 2 GPUs")
def test_nccl_ranks_match_oracle():
    import torch
    size = 4 if torch.cuda.device_count() >= 4 else 2
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes", "1", "--nproc-per-node", str(size), "--master-addr", "127.0.0.1",
           "--master-port", "29571", os.path.join(HERE, "shard_nccl_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=os.path.dirname(HERE))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "sharded-nccl-ok" in r.stdout


def test_emulated_ranks_row_sharded_qnn_match_oracle(runtime, oracle):
    """The batched QNN (10 qubits) with its rows split over 4 emulated ranks on one GPU."""
    from arcqml_b200.sharded import RuntimeBackend, ShardedBatchSimulator
    from arcqml_b200.workloads import half_mse_upstream, qnn
    n, b = 10, 64
    c, obs, init, labels = qnn(n, b, 4, seed=7)

    def body(rank, comm):
        sim = ShardedBatchSimulator(n, b, comm=comm, backend=RuntimeBackend())
        sim.load(init)
        vals = sim.run(c, obs)
        _, up = half_mse_upstream(vals, labels)
        return vals, sim.backward(up)

    res = run_threads(4, body)
    ops = c.compile_plan(1)
    psi = oracle.plan_apply(ops, init.reshape(-1), n, b).reshape(b, -1)
    terms = obs.compiled_terms()
    vals = np.array([oracle.expectation(terms, psi[i], n) for i in range(b)])
    lam = np.stack([oracle.expectation_and_apply(terms, psi[i], n)[1] for i in range(b)])
    _, up = half_mse_upstream(vals, labels)
    req = c.requires_grad_mask(True, False)
    _, _, g = oracle.adjoint_backward(ops, psi.reshape(-1), lam.reshape(-1), n, up, req, len(req), b)
    for v, gr in res:
        np.testing.assert_allclose(v, vals, rtol=0, atol=1e-10)
        np.testing.assert_allclose(gr, g[1:], rtol=0, atol=1e-10 * max(1.0, np.abs(g).max()))


def test_emulated_ranks_partner_terms_match_oracle(runtime, oracle):
    """Terms that flip more qubits than a shard holds (evaluated against the partner rank's
    shard, chunk by chunk) on 4 emulated ranks through the device backend."""
    from test_sharded_host import partner_terms
    n, size = 12, 4
    rng = np.random.Generator(np.random.PCG64(1212))
    npar = 8
    case = dict(n=n, ops=random_plan(rng, n, 80, npar),
                terms=partner_terms(n, rng, 10) + random_terms(rng, n, 20),
                init=random_state(rng, n), upstream=0.6, req=[1] * (npar + 1), chunk=1 << 7)
    res = thread_world(size, case)
    check_world(res, expected(oracle, case), size)
