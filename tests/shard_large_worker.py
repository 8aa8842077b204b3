"""One rank of the large sharded configurations over NCCL (launched by torchrun from
tests/test_gpu_large_sharded.py; one process per GPU).

* ``c4 <reference.npz>``: the 32-qubit, 20-layer brickwork with the 200-term sum, forward + <H> +
  adjoint gradient, sharded over the world; rank 0 compares <H> and all 1280 gradients with the
  same step run unsharded on one GPU (reference.npz: value, grads) at 1e-10, and the final
  state's norm with 1.
* ``c5 <fixture.npz>``: the 35-qubit configuration (10 layers with gates on the global qubits,
  50-term sum; 512 GiB over 8 GPUs): <H>, the norm after the circuit, then the reverse sweep with
  upstream 0 un-applies every gate and must return |0...0>; then the same generator at 30 qubits
  against the oracle's outputs (tests/golden/config_30q_brickwork10.npz): <H> at 1e-10 relative
  and sampled amplitudes of psi and H psi.

Rank 0 prints ``large-sharded-ok`` and each check's figures; any failed check exits non-zero.
"""
import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, HERE):
    sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from arcqml_b200.sharded import DistComm, RuntimeBackend, ShardedStateVectorSimulator  # noqa: E402
from arcqml_b200.workloads import brickwork, random_pauli_sum  # noqa: E402


def world_norm(sim):
    local = sim.backend.norm(sim.psi, sim.n_local)
    return float(sim.comm.allreduce_sum(np.array([local]))[0])


def c4(ref_path, rank, report):
    n = 32
    c = brickwork(n, 20, seed=1234)
    obs = random_pauli_sum(n, 200, seed=1235)
    sim = ShardedStateVectorSimulator(n)
    try:
        value = sim.run(c, obs)
        norm = world_norm(sim)
        grads = sim.backward(1.0)
        swaps = sim.stats.swaps
    finally:
        sim.close()
    if rank == 0:
        ref = np.load(ref_path)
        rv, rg = float(ref["value"]), np.asarray(ref["grads"])
        dv = abs(value - rv) / max(1.0, abs(rv))
        dg = float(np.max(np.abs(grads - rg))) / max(1.0, float(np.max(np.abs(rg))))
        report(f"c4 value {value!r} vs 1 GPU {rv!r}: rel {dv:.3e}; {len(grads)} gradients: max "
               f"rel {dg:.3e}; norm-1 {norm - 1:.3e}; swaps {swaps}",
               dv <= 1e-10 and dg <= 1e-10 and abs(norm - 1) <= 1e-10)


def c5(fixture, rank, report):
    n = 35
    c = brickwork(n, 10, seed=1234)
    ops = c.compile_plan(0)
    terms = random_pauli_sum(n, 50, seed=1235).compiled_terms()
    sim = ShardedStateVectorSimulator(n)
    try:
        sim.reset()
        sim.forward(ops)
        norm = world_norm(sim)
        value = sim.observe(terms, True)
        swaps = sim.stats.swaps
        req = np.zeros(c.num_parameters() + 1, dtype=np.uint8)  # no gradient requested
        sim.adjoint(ops, 0.0, req)
        back = sim.amplitudes_at([0, 1, 1 << (n - 1), (1 << n) - 1])
        norm0 = world_norm(sim)
    finally:
        sim.close()
    if rank == 0:
        err = float(np.max(np.abs(back - np.array([1, 0, 0, 0]))))
        report(f"c5 35q: <H> {value!r}, norm-1 {norm - 1:.3e}, swaps {swaps}; after the inverse "
               f"sweep |psi - |0>| at 4 indices {err:.3e}, norm-1 {norm0 - 1:.3e}",
               abs(norm - 1) <= 1e-10 and err <= 1e-10 and abs(norm0 - 1) <= 1e-10)
    fx = np.load(fixture)
    idx, want_psi, want_h = fx["indices"], fx["psi"], fx["hpsi"]
    n30 = int(fx["qubits"])
    c30 = brickwork(n30, int(fx["layers"]), seed=1234)
    t30 = random_pauli_sum(n30, int(fx["terms"]), seed=1235).compiled_terms()
    sim = ShardedStateVectorSimulator(n30)
    try:
        sim.reset()
        sim.forward(c30.compile_plan(0))
        v30 = sim.observe(t30, True)
        got_psi = sim.amplitudes_at(idx)
        got_h = sim.amplitudes_at(idx, "lam")
    finally:
        sim.close()
    if rank == 0:
        ref = float(fx["value"])
        dv = abs(v30 - ref) / max(1.0, abs(ref))
        dp = float(np.max(np.abs(got_psi - want_psi)))
        dh = float(np.max(np.abs(got_h - want_h)))
        report(f"c5 generator at 30q: <H> {v30!r} vs oracle {ref!r} (rel {dv:.3e}); sampled psi "
               f"max diff {dp:.3e}, H psi {dh:.3e}", dv <= 1e-10 and dp <= 1e-12 and dh <= 1e-12)


def main():
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                            device_id=torch.device("cuda", local))
    rank = dist.get_rank()
    ok = [True]

    def report(msg, good):
        print(("PASS " if good else "FAIL ") + msg, flush=True)
        ok[0] = ok[0] and good

    mode, path = sys.argv[1], sys.argv[2]
    (c4 if mode == "c4" else c5)(path, rank, report)
    flag = torch.tensor([0 if ok[0] else 1], device="cuda")
    dist.all_reduce(flag)
    dist.destroy_process_group()
    if flag.item() != 0:
        sys.exit(1)
    if rank == 0:
        print("large-sharded-ok", mode, flush=True)


if __name__ == "__main__":
    main()
