"""One rank of a sharded run over NCCL (launched by torchrun from test_gpu_sharded.py).

Every rank runs the same seeded case on its own GPU; rank 0 compares the gathered results with
the oracle at 1e-10 and prints ``sharded-nccl-ok``. Exit status is non-zero on any mismatch.
"""
import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, os.path.join(ROOT, "oracle"), HERE):
    sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import oracle as O  # noqa: E402
from arcqml_b200.sharded import DistComm, RuntimeBackend, ShardedStateVectorSimulator  # noqa: E402
from arcqml_b200.workloads import brickwork, random_pauli_sum  # noqa: E402
from plans import random_plan, random_state, random_terms  # noqa: E402
from shard_support import sharded_case  # noqa: E402
from test_sharded_host import check_world, expected  # noqa: E402


def main():
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    rank, size = dist.get_rank(), dist.get_world_size()
    if rank == 0:
        O.build()
    dist.barrier()
    rng = np.random.Generator(np.random.PCG64(4242))
    npar = 12
    n = 14
    cases = [
        dict(n=n, ops=random_plan(rng, n, 200, npar), terms=random_terms(rng, n, 40),
             init=random_state(rng, n), upstream=float(rng.normal()),
             req=[1] + [int(x) for x in (rng.uniform(size=npar) < 0.8)], chunk=1 << 10),
    ]
    c = brickwork(16, 8, seed=3)
    cases.append(dict(n=16, ops=c.compile_plan(1),
                      terms=random_pauli_sum(16, 50, seed=5).compiled_terms(),
                      init=random_state(rng, 16), upstream=1.25,
                      req=c.requires_grad_mask(True, False)))
    ok = True
    for case in cases:
        for transport in ("p2p", "peer", "nccl"):
            sim = ShardedStateVectorSimulator(case["n"], comm=DistComm(), backend=RuntimeBackend(),
                                              chunk_amplitudes=case.get("chunk", 1 << 20),
                                              transport=transport, peer_bytes=1 << 20)
            res = sharded_case(sim, case["ops"], case["terms"], case["init"], case["upstream"],
                               case["req"])
            sim.close()
            if rank == 0:
                try:
                    check_world({0: res}, expected(O, case), 1)
                except AssertionError as e:
                    print("mismatch", transport, e, flush=True)
                    ok = False
    flag = torch.tensor([0 if ok else 1], device="cuda")
    dist.all_reduce(flag)
    dist.destroy_process_group()
    if flag.item() != 0:
        sys.exit(1)
    if rank == 0:
        print("sharded-nccl-ok", size, flush=True)


if __name__ == "__main__":
    main()
