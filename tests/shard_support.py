"""Test support for the sharded statevector: a CPU shard backend over the oracle, the slice
packing rule in numpy, an in-process communicator for ranks run as threads, and the worker that
the gloo tests start once per rank.

Nothing here is used by the package: ``arcqml_b200.sharded`` runs its shards on the GPU runtime
(``RuntimeBackend``) and exchanges them over ``torch.distributed``.
"""
from __future__ import annotations

import os
import threading

import numpy as np


def slice_index(o: np.ndarray, y: int, positions) -> np.ndarray:
    """Local index of other-index o with slice value y (bit i of y at positions[i])."""
    o = np.asarray(o, dtype=np.int64)
    for p in sorted(positions):
        o = ((o >> p) << (p + 1)) | (o & ((1 << p) - 1))
    for i, p in enumerate(positions):
        if (y >> i) & 1:
            o = o | (1 << p)
    return o


def slices_numpy(shard: np.ndarray, positions, chunk_begin: int, chunk_len: int, skip: int,
                 staging: np.ndarray, unpack: bool) -> None:
    k = len(positions)
    o = np.arange(chunk_begin, chunk_begin + chunk_len, dtype=np.int64)
    blk = 0
    for y in range(1 << k):
        if y == skip:
            continue
        idx = slice_index(o, y, positions)
        st = staging[blk * chunk_len:(blk + 1) * chunk_len]
        if unpack:
            shard[idx] = st
        else:
            st[:] = shard[idx]
        blk += 1


class OracleShardBackend:
    """Shard compute on the CPU oracle (torch CPU tensors, numpy views)."""

    def __init__(self, oracle_module):
        import torch
        self.O = oracle_module
        self.torch = torch

    def empty(self, numel):
        return self.torch.empty(numel, dtype=self.torch.complex128)

    def zeros(self, numel):
        return self.torch.zeros(numel, dtype=self.torch.complex128)

    def from_numpy(self, a):
        return self.torch.from_numpy(np.ascontiguousarray(a, dtype=np.complex128).copy())

    def set_amplitude_one(self, shard, index):
        shard.zero_()
        shard[index] = 1.0

    def apply(self, ops, shard, n_local):
        if ops:
            rows = shard.numel() >> n_local
            out = self.O.plan_apply(ops, shard.numpy().reshape(-1), n_local, rows)
            shard.copy_(self.torch.from_numpy(out).reshape(shard.shape))

    def adjoint(self, ops, psi, lam, n_local, upstream, req, grads):
        rows = psi.numel() >> n_local
        up = np.broadcast_to(np.asarray(upstream, dtype=np.float64), (rows,))
        up = float(up[0]) if rows == 1 else np.ascontiguousarray(up)
        p, l, g = self.O.adjoint_backward(ops, psi.numpy().reshape(-1), lam.numpy().reshape(-1),
                                          n_local, up, req, len(grads), rows)
        psi.copy_(self.torch.from_numpy(p).reshape(psi.shape))
        lam.copy_(self.torch.from_numpy(l).reshape(lam.shape))
        grads += g

    def observable_rows(self, coef, flip, phase, psi, out, n_local):
        terms = [(float(c), int(f), int(p), bin(int(f) & int(p)).count("1") % 4)
                 for c, f, p in zip(coef, flip, phase)]
        rows = psi.numel() >> n_local
        a = psi.numpy().reshape(rows, -1)
        vals = np.zeros(rows)
        for b in range(rows):
            if out is None:
                vals[b] = self.O.expectation(terms, a[b], n_local)
            else:
                v, h = self.O.expectation_and_apply(terms, a[b], n_local)
                out.view(rows, -1)[b] += self.torch.from_numpy(h)
                vals[b] = v
        return vals

    def observable(self, coef, flip, phase, psi, out, n_local):
        return float(self.observable_rows(coef, flip, phase, psi, out, n_local)[0])

    def scale(self, x, factor, out, n_local):
        out.copy_(x * complex(factor))

    def marginal(self, shard, n_local, positions):
        return self.O.marginal_probabilities(shard.numpy(), n_local, list(positions))

    def bloch(self, shard, n_local, position):
        return self.O.bloch_vector(shard.numpy(), n_local, position)

    def overlap(self, a, b, n_local):
        return self.O.overlap_fidelity(a.numpy(), b.numpy(), n_local)[0]

    def norm(self, shard, n_local):
        a = shard.numpy()
        return float(np.vdot(a, a).real)

    def slices(self, shard, n_local, positions, chunk_begin, chunk_len, skip, staging, unpack):
        slices_numpy(shard.numpy(), positions, chunk_begin, chunk_len, skip, staging.numpy(),
                     unpack)


class ThreadHub:
    def __init__(self, size):
        self.size = size
        self.barrier = threading.Barrier(size, timeout=600)
        self.box = {}
        self.lock = threading.Lock()


class ThreadComm:
    """Ranks as threads of one process: exchanges are copies between the threads' buffers."""

    def __init__(self, hub: ThreadHub, rank: int):
        self.hub = hub
        self.rank = rank
        self.size = hub.size

    def _sync(self):
        import torch
        if torch.cuda.is_available():
            torch.cuda.synchronize()

    def exchange_start(self, sends, recvs):
        self._sync()
        with self.hub.lock:
            for peer, t in sends.items():
                self.hub.box[(self.rank, peer)] = t
        self.hub.barrier.wait()
        for peer, buf in recvs.items():
            buf.copy_(self.hub.box[(peer, self.rank)])
        self._sync()
        self.hub.barrier.wait()
        with self.hub.lock:
            for peer in sends:
                del self.hub.box[(self.rank, peer)]
        self.hub.barrier.wait()
        return []

    @staticmethod
    def wait(handle):
        pass

    def _gather(self, value, take=lambda v: v):
        """Every rank's value, each passed through take() while no rank can change it."""
        with self.hub.lock:
            self.hub.box[("g", self.rank)] = value
        self.hub.barrier.wait()
        vals = [take(self.hub.box[("g", r)]) for r in range(self.size)]
        self._sync()  # device copies done before any rank goes on
        self.hub.barrier.wait()
        with self.hub.lock:
            del self.hub.box[("g", self.rank)]
        self.hub.barrier.wait()
        return vals

    def allreduce_sum(self, values):
        vals = self._gather(np.array(values, dtype=np.float64, copy=True))
        out = np.zeros_like(vals[0])
        for v in vals:
            out = out + v
        return out

    def allgather(self, shard):
        self._sync()
        return self._gather(shard, lambda t: t.clone())

    # peer transport: the threads share one device, so buffers are used by address directly
    def barrier(self):
        self._sync()
        self.hub.barrier.wait()

    same_process = True

    def same_node(self):
        return True

    def allgather_object(self, obj):
        return list(self._gather(obj))


def run_threads(size, fn):
    """Runs fn(rank, comm) on `size` threads; returns the per-rank results (re-raises)."""
    hub = ThreadHub(size)
    out = [None] * size
    errs = []

    def body(r):
        try:
            out[r] = fn(r, ThreadComm(hub, r))
        except BaseException as e:  # noqa: BLE001 - re-raised below
            errs.append(e)
            hub.barrier.abort()

    ts = [threading.Thread(target=body, args=(r,)) for r in range(size)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    if errs:
        raise errs[0]
    return out


# ---------------------------------------------------------------------------- gloo worker


def sharded_case(sim, ops, terms, init, upstream, req):
    """Forward, observable and adjoint on the sharded simulator; returns what the tests
    compare: value, psi_m, H psi (logical order), gradients, psi_0, lambda_0."""
    sim.load(init)
    sim.forward(ops)
    psi_m = sim.amplitudes("psi")
    value = sim.observe(terms, True)
    hpsi = sim.amplitudes("lam")
    grads = sim.adjoint(ops, upstream, req)
    return dict(value=value, psi_m=psi_m, hpsi=hpsi, grads=grads,
                psi0=sim.amplitudes("psi"), lam0=sim.amplitudes("lam"),
                swaps=sim.stats.swaps)


def gloo_worker(rank, size, port, case, queue):
    """One rank of a world on gloo (CPU): runs `case` through the sharded simulator."""
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (root, os.path.join(root, "oracle"), here):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(size))
    import datetime

    import torch.distributed as dist

    import oracle as O
    from arcqml_b200.sharded import DistComm, ShardedStateVectorSimulator
    try:
        dist.init_process_group("gloo", rank=rank, world_size=size,
                                timeout=datetime.timedelta(seconds=120))
        sim = ShardedStateVectorSimulator(case["n"], comm=DistComm(),
                                          backend=OracleShardBackend(O),
                                          chunk_amplitudes=case.get("chunk", 1 << 24))
        res = sharded_case(sim, case["ops"], case["terms"], case["init"], case["upstream"],
                           case["req"])
        queue.put((rank, res))
    except BaseException as e:  # noqa: BLE001 - reported to the parent
        queue.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def gloo_batch_worker(rank, size, port, case, queue):
    """One rank of a gloo world running the row-sharded batch simulator on the oracle."""
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (root, os.path.join(root, "oracle"), here):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import torch.distributed as dist

    import oracle as O
    from arcqml_b200.sharded import DistComm, ShardedBatchSimulator
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=size, timeout=datetime.timedelta(seconds=120))
        from arcqml_b200.workloads import qnn
        circuit, obs, init, labels = qnn(case["n"], case["batch"], case["layers"], case["seed"])
        sim = ShardedBatchSimulator(circuit.num_qubits, init.shape[0], comm=DistComm(),
                                    backend=OracleShardBackend(O))
        sim.load(init)
        vals = sim.run(circuit, obs)
        up = (vals - labels) / len(labels)
        grads = sim.backward(up)
        queue.put((rank, dict(values=vals, grads=grads)))
    except BaseException as e:  # noqa: BLE001 - reported to the parent
        queue.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


class _FakePeerBuffer:
    address = 0

    def handle_bytes(self):
        return bytes(64)

    def destroy(self):
        pass


class FailingPeerBackend(OracleShardBackend):
    """Offers the peer transport, but rank `fail_rank` cannot create its peer buffer."""

    def __init__(self, oracle_module, rank, fail_rank):
        super().__init__(oracle_module)
        self.rank, self.fail_rank = rank, fail_rank

    def peer_buffer(self, nbytes):
        if self.rank == self.fail_rank:
            raise RuntimeError("no peer buffer on this rank")
        return _FakePeerBuffer()

    def gather_from(self, *args):
        raise AssertionError("the peer transport must not run after a failed setup")


def gloo_fallback_worker(rank, size, port, case, queue):
    """One rank of a gloo world whose peer-transport setup fails on rank 1."""
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (root, os.path.join(root, "oracle"), here):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import torch.distributed as dist

    import oracle as O
    from arcqml_b200.sharded import DistComm, ShardedStateVectorSimulator
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=size, timeout=datetime.timedelta(seconds=120))
        sim = ShardedStateVectorSimulator(case["n"], comm=DistComm(),
                                          backend=FailingPeerBackend(O, rank, 1),
                                          chunk_amplitudes=8, transport="peer")
        res = sharded_case(sim, case["ops"], case["terms"], case["init"], case["upstream"],
                           case["req"])
        res["transport"] = sim.transport
        queue.put((rank, res))
    except BaseException as e:  # noqa: BLE001 - reported to the parent
        queue.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()
