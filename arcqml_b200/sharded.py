"""One statevector sharded over the ranks of a process group on its highest ("global") qubits.

With P = 2^g ranks, rank r holds the 2^(n-g) amplitudes whose physical index has r in its top g
bits. A layout maps every logical qubit to a physical bit position; positions below
``n_local = n - g`` are local (inside every shard), the top g are global (the rank's bits).

* Gates run on the ranks' shards through the runtime's device entry points, with qubits renamed
  to their physical positions. An op that touches a global qubit first triggers a swap: the
  needed global qubits trade places with local qubits, chosen as those whose next use lies
  farthest ahead (the layout planner below). The ops between swaps are scheduled as a list over
  the circuit's dependency order (ops on disjoint qubits commute), so every op whose qubits are
  all local runs before a swap is paid.
* A swap of k qubits is an all-to-all among 2^k ranks: each rank packs the slices of its shard
  that belong to the other ranks (``arcqml_rt_v2_shard_slices``), exchanges them with
  point-to-point NCCL calls through ``torch.distributed``, and unpacks what it receives into the
  slots it emptied. Chunks are double-buffered so packing overlaps the transfer.
* The observable's terms are evaluated in groups, one per layout in which no flip bit (X/Y) of
  the group lies on a global qubit; a Z on a global qubit becomes a per-rank sign on the
  coefficient. ``H psi`` accumulates over the groups (``arcqml_rt_v2_expectation_and_accumulate``)
  and moves with psi when the layout changes. The value is summed over ranks. A group that flips
  more qubits than a shard holds (a global qubit is flipped in every layout) is evaluated against
  the partner rank's shard instead, exchanged chunk by chunk (``_partner_terms``).
* The adjoint sweep schedules the reversed op list from the observable's final layout, swaps psi
  and lambda together, and sums the per-rank gradient partials over ranks at the end.

Semantics follow the single-device path (``simulator.StateVectorSimulator``), i.e. the
reference's run/backward (``crates/arcqml-sim/src/statevector/execution/adjoint/single.rs:29-163``)
and observable (``crates/arcqml-observable/src/compiled_hamiltonian.rs:30-182``); results agree
to rounding (ops that commute may run in a different order).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from .circuit import Circuit, PlanOp
from .observable import SparsePauliOp

INF = 1 << 62


class ShardError(ValueError):
    pass


# ---------------------------------------------------------------------------- layout planning


class Layout:
    """Logical qubit -> physical bit position; positions >= n_local are global."""

    def __init__(self, num_qubits: int, global_qubits: int):
        if global_qubits < 0 or global_qubits >= num_qubits:
            raise ShardError(f"cannot shard {num_qubits} qubits over 2^{global_qubits} ranks")
        self.n = num_qubits
        self.g = global_qubits
        self.n_local = num_qubits - global_qubits
        self.pos = list(range(num_qubits))
        self.at = list(range(num_qubits))

    def copy(self) -> "Layout":
        c = Layout.__new__(Layout)
        c.n, c.g, c.n_local = self.n, self.g, self.n_local
        c.pos, c.at = list(self.pos), list(self.at)
        return c

    def is_local(self, q: int) -> bool:
        return self.pos[q] < self.n_local

    def global_qubits(self) -> List[int]:
        return [self.at[p] for p in range(self.n_local, self.n)]

    def apply_swap(self, pairs: Sequence[Tuple[int, int]]) -> None:
        for pg, pl in pairs:
            a, b = self.at[pg], self.at[pl]
            self.at[pg], self.at[pl] = b, a
            self.pos[a], self.pos[b] = pl, pg

    def physical_mask(self, mask: int) -> int:
        out = 0
        q = 0
        while mask:
            if mask & 1:
                out |= 1 << self.pos[q]
            mask >>= 1
            q += 1
        return out


@dataclass
class SwapStep:
    pairs: List[Tuple[int, int]]  # (global position, local position)


@dataclass
class OpsStep:
    ops: List[PlanOp]                                 # qubits renamed to physical positions
    indices: List[int] = field(default_factory=list)  # positions in the input op list


@dataclass
class TermsStep:
    groups: List[int]  # indices into the flip-mask group list


@dataclass
class PartnerStep:
    group: int  # a flip group that flips a global qubit in every layout (see _partner_terms)


def _pair(layout: Layout, bring: Sequence[int], evict: Sequence[int]) -> List[Tuple[int, int]]:
    gpos = sorted(layout.pos[q] for q in bring)
    lpos = sorted(layout.pos[q] for q in evict)
    return list(zip(gpos, lpos))


def schedule_ops(ops: Sequence[PlanOp], layout: Layout) -> Tuple[list, Layout]:
    """List-schedules ops (in dependency order) into OpsStep / SwapStep items.

    Returns the steps and the layout after them; ``layout`` itself is not modified.
    """
    L = layout.copy()
    n = L.n
    m = len(ops)
    for i, op in enumerate(ops):
        if len(set(op.qubits)) > L.n_local:
            raise ShardError(f"operation {i} acts on {len(op.qubits)} qubits, a shard holds "
                             f"only {L.n_local} local qubits")
        for q in op.qubits:
            if not 0 <= q < n:
                raise ShardError(f"operation {i} uses qubit {q} outside the {n}-qubit state")
    queues: List[List[int]] = [[] for _ in range(n)]
    for i, op in enumerate(ops):
        for q in dict.fromkeys(op.qubits):
            queues[q].append(i)
    head = [0] * n

    def is_ready(i):
        return all(head[q] < len(queues[q]) and queues[q][head[q]] == i
                   for q in dict.fromkeys(ops[i].qubits))

    ready = set(i for i in range(m) if is_ready(i))
    steps: list = []
    cur_ops: List[PlanOp] = []
    cur_idx: List[int] = []
    done = 0

    def emit(i):
        op = ops[i]
        cur_ops.append(PlanOp(op.opcode, tuple(L.pos[q] for q in op.qubits), op.params,
                              op.matrix, op.bindings, op.name))
        cur_idx.append(i)
        ready.discard(i)
        for q in dict.fromkeys(op.qubits):
            head[q] += 1
            if head[q] < len(queues[q]):
                j = queues[q][head[q]]
                if is_ready(j):
                    ready.add(j)

    while done < m:
        progressed = True
        while progressed:
            progressed = False
            for i in sorted(ready):
                if i in ready and all(L.is_local(q) for q in ops[i].qubits):
                    emit(i)
                    done += 1
                    progressed = True
        if done == m:
            break
        if cur_ops:
            steps.append(OpsStep(cur_ops, cur_idx))
            cur_ops, cur_idx = [], []
        # bring in the global qubits of as many blocked ops as fit, oldest first
        bring: List[int] = []
        protect: set = set()
        for i in sorted(ready):
            qs = list(dict.fromkeys(ops[i].qubits))
            need = [q for q in qs if not L.is_local(q) and q not in bring]
            prot = protect | {q for q in qs if L.is_local(q)}
            free = [q for q in L.at[:L.n_local] if q not in prot]
            if len(bring) + len(need) <= len(free):
                bring += need
                protect = prot
        assert bring, "scheduler made no progress"
        free = [q for q in L.at[:L.n_local] if q not in protect]

        def next_use(q):
            return queues[q][head[q]] if head[q] < len(queues[q]) else INF

        # farthest next use first; among equals the higher position (longer contiguous runs)
        free.sort(key=lambda q: (-next_use(q), -L.pos[q]))
        evict = free[:len(bring)]
        pairs = _pair(L, bring, evict)
        steps.append(SwapStep(pairs))
        L.apply_swap(pairs)
    if cur_ops:
        steps.append(OpsStep(cur_ops, cur_idx))
    return steps, L


def schedule_terms(flips: Sequence[int], layout: Layout) -> Tuple[list, Layout]:
    """Splits flip-mask groups into TermsStep items, each evaluable with no flip bit on a global
    qubit, separated by SwapStep items; a group that flips more qubits than a shard holds
    becomes a PartnerStep. Returns the steps and the final layout."""
    L = layout.copy()
    n = L.n
    remaining = list(range(len(flips)))
    steps: list = []
    while remaining:
        gmask = 0
        for q in L.global_qubits():
            gmask |= 1 << q
        ok = [i for i in remaining if not (flips[i] & gmask)]
        if ok:
            steps.append(TermsStep(ok))
            okset = set(ok)
            remaining = [i for i in remaining if i not in okset]
        if not remaining:
            break
        first = flips[remaining[0]]
        cand = [q for q in range(n) if not (first >> q) & 1]
        if len(cand) < L.g:  # no layout keeps its flips local
            steps.append(PartnerStep(remaining[0]))
            remaining = remaining[1:]
            continue
        count = [0] * n
        for i in remaining:
            f = flips[i]
            for q in range(n):
                if (f >> q) & 1:
                    count[q] += 1
        cand.sort(key=lambda q: (count[q], 0 if not L.is_local(q) else 1, -L.pos[q]))
        chosen = set(cand[:L.g])
        bring = [q for q in L.global_qubits() if q not in chosen]
        evict = [q for q in chosen if L.is_local(q)]
        pairs = _pair(L, bring, evict)
        steps.append(SwapStep(pairs))
        L.apply_swap(pairs)
    return steps, L


def flip_groups(terms) -> Tuple[List[int], List[List[int]]]:
    """Distinct flip masks in first-appearance order and the term indices of each."""
    flips: List[int] = []
    members: Dict[int, List[int]] = {}
    for k, (_, f, _, _) in enumerate(terms):
        if f not in members:
            members[f] = []
            flips.append(f)
        members[f].append(k)
    return flips, [members[f] for f in flips]


def local_terms(terms, member_lists, layout: Layout, rank: int):
    """(coefficients, local flip masks, local phase masks) of the given term groups on `rank`:
    masks renamed to physical positions; the phase bits on global positions (Z factors only,
    as the groups flip no global qubit) become the sign (-1)^popcount(rank bits & phase)."""
    coef, flip, phase = [], [], []
    local_mask = (1 << layout.n_local) - 1
    for ks in member_lists:
        for k in ks:
            c, f, p, _ = terms[k]
            fp = layout.physical_mask(f)
            pp = layout.physical_mask(p)
            assert fp & ~local_mask == 0
            sign = -1.0 if bin((pp >> layout.n_local) & rank).count("1") & 1 else 1.0
            coef.append(sign * c)
            flip.append(fp)
            phase.append(pp & local_mask)
    return (np.asarray(coef, dtype=np.float64), np.asarray(flip, dtype=np.uint64),
            np.asarray(phase, dtype=np.uint64))


# ---------------------------------------------------------------------------- communication


class DistComm:
    """Point-to-point exchange and sums over a torch.distributed process group."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self.nccl = dist.get_backend(group) == "nccl"

    def _global(self, r: int) -> int:
        if self.group is None:
            return r
        return self.dist.get_global_rank(self.group, r)

    def exchange_start(self, sends: Dict[int, object], recvs: Dict[int, object]):
        """Starts sends[peer] -> peer and recvs[peer] <- peer; returns a handle for wait()."""
        import torch
        ops = []
        for peer in sorted(set(sends) | set(recvs)):
            if peer in sends:
                ops.append(self.dist.P2POp(self.dist.isend, torch.view_as_real(sends[peer]),
                                           self._global(peer), self.group))
            if peer in recvs:
                ops.append(self.dist.P2POp(self.dist.irecv, torch.view_as_real(recvs[peer]),
                                           self._global(peer), self.group))
        return self.dist.batch_isend_irecv(ops) if ops else []

    @staticmethod
    def wait(handle) -> None:
        for w in handle:
            w.wait()

    def nccl_comm(self) -> Optional[int]:
        """The group's raw NCCL communicator (an ncclComm_t address) for the runtime's own
        swaps, or None when the group has none (gloo) or torch does not expose it."""
        if not self.nccl:
            return None
        import torch
        pg = self.group if self.group is not None else self.dist.distributed_c10d._get_default_group()
        try:
            backend = pg._get_backend(torch.device("cuda", torch.cuda.current_device()))
            ptr = int(backend._comm_ptr())
        except Exception:  # noqa: BLE001 - an older torch, or no communicator yet
            return None
        return ptr or None

    def allreduce_sum(self, values: np.ndarray) -> np.ndarray:
        import torch
        dev = torch.device("cuda", torch.cuda.current_device()) if self.nccl else torch.device("cpu")
        t = torch.from_numpy(np.ascontiguousarray(values, dtype=np.float64)).to(dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM, group=self.group)
        return t.cpu().numpy()

    def barrier(self) -> None:
        """Waits for this rank's device work, then for every rank."""
        import torch
        torch.cuda.synchronize()
        if self.nccl:
            self.dist.barrier(group=self.group, device_ids=[torch.cuda.current_device()])
        else:
            self.dist.barrier(group=self.group)

    def same_node(self) -> bool:
        import socket
        names = [None] * self.size
        self.dist.all_gather_object(names, socket.gethostname(), group=self.group)
        return len(set(names)) == 1

    def allgather_object(self, obj) -> list:
        out = [None] * self.size
        self.dist.all_gather_object(out, obj, group=self.group)
        return out

    def allgather(self, shard):
        import torch
        parts = [torch.empty_like(shard) for _ in range(self.size)]
        self.dist.all_gather([torch.view_as_real(p) for p in parts], torch.view_as_real(shard),
                             group=self.group)
        return parts


# ---------------------------------------------------------------------------- device backend


class RuntimeBackend:
    """Local compute on this rank's GPU through the runtime's v2 entry points."""

    def __init__(self, device=None):
        import torch
        from . import runtime as rt
        if not torch.cuda.is_available():
            raise ShardError("the sharded statevector runtime needs a CUDA device")
        self.rt = rt
        self.torch = torch
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())

    def empty(self, numel: int):
        return self.torch.empty(numel, dtype=self.torch.complex128, device=self.device)

    def zeros(self, numel: int):
        return self.torch.zeros(numel, dtype=self.torch.complex128, device=self.device)

    def from_numpy(self, a: np.ndarray):
        return self.torch.from_numpy(np.ascontiguousarray(a, dtype=np.complex128)).to(self.device)

    def set_amplitude_one(self, shard, index: int) -> None:
        """shard <- |index> (every other amplitude zero)."""
        self.rt.set_basis_state_device(shard, int(shard.numel()).bit_length() - 1, index)

    def _plan(self, ops: Sequence[PlanOp]):
        """A plan of these operations. Plans are kept by structure (rt.plan_structure_key): one
        seen before gets the operations' bound values (arcqml_rt_v2_plan_set_parameters)
        instead of every operation being marshalled through the C ABI again. Each plan is used
        at once by the call that asks for it."""
        key = self.rt.plan_structure_key(ops)
        plans = self.__dict__.setdefault("_plans", {})
        plan = plans.get(key)
        values = None if plan is None else self.rt.plan_bound_values(ops)
        if plan is not None and values is not None:
            plan.set_parameters(values)
            return plan
        plan = self.rt.CircuitPlan.create(ops)
        if len(plans) >= 256:
            plans.clear()
        plans[key] = plan
        return plan

    def apply(self, ops: Sequence[PlanOp], shard, n_local: int) -> None:
        if not ops:
            return
        self.rt.plan_apply_device(self._plan(ops), shard, n_local)

    def adjoint(self, ops: Sequence[PlanOp], psi, lam, n_local: int, upstream, req,
                grads: np.ndarray) -> None:
        """Reverse sweep over [rows, 2^n_local] psi/lambda; upstream is a scalar or one factor
        per row; gradients (summed over rows) are added to grads."""
        grads += self.rt.adjoint_backward_device(self._plan(ops), psi, lam, n_local, upstream,
                                                 req, len(grads))

    def observable(self, coef, flip, phase, psi, out, n_local: int) -> float:
        return float(self.observable_rows(coef, flip, phase, psi, out, n_local)[0])

    def scale(self, x, factor: complex, out, n_local: int) -> None:
        """out <- factor * x."""
        self.rt.scaled_copy_device(x, n_local, [factor], out=out)

    def observable_rows(self, coef, flip, phase, psi, out, n_local: int) -> np.ndarray:
        """Per-row <psi|H|psi>; adds H psi to out when given."""
        obs = self.rt.Observable(n_local, coef, flip, phase)
        if out is None:
            return obs.expectation(psi, n_local)
        return obs.expectation_and_accumulate(psi, out, n_local)

    def slices(self, shard, n_local, positions, chunk_begin, chunk_len, skip, staging,
               unpack) -> None:
        self.rt.shard_slices(shard, n_local, positions, chunk_begin, chunk_len, skip, staging,
                             unpack)

    # -- peer transport (device addresses) --
    def marginal(self, shard, n_local: int, positions) -> np.ndarray:
        return self.rt.marginal_probabilities_device(shard, n_local, list(positions)).cpu().numpy()

    def bloch(self, shard, n_local: int, position: int) -> np.ndarray:
        return self.rt.bloch_vector_device(shard, n_local, position)

    def overlap(self, a, b, n_local: int) -> complex:
        return self.rt.overlap_device(a, b, n_local)

    def norm(self, shard, n_local: int) -> float:
        return float(self.rt.norms_device(shard, n_local)[0])

    def peer_buffer(self, nbytes: int):
        return self.rt.PeerBuffer(nbytes)

    def pack_to(self, shard, n_local, positions, chunk_begin, chunk_len, skip, address) -> None:
        self.rt.shard_slices_ptr(shard, n_local, positions, chunk_begin, chunk_len, skip, address,
                                 False)

    def gather_from(self, shard, n_local, positions, chunk_begin, chunk_len, sources) -> None:
        self.rt.shard_slices_from(shard, n_local, positions, chunk_begin, chunk_len, sources)

    def swap_nccl(self, shard, n_local, global_bits, local_positions, comm_ptr, staging) -> None:
        self.rt.shard_swap_nccl(shard, n_local, global_bits, local_positions, comm_ptr, staging)

    def peer_open(self, handle: bytes) -> int:
        return self.rt.PeerBuffer.open(handle)

    def peer_close(self, address: int) -> None:
        self.rt.PeerBuffer.close(address)


# ---------------------------------------------------------------------------- simulator


@dataclass
class SwapStats:
    swaps: int = 0
    qubits: int = 0
    bytes_sent: int = 0


class ShardedStateVectorSimulator:
    """A single n-qubit state over all ranks of ``comm`` (a power-of-two count).

    ``run(circuit, observable)`` returns ``(value, ctx)``-style results like
    ``StateVectorSimulator.run``; ``backward(upstream)`` returns the parameter gradients summed
    over ranks (same on every rank).
    """

    def __init__(self, num_qubits: int, comm=None, backend=None, chunk_amplitudes: int = 1 << 24,
                 transport: Optional[str] = None, peer_bytes: int = 2 << 30):
        self.comm = comm if comm is not None else DistComm()
        self.backend = backend if backend is not None else RuntimeBackend()
        size = self.comm.size
        if size & (size - 1):
            raise ShardError(f"world size {size} is not a power of two")
        g = size.bit_length() - 1
        if num_qubits - g < 1:
            raise ShardError(f"{num_qubits} qubits cannot be sharded over {size} ranks")
        self.num_qubits = num_qubits
        self.layout = Layout(num_qubits, g)
        self.rank = self.comm.rank
        self.chunk = max(1, int(chunk_amplitudes))
        self.stats = SwapStats()
        self._events = None
        self._staging = None
        # Swap transport: "peer" (each rank gathers its slices from the peers' packed buffers
        # over NVLink with its own kernel) when every rank can map the others' memory, else
        # "p2p" (point-to-point sends through the communicator); "nccl" (the runtime's
        # arcqml_rt_v2_shard_swap_nccl on the group's own NCCL communicator) on request.
        # ARCQML_SWAP overrides.
        import os
        want = transport or os.environ.get("ARCQML_SWAP") or "auto"
        if want not in ("auto", "peer", "p2p", "nccl"):
            raise ShardError(f"unknown swap transport {want!r}")
        if want == "nccl" and not (hasattr(self.backend, "swap_nccl") and
                                   getattr(self.comm, "nccl_comm", lambda: None)() is not None):
            raise ShardError("the nccl swap transport needs an NCCL process group and the "
                             "GPU backend")
        can_peer = (size > 1 and hasattr(self.comm, "allgather_object") and
                    hasattr(self.backend, "gather_from"))
        if want == "auto":
            want = "peer" if can_peer and self.comm.same_node() else "p2p"
        if want == "peer" and not can_peer:
            raise ShardError("the peer swap transport needs allgather_object and gather_from")
        self.transport = want
        self._peer_bytes = int(peer_bytes)
        self._peer = None  # (buffer, {rank: address})
        self.psi = None
        self.lam = None
        self._ctx = None

    @property
    def n_local(self) -> int:
        return self.layout.n_local

    # -- state ---------------------------------------------------------------------------
    def reset(self) -> None:
        """|0...0>: amplitude 1 at physical index 0, which rank 0 holds."""
        self.layout = Layout(self.num_qubits, self.layout.g)
        d = 1 << self.n_local
        if self.psi is None or self.psi.numel() != d:
            self.psi = self.backend.empty(d)
        if self.rank == 0:
            self.backend.set_amplitude_one(self.psi, 0)
        else:
            self.psi.zero_()

    def load(self, full_amplitudes) -> None:
        """Takes this rank's part of a full state given in logical order (tests, small n)."""
        self.layout = Layout(self.num_qubits, self.layout.g)
        a = np.ascontiguousarray(full_amplitudes, dtype=np.complex128).reshape(-1)
        d = 1 << self.n_local
        self.psi = self.backend.from_numpy(a[self.rank * d:(self.rank + 1) * d])

    def amplitudes(self, which: str = "psi") -> np.ndarray:
        """Full state in logical order on every rank (gathers all shards; tests, small n)."""
        shard = self.psi if which == "psi" else self.lam
        parts = self.comm.allgather(shard.contiguous())
        full = np.concatenate([p.cpu().numpy() for p in parts])
        n = self.num_qubits
        idx = np.arange(1 << n, dtype=np.int64)
        phys = np.zeros_like(idx)
        for q in range(n):
            phys |= ((idx >> q) & 1) << self.layout.pos[q]
        return full[phys]

    def amplitudes_at(self, indices, which: str = "psi") -> np.ndarray:
        """Amplitudes at the given logical basis indices, on every rank (collective): each rank
        reads the ones its shard holds, and one all-reduce assembles them. For checks of
        states too large to gather whole."""
        shard = self.psi if which == "psi" else self.lam
        idx = np.asarray(indices, dtype=np.int64).reshape(-1)
        if idx.size and (idx.min() < 0 or idx.max() >= (1 << self.num_qubits)):
            raise ShardError("basis index outside the state")
        phys = np.zeros_like(idx)
        for q in range(self.num_qubits):
            phys |= ((idx >> q) & 1) << self.layout.pos[q]
        n_local = self.n_local
        mine = (phys >> n_local) == self.rank
        out = np.zeros(2 * idx.size, dtype=np.float64)
        if mine.any():
            import torch
            local = torch.from_numpy(phys[mine] & ((1 << n_local) - 1)).to(shard.device)
            vals = shard.index_select(0, local).cpu().numpy()
            out[0::2][mine] = vals.real
            out[1::2][mine] = vals.imag
        tot = self.comm.allreduce_sum(out)
        return tot[0::2] + 1j * tot[1::2]

    # -- swaps ---------------------------------------------------------------------------
    def timing(self, on: bool):
        """Starts (True) or stops (False) timing the swaps with CUDA events on the current
        stream; stopping returns {swaps, qubits, bytes_sent, ms} since the start."""
        import torch
        if on:
            self.stats = SwapStats()
            self._events = []
            return None
        torch.cuda.synchronize()
        ms = sum(a.elapsed_time(b) for a, b in (self._events or []))
        self._events = None
        return dict(swaps=self.stats.swaps, qubits=self.stats.qubits,
                    bytes_sent=self.stats.bytes_sent, ms=ms)

    def _staging_for(self, numel: int):
        if self._staging is None or self._staging[0][0].numel() < numel:
            self._staging = [(self.backend.empty(numel), self.backend.empty(numel))
                             for _ in range(2)]
        return self._staging

    def close(self) -> None:
        """Releases the peer mappings and buffer (collective: every rank calls it)."""
        if self._peer is not None:
            buf, addrs = self._peer
            self.comm.barrier()
            if not getattr(self.comm, "same_process", False):
                for r, a in addrs.items():
                    if r != self.rank:
                        self.backend.peer_close(a)
            self.comm.barrier()
            buf.destroy()
            self._peer = None

    def _share_peer_buffer(self):
        """Creates this rank's peer buffer and maps every other rank's (collective); None on
        every rank if any rank failed, after undoing what succeeded."""
        same = getattr(self.comm, "same_process", False)
        buf, handle = None, None
        try:
            buf = self.backend.peer_buffer(self._peer_bytes)
            handle = buf.address if same else buf.handle_bytes()
        except Exception:  # noqa: BLE001 - reported to the other ranks below
            handle = None
        handles = self.comm.allgather_object(handle)
        addrs, ok = {}, all(h is not None for h in handles)
        if ok:
            try:
                for r, h in enumerate(handles):
                    addrs[r] = buf.address if r == self.rank else (h if same else
                                                                    self.backend.peer_open(h))
            except Exception:  # noqa: BLE001 - reported to the other ranks below
                ok = False
        failed = float(self.comm.allreduce_sum(np.array([0.0 if ok else 1.0]))[0])
        if failed == 0.0:
            return buf, addrs
        if not same:
            for r, a in addrs.items():
                if r != self.rank:
                    self.backend.peer_close(a)
        if buf is not None:
            buf.destroy()
        return None

    def _pack_stream(self):
        """A second CUDA stream for the peer transport's packs (None off the GPU backend)."""
        if not isinstance(self.backend, RuntimeBackend):
            return None
        if getattr(self, "_packs", None) is None:
            import torch
            self._packs = torch.cuda.Stream()
        return self._packs

    def _peer_swap(self, t, n_l, lpos, x, peers, others) -> int:
        """Moves one tensor's slices through the peers' buffers; returns the chunk length."""
        buf, addrs = self._peer
        half = self._peer_bytes // 2
        chunk = min(others, max(1, half // (16 * ((1 << self.layout.g) - 1))))
        chunk = 1 << (chunk.bit_length() - 1)
        starts = list(range(0, others, chunk))
        be = self.backend

        def region(rank, c):  # buffer half of chunk c in `rank`'s buffer
            return addrs[rank] + (c & 1) * half

        # On a GPU the packs run on their own stream, so that packing chunk c + 1 (local HBM)
        # overlaps gathering chunk c (NVLink): they touch disjoint slots of the shard and
        # different buffer halves, and every barrier synchronises the whole device.
        ps = self._pack_stream()
        if ps is not None:
            import torch
            ps.wait_stream(torch.cuda.current_stream())

        def pack(c):
            if ps is None:
                be.pack_to(t, n_l, lpos, starts[c], chunk, x, region(self.rank, c))
            else:
                import torch
                with torch.cuda.stream(ps):
                    be.pack_to(t, n_l, lpos, starts[c], chunk, x, region(self.rank, c))

        # Pack chunk c into half c % 2 of this rank's buffer (block order: slice values but
        # this rank's own); after a barrier every rank gathers chunk c from the peers' halves
        # while packing chunk c + 1 into its other half; one barrier per chunk.
        pack(0)
        self.comm.barrier()
        for c, c0 in enumerate(starts):
            if c + 1 < len(starts):
                pack(c + 1)
            sources = [None] * (1 << len(lpos))
            for y, r in peers.items():
                blk = x - (1 if x > y else 0)  # rank r skipped its own value y when packing
                sources[y] = region(r, c) + blk * chunk * 16
            be.gather_from(t, n_l, lpos, c0, chunk, sources)
            self.comm.barrier()
        return chunk

    def _swap(self, pairs: Sequence[Tuple[int, int]], tensors: Sequence) -> None:
        L = self.layout
        n_l = L.n_local
        k = len(pairs)
        gbits = [pg - n_l for pg, _ in pairs]
        lpos = [pl for _, pl in pairs]
        x = 0
        for i, b in enumerate(gbits):
            x |= ((self.rank >> b) & 1) << i
        peers = {}
        for y in range(1 << k):
            if y == x:
                continue
            r = self.rank
            for i, b in enumerate(gbits):
                r = (r & ~(1 << b)) | (((y >> i) & 1) << b)
            peers[y] = r
        others = 1 << (n_l - k)
        nblk = (1 << k) - 1
        be = self.backend
        ev = None
        if self._events is not None:
            import torch
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        if self.transport == "peer" and self._peer is None:
            self._peer = self._share_peer_buffer()
            if self._peer is None:
                self.transport = "p2p"
        if self.transport == "nccl":
            # the runtime's own swap (arcqml_rt_v2_shard_swap_nccl) over the group's communicator
            chunk = min(others, max(1, self.chunk // nblk))
            chunk = 1 << (chunk.bit_length() - 1)
            if getattr(self, "_nccl_stage", None) is None or \
                    self._nccl_stage.numel() < 2 * nblk * chunk:
                self._nccl_stage = be.empty(2 * nblk * chunk)
            ptr = self.comm.nccl_comm()
            for t in tensors:
                be.swap_nccl(t, n_l, gbits, lpos, ptr, self._nccl_stage)
            if ev is not None:
                ev[1].record()
                self._events.append(ev)
            self.stats.swaps += 1
            self.stats.qubits += k
            self.stats.bytes_sent += len(tensors) * nblk * others * 16
            L.apply_swap(pairs)
            return
        if self.transport == "peer":
            for t in tensors:
                self._peer_swap(t, n_l, lpos, x, peers, others)
            if ev is not None:
                ev[1].record()
                self._events.append(ev)
            self.stats.swaps += 1
            self.stats.qubits += k
            self.stats.bytes_sent += len(tensors) * nblk * others * 16
            L.apply_swap(pairs)
            return
        chunk = min(others, max(1, self.chunk // nblk))
        chunk = 1 << (chunk.bit_length() - 1)
        stage = self._staging_for(nblk * chunk)

        def views(buf):
            return {peers[y]: buf[(y - (1 if y > x else 0)) * chunk:
                                  (y - (1 if y > x else 0) + 1) * chunk] for y in peers}

        # Two staging sets: chunk j is packed and put on the wire while chunk j-1, already
        # received, is unpacked.
        jobs = [(t, c0) for t in tensors for c0 in range(0, others, chunk)]
        pending = None  # (tensor, c0, recv buffer, handle)
        for j, (t, c0) in enumerate(jobs):
            send, recv = stage[j & 1]
            be.slices(t, n_l, lpos, c0, chunk, x, send, False)
            h = self.comm.exchange_start(views(send), views(recv))
            if pending is not None:
                pt, pc0, precv, ph = pending
                self.comm.wait(ph)
                be.slices(pt, n_l, lpos, pc0, chunk, x, precv, True)
            pending = (t, c0, recv, h)
        if pending is not None:
            pt, pc0, precv, ph = pending
            self.comm.wait(ph)
            be.slices(pt, n_l, lpos, pc0, chunk, x, precv, True)
        if ev is not None:
            ev[1].record()
            self._events.append(ev)
        self.stats.swaps += 1
        self.stats.qubits += k
        self.stats.bytes_sent += len(tensors) * nblk * others * 16
        L.apply_swap(pairs)

    # -- forward / observable / adjoint on plan ops -------------------------------------------
    def forward(self, ops: Sequence[PlanOp]) -> None:
        """psi <- U_m ... U_1 psi for plan ops in logical qubits (starts from |0...0> if unset)."""
        if self.psi is None:
            self.reset()
        steps, _ = schedule_ops(ops, self.layout)
        for st in steps:
            if isinstance(st, SwapStep):
                self._swap(st.pairs, [self.psi])
            else:
                self.backend.apply(st.ops, self.psi, self.n_local)

    def observe(self, terms, keep_lambda: bool) -> float:
        """<psi|H|psi> summed over ranks for compiled terms (coef, flip, phase, y); with
        keep_lambda the shards of H psi are kept (as lambda) for ``adjoint``."""
        flips, members = flip_groups(terms)
        if keep_lambda:
            if self.lam is None or self.lam.numel() != self.psi.numel():
                self.lam = self.backend.empty(self.psi.numel())
            self.lam.zero_()
        else:
            self.lam = None
        tsteps, _ = schedule_terms(flips, self.layout)
        partial = 0.0
        for st in tsteps:
            if isinstance(st, SwapStep):
                self._swap(st.pairs, [self.psi] + ([self.lam] if keep_lambda else []))
            elif isinstance(st, PartnerStep):
                partial += self._partner_terms(terms, members[st.group], flips[st.group],
                                               keep_lambda)
            else:
                coef, flip, phase = local_terms(terms, [members[i] for i in st.groups],
                                                self.layout, self.rank)
                partial += self.backend.observable(coef, flip, phase, self.psi, self.lam,
                                                   self.n_local)
        return float(self.comm.allreduce_sum(np.array([partial]))[0])

    def _partner_terms(self, terms, ks, flip: int, keep_lambda: bool) -> float:
        """This rank's part of <psi|H_g|psi> (and H_g psi into lambda) for the terms ks of one
        flip group whose flips cover a global qubit in every layout.

        With physical masks split into the rank bits (fg, pg), the chunk bits above the low
        n_c local bits (ftop, ptop) and the low bits (flow, plow), a Pauli string P with
        y = popcount(f & p) acts on index t = (R, c, j) as
        (P psi)[t] = i^y (-1)^popcount((t ^ f) & p) psi[t ^ f], and t ^ f = (R ^ fg, c ^ ftop,
        j ^ flow) lies on the partner rank R' = R ^ fg. So chunk c of (P psi) on this rank is
        alpha * P_low b, where b is chunk c ^ ftop of the partner's shard, P_low the string with
        masks (flow, plow) on n_c qubits (the runtime's observable, with its own i^y) and
        alpha = i^(popcount(fg & pg) + popcount(ftop & ptop)) (-1)^popcount(R' & pg)
        (-1)^popcount((c ^ ftop) & ptop). Terms are grouped by the power of i: for each power
        the received chunk is multiplied by it (exact) and the real-coefficient sum is applied
        once into lambda and once into a zeroed chunk x, whose overlap with this rank's chunk c
        of psi gives the value. The partner computes the complex conjugate contributions, so
        each rank adds the real part. Every rank sends its chunk c ^ ftop to its partner while
        receiving the partner's, chunk by chunk, in the same order on every rank."""
        L = self.layout
        n_l = L.n_local
        be = self.backend
        fp = L.physical_mask(flip)
        fg, fl = fp >> n_l, fp & ((1 << n_l) - 1)
        partner = self.rank ^ fg
        n_c = min(n_l, max(1, self.chunk.bit_length() - 1))  # chunks of at least one qubit
        cs = 1 << n_c
        ftop, flow = fl >> n_c, fl & (cs - 1)
        # per term: coefficient, rank-bit phase mask, chunk-bit phase mask, low phase mask, i power
        rows = []
        for k in ks:
            c, _, p, _ = terms[k]
            pp = L.physical_mask(p)
            pg, pl = pp >> n_l, pp & ((1 << n_l) - 1)
            ptop, plow = pl >> n_c, pl & (cs - 1)
            m = (bin(fg & pg).count("1") + bin(ftop & ptop).count("1")) % 4
            sign = -1.0 if bin(partner & pg).count("1") & 1 else 1.0
            rows.append((sign * float(c), ptop, plow, m))
        powers = sorted({r[3] for r in rows})
        unit = [1.0, 1j, -1.0, -1j]
        b = be.empty(cs)
        b2 = be.empty(cs)
        x = be.empty(cs)
        value = 0.0
        for c in range(1 << (n_l - n_c)):
            src = c ^ ftop
            h = self.comm.exchange_start({partner: self.psi[src * cs:(src + 1) * cs]},
                                         {partner: b})
            self.comm.wait(h)
            for m in powers:
                sel = [r for r in rows if r[3] == m]
                coef = np.array([r[0] * (-1.0 if bin(src & r[1]).count("1") & 1 else 1.0)
                                 for r in sel], dtype=np.float64)
                fmask = np.full(len(sel), flow, dtype=np.uint64)
                pmask = np.array([r[2] for r in sel], dtype=np.uint64)
                be.scale(b, unit[m], b2, n_c)
                if keep_lambda:
                    be.observable(coef, fmask, pmask, b2, self.lam[c * cs:(c + 1) * cs], n_c)
                x.zero_()
                be.observable(coef, fmask, pmask, b2, x, n_c)
                value += be.overlap(self.psi[c * cs:(c + 1) * cs], x, n_c).real
        return value

    def adjoint(self, ops: Sequence[PlanOp], upstream: float, requires_grad) -> np.ndarray:
        """Reverse sweep over ops from (psi, lambda = H psi): lambda <- g lambda, then per op
        psi <- U^dag psi, grads[parent] += 2 Re<lambda|dU psi>, lambda <- U^dag lambda. Returns
        the gradients summed over ranks (len(requires_grad) entries, index = parent)."""
        if self.lam is None:
            raise ShardError("adjoint needs lambda: call observe(..., keep_lambda=True) first")
        req = list(requires_grad)
        steps, _ = schedule_ops(list(reversed(ops)), self.layout)
        grads = np.zeros(len(req), dtype=np.float64)
        first = True
        for st in steps:
            if isinstance(st, SwapStep):
                self._swap(st.pairs, [self.psi, self.lam])
            else:
                self.backend.adjoint(list(reversed(st.ops)), self.psi, self.lam, self.n_local,
                                     upstream if first else 1.0, req, grads)
                first = False
        if first:
            self.backend.adjoint([], self.psi, self.lam, self.n_local, upstream, req, grads)
        return self.comm.allreduce_sum(grads)

    # -- run / backward (circuit API) ----------------------------------------------------------
    def run(self, circuit: Circuit, observable: SparsePauliOp, grad: bool = True,
            initial_shard=None) -> float:
        """Applies the circuit to |0...0> (or to ``initial_shard``: this rank's 2^n_local
        amplitudes of the initial state in logical order, e.g. a pinned host tensor, copied on
        the current stream) and returns <H>; keeps psi and H psi for ``backward``."""
        if circuit.num_qubits != self.num_qubits or observable.num_qubits != self.num_qubits:
            raise ShardError("circuit, observable and simulator qubit counts differ")
        records = grad and any(p.requires_grad for p in circuit.parameters)
        ops = circuit.compile_plan(1 if records else 0)
        if initial_shard is None:
            self.reset()
        else:
            if initial_shard.numel() != (1 << self.n_local):
                raise ShardError(f"initial shard must hold 2^{self.n_local} amplitudes")
            self.layout = Layout(self.num_qubits, self.layout.g)
            if self.psi is None or self.psi.numel() != initial_shard.numel():
                self.psi = self.backend.empty(initial_shard.numel())
            self.psi.copy_(initial_shard.reshape(-1), non_blocking=True)
        self.forward(ops)
        value = self.observe(observable.compiled_terms(), records)
        self._ctx = (ops, circuit) if records else None
        return value

    def backward(self, upstream: float = 1.0) -> np.ndarray:
        """Adjoint sweep; returns the parameter gradients (index i = circuit parameter i)."""
        if self._ctx is None:
            raise ShardError("run was executed without gradient recording")
        ops, circuit = self._ctx
        grads = self.adjoint(ops, upstream, circuit.requires_grad_mask(True, False))
        self._ctx = None
        pgrads = grads[1:].copy()
        for p, g in zip(circuit.parameters, pgrads):
            if p.requires_grad:
                g = float(np.float32(g)) if p.dtype == "f32" else float(g)
                p.grad = g if getattr(p, "grad", None) is None else p.grad + g
        return pgrads


    # -- analysis (crates/arcqml-analysis/src/statevector on the sharded state) -----------
    def _check_qubit(self, q: int) -> None:
        if not 0 <= q < self.num_qubits:
            raise ShardError(f"qubit index out of range: simulator has {self.num_qubits} "
                             f"qubits, got {q}")

    def marginal_probabilities(self, qubits) -> np.ndarray:
        """Marginal probabilities of logical qubits, the highest selected qubit as the most
        significant output bit (marginal.rs:9-32), on every rank. Each rank sums its shard over
        the selected local qubits at their physical positions; a selected global qubit reads the
        rank's own bit; one all-reduce of the 2^k bins. No amplitude moves between ranks."""
        qubits = [int(q) for q in qubits]
        if not qubits:
            raise ShardError("at least one qubit must be selected")
        seen = set()
        for q in qubits:
            self._check_qubit(q)
            if q in seen:
                raise ShardError(f"duplicate qubit in selection: {q}")
            seen.add(q)
        if self.psi is None:
            self.reset()
        L = self.layout
        disp = sorted(qubits, reverse=True)
        lphys = sorted((L.pos[q] for q in disp if L.is_local(q)), reverse=True)
        if lphys:
            part = np.asarray(self.backend.marginal(self.psi, self.n_local, lphys))
        else:
            part = np.array([self.backend.norm(self.psi, self.n_local)])
        out = np.zeros(1 << len(disp))
        mm = np.arange(part.size)
        m = np.zeros(part.size, dtype=np.int64)
        for q in disp:  # logical bin of every local bin
            if L.is_local(q):
                bit = (mm >> (len(lphys) - 1 - lphys.index(L.pos[q]))) & 1
            else:
                bit = np.full(part.size, (self.rank >> (L.pos[q] - self.n_local)) & 1)
            m = (m << 1) | bit
        np.add.at(out, m, part)
        return self.comm.allreduce_sum(out)

    def bloch_vector(self, qubit: int) -> np.ndarray:
        """(<X>, <Y>, <Z>) of a logical qubit (bloch.rs:23-56), on every rank. A global qubit
        is first swapped with the highest local position (psi and a kept lambda together), since
        its X and Y parts pair amplitudes of different ranks."""
        q = int(qubit)
        self._check_qubit(q)
        if self.psi is None:
            self.reset()
        if not self.layout.is_local(q):
            tensors = [self.psi] + ([self.lam] if self.lam is not None else [])
            self._swap([(self.layout.pos[q], self.n_local - 1)], tensors)
        v = np.asarray(self.backend.bloch(self.psi, self.n_local, self.layout.pos[q]), float)
        return self.comm.allreduce_sum(v)

    def overlap(self, other: "ShardedStateVectorSimulator") -> complex:
        """<self|other> over all ranks; both states must be in the same qubit layout (two states
        from circuits of the same structure, or freshly loaded ones are)."""
        if other.num_qubits != self.num_qubits:
            raise ShardError("cannot compare states with different qubit counts: "
                             f"{self.num_qubits} and {other.num_qubits}")
        if other.layout.pos != self.layout.pos:
            raise ShardError("overlap needs both states in the same qubit layout")
        if self.psi is None:
            self.reset()
        if other.psi is None:
            other.reset()
        s = self.backend.overlap(self.psi, other.psi, self.n_local)
        v = self.comm.allreduce_sum(np.array([s.real, s.imag]))
        return complex(v[0], v[1])

    def fidelity(self, other: "ShardedStateVectorSimulator") -> float:
        """|<self|other>|^2 (fidelity.rs:14-30)."""
        s = self.overlap(other)
        h = float(np.hypot(s.real, s.imag))
        return h * h


# ---------------------------------------------------------------------------- batch rows


class ShardedBatchSimulator:
    """[batch, 2^n] rows split over the ranks of ``comm`` in contiguous blocks.

    Mirrors ``BatchStateVectorSimulator`` (rows independent, per-row upstream factors, gradients
    summed over rows: ``crates/arcqml-sim/src/statevector/execution/adjoint/row_major.rs:108-162``)
    with the rows of each rank on its own GPU: ``run`` returns all B values (gathered), and
    ``backward`` returns the gradients summed over every row of every rank.
    """

    def __init__(self, num_qubits: int, batch_size: int, comm=None, backend=None):
        self.comm = comm if comm is not None else DistComm()
        self.backend = backend if backend is not None else RuntimeBackend()
        size = self.comm.size
        if batch_size < size:
            raise ShardError(f"batch of {batch_size} rows cannot be split over {size} ranks")
        self.num_qubits = num_qubits
        self.batch_size = batch_size
        counts = [batch_size // size + (1 if r < batch_size % size else 0) for r in range(size)]
        self.row_begin = sum(counts[:self.comm.rank])
        self.rows = counts[self.comm.rank]
        self.state = None
        self._ctx = None

    def load(self, full_rows) -> None:
        """Takes this rank's rows of a [batch, 2^n] initial state."""
        a = np.ascontiguousarray(full_rows, dtype=np.complex128).reshape(self.batch_size, -1)
        if a.shape[1] != (1 << self.num_qubits):
            raise ShardError(f"batch state must have shape [{self.batch_size}, {1 << self.num_qubits}]")
        self.state = self.backend.from_numpy(a[self.row_begin:self.row_begin + self.rows])

    def _gather_rows(self, local: np.ndarray) -> np.ndarray:
        full = np.zeros(self.batch_size, dtype=np.float64)
        full[self.row_begin:self.row_begin + self.rows] = local
        return self.comm.allreduce_sum(full)

    def run(self, circuit: Circuit, observable: SparsePauliOp, grad: bool = True) -> np.ndarray:
        """Values of all B rows; keeps psi and H psi of this rank's rows for ``backward``."""
        if circuit.num_qubits != self.num_qubits or observable.num_qubits != self.num_qubits:
            raise ShardError("circuit, observable and state qubit counts differ")
        if self.state is None:
            raise ShardError("load the batch state first")
        records = grad and any(p.requires_grad for p in circuit.parameters)
        ops = circuit.compile_plan(1 if records else 0)
        n = self.num_qubits
        psi = self.state.clone()
        self.backend.apply(ops, psi, n)
        coef, flip, phase = (np.asarray(x) for x in observable.masks())
        lam = None
        if records:
            lam = self.backend.zeros(psi.numel()).reshape(psi.shape)
        vals = self.backend.observable_rows(coef, flip, phase, psi, lam, n)
        self._ctx = (ops, circuit, psi, lam) if records else None
        return self._gather_rows(np.asarray(vals, dtype=np.float64))

    def backward(self, upstream) -> np.ndarray:
        """Per-row upstream factors (length B, or a scalar); returns the parameter gradients
        summed over all rows of all ranks."""
        if self._ctx is None:
            raise ShardError("run was executed without gradient recording")
        ops, circuit, psi, lam = self._ctx
        up = np.broadcast_to(np.asarray(upstream, dtype=np.float64), (self.batch_size,))
        mine = np.ascontiguousarray(up[self.row_begin:self.row_begin + self.rows])
        req = circuit.requires_grad_mask(True, False)
        grads = np.zeros(len(req), dtype=np.float64)
        self.backend.adjoint(ops, psi, lam, self.num_qubits, mine, req, grads)
        grads = self.comm.allreduce_sum(grads)
        self._ctx = None
        pgrads = grads[1:].copy()
        for p, g in zip(circuit.parameters, pgrads):
            if p.requires_grad:
                g = float(np.float32(g)) if p.dtype == "f32" else float(g)
                p.grad = g if getattr(p, "grad", None) is None else p.grad + g
        return pgrads
