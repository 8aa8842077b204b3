"""Benchmark: 32-qubit brickwork circuit, forward + <H> + full adjoint gradient on B200.

Workload (one step): |0...0> on 32 qubits (complex128, 64 GiB per state); 20 brickwork layers
(two random-axis rotations per qubit per layer, CZ on alternating neighbour pairs: 1280
parameters, 1590 gates); a 200-term random Pauli observable; forward pass, expectation and
H|psi> in one pass, then the adjoint reverse sweep producing all 1280 parameter gradients.
Inputs are seeded synthetic data (no dataset). The state (64 GiB) is far larger than L2, so no
L2 flush is needed between steps.

Reported value: gate passes per second = (gates applied forward + gates un-applied in the
adjoint sweep) x steps / device time. ``e2e`` times the same step through the public simulator
API with the initial state copied from pinned host memory every step and the value and
gradients read back to the host.

With ``--gpus N`` (N > 1, one process per GPU under torchrun) the same 32-qubit state is sharded
over the N GPUs on its top log2(N) qubits (``arcqml_b200.sharded``): strong scaling, the
whole-job rate over the max-over-ranks device time. Global-qubit swaps gather the peers'
packed slices over NVLink from CUDA IPC buffers (``ARCQML_SWAP=p2p|nccl`` for NCCL
point-to-point instead); their count, bytes and time are reported under ``swaps``.

``--impl reference`` times the CPU oracle (the f64 restatement of the reference's algorithm;
the reference's own runtime is a closed Windows library) on the host cores: each step a bounded
sample of the same workload at 28 qubits (per-gate forward and adjoint costs of each gate kind,
the observable's per-term cost), the 32-qubit step extrapolated from it by state size.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# DRAM bytes per amplitude of one pass from ncu (dram__bytes_read.sum + dram__bytes_write.sum)
# on 26-qubit passes of this workload: forward 1.106 + 1.032 GB, adjoint 2.206 + 2.088 GB,
# observable tile pass 2.801 + 1.030 GB per 2^26 amplitudes; a pass's traffic grows with the
# state it streams.
NCU_DRAM_BYTES_PER_AMP = {"fused_forward": 2.138e9 / 2 ** 26, "fused_adjoint": 4.294e9 / 2 ** 26,
                          "observable": 3.831e9 / 2 ** 26}

METRIC = "gate passes/s (32q 20-layer brickwork forward + adjoint gradient, 200-term <H>)"
UNIT = "gate_passes/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--qubits", type=int, default=32)
    ap.add_argument("--layers", type=int, default=20)
    ap.add_argument("--terms", type=int, default=200)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--forward-only", action="store_true",
                    help="forward + <H> without the adjoint sweep (the 35-qubit sharded config)")
    ap.add_argument("--workload", default="brickwork",
                    choices=["brickwork", "vqe4", "qnn", "analysis"],
                    help="vqe4: the 4-qubit VQE's 100 Adam steps; qnn: the batched QNN gradient")
    return ap.parse_args()


def workload(n, layers, terms, seed):
    from arcqml_b200 import workloads
    c = workloads.brickwork(n, layers, seed=seed)
    obs = workloads.random_pauli_sum(n, terms, seed=seed + 1)
    return c, obs


def config(args, c):
    what = "fwd + <H>" if args.forward_only else "fwd + adjoint"
    return {"workload": f"{args.qubits}q brickwork x{args.layers} {what}, "
                        f"{args.terms}-term Pauli sum",
            "qubits": args.qubits, "layers": args.layers, "pauli_terms": args.terms,
            "gates": len(c.operations), "parameters": c.num_parameters(),
            "state_bytes": 16 << args.qubits,
            "l2": "state (16 * 2^n bytes) larger than the 126 MB L2; no flush needed",
            "parallelism": "1 GPU" if args.gpus == 1 else
            f"state sharded over {args.gpus} GPUs on its top {args.gpus.bit_length() - 1} qubits"}


# ------------------------------------------------------------------ CPU oracle sample


def cpu_sample(args, sample_qubits=28, rot=(4, 2), cz=(2, 1), term_counts=(2, 16)):
    """Times the oracle (all host threads) on a bounded sample of the workload at
    min(28, --qubits) qubits and returns the gate passes/s of the whole step, extrapolated to
    --qubits by state size, with a description.

    Measured at the sample size, in place on one state, for each gate kind of the workload
    (parametrised rotations, CZ): the forward cost per gate (rot[0] / cz[0] gates) and the
    adjoint sweep's cost per gate (a sweep over rot[1] / cz[1] gates minus an empty sweep, which
    is the sweep's fixed part); and the observable's cost per term and its fixed part (two calls
    with term_counts terms). The step at the sample size is the --qubits workload's gate counts
    times these costs plus the fixed parts plus its terms times the per-term cost; every part
    scales with the state, so the --qubits step takes 2^(qubits - sample) times as long."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ctypes
    import oracle as O

    O.build()
    L = O.lib()
    n = min(sample_qubits, args.qubits)
    c, obs = workload(n, args.layers, args.terms, args.seed)
    ops = c.compile_plan(1)
    kinds = {"rot": [o for o in ops if o.bindings], "cz": [o for o in ops if not o.bindings]}
    full = workload(args.qubits, args.layers, args.terms, args.seed)[0].compile_plan(1)
    counts = {"rot": sum(1 for o in full if o.bindings), "cz": sum(1 for o in full if not o.bindings)}
    take = {"rot": rot, "cz": cz}
    psi = np.zeros(1 << n, np.complex128)
    psi[0] = 1.0  # the oracle's loops cost the same for any amplitude values
    lam = psi.copy()
    req = np.ascontiguousarray(c.requires_grad_mask(True), dtype=np.uint8)
    grads = np.zeros(len(req))

    def forward(packed):
        t = time.perf_counter()
        L.oracle_plan_apply(packed.ptr, packed.n, psi.ctypes.data, n)
        return time.perf_counter() - t

    def sweep(packed):
        t = time.perf_counter()
        L.oracle_adjoint_backward(packed.ptr, packed.n, psi.ctypes.data, lam.ctypes.data, n, 1.0,
                                  req.ctypes.data, len(req), grads.ctypes.data, len(grads))
        return time.perf_counter() - t

    t_start = time.perf_counter()
    adj_fixed = sweep(O._Packed([]))
    fwd, adj = {}, {}
    for k in ("rot", "cz"):
        pf = O._Packed(kinds[k][:take[k][0]])
        fwd[k] = forward(pf) / pf.n
        pa = O._Packed(kinds[k][:take[k][1]])
        adj[k] = max(0.0, sweep(pa) - adj_fixed) / pa.n
    terms = obs.compiled_terms()
    out = np.zeros_like(psi)  # touched before the timed calls
    t_obs = []
    for k in term_counts:
        arr, nt = O._terms(terms[:k])
        t0 = time.perf_counter()
        L.oracle_expectation_and_apply(ctypes.addressof(arr), nt, psi.ctypes.data,
                                       out.ctypes.data, n)
        t_obs.append(time.perf_counter() - t0)
    per_term = max(0.0, (t_obs[1] - t_obs[0]) / (term_counts[1] - term_counts[0]))
    obs_fixed = max(0.0, t_obs[0] - term_counts[0] * per_term)
    sample_dt = time.perf_counter() - t_start
    step_at_n = (sum(counts[k] * (fwd[k] + adj[k]) for k in counts) + adj_fixed + obs_fixed +
                 args.terms * per_term)
    step = step_at_n * 2.0 ** (args.qubits - n)
    gates = counts["rot"] + counts["cz"]
    rate = 2 * gates / step
    ms = lambda x: f"{x * 1e3:.0f} ms"  # noqa: E731
    sample = (f"oracle at {n} qubits in place on one state, {sample_dt:.1f} s of timing: per "
              f"rotation {ms(fwd['rot'])} forward / {ms(adj['rot'])} adjoint, per CZ "
              f"{ms(fwd['cz'])} / {ms(adj['cz'])}, adjoint sweep fixed {ms(adj_fixed)}, <H> and "
              f"H psi {ms(per_term)} per term + {ms(obs_fixed)}; the {args.qubits}-qubit step "
              f"({counts['rot']} rotations, {counts['cz']} CZ, forward and adjoint, {args.terms} "
              f"terms) extrapolated by state size x2^{args.qubits - n}: {step:.0f} s")
    return rate, O.num_threads(), sample, sample_dt


# ------------------------------------------------------------------ clocks


class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        # samples go to ARCQML_CLOCKS_DIR when set (to keep them), else the temp directory
        out_dir = os.environ.get("ARCQML_CLOCKS_DIR") or tempfile.gettempdir()
        self.path = os.path.join(out_dir, f"clocks_{os.getpid()}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                stderr=subprocess.DEVNULL)
        except Exception:  # nvidia-smi missing
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        self.proc.wait()
        self.f.close()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "samples": len(rows), "reasons": reasons}


# ------------------------------------------------------------------ GPU arm


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return {}


def gpu_arm(args):
    import torch
    from arcqml_b200 import build, runtime as rt
    from arcqml_b200.simulator import StateVectorSimulator

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    build.build()
    rt.load()
    n = args.qubits
    c, obs = workload(n, args.layers, args.terms, args.seed)
    gates = len(c.operations)
    if world == 1:
        sim = StateVectorSimulator(n)

        def step(initial=None):
            res = sim.run(c, obs, grad=not args.forward_only, initial_state=initial)
            if args.forward_only:
                return res.value, np.zeros(0)
            pgrads, _ = res.backward(1.0)
            return res.value, pgrads
    else:
        from arcqml_b200.sharded import ShardedStateVectorSimulator
        sim = ShardedStateVectorSimulator(n)

        def step(initial=None):
            value = sim.run(c, obs, grad=not args.forward_only, initial_shard=initial)
            return value, (np.zeros(0) if args.forward_only else sim.backward(1.0))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    clocks = Clocks(local)
    rt.profile_enable(True)
    if world > 1:
        sim.timing(True)
    launches0 = rt.launch_count()
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        value, grads = step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    launches = rt.launch_count() - launches0
    if world > 1:
        t = torch.tensor([launches], device="cuda", dtype=torch.int64)
        torch.distributed.all_reduce(t)
        launches = int(t.item())
    prof = rt.profile_read()
    rt.profile_enable(False)
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    passes = (1 if args.forward_only else 2) * gates
    value_rate = passes * args.steps / (ms / 1e3)
    swaps = None
    if world > 1:
        st = sim.timing(False)
        link = 770.0  # NVLink peer copy measured on this GPU type, GB/s per direction
        sent = st["bytes_sent"] / args.steps
        swap_ms = st["ms"] / args.steps
        swaps = {"transport": sim.transport,
                 "per_step": st["swaps"] / args.steps, "qubits_per_step": st["qubits"] / args.steps,
                 "bytes_sent_per_step": sent, "ms_per_step": round(swap_ms, 3),
                 "achieved_gbs": round(sent / (swap_ms * 1e-3) / 1e9, 1) if swap_ms else None,
                 "peak_gbs": link, "peak_source": "measured NVLink peer copy",
                 "frac": round(sent / (swap_ms * 1e-3) / 1e9 / link, 4) if swap_ms else None}

    # dominant kernel category and its roofline
    dom = max(prof.items(), key=lambda kv: kv[1][1])
    dname, (dl, dms, dbytes) = dom
    pk = peaks()
    hbm = pk.get("hbm_gbs")
    achieved = (dbytes / dl) / (dms / dl * 1e-3) / 1e9 if dl else 0.0
    peak = hbm if hbm else 6650.0
    local_amps = 2.0 ** (n - (world.bit_length() - 1))
    traffic = NCU_DRAM_BYTES_PER_AMP.get(dname)
    label = {"fused_adjoint": "arcqml_pass (fused adjoint passes, run-time compiled)",
             "fused_forward": "arcqml_pass (fused forward passes, run-time compiled)",
             "observable": "k_pauli_tile (observable tile passes)"}.get(dname, dname)
    roofline = {"kernel": label,
                "bound": "hbm", "achieved": round(achieved, 1),
                "peak": peak, "unit": "GB/s",
                "peak_source": "measured" if hbm else "fallback",
                "frac": round(achieved / peak, 4),
                "bytes_per_launch": dbytes / dl if dl else 0, "avg_launch_ms": dms / dl if dl else 0,
                "traffic": traffic * local_amps if traffic else None,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                  "26-qubit pass of this kernel, scaled per amplitude"
                                  if traffic else None}
    # FP64 roofline of the fused passes, which are bound by FP64 issue rather than HBM. The
    # algorithmic FP64 work of a Pauli rotation in the scaled unit-diagonal form is one FMA per
    # amplitude component: 4 flop per amplitude forward; the adjoint un-applies it from psi and
    # lambda and forms the gradient sum: 12 flop. CZ and the other sign flips take none. The
    # count is of the rotation ops the schedules execute: forward passes merge same-axis
    # rotations on a qubit inside a register sub-block, adjoint passes across the pass (with one
    # gradient sum for the merged parameters), so fewer ops run than the circuit has rotations.
    # Peak: 148 SMs x 64 FP64 FMA per clock x 2 flop at the median SM clock sampled under load
    # (no measured FP64 figure exists for these GPUs).
    plan0 = rt.CircuitPlan.create(c.compile_plan(1))
    sched = {"fused_forward": rt.plan_schedule_summary(plan0, n, False),
             "fused_adjoint": rt.plan_schedule_summary(
                 plan0, n, True, np.asarray(c.requires_grad_mask(True), np.uint8))}
    sm_mhz = (clk or {}).get("sm_mhz") or 1965.0
    fp64_peak = 148 * 64 * 2 * sm_mhz * 1e6 / 1e12
    roofline_fp64 = {}
    for cat, per_amp in (("fused_forward", 4.0), ("fused_adjoint", 12.0)):
        if cat not in prof or not prof[cat][0] or (cat == "fused_adjoint" and args.forward_only):
            continue
        cl, cms, _ = prof[cat]
        rot_ops = sched[cat]["rotations"]
        flops = per_amp * rot_ops * local_amps * args.steps
        tf = flops / (cms * 1e-3) / 1e12
        roofline_fp64[cat] = {"bound": "fp64", "achieved": round(tf, 2), "peak": round(fp64_peak, 2),
                              "unit": "TFLOP/s", "frac": round(tf / fp64_peak, 4),
                              "flop_per_launch": flops / cl, "avg_launch_ms": cms / cl,
                              "rotation_ops_executed": rot_ops,
                              "schedule": sched[cat] if world == 1 else
                              dict(sched[cat], note="unsharded schedule of the same circuit"),
                              "peak_source": f"nominal at the sampled {sm_mhz:.0f} MHz"}
    # The rate per-gate kernels would reach at the HBM roofline: every gate one pass over the
    # state (32 B per amplitude forward, 64 B adjoint), all GPUs streaming their shards.
    step_bytes = gates * (32.0 if args.forward_only else 96.0) * 2.0 ** n
    unfused = passes * world * peak * 1e9 / step_bytes

    e2e = None
    if not args.no_e2e:
        e2e = e2e_arm(args, step, n, world, passes)

    line = {"metric": METRIC, "value": round(value_rate, 3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "complex128 (f64)", "data": "synthetic (seeded brickwork + random Pauli sum)",
            "config": config(args, c), "roofline": roofline, "roofline_fp64": roofline_fp64,
            "swaps": swaps,
            "kernels": {k: {"launches": v[0], "ms": round(v[1], 3),
                            "gbs": round(v[2] / (v[1] * 1e-3) / 1e9, 1) if v[1] else 0}
                        for k, v in prof.items() if v[0]},
            "gpu_launches": launches, "e2e": e2e, "clocks": clk,
            "unfused_hbm_roofline_value": round(unfused, 3),
            "vs_unfused_hbm_roofline": round(value_rate / unfused, 3),
            "adjoint_grads_per_s": round(args.steps / (ms / 1e3), 5),
            "param_grads_per_s": round(c.num_parameters() * args.steps / (ms / 1e3), 2),
            "check": {"value": value, "grad_norm": float(np.linalg.norm(grads))}}
    if rank == 0 and world == 1 and not args.no_cpu:
        rate, cores, sample, _ = cpu_sample(args)
        line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
                                "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        sim.close()
        torch.distributed.destroy_process_group()


def e2e_arm(args, step, n, world, passes):
    import torch
    g = world.bit_length() - 1
    rank = int(os.environ.get("RANK", "0"))
    try:
        host = torch.zeros(1 << (n - g), dtype=torch.complex128, pin_memory=True)
    except Exception as exc:  # pinned host memory unavailable
        return {"value": None, "unit": UNIT, "unavailable": f"pinned host buffer: {exc}"}
    if rank == 0:
        host[0] = 1.0
    step(host)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _, grads = step(host)  # value and gradients come back to the host inside step
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([dt], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        dt = float(t.item())
    return {"value": round(passes * args.steps / dt, 3), "unit": UNIT,
            "h2d_bytes_per_step": int(16 << n), "d2h_bytes_per_step": int(8 * (len(grads) + 2)),
            "path": "StateVectorSimulator.run(initial_state=pinned host) + backward" if world == 1
            else "ShardedStateVectorSimulator.run(initial_shard=pinned host) + backward, "
                 "every rank its shard"}


# ------------------------------------------------------------------ reference arm


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from arcqml_b200 import workloads  # noqa: F401 (generators only)
    rates, samples = [], []
    # each step: a bounded sample of the workload at 28 qubits (a few seconds on the host)
    small = dict(rot=(1, 1), cz=(1, 1), term_counts=(1, 4))
    for _ in range(args.warmup):
        cpu_sample(args, **small)
    for _ in range(args.steps):
        rate, cores, sample, _ = cpu_sample(args, **small)
        rates.append(rate)
    value = statistics.median(rates)
    c, _ = workload(args.qubits, args.layers, args.terms, args.seed)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "complex128 (f64)", "data": "synthetic (seeded brickwork + random Pauli sum)",
            "config": config(args, c),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference runtime ships only as a closed Windows static library; this arm "
                    "times the f64 CPU oracle that restates its algorithm"}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ small configurations


def small_arm(args):
    """One GPU: the 4-qubit VQE (steps of run -> backward -> Adam, lr 0.05, 100 per timed
    repetition: the device optimizer loop, one launch and one read-back of the 100 energies and
    the parameters per repetition; the host loop through StateVectorSimulator is timed beside
    it) or the batched QNN (full-batch gradient of 1024 rows x 10 qubits), with the oracle timed
    on the same work beside it. Device time with CUDA events around host-driven calls."""
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    from arcqml_b200 import build, runtime as rt, workloads
    from arcqml_b200.simulator import BatchStateVectorSimulator, StateVectorSimulator
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    build.build()
    O.build()
    rt.load()
    if args.workload == "vqe4":
        c, obs = workloads.vqe4(seed=1)
        sim = StateVectorSimulator(4)
        theta0 = c.parameter_values().astype(np.float64)

        plan = rt.CircuitPlan.create(c.compile_plan(1))
        robs = rt.Observable.from_sparse_pauli_op(obs)
        req0 = c.requires_grad_mask(True)
        p0 = np.concatenate([[0.0], theta0])

        def unit():  # 100 Adam steps in one launch
            e, _ = rt.small_adam_device(plan, robs, 4, p0, req0, 100, lr=0.05)
            return float(e[-1])

        def host_unit():  # the same 100 steps, one run + backward per step, Adam on the host
            theta, st = theta0.copy(), rt.AdamState(theta0.size)
            for _ in range(100):
                c.set_parameter_values(theta)
                res = sim.run(c, obs)
                g, _ = res.backward(1.0)
                theta = st.update(theta, g, lr=0.05)
            c.set_parameter_values(theta0)
            return res.value

        per_unit, unit_name, metric = 100, "steps/s", "4-qubit VQE Adam steps/s (15-term H)"
        terms, ops_n = obs.compiled_terms(), 4

        def cpu_unit():
            theta, st = theta0.copy(), {}
            init = np.zeros(16, np.complex128)
            init[0] = 1
            for _ in range(100):
                c.set_parameter_values(theta)
                ops = c.compile_plan(1)
                psi = O.plan_apply(ops, init, 4)
                _, lam = O.expectation_and_apply(terms, psi, 4)
                req = c.requires_grad_mask(True)
                _, _, g = O.adjoint_backward(ops, psi, lam, 4, 1.0, req, len(req))
                theta = O.adam_step(theta, g[1:], st, lr=0.05)
    else:
        host_unit = None
        c, obs, init, labels = workloads.qnn(10, 1024, 4, seed=7)
        sim = BatchStateVectorSimulator.from_amplitudes(10, init)

        def unit():  # one full-batch gradient
            res = sim.run(c, obs)
            _, up = workloads.half_mse_upstream(res.values, labels)
            g, _ = res.backward(up)
            return float(np.sum(g))

        per_unit, unit_name = 1, "gradients/s"
        metric = "batched QNN full-batch gradients/s (1024 rows x 10 qubits, 80 parameters)"
        ops = c.compile_plan(1)
        terms = obs.compiled_terms()
        req = c.requires_grad_mask(True, False)

        def cpu_unit():
            psi = O.plan_apply(ops, init.reshape(-1), 10, 1024).reshape(1024, -1)
            vals = np.array([O.expectation(terms, psi[i], 10) for i in range(1024)])
            lam = np.stack([O.expectation_and_apply(terms, psi[i], 10)[1] for i in range(1024)])
            _, up = workloads.half_mse_upstream(vals, labels)
            O.adjoint_backward(ops, psi.reshape(-1), lam.reshape(-1), 10, up, req, len(req), 1024)
    for _ in range(args.warmup):
        unit()
    torch.cuda.synchronize()
    launches0 = rt.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        check = unit()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    launches = rt.launch_count() - launches0
    host_loop = None
    if host_unit is not None:
        host_unit()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            host_unit()
        e1.record()
        torch.cuda.synchronize()
        host_loop = {"value": round(per_unit * args.steps / (e0.elapsed_time(e1) / 1e3), 3),
                     "unit": unit_name,
                     "path": "StateVectorSimulator.run + backward per step, Adam on the host"}
    if args.workload == "vqe4":
        O.set_num_threads(1)  # 16 amplitudes: threads only add overhead
    t0 = time.perf_counter()
    cpu_unit()
    cpu_dt = time.perf_counter() - t0
    line = {"metric": metric, "value": round(per_unit * args.steps / (ms / 1e3), 3),
            "unit": unit_name, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "complex128 (f64)",
            "data": "synthetic (seeded workload generator)", "config": {"workload": args.workload},
            "gpu_launches": launches, "check": check,
            "path": ("arcqml_rt_v2_small_adam: 100 steps per launch" if host_unit is not None
                     else "BatchStateVectorSimulator.run + backward"),
            "host_loop": host_loop,
            "cpu_baseline": {"value": round(per_unit / cpu_dt, 3), "unit": unit_name,
                             "cores": O.num_threads(), "kind": "port",
                             "sample": f"one unit of the same work on the oracle in {cpu_dt:.3f} s"}}
    if args.workload == "qnn":
        # FP64 lower bound of one full-batch gradient: every row runs the 120 gates forward, 240
        # gate applications in the reverse sweep and one observable pass, ~14 flop per
        # amplitude each (a complex 2x2 on a pair): B (m_fwd + 2 m_bwd + 1) 14 D flop.
        flop = 1024 * (120 + 2 * 120 + 1) * 14 * 1024
        tf = flop * args.steps / (ms * 1e-3) / 1e12
        line["fp64"] = {"flop_per_gradient": flop, "achieved_tflops": round(tf, 3),
                        "peak_tflops": 37.2, "frac": round(tf / 37.2, 4),
                        "peak_source": "nominal: 148 SMs x 64 FP64 FMA/clock x 2 x 1965 MHz"}
    print(json.dumps(line), flush=True)


def analysis_arm(args):
    """One GPU: the state-analysis kernels on random states of min(--qubits, 28) qubits (4 GiB,
    beyond L2), each timed over --steps calls with CUDA events after --warmup calls; GB/s of
    algorithmic bytes (every amplitude read once, outputs written once) against the measured
    HBM copy rate. Bloch vector and overlap calls include their 16-24-byte read-back."""
    import torch
    from arcqml_b200 import build, runtime as rt
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    build.build()
    rt.load()
    n = min(args.qubits, 28)
    dim = 1 << n
    gen = torch.Generator(device="cuda").manual_seed(args.seed)
    a = torch.randn(dim, dtype=torch.complex128, device="cuda", generator=gen)
    a /= torch.linalg.vector_norm(a)
    b = torch.randn(dim, dtype=torch.complex128, device="cuda", generator=gen)
    b /= torch.linalg.vector_norm(b)
    probs = torch.empty(dim, dtype=torch.float64, device="cuda")
    lam = torch.empty_like(a)
    up = torch.randn(dim, dtype=torch.float64, device="cuda", generator=gen)
    ops = {
        "probabilities": (lambda: rt.probabilities_device(a, n, out=probs), 24.0),
        "marginal_top3": (lambda: rt.marginal_probabilities_device(a, n, [n - 1, n - 2, n - 3]),
                          16.0),
        "marginal_low2": (lambda: rt.marginal_probabilities_device(a, n, [0, 1]), 16.0),
        "bloch_vector": (lambda: rt.bloch_vector_device(a, n, n // 2), 16.0),
        "overlap": (lambda: rt.overlap_device(a, b, n), 32.0),
        "probability_cotangent": (lambda: rt.probability_cotangent_device(a, n, up, out=lam),
                                  40.0),
    }
    hbm = peaks().get("hbm_gbs") or 6650.0
    launches0 = rt.launch_count()
    out = {}
    for name, (fn, per_amp) in ops.items():
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        gbs = per_amp * dim / (ms * 1e-3) / 1e9
        out[name] = {"ms": round(ms, 4), "gbs": round(gbs, 1), "frac": round(gbs / hbm, 4),
                     "bytes_per_amplitude": per_amp}
    line = {"metric": f"state-analysis kernels, HBM GB/s ({n} qubits)",
            "value": out["probabilities"]["gbs"], "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "complex128 (f64)",
            "data": "synthetic (random normalised states)",
            "config": {"workload": "analysis", "qubits": n, "l2": "inputs larger than L2"},
            "peak": hbm, "peak_source": "measured" if peaks().get("hbm_gbs") else "fallback",
            "kernels": out, "gpu_launches": rt.launch_count() - launches0}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
    elif args.workload == "analysis":
        analysis_arm(args)
    elif args.workload != "brickwork":
        small_arm(args)
    else:
        gpu_arm(args)


if __name__ == "__main__":
    main()
