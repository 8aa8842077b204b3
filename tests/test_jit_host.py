"""Run-time compiled pass kernels on CPU: the generated sources of a forward and an adjoint
schedule compile for sm_100a with NVRTC (no GPU needed)."""
import numpy as np
import pytest

from arcqml_b200 import workloads


def test_generated_pass_kernels_compile(runtime):
    c = workloads.brickwork(10, 3, seed=5)
    plan = runtime.CircuitPlan.create(c.compile_plan(1))
    for adjoint in (False, True):
        r = plan.jit_check(10, adjoint)
        if r["eligible"] == 0 and "not found" in r["message"]:
            pytest.skip("NVRTC is not available: " + r["message"])
        assert r["eligible"] >= 1
        assert r["compiled"] == r["eligible"], r["message"]


def test_jit_check_rejects_small_states(runtime):
    c = workloads.brickwork(4, 1, seed=5)
    plan = runtime.CircuitPlan.create(c.compile_plan(1))
    with pytest.raises(runtime.RuntimeError, match="below 8 qubits"):
        plan.jit_check(4, False)


def test_scaled_and_plain_rotation_forms_compile(runtime):
    """Passes mixing scaled rotation forms with the plain forms kept for angles at pi (and
    past the per-pass growth cap) compile, forward and adjoint; ARCQML_SCALED=0 (subprocess)
    compiles the all-plain sources."""
    import math
    import os
    import subprocess
    import sys

    from arcqml_b200 import circuit as cm
    c = cm.Circuit(12)
    for layer in range(6):
        for q in range(12):
            c.rot(("rx", "ry", "rz")[(q + layer) % 3], math.pi if q % 4 == 0 else 0.3 * q, q)
            c.append("phase", (q,), math.pi * (1 - 1e-9))  # fixed: no gradient slot
        for a in range(layer % 2, 11, 2):
            c.append("cz", (a, a + 1))
    for _ in range(30):
        c.rot("ry", math.pi * (1 - 1e-9), 5)
    plan = runtime.CircuitPlan.create(c.compile_plan(1))
    for adjoint in (False, True):
        r = plan.jit_check(12, adjoint)
        if r["eligible"] == 0 and "not found" in r["message"]:
            pytest.skip("NVRTC is not available: " + r["message"])
        assert r["eligible"] >= 1 and r["compiled"] == r["eligible"], r["message"]
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = ("import sys; sys.path.insert(0, %r)\n"
            "from arcqml_b200 import runtime as rt, workloads as W\n"
            "p = rt.CircuitPlan.create(W.brickwork(10, 3, seed=5).compile_plan(1))\n"
            "for adj in (False, True):\n"
            "    r = p.jit_check(10, adj)\n"
            "    assert r['compiled'] == r['eligible'] >= 1, r\n"
            "print('plain-ok')\n") % root
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       env=dict(os.environ, ARCQML_SCALED="0"), timeout=600)
    assert r.returncode == 0 and "plain-ok" in r.stdout, r.stdout + r.stderr


@pytest.mark.parametrize("n,seed", [(8, 1), (11, 2), (14, 3)])
def test_random_fast_path_circuits_compile(runtime, n, seed):
    """Every pass of random circuits built from fast-path gates (rotations at random and edge
    angles, fixed phases, H / SX / S / T / Z, U3 as a dense 2x2, RXX / RYY as dense 4x4s, CZ
    between any qubits) has a compiled form that compiles, forward and adjoint."""
    import math

    import numpy as np

    from arcqml_b200 import circuit as cm
    g = np.random.Generator(np.random.PCG64(seed))
    c = cm.Circuit(n)
    edge = (math.pi, -math.pi, 0.0, 3 * math.pi, math.pi * (1 - 1e-9))
    for _ in range(4):
        for q in range(n):
            r = g.uniform()
            a = float(edge[int(g.integers(0, len(edge)))] if g.uniform() < 0.3
                      else g.uniform(-3, 3))
            if r < 0.45:
                c.rot(("rx", "ry", "rz")[int(g.integers(0, 3))], a, q)
            elif r < 0.6:
                c.append(("h", "sx", "s", "t", "z")[int(g.integers(0, 5))], (q,))
            elif r < 0.7:
                c.append("phase", (q,), a)
            elif r < 0.8:
                c.append("u3", (q,), a, float(g.uniform(-3, 3)), float(g.uniform(-3, 3)))
        for _ in range(n // 2):
            a, b = (int(x) for x in g.choice(n, size=2, replace=False))
            if g.uniform() < 0.7:
                c.append("cz", (a, b))
            elif abs(a - b) == 1:
                c.append(("rxx", "ryy")[int(g.integers(0, 2))], (a, b), float(g.uniform(-3, 3)))
    plan = runtime.CircuitPlan.create(c.compile_plan(1))
    for adjoint in (False, True):
        r = plan.jit_check(n, adjoint)
        if r["eligible"] == 0 and "not found" in r["message"]:
            pytest.skip("NVRTC is not available: " + r["message"])
        assert r["compiled"] == r["eligible"], r["message"]
        if not adjoint:
            assert r["eligible"] >= 1


def test_benchmark_schedule_compiles_completely(runtime):
    """Every pass of the 32-qubit 20-layer brickwork (the bench's step), forward and adjoint,
    has a compiled form that compiles: none falls back to the table-driven kernel."""
    c = workloads.brickwork(32, 20, seed=1234)
    plan = runtime.CircuitPlan.create(c.compile_plan(1))
    for adjoint in (False, True):
        r = plan.jit_check(32, adjoint)
        if r["eligible"] == 0 and "not found" in r["message"]:
            pytest.skip("NVRTC is not available: " + r["message"])
        assert r["eligible"] >= 15 and r["compiled"] == r["eligible"], r
        assert plan.schedule_stats(32, adjoint)["passes"] == r["eligible"]


def test_default_pass_code_is_pinned():
    """The compiled pass code of the default configuration equals the pinned digests
    (tests/golden/pass_code_pins.json, last run on a B200): a planner or code-generator change
    shows up here first and needs the GPU parity tests before the pins are regenerated."""
    import json
    import os
    if any(k.startswith("ARCQML_") for k in os.environ):
        pytest.skip("an ARCQML_* switch is set")
    from golden import pass_code_pins
    with open(pass_code_pins.PINS) as f:
        pinned = json.load(f)
    assert pass_code_pins.digests() == pinned


def warp_local_layouts(runtime, c, n, adjoint):
    """(sub-blocks, warp-local exchanges) of the plan's schedule, checking every warp-local pair:
    the same warp bits (thread bits 5 and up, same tile bits in the same order), outside both
    sub-blocks' register bits, and lane bits holding all three swizzle residues."""
    import struct

    import jit_host_run as J
    ops = c.compile_plan(1)
    req = np.asarray(c.requires_grad_mask(True), np.uint8) if adjoint else None
    plan = runtime.CircuitPlan.create(ops)
    steps = J.parse(runtime.plan_schedule_export(plan, n, adjoint, req))
    nsub = nwarp = 0
    for kind, p in steps:
        if kind != "pass":
            continue
        k, _, _, _, _, _, rb = struct.unpack_from("<7I", p.header, 0)
        tbits = k - rb
        subs = []
        for i in range(len(p.subs) // 24):
            b = p.subs[24 * i:24 * (i + 1)]
            R = set(b[:rb])
            perm = list(b[4:4 + tbits])
            flags = struct.unpack_from("<I", b, 20)[0]
            subs.append((R, perm, flags))
        nsub += len(subs)
        for i, (R, perm, flags) in enumerate(subs):
            assert sorted(set(perm) | R) == list(range(k))  # a permutation of the tile bits
            assert len({q % 3 for q in perm[:3]}) == 3 or tbits < 3
            if not flags & 4:
                continue
            assert i + 1 < len(subs), "the last sub-block of a pass must end with a CTA barrier"
            R2, perm2, _ = subs[i + 1]
            assert perm[5:] == perm2[5:] and not (set(perm[5:]) & (R | R2))
            nwarp += 1
    return nsub, nwarp


def test_warp_local_exchanges_keep_elements_in_their_warp(runtime):
    for n, layers, adjoint in ((32, 20, False), (32, 20, True), (20, 6, True), (14, 5, False)):
        c = workloads.brickwork(n, layers, seed=1234)
        nsub, nwarp = warp_local_layouts(runtime, c, n, adjoint)
        assert nsub > 0
        if n == 32:
            assert nwarp >= nsub // 3, (nsub, nwarp)
