"""Pins of the run-time compiled pass code in the default configuration.

The compiled pass kernels are generated from each fused pass; a change to the planner or the
code generator changes them, and such a change needs the GPU parity tests again. This module
lists the circuits whose generated code is pinned and computes a SHA-256 digest of every pass's
source (forward and adjoint schedules). ``tests/test_jit_host.py`` compares the digests with
``pass_code_pins.json``; after a deliberate change (and its GPU run) regenerate the file with

    python tests/golden/pass_code_pins.py

with none of the ARCQML_* switches set.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PINS = os.path.join(HERE, "pass_code_pins.json")
for _p in (os.path.dirname(os.path.dirname(HERE)), os.path.dirname(HERE)):
    if _p not in sys.path:
        sys.path.insert(0, _p)


def cases():
    import numpy as np
    from arcqml_b200 import workloads
    from plans import random_plan
    out = [("brickwork 32q x20", workloads.brickwork(32, 20, seed=1234), 32),
           ("brickwork 12q x4", workloads.brickwork(12, 4, seed=9), 12),
           ("brickwork 20q x6", workloads.brickwork(20, 6, seed=5), 20)]
    for n in (8, 10, 13, 16):
        g = np.random.Generator(np.random.PCG64(n))
        out.append((f"random plan {n}q", random_plan(g, n, 150, 8), n))
    return out


def digests():
    """{case: {"forward": [sha256 per pass], "adjoint": [...]}} (empty string: no compiled form)."""
    import numpy as np
    import jit_host_run as J
    from arcqml_b200 import runtime
    res = {}
    for name, c, n in cases():
        ops = c if isinstance(c, list) else c.compile_plan(1)
        if not isinstance(c, list):
            req = np.asarray(c.requires_grad_mask(True), np.uint8)
        else:
            req = np.ones(1 + max((b[1] for o in ops for b in o.bindings), default=0), np.uint8)
        plan = runtime.CircuitPlan.create(ops)
        entry = {}
        for adj in (False, True):
            steps = J.parse(runtime.plan_schedule_export(plan, n, adj, req if adj else None))
            entry["adjoint" if adj else "forward"] = [
                hashlib.sha256(p.code.encode()).hexdigest() if kind == "pass" and p.code else ""
                for kind, p in steps]
        res[name] = entry
    return res


if __name__ == "__main__":
    if any(k.startswith("ARCQML_") for k in os.environ):
        sys.exit("unset the ARCQML_* switches first")
    pins = digests()
    with open(PINS, "w") as f:
        json.dump(pins, f, indent=1, sort_keys=True)
        f.write("\n")
    print("wrote", PINS)
