"""Plan reuse in the simulators (arcqml_b200/simulator.py `_PlanPool`; host code, no GPU).

A run whose circuit has the structure of an earlier one (gates, qubits, parameter bindings,
constant values) takes a plan of that structure that no live result holds and replaces its bound
parameter values (arcqml_rt_v2_plan_set_parameters); a plan a result still holds is never
changed under it. The reused plan's schedule is run on the CPU (arcqml_rt_v2_plan_emulate)
against the oracle with the new values.
"""
import gc
import math

import numpy as np

from arcqml_b200 import circuit as cm
from arcqml_b200.simulator import _Context, _PlanPool
from arcqml_b200.workloads import brickwork
from plans import random_state


def test_free_plans_are_reused_with_new_values(runtime, oracle):
    n = 9
    c = brickwork(n, 3, seed=11)
    pool = _PlanPool()
    p1, users1 = pool.get(c, 1)
    holder = _Context(n, None, None, None, p1, c, False)  # a live result holds p1
    users1.add(holder)
    p2, _ = pool.get(c, 1)
    assert p2 is not p1  # p1 is held
    del holder
    gc.collect()
    g = np.random.Generator(np.random.PCG64(3))
    c.set_parameter_values(g.uniform(-math.pi, math.pi, size=c.num_parameters()))
    p3, _ = pool.get(c, 1)
    assert p3 is p1 or p3 is p2
    init = random_state(g, n)
    got = runtime.plan_emulate(p3, init, n)
    ref = oracle.plan_apply(c.compile_plan(1), init, n)
    assert float(np.max(np.abs(got - ref))) < 1e-12


def test_other_structures_get_other_plans():
    c1 = cm.Circuit(8)
    c1.rot("rx", 0.3, 0)
    c1.append("rz", (1,), 0.25)  # a constant angle belongs to the structure
    c2 = cm.Circuit(8)
    c2.rot("rx", 0.3, 0)
    c2.append("rz", (1,), 0.5)
    pool = _PlanPool()
    a, _ = pool.get(c1, 1)
    b, _ = pool.get(c2, 1)
    assert a is not b
    a2, _ = pool.get(c1, 1)
    assert a2 is a
    z, _ = pool.get(c1, 0)  # another parent offset: another plan
    assert z is not a


class _Stand:  # the attributes RuntimeBackend._plan uses (the backend itself needs a GPU)
    pass


def test_sharded_backend_reuses_plans_by_structure(runtime, oracle):
    from arcqml_b200.sharded import RuntimeBackend
    be = _Stand()
    be.rt = runtime
    n = 9
    c = brickwork(n, 2, seed=4)
    p1 = RuntimeBackend._plan(be, c.compile_plan(1))
    g = np.random.Generator(np.random.PCG64(8))
    c.set_parameter_values(g.uniform(-math.pi, math.pi, size=c.num_parameters()))
    ops = c.compile_plan(1)
    p2 = RuntimeBackend._plan(be, ops)
    assert p2 is p1
    init = random_state(g, n)
    got = runtime.plan_emulate(p2, init, n)
    assert float(np.max(np.abs(got - oracle.plan_apply(ops, init, n)))) < 1e-12


def test_bound_values_of_a_parent_must_agree(runtime):
    c = cm.Circuit(8)
    p = c.add_parameter(0.4)
    c.append("rx", (0,), p)
    c.append("ry", (1,), p)
    ops = c.compile_plan(1)
    assert list(runtime.plan_bound_values(ops)) == [0.0, 0.4]
    bad = [ops[0], cm.PlanOp(ops[1].opcode, ops[1].qubits, (0.7, 0.0, 0.0), None,
                             ops[1].bindings, ops[1].name)]
    assert runtime.plan_bound_values(bad) is None
    assert runtime.plan_structure_key(bad) == runtime.plan_structure_key(ops)


def test_schedule_summary_counts(runtime):
    """plan_schedule_summary (the counts bench.py's FP64 roofline uses) agrees with the
    schedule's own statistics: passes, ops (= gates after merges), one gradient row per
    rotation op that has a gradient, merged parameters as aliases."""
    from arcqml_b200.workloads import brickwork
    n = 20
    c = brickwork(n, 6, seed=3)
    plan = runtime.CircuitPlan.create(c.compile_plan(1))
    req = np.asarray(c.requires_grad_mask(True), np.uint8)
    for adj in (False, True):
        summ = runtime.plan_schedule_summary(plan, n, adj, req if adj else None)
        stats = plan.schedule_stats(n, adj)
        assert summ["passes"] == stats["passes"] and summ["ops"] == stats["gates"]
        assert summ["custom"] == 0 and summ["rotations"] <= summ["ops"]
        if adj:
            # every rotation of the brickwork has a parameter: rows + aliases = rotations
            assert summ["rows"] + summ["aliases"] == c.num_parameters()
            assert summ["rows"] == summ["rotations"]
        else:
            assert summ["rows"] == 0 and summ["aliases"] == 0
