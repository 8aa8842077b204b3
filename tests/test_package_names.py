"""Static check: every global name a function of the package, the benchmark or the oracle
wrapper reads is defined at module level or is a builtin (a name bound only inside another
function fails at run time, on paths the CPU tests may not reach, such as the device backends)."""
import builtins
import glob
import os
import symtable

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MODULE_ATTRS = {"__file__", "__name__", "__doc__", "__spec__", "__package__", "__loader__"}
FILES = sorted(glob.glob(os.path.join(ROOT, "arcqml_b200", "*.py")) +
               [os.path.join(ROOT, "bench.py"), os.path.join(ROOT, "__graft_entry__.py")] +
               glob.glob(os.path.join(ROOT, "oracle", "*.py")))


def undefined_globals(path):
    with open(path) as f:
        top = symtable.symtable(f.read(), path, "exec")
    defined = {s.get_name() for s in top.get_symbols()
               if s.is_assigned() or s.is_imported() or s.is_namespace()}
    bad = []

    def walk(t):
        if t.get_type() != "module":
            for s in t.get_symbols():
                name = s.get_name()
                if (s.is_referenced() and s.is_global() and not s.is_declared_global() and
                        name not in defined and name not in MODULE_ATTRS and
                        not hasattr(builtins, name)):
                    bad.append(f"{t.get_name()} (line {t.get_lineno()}): {name}")
        for c in t.get_children():
            walk(c)

    walk(top)
    return bad


@pytest.mark.parametrize("path", FILES, ids=[os.path.relpath(p, ROOT) for p in FILES])
def test_no_undefined_globals(path):
    assert undefined_globals(path) == []


def test_runtime_binding_attributes_exist():
    """Every attribute read from the ctypes binding (``rt.X``, ``self.rt.X``, ``runtime.X``) in
    the package, the benchmark and the tests is defined by ``arcqml_b200.runtime``."""
    import ast

    from arcqml_b200 import runtime
    files = FILES + sorted(glob.glob(os.path.join(ROOT, "tests", "*.py")))
    bad = []
    for path in files:
        with open(path) as f:
            tree = ast.parse(f.read())
        for node in ast.walk(tree):
            if not isinstance(node, ast.Attribute):
                continue
            v = node.value
            on_rt = isinstance(v, ast.Name) and v.id in ("rt", "runtime")
            on_rt = on_rt or (isinstance(v, ast.Attribute) and v.attr == "rt" and
                              isinstance(v.value, ast.Name) and v.value.id == "self")
            if on_rt and not hasattr(runtime, node.attr):
                bad.append(f"{os.path.relpath(path, ROOT)}:{node.lineno}: {node.attr}")
    assert bad == []
