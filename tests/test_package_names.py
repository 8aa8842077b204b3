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
