"""Builds the sm_100a runtime library in-tree.

Outputs (next to this file):
  libarcqml_runtime_private.so — the shared C-ABI library loaded by the Python layer and tests;
  libarcqml_runtime_private.a  — the static twin that ArcQML's ``arcqml-runtime-sys`` links
                                 (``cargo:rustc-link-lib=static=arcqml_runtime_private``).
Every translation unit is compiled by nvcc with ``-gencode arch=compute_100a,code=sm_100a``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
OBJ = os.path.join(HERE, "_build")
SO = os.path.join(HERE, "libarcqml_runtime_private.so")
ARCHIVE = os.path.join(HERE, "libarcqml_runtime_private.a")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")] + ARCH


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC)
                  if f.endswith((".cu", ".cpp")))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    inc = os.path.join(ROOT, "include")
    hs += [os.path.join(inc, f) for f in os.listdir(inc) if f.endswith(".h")]
    return hs


JIT_INC = os.path.join(OBJ, "jit_source.inc")


def write_jit_source() -> None:
    """Embeds fused.h and fused_core.cuh as string literals for the run-time pass compiler."""
    parts = []
    for var, name in (("kJitFusedH", "fused.h"), ("kJitCore", "fused_core.cuh")):
        text = open(os.path.join(CSRC, name)).read()
        if ")ARCQMLSRC" in text:
            raise RuntimeError(f"{name} contains the raw-string delimiter")
        parts.append(f'static const char {var}[] = R"ARCQMLSRC({text})ARCQMLSRC";\n')
    body = "".join(parts)
    if not os.path.exists(JIT_INC) or open(JIT_INC).read() != body:
        with open(JIT_INC, "w") as f:
            f.write(body)


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    newest_dep = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in headers()])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest_dep:
        return obj
    cmd = [nvcc()] + NVCC_FLAGS + ["-I", OBJ, "-x", "cu", "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    if force:
        for f in os.listdir(OBJ):
            os.remove(os.path.join(OBJ, f))
    write_jit_source()
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), sources()))
    newest = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(SO) or os.path.getmtime(SO) < newest:
        cmd = [nvcc()] + ARCH + ["-shared", "-o", SO] + objs + ["-lcudart_static", "-lrt", "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if force or not os.path.exists(ARCHIVE) or os.path.getmtime(ARCHIVE) < newest:
        if os.path.exists(ARCHIVE):
            os.remove(ARCHIVE)
        subprocess.run(["ar", "rcs", ARCHIVE] + objs, check=True)
    return SO


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="--force" in sys.argv))
