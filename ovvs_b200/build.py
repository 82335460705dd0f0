"""Builds ovvs_b200/libovvs.so: the ovvs C ABI on B200 (sm_100a only).

Every .cu / .cpp under ovvs_b200/csrc is compiled by nvcc (device code for sm_100a, host code by
the system g++) and linked into one shared library with a static CUDA runtime; at run time it
needs only the NVIDIA driver; NCCL (libnccl.so.2) is opened on first use by a sharded
Resources. Objects go to ovvs_b200/_build/.

    python -m ovvs_b200.build          # incremental
    python -m ovvs_b200.build --clean
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libovvs.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden,-Wall,-Wno-unused-function",
    "-DOVVS_BUILD", "-I" + os.path.join(ROOT, "include"), "-I" + CSRC,
]


def sources():
    out = []
    for d, _, files in os.walk(CSRC):
        for f in sorted(files):
            if f.endswith((".cu", ".cpp")):
                out.append(os.path.join(d, f))
    return sorted(out)


def headers():
    out = []
    for base in (CSRC, os.path.join(ROOT, "include")):
        for d, _, files in os.walk(base):
            out += [os.path.join(d, f) for f in files if f.endswith((".h", ".hpp", ".cuh"))]
    return out


def _obj(src):
    rel = os.path.relpath(src, CSRC).replace(os.sep, "__")
    return os.path.join(BUILD, rel + ".o")


def _compile(src, verbose):
    obj = _obj(src)
    cmd = [NVCC] + ARCH + COMMON + ["-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [NVCC, "-x", "cu"] + ARCH + COMMON + ["-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    return src, r.returncode, r.stdout + r.stderr


def build(verbose: bool = False, jobs: int | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    newest_header = max((os.path.getmtime(h) for h in headers()), default=0.0)
    todo = []
    for s in sources():
        o = _obj(s)
        if (not os.path.exists(o) or os.path.getmtime(o) < os.path.getmtime(s)
                or os.path.getmtime(o) < newest_header):
            todo.append(s)
    failed = []
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        for src, rc, log in ex.map(lambda s: _compile(s, verbose), todo):
            if rc != 0 or verbose:
                sys.stderr.write(f"--- {os.path.relpath(src, ROOT)}\n{log}")
            if rc != 0:
                failed.append(src)
    if failed:
        raise RuntimeError("nvcc failed: " + ", ".join(os.path.relpath(f, ROOT) for f in failed))
    objs = [_obj(s) for s in sources()]
    if todo or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(map(os.path.getmtime, objs)):
        vscript = os.path.join(BUILD, "exports.map")
        with open(vscript, "w") as f:
            f.write("{ global: ovvs*; local: *; };\n")  # only the C ABI leaves the library
        cmd = [NVCC] + ARCH + ["-shared", "-cudart=static", "-o", LIB] + objs + [
            "-ldl", "-Xlinker", "-Bsymbolic", "-Xlinker", "--exclude-libs,ALL",
            "-Xlinker", "--version-script=" + vscript]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    if a.clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    print(build(verbose=a.verbose))


if __name__ == "__main__":
    main()
