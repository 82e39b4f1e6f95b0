"""Build libsupra_attn.so in-tree for sm_100a with nvcc.

    python supra2-img-web_b200/supra_attn/build.py [--force] [-v]

(Run it as a script or load it by path, as __graft_entry__.build() does: importing it as
supra_attn.build would first run the package's __init__, which loads the library.)

Every csrc/*.cu and csrc/*.cpp is compiled to an object under _build/ (skipped when the object
is newer than its source and the headers), then linked into supra_attn/libsupra_attn.so.
The CUDA runtime is linked statically so the library does not depend on which libcudart the
host process loaded first.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)               # supra2-img-web_b200/
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libsupra_attn.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I", CSRC, "-I", INCLUDE]


def _nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: libsupra_attn needs the CUDA toolkit to build")


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _compile(nvcc, src, obj, verbose):
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> str:
    """Compiles and links the library if anything changed; returns its path."""
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    hdr_time = max(os.path.getmtime(h) for h in _headers())
    todo, objs = [], []
    for s in srcs:
        obj = os.path.join(BUILD, os.path.basename(s) + ".o")
        objs.append(obj)
        if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(s), hdr_time):
            todo.append((s, obj))
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            for log in ex.map(lambda so: _compile(nvcc, so[0], so[1], verbose), todo):
                logs.append(log)
    if todo or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc, *ARCH, "-shared", "-o", tmp, *objs, "-cudart", "static", "-Xcompiler", "-fPIC"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        sys.stderr.write("".join(logs))
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
