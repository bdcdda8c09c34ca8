"""Build recipe of libqmoe_b200.so: nvcc for sm_100a only, in-tree output next to this file.

    python nemotron-super-8gb_b200/qmoe_build.py          # or __graft_entry__.build()

Each csrc/*.cu is compiled to an object in _build/ (in parallel), then linked into one shared library
against the shared CUDA runtime: inside a torch process the library binds to the libcudart.so.12 torch
already loaded, so both see the same current device and streams; standalone it finds the toolkit's
runtime through its rpath.
"""
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libqmoe_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc():
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _stale(obj, deps):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose=False, extra=()):
    os.makedirs(BUILD, exist_ok=True)
    nv = nvcc()
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(os.path.dirname(HERE), "include", "qmoe_b200.h"))
    jobs = []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        if _stale(obj, [src] + headers):
            jobs.append([nv, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0 or verbose:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError("nvcc failed: " + " ".join(cmd))
        return r.stdout + r.stderr

    with cf.ThreadPoolExecutor(max(1, min(len(jobs), os.cpu_count() or 4))) as ex:
        logs = list(ex.map(run, jobs))
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in sources()]
    if jobs or not os.path.exists(LIB):
        tmp = LIB + ".tmp"
        run([nv, *ARCH, "-shared", "-o", tmp, *objs, "-cudart", "shared",
             "-Xlinker", "-rpath=/usr/local/cuda/lib64"])
        os.replace(tmp, LIB)
    return logs


if __name__ == "__main__":
    for line in build(verbose="-v" in sys.argv):
        pass
    print(LIB)
