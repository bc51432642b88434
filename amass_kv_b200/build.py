"""Build libamass_b200.so in-tree with nvcc for sm_100a.

    python -m amass_kv_b200.build

The library is written next to this file; the Python host layer loads it with
ctypes.  The build is a plain nvcc invocation (no torch extension machinery):
every .cu under csrc/ is compiled into one shared object.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libamass_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-O3"]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def build(verbose: bool = False, ptxas_v: bool = False, force: bool = False):
    srcs = sources()
    hdrs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(
        os.path.join(os.path.dirname(HERE), "include", "*.h"))
    if (not force and os.path.exists(LIB) and os.path.getmtime(LIB) >=
            max(os.path.getmtime(p) for p in srcs + hdrs)):
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    extra = ["-Xptxas", "-v"] if ptxas_v else []
    procs = []
    for s in srcs:
        o = os.path.join(objdir, os.path.basename(s)[:-3] + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", s, "-o", o]
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE,
                                            stderr=subprocess.STDOUT,
                                            text=True)))
        objs.append(o)
    failed = False
    for cmd, p in procs:
        out, _ = p.communicate()
        if verbose or ptxas_v or p.returncode:
            sys.stdout.write(out)
        if p.returncode:
            failed = True
            sys.stdout.write("FAILED: " + " ".join(cmd) + "\n")
    if failed:
        raise RuntimeError("nvcc failed")
    cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart"]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_v="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
