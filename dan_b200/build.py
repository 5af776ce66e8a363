"""Build ``libdan_b200.so`` in-tree with nvcc for sm_100a.

    python -m dan_b200.build [-v]

Every ``csrc/*.cu`` is compiled in parallel (``-gencode arch=compute_100a,code=sm_100a
-O3 -lineinfo``) into ``_build/`` and linked into ``dan_b200/libdan_b200.so`` with
the CUDA runtime linked statically, so the library does not depend on which
libcudart the host process (e.g. torch) has loaded. Objects are rebuilt only when
their source or a header is newer.
"""
import argparse
import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(os.path.dirname(HERE), "_build")
LIB = os.path.join(HERE, "libdan_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build libdan_b200.so")


def _stale(obj, src, headers):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or any(os.path.getmtime(h) > t for h in headers)


def build(verbose=False, ptxas_info=False):
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(os.path.dirname(HERE), "include", "*.h"))
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    jobs = []
    objs = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if ptxas_info or _stale(obj, src, headers):
            jobs.append([cc, *ARCH, *FLAGS, *extra, "-I", CSRC, "-I", os.path.join(os.path.dirname(HERE), "include"),
                         "-c", src, "-o", obj])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    failed = []
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for cmd, r in ex.map(run, jobs):
            out = (r.stdout + r.stderr).strip()
            if out and (verbose or ptxas_info or r.returncode):
                print(out, file=sys.stderr)
            if r.returncode:
                failed.append(cmd[-1])
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    if jobs or not os.path.exists(LIB):
        cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs, "-lcuda" if False else "-ldl", "-lrt",
               "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills / shared memory per kernel")
    a = ap.parse_args()
    print(build(a.verbose, a.ptxas_info))
