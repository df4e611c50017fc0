"""Builds libbt_ops.so (the sm_100a C-ABI library) in-tree with nvcc.

    python best-tts-godot_b200/build.py [--force] [--verbose]

Sources: best-tts-godot_b200/csrc/*.cu, *.cpp.  Output:
best-tts-godot_b200/bt_b200/libbt_ops.so (git-ignored; it travels with the
working tree).  The CUDA runtime is linked statically, so the library loads
on a machine without a GPU (its compute entry points then return BT_ECUDA).

Numerics flags: --fmad=false (no a*b+c contraction -- every op of the
reference rounds separately; kernels that want a fused multiply-add call
__fmaf_rn explicitly), IEEE division and square root (the nvcc defaults
without --use_fast_math), denormals preserved; the host compiler gets
-ffp-contract=off for the host-side math self-test.
"""
import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "bt_b200", "libbt_ops.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "--fmad=false", "-prec-div=true",
          "-prec-sqrt=true", "-ftz=false", "-I", INCLUDE, "-I", CSRC,
          "-Xcompiler", "-fPIC,-ffp-contract=off,-O2"]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the sm_100a library cannot be built")
    return path


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC)
                  if f.endswith((".cu", ".cpp")))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(INCLUDE, "bt_ops.h"))
    return hs


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    cc = nvcc()
    hdrs = headers()
    objs, jobs = [], []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            cmd = [cc] + ARCH + COMMON + ["-c", src, "-o", obj]
            if src.endswith(".cpp"):
                cmd = [cc] + COMMON + ["-x", "c++", "-c", src, "-o", obj]
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)

    if jobs:
        with ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            list(ex.map(run, jobs))
    if force or jobs or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        run([cc] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs)
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    try:
        print(build(force=args.force, verbose=args.verbose))
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
