"""Build libknx.so (all sm_100a CUDA kernels behind the C ABI in include/knx.h).

    python build.py            # incremental: rebuild objects whose sources changed
    python build.py --force    # rebuild everything

Objects go to _build/ next to this file; the shared library to lib/libknx.so.  Only nvcc is
needed (no GPU): the code is compiled for sm_100a exclusively.
"""
import argparse
import hashlib
import os
import pathlib
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "lib" / "libknx.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", f"-I{REPO / 'include'}", f"-I{CSRC}"]


def _digest(paths):
    h = hashlib.sha256()
    for p in sorted(paths):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(ARCH + FLAGS).encode())
    return h.hexdigest()[:16]


def build(force=False, verbose=False, extra=()):
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list((REPO / "include").glob("*.h"))
    objs = []
    for cu in sorted(CSRC.glob("*.cu")):
        tag = _digest([cu] + headers)
        obj = BUILD / f"{cu.stem}.{tag}.o"
        objs.append(obj)
        if obj.exists() and not force:
            continue
        for old in BUILD.glob(f"{cu.stem}.*.o"):
            old.unlink()
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", str(cu), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    stamp = BUILD / "lib.stamp"
    key = ",".join(o.name for o in objs)
    if force or not LIB.exists() or not stamp.exists() or stamp.read_text() != key:
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        stamp.write_text(key)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    a = ap.parse_args()
    extra = ("-Xptxas", "-v") if a.ptxas_v else ()
    print(build(force=a.force or a.ptxas_v, verbose=a.verbose, extra=extra))
    sys.exit(0)
