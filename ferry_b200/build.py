"""Build libferry_cuda.so in-tree for sm_100a (nvcc, no JIT cache).

``python -m ferry_b200.build`` compiles every ``csrc/*.cu`` (one nvcc per
file, in parallel) and links ``ferry_b200/libferry_cuda.so``. The library is git-ignored but travels with
the working tree, so a GPU box runs exactly what was compiled here.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libferry_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + [
        os.path.join(ROOT, "include", "ferry_cuda.h")]
    return any(os.path.getmtime(p) > t for p in deps)


DRIVERS = os.path.join(HERE, "drivers")
DRIVER_BIN = os.path.join(DRIVERS, "bin")


def build_drivers(force: bool = False) -> list[str]:
    """The C++ drivers (drivers/*.cpp) against include/ferry_cuda.h and the
    built library (rpath to it), into drivers/bin/."""
    os.makedirs(DRIVER_BIN, exist_ok=True)
    out = []
    for src in sorted(glob.glob(os.path.join(DRIVERS, "*.cpp"))):
        exe = os.path.join(DRIVER_BIN, os.path.splitext(os.path.basename(src))[0])
        if force or not os.path.exists(exe) or os.path.getmtime(exe) < max(os.path.getmtime(src), os.path.getmtime(LIB)):
            cmd = [NVCC, "-O2", "-std=c++17", "-I" + os.path.join(ROOT, "include"), "-o", exe, src,
                   "-L" + HERE, "-lferry_cuda", "-Xlinker", "-rpath", "-Xlinker", "$ORIGIN/../.."]
            res = subprocess.run(cmd, capture_output=True, text=True)
            if res.returncode != 0:
                raise RuntimeError("driver build failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
        out.append(exe)
    return out


def _compile(src: str, obj: str, verbose: bool) -> str:
    cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-c",
           "-I" + os.path.join(ROOT, "include"), "-I" + CSRC, "-o", obj, src]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    return res.stdout + res.stderr


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every csrc/*.cu to an object (in parallel, objects under
    _build/), then link libferry_cuda.so."""
    if not force and not _stale():
        build_drivers()
        return LIB
    from concurrent.futures import ThreadPoolExecutor

    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    srcs = sources()
    objs = [os.path.join(objdir, os.path.splitext(os.path.basename(p))[0] + ".o") for p in srcs]
    with ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        logs = list(ex.map(lambda so: _compile(so[0], so[1], verbose), zip(srcs, objs)))
    cmd = [NVCC, *ARCH, "-shared", "-o", LIB + ".tmp", *objs]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc link failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    os.replace(LIB + ".tmp", LIB)
    if verbose:
        print("".join(logs))
    build_drivers(force=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
