"""Build libyabt_b200.so in-tree with nvcc for sm_100a.

    python -m yabt_b200.build [--force]

Every ``csrc/*.cu`` file is compiled to an object and linked into
``yabt_b200/libyabt_b200.so`` (static CUDA runtime, no torch dependency).
Rebuilds only when a source or header is newer than the library.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libyabt_b200.so")
BUILD = os.path.join(HERE, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I" + os.path.join(ROOT, "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return _sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + [
        os.path.join(ROOT, "include", "yabt_b200.h"), os.path.abspath(__file__)]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in _deps())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    cc = nvcc()
    objs = []
    procs = []
    for src in _sources():
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        cmd = [cc, *ARCH, *FLAGS, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd))
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(obj)
    failed = []
    for src, pr in procs:
        out, _ = pr.communicate()
        if pr.returncode != 0:
            failed.append((src, out.decode(errors="replace")))
        elif verbose and out:
            print(out.decode(errors="replace"))
    if failed:
        msg = "\n".join(f"--- {s}\n{o}" for s, o in failed)
        raise RuntimeError("nvcc failed:\n" + msg)
    tmp = LIB + ".tmp"
    cmd = [cc, *ARCH, "-shared", "-o", tmp, *objs]
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    if r.returncode != 0:
        raise RuntimeError("link failed:\n" + r.stdout.decode(errors="replace"))
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
