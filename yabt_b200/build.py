"""Build libyabt_b200.so in-tree with nvcc for sm_100a.

    python -m yabt_b200.build [--force] [--bounds-check]

Every ``csrc/*.cu`` file is compiled to an object and linked into
``yabt_b200/libyabt_b200.so`` (static CUDA runtime, no torch dependency).
Rebuilds only when a source or header is newer than the library.
``--bounds-check`` builds the same sources with ``-DYABT_BOUNDS_CHECK`` into
``yabt_b200/libyabt_b200_checked.so`` (device-side index checks that report
through the kernels' error words); ``YABT_LIB_VARIANT=checked`` makes the
package load it instead of the ordinary library.
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
LIB_CHECKED = os.path.join(HERE, "libyabt_b200_checked.so")
BUILD_CHECKED = os.path.join(HERE, "_build_checked")
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


def up_to_date(lib: str = LIB) -> bool:
    if not os.path.exists(lib):
        return False
    t = os.path.getmtime(lib)
    return all(os.path.getmtime(p) <= t for p in _deps())


def build(force: bool = False, verbose: bool = False, bounds_check: bool = False) -> str:
    lib_out = LIB_CHECKED if bounds_check else LIB
    build_dir = BUILD_CHECKED if bounds_check else BUILD
    extra = ["-DYABT_BOUNDS_CHECK"] if bounds_check else []
    if not force and up_to_date(lib_out):
        return lib_out
    os.makedirs(build_dir, exist_ok=True)
    cc = nvcc()
    objs = []
    procs = []
    for src in _sources():
        obj = os.path.join(build_dir, os.path.basename(src)[:-3] + ".o")
        cmd = [cc, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
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
    tmp = lib_out + ".tmp"
    cmd = [cc, *ARCH, "-shared", "-o", tmp, *objs]
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    if r.returncode != 0:
        raise RuntimeError("link failed:\n" + r.stdout.decode(errors="replace"))
    os.replace(tmp, lib_out)
    return lib_out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv, bounds_check="--bounds-check" in sys.argv))
