"""Builds the reference's own CUDA histogram extension (test infrastructure only).

    python oracle/build_ref_hist.py [REFERENCE_ROOT]

Compiles ``yabt/_cuda/hist.cu`` of the reference (grafael/yabt) from its source,
the way its loader does on first use (``torch.utils.cpp_extension.load`` with
``extra_cuda_cflags=["-O3"]``, yabt/cuda_hist.py:42-67), for the B200's
architecture (compute capability 10.0, what the loader targets on a B200), into
``oracle/_ref/yabt_hist_cuda.so``. Nothing is copied from the reference tree:
the source is compiled where it lies, and the output stays out of version
control (it travels to the GPU box with the working tree). The GPU timing test
(tests/test_gpu_ref_hist.py) loads it to time the reference's kernels
(``hist_kernel`` / ``hist_priv_kernel``) beside this library's on the same
B200; nothing in the library imports it.
"""

from __future__ import annotations

import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NAME = "yabt_hist_cuda"          # the module name the reference's loader uses


def build(ref: str = "/root/reference") -> str | None:
    src = os.path.join(ref, "yabt", "_cuda", "hist.cu")
    dst = os.path.join(OUT, NAME + ".so")
    if not os.path.exists(src):
        return None
    if os.path.exists(dst) and os.path.getmtime(dst) >= os.path.getmtime(src):
        return dst
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    bindir = os.path.dirname(os.path.abspath(sys.executable))   # ninja next to the interpreter
    os.environ["PATH"] = bindir + os.pathsep + os.environ.get("PATH", "")
    from torch.utils.cpp_extension import load
    work = os.path.join(OUT, "_hist_build")
    os.makedirs(work, exist_ok=True)
    load(name=NAME, sources=[src], extra_cuda_cflags=["-O3"], build_directory=work, verbose=False)
    shutil.copy2(os.path.join(work, NAME + ".so"), dst)
    shutil.rmtree(work, ignore_errors=True)
    return dst


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else "/root/reference"))
