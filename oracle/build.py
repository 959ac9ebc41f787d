"""Build recipes for the test oracle (TEST INFRASTRUCTURE ONLY).

* ``build_oracle()`` compiles this project's CPU restatement ``hq_oracle.c`` into
  ``oracle/liboracle.so`` with gcc.
* ``build_ref()`` compiles the reference's own ``hydrogen/src/model/marlin_gemm.cu``
  where it lies (nothing is copied) together with ``ref_shim.cu`` into
  ``oracle/_ref/libref_marlin.so``.  It needs the reference tree, so it runs only
  where that tree is present; the built ``.so`` is kept out of version control
  (``oracle/_ref/`` is git-ignored) and is copied along with the working tree to
  the machine that runs the GPU tests.

The product library never loads either file.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_ROOT = os.environ.get("HQ_REFERENCE_ROOT", "/root/reference")
NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")


def _stale(out: str, srcs: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(s) > t for s in srcs)


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "hq_oracle.c")
    hdr = os.path.join(HERE, "hq_oracle.h")
    out = os.path.join(HERE, "liboracle.so")
    if force or _stale(out, [src, hdr, __file__]):
        cmd = ["gcc", "-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fopenmp",
               "-std=c11", "-Wall", "-shared", "-fPIC", src, "-o", out + ".tmp", "-lm"]
        subprocess.run(cmd, check=True)
        os.replace(out + ".tmp", out)
    return out


def ref_sources() -> list[str]:
    return [os.path.join(REF_ROOT, "hydrogen", "src", "model", "marlin_gemm.cu")]


def build_ref(force: bool = False) -> str | None:
    """Compile the reference Marlin engine from its own source tree.

    Flags follow hydrogen/CMakeLists.txt:39-46 (-O3 --use_fast_math, C++20);
    the architecture is sm_100a instead of the reference's sm_89 so that the
    reference kernels run on a B200.  Returns None when the reference tree is
    absent (GPU box): the prebuilt library is then used if present.
    """
    out_dir = os.path.join(HERE, "_ref")
    out = os.path.join(out_dir, "libref_marlin.so")
    srcs = ref_sources()
    if not all(os.path.exists(s) for s in srcs):
        return out if os.path.exists(out) else None
    shim = os.path.join(HERE, "ref_shim.cu")
    if force or _stale(out, srcs + [shim, __file__]):
        os.makedirs(out_dir, exist_ok=True)
        cmd = [NVCC, "-std=c++20", "-O3", "--use_fast_math", "--expt-relaxed-constexpr",
               "-gencode", "arch=compute_100a,code=sm_100a",
               "-Xcompiler", "-fPIC", "-shared",
               "-I", os.path.join(REF_ROOT, "hydrogen", "include"),
               srcs[0], shim, "-o", out + ".tmp", "-lcudart"]
        subprocess.run(cmd, check=True)
        os.replace(out + ".tmp", out)
    return out


if __name__ == "__main__":
    print(build_oracle(force="--force" in sys.argv))
    print(build_ref(force="--force" in sys.argv))
