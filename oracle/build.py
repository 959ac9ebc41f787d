"""Build recipes for the test oracle (TEST INFRASTRUCTURE ONLY).

* ``build_oracle()`` compiles this project's CPU restatement ``hq_oracle.c`` into
  ``oracle/liboracle.so`` with gcc.
* ``build_ref()`` compiles the reference's own sources where they lie (nothing is
  copied): ``hydrogen/src/model/marlin_gemm.cu`` with ``ref_shim.cu`` into
  ``oracle/_ref/libref_marlin.so``, and ``hydrogen/src/batcher/split_fuse.cpp``
  with ``ref_batcher_shim.cpp`` into ``oracle/_ref/libref_batcher.so``.
* ``build_ref_h08()`` compiles the reference's H08 harness
  ``hydrogen/src/tools/bench_marlin_gemm.cpp`` against this library's drop-in
  header and links it to ``nebula_b200/libhq.so``.  These need
  the reference tree: the directory named by ``HQ_REFERENCE_ROOT``, else a
  checkout named ``reference`` beside this repository.  Where neither exists
  (the GPU machine) the prebuilt libraries are used; they are kept out of
  version control (``oracle/_ref/`` is git-ignored) and travel with the working
  tree.

The product library never loads either file.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def ref_root() -> str:
    """The reference tree: $HQ_REFERENCE_ROOT, else a checkout named `reference` beside this repository."""
    return os.environ.get("HQ_REFERENCE_ROOT") or os.path.join(os.path.dirname(ROOT), "reference")


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
    return [os.path.join(ref_root(), "hydrogen", "src", "model", "marlin_gemm.cu")]


def ref_batcher_sources() -> list[str]:
    return [os.path.join(ref_root(), "hydrogen", "src", "batcher", "split_fuse.cpp")]


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
               "-I", os.path.join(ref_root(), "hydrogen", "include"),
               srcs[0], shim, "-o", out + ".tmp", "-lcudart"]
        subprocess.run(cmd, check=True)
        os.replace(out + ".tmp", out)
    build_ref_batcher(force)
    return out


def build_ref_batcher(force: bool = False) -> str | None:
    """Compile the reference split-fuse scheduler (split_fuse.cpp, C++20 as hydrogen/CMakeLists.txt builds
    it) with the C shim; None when neither the reference tree nor a prebuilt library is present."""
    out = os.path.join(HERE, "_ref", "libref_batcher.so")
    srcs = ref_batcher_sources()
    if not all(os.path.exists(s) for s in srcs):
        return out if os.path.exists(out) else None
    shim = os.path.join(HERE, "ref_batcher_shim.cpp")
    if force or _stale(out, srcs + [shim, __file__]):
        os.makedirs(os.path.dirname(out), exist_ok=True)
        cmd = [NVCC, "-std=c++20", "-O2", "-x", "cu", "-gencode", "arch=compute_100a,code=sm_100a",
               "-Xcompiler", "-fPIC", "-shared", "-I", os.path.join(ref_root(), "hydrogen", "include"),
               srcs[0], shim, "-o", out + ".tmp", "-lcudart"]
        subprocess.run(cmd, check=True)
        os.replace(out + ".tmp", out)
    return out


def build_ref_h08(force: bool = False) -> str | None:
    """Compile the reference's H08 harness, hydrogen/src/tools/bench_marlin_gemm.cpp, unmodified,
    against this library's drop-in header (oracle/h08/marlin_gemm.hpp includes
    include/hq_marlin_gemm.hpp) and link it to nebula_b200/libhq.so: the reference's acceptance
    program for the MarlinGemmEngine API, run on the drop-in.  Output:
    oracle/_ref/hydrogen_bench_marlin_gemm (rpath to the in-tree libhq.so).  None when the
    reference tree or libhq.so is absent and no prebuilt harness exists."""
    out = os.path.join(HERE, "_ref", "hydrogen_bench_marlin_gemm")
    src = os.path.join(ref_root(), "hydrogen", "src", "tools", "bench_marlin_gemm.cpp")
    lib = os.path.join(ROOT, "nebula_b200", "libhq.so")
    hdrs = [os.path.join(HERE, "h08", "marlin_gemm.hpp"), os.path.join(ROOT, "include", "hq_marlin_gemm.hpp")]
    if not (os.path.exists(src) and os.path.exists(lib)):
        return out if os.path.exists(out) else None
    if force or _stale(out, [src, lib, __file__] + hdrs):
        os.makedirs(os.path.dirname(out), exist_ok=True)
        cmd = ["g++", "-std=c++20", "-O2", "-I", os.path.join(HERE, "h08"), "-I", os.path.join(ROOT, "include"),
               src, "-o", out + ".tmp", "-L", os.path.dirname(lib), "-lhq",
               "-Wl,-rpath,$ORIGIN/../../nebula_b200"]
        subprocess.run(cmd, check=True)
        os.replace(out + ".tmp", out)
    return out


if __name__ == "__main__":
    print(build_oracle(force="--force" in sys.argv))
    print(build_ref(force="--force" in sys.argv))
    print(build_ref_h08(force="--force" in sys.argv))
