"""Build the native extension ``xnn_b200/_C.so`` in-tree (sm_100a CUDA + C++/OpenMP).

``python -m xnn_b200.build`` compiles every source of ``xnn_b200/csrc`` with nvcc for
``sm_100a`` only (``-gencode arch=compute_100a,code=sm_100a``) and ``g++ -fopenmp``,
through ``torch.utils.cpp_extension`` (ninja, incremental), into ``xnn_b200/_build``,
and places the module next to the package so that it ships with the source tree.
nvcc cross-compiles: no GPU is needed to build.
"""
from __future__ import annotations

import glob
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")

CUDA_FLAGS = ["-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
              "--expt-relaxed-constexpr", "-Xptxas=-warn-spills"]
CXX_FLAGS = ["-O3", "-std=c++17", "-fopenmp"]


def sources():
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    srcs += sorted(glob.glob(os.path.join(CSRC, "*.cpp")))
    srcs += sorted(glob.glob(os.path.join(CSRC, "cpu", "*.cpp")))
    return srcs


def _openmp_ok(cxx: str) -> bool:
    import subprocess
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "t.cpp")
        with open(src, "w") as f:
            f.write("#include <omp.h>\nint main(){return omp_get_max_threads() > 0 ? 0 : 1;}\n")
        r = subprocess.run([cxx, "-fopenmp", src, "-o", os.path.join(d, "t")], capture_output=True)
        return r.returncode == 0


def _pick_openmp_compiler() -> None:
    """Use a C++ compiler whose OpenMP runtime links (the CPU twins need it)."""
    cxx = os.environ.get("CXX", "c++")
    if _openmp_ok(cxx):
        return
    for cand in ("/usr/bin/g++", "/usr/bin/c++"):
        if os.path.exists(cand) and _openmp_ok(cand):
            os.environ["CXX"] = cand
            os.environ["CC"] = cand.replace("g++", "gcc").replace("c++", "cc")
            return
    raise RuntimeError("no C++ compiler with a working OpenMP runtime")


def build(verbose: bool = False) -> str:
    """Compile (incrementally) and return the path of the in-tree module."""
    os.makedirs(BUILD, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
    _pick_openmp_compiler()
    from torch.utils.cpp_extension import load
    load(name="_C", sources=sources(), extra_cflags=CXX_FLAGS, extra_cuda_cflags=CUDA_FLAGS,
         extra_ldflags=["-fopenmp"], extra_include_paths=[CSRC], build_directory=BUILD,
         verbose=verbose, with_cuda=True, is_python_module=True)
    built = os.path.join(BUILD, "_C.so")
    if not os.path.exists(built):
        cands = glob.glob(os.path.join(BUILD, "_C*.so"))
        if not cands:
            raise RuntimeError("extension build produced no module")
        built = cands[0]
    target = os.path.join(HERE, "_C.so")
    tmp = target + ".tmp"
    shutil.copyfile(built, tmp)
    os.replace(tmp, target)
    return target


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv)
    print(path)
