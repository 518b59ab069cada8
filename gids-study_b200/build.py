"""Build the B200 GIDS libraries in-tree (no GPU needed: nvcc cross-compiles).

Outputs (git-ignored, shipped with the source tree):
  lib/libgids_b200.so                      C ABI (include/gids_b200.h), sm_100a kernels,
                                           CUDA runtime linked statically, only gids_* exported
  BAM_Feature_Store/BAM_Feature_Store*.so  pybind11 module over the C ABI

Usage: python gids-study_b200/build.py [--force]
       GIDS_PHASE_TIMERS=1 python gids-study_b200/build.py   (diagnosis build: per-phase timers)
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "lib", "libgids_b200.so")
PYMOD_DIR = os.path.join(HERE, "BAM_Feature_Store")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

CU_SOURCES = ["gather.cu", "store.cu", "noalloc.cu", "sampler.cu"]
CPP_SOURCES = ["backing.cpp", "abi.cpp"]
HEADERS = [os.path.join(CSRC, "gids_internal.hpp"), os.path.join(INCLUDE, "gids_b200.h")]


def _pymod_path() -> str:
    return os.path.join(PYMOD_DIR, "BAM_Feature_Store" + sysconfig.get_config_var("EXT_SUFFIX"))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(force: bool = False) -> dict:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    # GIDS_PHASE_TIMERS=1: the diagnosis build (per-phase gather timers in the stats)
    defines = ["-DGIDS_PHASE_TIMERS"] if os.environ.get("GIDS_PHASE_TIMERS") == "1" else []
    stamp = os.path.join(BUILD, "defines.txt")
    if not os.path.exists(stamp) or open(stamp).read() != " ".join(defines):
        force = True
        with open(stamp, "w") as f:
            f.write(" ".join(defines))
    objs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        if force or _stale(o, [s] + HEADERS):
            _run([NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                  "-Xptxas", "-v", *defines, f"-I{INCLUDE}", "-c", s, "-o", o])
        objs.append(o)
    for src in CPP_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        if force or _stale(o, [s] + HEADERS):
            _run(["g++", "-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-Wall", f"-I{INCLUDE}",
                  f"-I{CUDA_HOME}/include", "-c", s, "-o", o])
        objs.append(o)
    vscript = os.path.join(BUILD, "exports.map")
    with open(vscript, "w") as f:
        f.write("{ global: gids_*; local: *; };\n")
    if force or _stale(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs,
              "-Xlinker", f"--version-script={vscript}", "-Xlinker", "-Bsymbolic", "-lpthread"])

    import pybind11

    pymod = _pymod_path()
    src = os.path.join(CSRC, "bam_feature_store_py.cpp")
    if force or _stale(pymod, [src, LIB, os.path.join(INCLUDE, "gids_b200.h")]):
        py_inc = sysconfig.get_paths()["include"]
        _run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden", f"-I{INCLUDE}",
              f"-I{pybind11.get_include()}", f"-I{py_inc}", src, "-o", pymod, f"-L{os.path.dirname(LIB)}",
              "-lgids_b200", "-Wl,-rpath,$ORIGIN/../lib"])
    return {"lib": LIB, "pymod": pymod}


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
