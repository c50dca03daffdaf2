"""In-tree build of the native extension ``arc_forge_2026_b200/_C.so`` (sm_100a only).

Kernels live in ``csrc/*.cu`` and include only CUDA headers, so each compiles in seconds with nvcc;
``csrc/bindings.cpp`` is the one translation unit that includes torch. A generated ninja file gives
incremental, parallel builds. The result sits next to this file, so it travels with the repository
snapshot and ``import arc_forge_2026_b200._C`` finds it without any JIT cache.

    python -m arc_forge_2026_b200.build          # build (incremental)
    python -m arc_forge_2026_b200.build --clean  # rebuild from scratch
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG.parent / "_build"
TARGET = PKG / "_C.so"
ARCH = "-gencode arch=compute_100a,code=sm_100a"
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _torch_paths():
    import torch
    import torch.utils.cpp_extension as ce  # noqa: F401  (only for the paths)
    root = Path(torch.__file__).resolve().parent
    incs = [root / "include", root / "include/torch/csrc/api/include"]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    return incs, root / "lib", abi


def write_ninja() -> Path:
    incs, tlib, abi = _torch_paths()
    py_inc = sysconfig.get_paths()["include"]
    cutlass = None  # CuTe headers are optional; kernels here use inline PTX
    BUILD.mkdir(exist_ok=True)
    cu = sorted(CSRC.glob("*.cu"))
    cpp = sorted(CSRC.glob("*.cpp"))
    nvflags = (f"{ARCH} -lineinfo -O3 -std=c++17 --expt-relaxed-constexpr -Xcompiler -fPIC "
               f"-I{CSRC} -I{CUDA_HOME}/include -Xptxas -warn-spills")
    cxxflags = (f"-O2 -std=c++17 -fPIC -D_GLIBCXX_USE_CXX11_ABI={abi} -DTORCH_EXTENSION_NAME=_C "
                f"-DTORCH_API_INCLUDE_EXTENSION_H -I{CSRC} -I{CUDA_HOME}/include -I{py_inc} "
                + " ".join(f"-isystem {p}" for p in incs))
    ldflags = (f"-shared -L{tlib} -L{CUDA_HOME}/lib64 -Wl,-rpath,{tlib} -lc10 -ltorch -ltorch_cpu -ltorch_python "
               f"-lc10_cuda -ltorch_cuda -lcudart")
    lines = [
        f"nvflags = {nvflags}",
        f"cxxflags = {cxxflags}",
        f"ldflags = {ldflags}",
        f"rule nvcc\n  command = {CUDA_HOME}/bin/nvcc $nvflags -MD -MF $out.d -c $in -o $out\n  depfile = $out.d\n"
        f"  deps = gcc\n  description = NVCC $in",
        "rule cxx\n  command = c++ $cxxflags -MD -MF $out.d -c $in -o $out\n  depfile = $out.d\n  deps = gcc\n"
        "  description = CXX $in",
        "rule link\n  command = c++ $in $ldflags -o $out\n  description = LINK $out",
    ]
    objs = []
    for src in cu:
        obj = BUILD / (src.stem + ".cu.o")
        lines.append(f"build {obj}: nvcc {src}")
        objs.append(obj)
    for src in cpp:
        obj = BUILD / (src.stem + ".o")
        lines.append(f"build {obj}: cxx {src}")
        objs.append(obj)
    lines.append(f"build {TARGET}: link {' '.join(map(str, objs))}")
    lines.append(f"default {TARGET}")
    path = BUILD / "build.ninja"
    text = "\n".join(lines) + "\n"
    if not path.exists() or path.read_text() != text:
        path.write_text(text)
    return path


def build(clean: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    if clean and BUILD.exists():
        shutil.rmtree(BUILD)
    nf = write_ninja()
    cmd = ["ninja", "-f", str(nf)]
    if jobs:
        cmd += ["-j", str(jobs)]
    if verbose:
        cmd.append("-v")
    r = subprocess.run(cmd, cwd=str(BUILD), capture_output=not verbose, text=True)
    if r.returncode != 0:
        sys.stderr.write((r.stdout or "") + (r.stderr or ""))
        raise RuntimeError("native build failed")
    return TARGET


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("-j", "--jobs", type=int)
    a = ap.parse_args()
    print(build(a.clean, a.verbose, a.jobs))
