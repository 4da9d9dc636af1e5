"""Build the hif8_b200 native libraries in place.

* ``hif8_b200/libhif8_b200.so`` -- the C ABI (include/hif8_b200.h) and every
  CUDA kernel, compiled for sm_100a only; no PyTorch dependency.
* ``hif8_b200/_C_ops.so`` -- the PyTorch operator registrations
  (torch.ops.vllm_ascend_hif8.* and torch.ops.hif8_b200.*), a thin C++ layer
  that links the C ABI library (rpath $ORIGIN).

Usage: ``python build.py [--force] [-j N]``.  nvcc cross-compiles, so this
runs on a machine without a GPU.  Objects go to ``_build/`` (not committed).
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
PKG = HERE / "hif8_b200"
BUILD = HERE / "_build"
INCLUDE = REPO / "include"

CU_SOURCES = ["cabi.cu", "quant.cu", "gemv.cu", "gemm_tc.cu", "kv.cu", "noalloc.cu", "model.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# No --use_fast_math / -ftz: the static quantiser and the decode paths rely on
# IEEE division, denormals and round-to-nearest conversions.
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xptxas", "-O3",
              "-I", str(INCLUDE), "-I", str(CSRC)]


def _newer(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} ... {cmd[-1]}")


def build(force: bool = False, jobs: int | None = None) -> dict[str, Path]:
    BUILD.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    objects = []
    work = []
    for src in CU_SOURCES:
        obj = BUILD / (Path(src).stem + ".o")
        objects.append(obj)
        if force or _newer(obj, [CSRC / src, *headers]):
            work.append([NVCC, *ARCH, *NVCC_FLAGS, "-c", str(CSRC / src), "-o", str(obj)])
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as pool:
        for future in [pool.submit(_run, cmd) for cmd in work]:
            future.result()

    lib = PKG / "libhif8_b200.so"
    if force or work or not lib.exists():
        _run([NVCC, *ARCH, "-shared", "-cudart", "shared", "-o", str(lib), *map(str, objects),
              "-Xlinker", "-soname=libhif8_b200.so"])

    ops = PKG / "_C_ops.so"
    ops_src = CSRC / "torch_ops.cpp"
    if force or _newer(ops, [ops_src, lib, *INCLUDE.glob("*.h")]):
        import torch.utils.cpp_extension as ext

        torch_inc = ext.include_paths()
        torch_lib = ext.library_paths()[0]
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-D_GLIBCXX_USE_CXX11_ABI=1",
               "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=_C_ops",
               *[f"-I{p}" for p in torch_inc], "-I/usr/local/cuda/include", f"-I{INCLUDE}",
               str(ops_src), "-o", str(ops), f"-L{torch_lib}", f"-L{PKG}",
               "-lhif8_b200", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch",
               "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
        import torch

        abi = int(torch.compiled_with_cxx11_abi())
        cmd[5] = f"-D_GLIBCXX_USE_CXX11_ABI={abi}"
        _run(cmd)
    return {"lib": lib, "ops": ops}


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    parser.add_argument("-j", type=int, default=None)
    args = parser.parse_args()
    out = build(force=args.force, jobs=args.j)
    for name, path in out.items():
        print(f"{name}: {path}")


if __name__ == "__main__":
    main()
