"""Build the in-tree native libraries of multi_lora_b200.

* ``libmlora_b200.so`` — every CUDA kernel plus the C ABI of
  ``include/mlora_b200.h``; compiled by nvcc for sm_100a only, static cudart,
  no torch dependency.
* ``_mlora_torch.so`` — the ``torch.ops.mlora`` binding (torch_ops.cpp),
  linked against ``libmlora_b200.so`` through an ``$ORIGIN`` rpath.

Both land next to this file so that they travel with the source tree. A
library is rebuilt only when one of its sources is newer than it.

    python -m multi_lora_b200.build [--force]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = ROOT / "_build"
CUDA_LIB = PKG / "libmlora_b200.so"
TORCH_LIB = PKG / "_mlora_torch.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _cuda_sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "mlora_b200.h"]


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def build_cuda_lib(force: bool = False, verbose: bool = False) -> Path:
    srcs = _cuda_sources()
    hdrs = _headers()
    if not force and not _stale(CUDA_LIB, srcs + hdrs):
        return CUDA_LIB
    OBJ.mkdir(exist_ok=True)
    nvcc = _nvcc()
    objs = []
    jobs = []
    for src in srcs:
        obj = OBJ / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            jobs.append([nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(ROOT / "include"), "-c", str(src), "-o", str(obj)])
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 4))) as ex:
        for cmd, fut in [(c, ex.submit(_run, c)) for c in jobs]:
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            fut.result()
    tmp = CUDA_LIB.with_suffix(".so.tmp")
    _run([nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)])
    os.replace(tmp, CUDA_LIB)
    return CUDA_LIB


def build_torch_lib(force: bool = False, verbose: bool = False) -> Path:
    src = CSRC / "torch_ops.cpp"
    if not force and not _stale(TORCH_LIB, [src, CUDA_LIB, ROOT / "include" / "mlora_b200.h"]):
        return TORCH_LIB
    import torch
    import torch.utils.cpp_extension as ext

    incs = ext.include_paths("cuda")
    libs = ext.library_paths("cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [
        os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-shared", "-fPIC",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H",
        *[f"-I{p}" for p in incs], str(src), "-o", str(TORCH_LIB.with_suffix(".so.tmp")),
        *[f"-L{p}" for p in libs], f"-L{PKG}",
        "-lmlora_b200", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
        "-Wl,-rpath,$ORIGIN",
    ]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    _run(cmd)
    os.replace(TORCH_LIB.with_suffix(".so.tmp"), TORCH_LIB)
    return TORCH_LIB


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_cuda_lib(force=force, verbose=verbose)
    build_torch_lib(force=force, verbose=verbose)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    build_all(force=args.force, verbose=args.verbose)
    print(f"built {CUDA_LIB.name} and {TORCH_LIB.name}")


if __name__ == "__main__":
    main()
