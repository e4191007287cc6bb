"""Build the native parts of relmo_b200 in-tree.

1. ``librelm_mp_b200.so`` - the C-ABI CUDA library (``include/relm_mp.h``),
   compiled with nvcc for sm_100a only. No torch dependency.
2. ``relm_mp_ops.so`` - the ``torch.ops.relm_mp`` registration (same schemas
   as the reference library), a thin C++ layer over (1), linked with g++
   against the installed torch.

Both land in the package directory, where ``relmo_b200.ops.mp_runtime`` looks
for them (the reference loader globs ``relm_mp_ops*.so`` in its package
directory, ``src/relmo/ops/mp_runtime.py:97-125``).

Usage: ``python -m relmo_b200.build [--force] [--verbose-ptxas]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
CUDA_LIB = PKG / "librelm_mp_b200.so"
TORCH_LIB = PKG / "relm_mp_ops.so"

CUDA_SOURCES = [
    "relm_mp_plan.cu",
    "relm_mp_sort.cu",
    "relm_mp_ops.cu",
    "relm_mp_seg_f32.cu",
    "relm_mp_seg_f64.cu",
    "relm_mp_seg_bf16.cu",
    "relm_mp_seg_f16.cu",
    "relm_mp_noalloc.cu",
    "relm_mp_lgan.cu",
]
TORCH_SOURCES = ["relm_mp_torch.cpp", "relm_mp_cpu.cpp"]
HEADERS = ["relm_mp_internal.cuh", "relm_mp_segment.cuh", "relm_mp_seg_impl.cuh"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def cuda_home() -> Path:
    env = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if env:
        return Path(env)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    return Path("/usr/local/cuda")


def nvcc_version(nvcc: str) -> str:
    out = subprocess.run([nvcc, "--version"], capture_output=True, text=True, check=True).stdout
    m = re.search(r"release (\d+\.\d+)", out)
    return m.group(1) if m else "unknown"


def _newer(target: Path, deps: list[Path]) -> bool:
    if not target.is_file():
        return False
    t = target.stat().st_mtime
    return all(d.stat().st_mtime <= t for d in deps if d.exists())


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} {cmd[-1]}")
    if proc.stderr.strip():
        sys.stderr.write(proc.stderr)


def build_cuda(force: bool = False, verbose_ptxas: bool = False) -> Path:
    headers = [CSRC / h for h in HEADERS] + [INCLUDE / "relm_mp.h"]
    sources = [CSRC / s for s in CUDA_SOURCES]
    if not force and _newer(CUDA_LIB, sources + headers + [Path(__file__)]):
        return CUDA_LIB
    nvcc = str(cuda_home() / "bin" / "nvcc")
    version = nvcc_version(nvcc)
    BUILD.mkdir(parents=True, exist_ok=True)
    common = [
        nvcc, "-O3", "-std=c++17", *ARCH_FLAGS, "-lineinfo", "-Xcompiler", "-fPIC",
        "-Xcompiler", "-fvisibility=hidden", f"-I{INCLUDE}", f"-I{CSRC}",
        f'-DRELM_MP_KERNEL_CUDA_VERSION="{version}"',
    ]
    if verbose_ptxas:
        common += ["-Xptxas", "-v"]
    objs = []
    jobs = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        for src in sources:
            obj = BUILD / (src.stem + ".o")
            objs.append(obj)
            if force or not _newer(obj, [src] + headers + [Path(__file__)]):
                jobs.append(pool.submit(_run, common + ["-c", str(src), "-o", str(obj)]))
        for j in jobs:
            j.result()
    tmp = str(CUDA_LIB) + f".tmp{os.getpid()}"
    _run([nvcc, *ARCH_FLAGS, "-shared", "-o", tmp, *map(str, objs), "-cudart", "static"])
    os.replace(tmp, CUDA_LIB)
    return CUDA_LIB


def build_torch(force: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    sources = [CSRC / s for s in TORCH_SOURCES]
    deps = sources + [CSRC / "relm_mp_torch.h", INCLUDE / "relm_mp.h", CUDA_LIB, Path(__file__)]
    if not force and _newer(TORCH_LIB, deps):
        return TORCH_LIB
    version = str(torch.__version__).split("+")[0]
    major, minor = version.split(".")[:2]
    tcuda = getattr(torch.version, "cuda", None)
    cuda_tag = f"cu{tcuda.replace('.', '')}" if tcuda else "cpu"
    includes = [f"-I{p}" for p in cpp_extension.include_paths()]
    includes += [f"-I{cuda_home() / 'include'}", f"-I{INCLUDE}"]
    libdirs = cpp_extension.library_paths()
    link = [f"-L{p}" for p in libdirs] + [f"-Wl,-rpath,{p}" for p in libdirs]
    link += ["-lc10", "-ltorch", "-ltorch_cpu", "-lc10_cuda", "-ltorch_cuda"]
    link += [f"-L{PKG}", "-l:librelm_mp_b200.so", "-Wl,-rpath,$ORIGIN"]
    tmp = str(TORCH_LIB) + f".tmp{os.getpid()}"
    cmd = [
        "g++", "-O2", "-std=c++17", "-fPIC", "-shared",
        f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
        f'-DRELM_MP_BUILD_TORCH_VERSION="{version}"',
        f'-DRELM_MP_BUILD_CUDA_TAG="{cuda_tag}"',
        f'-DRELM_MP_ABI_TARGET="{major}.{minor}"',
        *includes, *map(str, sources), "-o", tmp, *link,
    ]
    _run(cmd)
    os.replace(tmp, TORCH_LIB)
    return TORCH_LIB


def build(force: bool = False, verbose_ptxas: bool = False) -> tuple[Path, Path]:
    return build_cuda(force, verbose_ptxas), build_torch(force)


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose-ptxas", action="store_true")
    parser.add_argument("--cuda-only", action="store_true")
    args = parser.parse_args()
    if args.cuda_only:
        print(build_cuda(args.force, args.verbose_ptxas))
    else:
        for p in build(args.force, args.verbose_ptxas):
            print(p)
    return 0


if __name__ == "__main__":
    sys.exit(main())
