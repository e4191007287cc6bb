"""Build the reference's own CPU ``relm_mp`` op library as a test oracle.

TEST INFRASTRUCTURE ONLY. Nothing in the ``relmo_b200`` product imports, links or
runs this. It compiles ``src/_ops/mp/mp_ops.cpp`` of maichmueller/relmo straight
from the reference checkout (read-only; nothing is copied into this repository)
with ``g++`` against the installed torch headers, CPU only
(``RELM_MP_HAS_CUDA=0``), into ``oracle/_ref/relm_mp_ref.so``.

The reference's own build (``src/CMakeLists.txt:104-160``) passes four string
macros and ``RELM_MP_HAS_CUDA``; the same macros are given here on the command
line instead of through CMake.

The library registers ``TORCH_LIBRARY(relm_mp, ...)``, the same namespace as the
B200 library, so it is only ever loaded in a process that does not load
``relmo_b200`` (the golden-vector generator and ``bench.py --impl reference``).

``--cuda`` also builds the reference's GPU library the same way, with
``src/_ops/mp/mp_cuda_kernels.cu`` compiled by nvcc for sm_100a and
``RELM_MP_HAS_CUDA=1`` (``src/CMakeLists.txt:146``), into
``oracle/_ref/relm_mp_ref_cuda.so``: the reference's own SIMT kernels, timed on
the B200 beside the new ones by ``oracle/ref_gpu_ops.py`` (a separate process,
for the same namespace reason). It is a baseline only; nothing of the product
loads it.

Usage: ``python oracle/build_ref.py [--reference-root PATH] [--force] [--cuda]``.
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
OUT_LIB = OUT_DIR / "relm_mp_ref.so"
# the reference checkout: $RELMO_REFERENCE_ROOT, else a `reference` directory beside this repository
DEFAULT_REFERENCE_ROOT = Path(os.environ.get("RELMO_REFERENCE_ROOT", str(HERE.parents[1] / "reference")))
REFERENCE_SOURCE = Path("src/_ops/mp/mp_ops.cpp")
REFERENCE_CUDA_SOURCE = Path("src/_ops/mp/mp_cuda_kernels.cu")
OUT_CUDA_LIB = OUT_DIR / "relm_mp_ref_cuda.so"
CUDA_BUILD_DIR = OUT_DIR / "cuda_obj"


def _torch_flags() -> tuple[list[str], list[str], str, str]:
    import torch
    from torch.utils import cpp_extension

    includes = [f"-I{p}" for p in cpp_extension.include_paths()]
    libdirs = cpp_extension.library_paths()
    link = [f"-L{p}" for p in libdirs] + [f"-Wl,-rpath,{p}" for p in libdirs]
    link += ["-lc10", "-ltorch", "-ltorch_cpu"]
    abi = f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"
    version = str(torch.__version__).split("+")[0]
    major, minor = version.split(".")[:2]
    return includes + [abi], link, version, f"{major}.{minor}"


def build(reference_root: Path = DEFAULT_REFERENCE_ROOT, force: bool = False) -> Path | None:
    """Compile the reference CPU op library; return its path, or None when the
    reference checkout is absent (e.g. on a GPU box)."""

    source = reference_root / REFERENCE_SOURCE
    if not source.is_file():
        return OUT_LIB if OUT_LIB.is_file() else None
    if OUT_LIB.is_file() and not force and OUT_LIB.stat().st_mtime >= source.stat().st_mtime:
        return OUT_LIB
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    cflags, link, torch_version, abi_target = _torch_flags()
    cmd = [
        "g++",
        "-O2",
        "-std=c++17",
        "-fPIC",
        "-shared",
        "-fopenmp",
        "-DRELM_MP_HAS_CUDA=0",
        f'-DRELM_MP_BUILD_TORCH_VERSION="{torch_version}"',
        '-DRELM_MP_BUILD_CUDA_TAG="cpu"',
        f'-DRELM_MP_ABI_TARGET="{abi_target}"',
        '-DRELM_MP_ABI_LANE="nonstable"',
        *cflags,
        str(source),
        "-o",
        str(OUT_LIB) + ".tmp",
        *link,
    ]
    subprocess.run(cmd, check=True)
    os.replace(str(OUT_LIB) + ".tmp", OUT_LIB)
    return OUT_LIB


def build_cuda(reference_root: Path = DEFAULT_REFERENCE_ROOT, force: bool = False) -> Path | None:
    """Compile the reference's GPU op library (mp_ops.cpp + mp_cuda_kernels.cu,
    sm_100a); return its path, or None when the reference checkout is absent."""

    import torch
    from torch.utils import cpp_extension

    cpp, cu = reference_root / REFERENCE_SOURCE, reference_root / REFERENCE_CUDA_SOURCE
    if not (cpp.is_file() and cu.is_file()):
        return OUT_CUDA_LIB if OUT_CUDA_LIB.is_file() else None
    newest = max(cpp.stat().st_mtime, cu.stat().st_mtime, Path(__file__).stat().st_mtime)
    if OUT_CUDA_LIB.is_file() and not force and OUT_CUDA_LIB.stat().st_mtime >= newest:
        return OUT_CUDA_LIB
    CUDA_BUILD_DIR.mkdir(parents=True, exist_ok=True)
    cflags, link, torch_version, abi_target = _torch_flags()
    tcuda = getattr(torch.version, "cuda", None) or "12.8"
    tag = f"cu{tcuda.replace('.', '')}"
    defs = [
        "-DRELM_MP_HAS_CUDA=1", "-DUSE_CUDA", f'-DRELM_MP_BUILD_TORCH_VERSION="{torch_version}"',
        f'-DRELM_MP_BUILD_CUDA_TAG="{tag}"', f'-DRELM_MP_ABI_TARGET="{abi_target}"', '-DRELM_MP_ABI_LANE="nonstable"',
    ]
    cuda_home = Path(cpp_extension.CUDA_HOME or "/usr/local/cuda")
    cu_obj, cpp_obj = CUDA_BUILD_DIR / "mp_cuda_kernels.o", CUDA_BUILD_DIR / "mp_ops.o"
    subprocess.run(
        [str(cuda_home / "bin" / "nvcc"), "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
         "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", *defs, *cflags, "-c", str(cu), "-o", str(cu_obj)],
        check=True,
    )
    subprocess.run(
        ["g++", "-O2", "-std=c++17", "-fPIC", "-fopenmp", *defs, *cflags, f"-I{cuda_home / 'include'}", "-c",
         str(cpp), "-o", str(cpp_obj)],
        check=True,
    )
    tmp = str(OUT_CUDA_LIB) + ".tmp"
    subprocess.run(
        ["g++", "-shared", "-fopenmp", str(cpp_obj), str(cu_obj), "-o", tmp, *link, "-lc10_cuda", "-ltorch_cuda",
         f"-L{cuda_home / 'lib64'}", "-lcudart"],
        check=True,
    )
    os.replace(tmp, OUT_CUDA_LIB)
    return OUT_CUDA_LIB


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference-root", type=Path, default=DEFAULT_REFERENCE_ROOT)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--cuda", action="store_true", help="also build the reference's GPU library (sm_100a)")
    args = parser.parse_args()
    out = build(args.reference_root, args.force)
    if out is not None and args.cuda:
        out = build_cuda(args.reference_root, args.force)
    if out is None:
        print("reference checkout not found; nothing built", file=sys.stderr)
        return 1
    print(out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
