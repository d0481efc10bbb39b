"""In-tree build of the native libraries (no JIT cache, no pip install).

    python -m zcutlass_b200.build            # core library + torch operators
    python -m zcutlass_b200.build --oracle   # also the test oracle (oracle/Makefile)

Outputs (git-ignored, shipped alongside the sources):
    zcutlass_b200/libzcutlass.so        kernels, dispatcher, C ABI (include/zcutlass_c.h)
    zcutlass_b200/libzcutlass_torch.so  torch.ops.zcutlass_torch.* / torch.ops.zcutlass.*

Every CUDA source is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a); host sources go through g++.
Each output is rebuilt unless a stamp beside it (zcutlass_b200/_build/*.sha256)
records the SHA-256 of the exact command and of every input file it was made
from, so a prebuilt library that does not match the committed sources is
always recompiled, whatever the file times say.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
CORE_SO = PKG / "libzcutlass.so"
TORCH_SO = PKG / "libzcutlass_torch.so"
BENCH_BIN = PKG / "zcutlass_bench"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
CXX = os.environ.get("CXX", "g++")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]

CORE_HOST_SRCS = ["foundation.cpp", "gemm.cpp", "c_abi.cpp", "tma_desc.cpp"]
CORE_CUDA_SRCS = ["launchers.cu", "collectives.cu"]


def _headers() -> list[Path]:
    return sorted(list(CSRC.rglob("*.hpp")) + list(CSRC.rglob("*.cuh")) + list(INCLUDE.rglob("*.h*")))


def _digest(cmd: list[str], deps: list[Path]) -> str:
    h = hashlib.sha256("\0".join(cmd).encode())
    for d in sorted(set(deps)):
        h.update(str(d.relative_to(ROOT) if d.is_relative_to(ROOT) else d).encode())
        h.update(d.read_bytes())
    return h.hexdigest()


def _stamp(target: Path) -> Path:
    return BUILD / (target.name + ".sha256")


def _make(target: Path, cmd: list[str], deps: list[Path], verbose: bool) -> None:
    """Runs `cmd` (which writes `target`) unless target exists and its stamp
    matches the digest of cmd and deps."""
    BUILD.mkdir(exist_ok=True)
    want = _digest(cmd, deps)
    stamp = _stamp(target)
    if target.exists() and stamp.exists() and stamp.read_text().strip() == want:
        return
    if verbose:
        print(" ".join(cmd), flush=True)
    stamp.unlink(missing_ok=True)
    subprocess.run(cmd, check=True)
    stamp.write_text(want + "\n")


def build_core(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = _headers()
    objs: list[Path] = []
    incs = [f"-I{INCLUDE}", f"-I{CSRC}", f"-I{CUDA_HOME / 'include'}"]
    for src in CORE_HOST_SRCS:
        s = CSRC / src
        o = BUILD / (s.stem + ".o")
        _make(o, [CXX, "-std=c++17", "-O2", "-fPIC", "-Wall", "-c", str(s), "-o", str(o), *incs], [s, *headers],
              verbose)
        objs.append(o)
    for src in CORE_CUDA_SRCS:
        s = CSRC / src
        o = BUILD / (s.stem + ".cu.o")
        _make(o, [NVCC, "-std=c++17", "-O3", "-lineinfo", *ARCH_FLAGS, "-Xcompiler", "-fPIC",
                  "-c", str(s), "-o", str(o), *incs], [s, *headers], verbose)
        objs.append(o)
    _make(CORE_SO, [NVCC, "-shared", *ARCH_FLAGS, "-o", str(CORE_SO), *map(str, objs),
                    "-Xlinker", "-Bsymbolic", "-lcudart"], objs, verbose)
    return CORE_SO


def build_torch_ops(verbose: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    build_core(verbose)
    src = CSRC / "torch_ext.cpp"
    obj = BUILD / "torch_ext.o"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = [f"-I{p}" for p in cpp_extension.include_paths()] + [f"-I{INCLUDE}", f"-I{CUDA_HOME / 'include'}"]
    _make(obj, [CXX, "-std=c++17", "-O2", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
                "-DTORCH_API_INCLUDE_EXTENSION_H", "-c", str(src), "-o", str(obj), *incs], [src, *_headers()], verbose)
    libdirs = [f"-L{p}" for p in cpp_extension.library_paths()]
    _make(TORCH_SO, [CXX, "-shared", "-o", str(TORCH_SO), str(obj), *libdirs, f"-L{PKG}", "-lzcutlass",
                     "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
                     f"-L{CUDA_HOME / 'lib64'}", "-lcudart", "-Wl,-rpath,$ORIGIN"], [obj, CORE_SO], verbose)
    return TORCH_SO


def build_bench(verbose: bool = False) -> Path:
    """zcutlass_b200/zcutlass_bench: the native benchmark (cuBLAS as comparator)."""
    build_core(verbose)
    src = CSRC / "bin" / "bench_gemm.cpp"
    _make(BENCH_BIN, [CXX, "-std=c++17", "-O2", "-o", str(BENCH_BIN), str(src), f"-I{INCLUDE}",
                      f"-I{CUDA_HOME / 'include'}", f"-L{PKG}", "-lzcutlass", f"-L{CUDA_HOME / 'lib64'}",
                      "-lcublas", "-lcudart", "-Wl,-rpath,$ORIGIN"], [src, CORE_SO, *_headers()], verbose)
    return BENCH_BIN


def build_oracle(ref_root: Path | None = None, verbose: bool = False) -> None:
    """Builds oracle/liboracle.so and, when `ref_root` (default: the
    ZCUTLASS_REF_ROOT environment variable) holds the reference's sources,
    oracle/_ref/libzcutlass_ref.so. Test infrastructure only: the library
    never loads either."""
    oracle = ROOT / "oracle"
    make = shutil.which("make")
    if make is None:
        raise RuntimeError("make is required to build the oracle")
    subprocess.run([make, "-s", "-C", str(oracle)], check=True)
    if ref_root is None and os.environ.get("ZCUTLASS_REF_ROOT"):
        ref_root = Path(os.environ["ZCUTLASS_REF_ROOT"])
    if ref_root is not None and (ref_root / "src" / "gemm.cu").exists():
        subprocess.run([make, "-s", "-C", str(oracle), "ref", f"REF_ROOT={ref_root}"], check=True)


def build_all(oracle: bool = True, verbose: bool = False, ref_root: Path | None = None) -> None:
    build_core(verbose)
    build_torch_ops(verbose)
    build_bench(verbose)
    if oracle:
        build_oracle(ref_root, verbose)


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--oracle", action="store_true", help="also build the test oracle")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args(argv)
    build_all(oracle=args.oracle, verbose=args.verbose)
    return 0


if __name__ == "__main__":
    sys.exit(main())
