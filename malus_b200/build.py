"""Build libmalus_runtime_cuda.so in-tree for sm_100a (B200).

Every .cu under malus_b200/csrc is compiled with nvcc for
`-gencode arch=compute_100a,code=sm_100a` (object files under
malus_b200/_build, rebuilt only when a source or header is newer), then
linked into malus_b200/libmalus_runtime_cuda.so against NCCL.  No GPU is
needed: nvcc cross-compiles.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libmalus_runtime_cuda.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wno-unused-function",
          "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}"]


def _nccl_dir() -> Path | None:
    """The NCCL that torch itself loads (the nvidia-nccl wheel), so that this
    library and torch share one libnccl.so.2 whichever is loaded first."""
    try:
        import importlib.util
        spec = importlib.util.find_spec("nvidia")
        for base in (spec.submodule_search_locations if spec else []):
            d = Path(base) / "nccl"
            if (d / "lib" / "libnccl.so.2").exists() and (d / "include" / "nccl.h").exists():
                return d
    except Exception:
        pass
    return None


NCCL = _nccl_dir()
if NCCL is not None:
    CFLAGS.append(f"-I{NCCL / 'include'}")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _needs(obj: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


# HBM-bound kernels keep the reference's separate multiply/add rounding
# (no FMA contraction); it costs nothing when bandwidth is the bound.
NO_FMAD = {"elementwise", "rows", "reduce"}


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if _needs(obj, [src] + _headers() + [Path(__file__)]):
        extra = ["-fmad=false"] if src.stem in NO_FMAD else []
        cmd = [NVCC, *ARCH, *CFLAGS, *extra, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip() and verbose:
            print(r.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if _needs(LIB, objs + [Path(__file__)]):
        if NCCL is not None:
            nccl = [f"-L{NCCL / 'lib'}", "-l:libnccl.so.2", "-Xlinker", f"-rpath={NCCL / 'lib'}"]
        else:
            nccl = ["-lnccl"]
        cuda_lib = Path(NVCC).resolve().parent.parent / "lib64"
        nvrtc = [f"-L{cuda_lib}", "-lnvrtc", "-Xlinker", f"-rpath={cuda_lib}"]
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), *nccl, *nvrtc]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
