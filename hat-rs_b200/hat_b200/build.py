"""Build `libhat_b200.so` in-tree from `hat-rs_b200/csrc` with nvcc for sm_100a.

    python -m hat_b200.build        (from hat-rs_b200/)   or   build.build()

Objects go to `hat-rs_b200/_build/`; a source is recompiled when it or any header in
csrc/ or include/ is newer than its object. The CUDA runtime is linked statically, so
the library needs only the driver at run time.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
SRC = PKG.parent / "csrc"
INC = PKG.parent.parent / "include"
OUT_DIR = PKG.parent / "_build"
LIB = PKG / "libhat_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", str(INC), "-I", str(SRC)]


def _nccl_dirs():
    """nccl.h and libnccl.so.2 of the NCCL wheel torch uses (strip sharding binds NCCL at
    run time; the header gives the types, the path is the last place it looks)."""
    try:
        import nvidia.nccl as nc
        root = Path(list(nc.__path__)[0])
    except Exception:
        root = Path("/usr")
    return root / "include", root / "lib" / "libnccl.so.2"


_NCCL_INC, _NCCL_LIB = _nccl_dirs()
FLAGS += ["-I", str(_NCCL_INC), f'-DHAT_NCCL_LIB="{_NCCL_LIB}"']


def _sources():
    return sorted([p for p in SRC.iterdir() if p.suffix in (".cu", ".cpp")])


def _headers_mtime():
    hs = [p for p in SRC.iterdir() if p.suffix in (".h", ".cuh")] + list(INC.glob("*.h"))
    return max((p.stat().st_mtime for p in hs), default=0.0)


def _compile(src: Path, verbose: bool) -> Path:
    obj = OUT_DIR / (src.name + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime()):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [NVCC, *FLAGS, "-x", "c++", "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr.strip():
        print(r.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    """Compile every source in csrc/ and link the shared library; returns its path."""
    OUT_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if LIB.exists() and LIB.stat().st_mtime >= newest:
        return LIB
    cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-cudart", "static", "-ldl", "-lz"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
