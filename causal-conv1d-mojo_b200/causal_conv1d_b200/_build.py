"""Ahead-of-time build of libcc1d_sm100.so (the C ABI in include/cc1d.h).

Compiles every CUDA source under ``csrc/`` for sm_100a with nvcc and links
them into ``libcc1d_sm100.so`` next to this file.  The CUDA runtime is linked
statically, so the library only needs the NVIDIA driver at run time and can
be loaded (for symbol checks) on a machine without a GPU.

Run ``python -m causal_conv1d_b200._build`` (with the project directory on
``sys.path``) or call :func:`build`.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
PROJECT_DIR = PKG_DIR.parent
CSRC_DIR = PROJECT_DIR / "csrc"
INCLUDE_DIR = PROJECT_DIR.parent / "include"
BUILD_DIR = PROJECT_DIR / "_build"
LIB_NAME = "libcc1d_sm100.so"
LIB_PATH = PKG_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden,-O3",
    "-Xptxas",
    "-O3",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    if cand.is_file():
        return str(cand)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cuh")) + sorted(CSRC_DIR.glob("*.h")) + sorted(INCLUDE_DIR.glob("*.h"))


def _compile(nvcc: str, src: Path, obj: Path, extra: list[str], verbose: bool) -> None:
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *extra, f"-I{INCLUDE_DIR}", f"-I{CSRC_DIR}", "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile (if stale) and link the library; returns its path."""
    extra = list(extra_flags or [])
    nvcc = _nvcc()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    srcs = sources()
    hdr_mtime = max((h.stat().st_mtime for h in _headers()), default=0.0)
    objs = []
    todo = []
    for s in srcs:
        o = BUILD_DIR / (s.stem + ".o")
        objs.append(o)
        if force or extra or not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, hdr_mtime):
            todo.append((s, o))
    if todo:
        workers = min(len(todo), os.cpu_count() or 1)
        with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, extra, verbose) for s, o in todo]
            for f in futs:
                f.result()
    newest_obj = max(o.stat().st_mtime for o in objs)
    if force or todo or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < newest_obj:
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB_PATH)
