"""Builds libb200ops.so in-tree from csrc/*.cu for sm_100a.

Usage: python triton-agent_b200/build.py [--force] [--jobs N] [--verbose]

Every translation unit is compiled with
    nvcc -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo
into _build/, then linked into lib/libb200ops.so.  The CUDA runtime is linked
statically so the library does not depend on which libcudart the host
process has loaded; the driver API is reached through
cudaGetDriverEntryPoint, so there is no -lcuda either.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
CSRC = PKG_ROOT / "csrc"
BUILD = PKG_ROOT / "_build"
LIB_DIR = PKG_ROOT / "lib"
LIB = LIB_DIR / "libb200ops.so"
REPO_ROOT = PKG_ROOT.parent
INCLUDE = REPO_ROOT / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O3,-Wall,-Wno-unused-function",
    "-Xptxas=-warn-spills",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _deps_mtime() -> float:
    headers = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((p.stat().st_mtime for p in headers), default=0.0)


def _compile(src: Path, verbose: bool, extra: list[str]) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stderr


def needs_build() -> bool:
    if not LIB.exists():
        return True
    lib_t = LIB.stat().st_mtime
    srcs = list(CSRC.glob("*.cu"))
    newest = max([p.stat().st_mtime for p in srcs] + [_deps_mtime(), Path(__file__).stat().st_mtime])
    return newest > lib_t


def build(force: bool = False, jobs: int | None = None, verbose: bool = False,
          extra: list[str] | None = None) -> Path:
    """Compiles and links the library; returns its path."""
    extra = list(extra or [])
    if not force and not extra and not needs_build():
        return LIB
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    objs: list[Path] = []
    logs: list[str] = []
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        futs = [ex.submit(_compile, s, verbose, extra) for s in srcs]
        for f in futs:
            obj, log = f.result()
            objs.append(obj)
            if log.strip():
                logs.append(log)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, LIB)
    if verbose:
        sys.stderr.write("\n".join(logs))
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill report")
    args = ap.parse_args()
    path = build(force=args.force, jobs=args.jobs, verbose=args.verbose)
    print(path)


if __name__ == "__main__":
    main()
