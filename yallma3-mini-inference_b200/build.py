"""Builds libyallma3_b200.so in-tree for sm_100a.

Every .cu/.cpp under csrc/ is compiled by nvcc with
`-gencode arch=compute_100a,code=sm_100a -lineinfo` into _build/ and linked
into this package directory, so the library travels with the source tree.
Rebuilds only objects whose sources or headers changed.

    python build.py            # build
    python build.py --clean    # remove objects and the library
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libyallma3_b200.so"
INCLUDE = PKG.parent / "include"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-ccbin", "/usr/bin/g++",
          f"-I{INCLUDE}", "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]
# host code rounds every f32 operation on its own (no contraction into fused multiply-adds)
HOST_FLAGS = ["-Xcompiler", "-ffp-contract=off"]


def sources() -> list[Path]:
    return sorted(list(CSRC.rglob("*.cu")) + list(CSRC.rglob("*.cpp")))


def headers() -> list[Path]:
    return sorted(list(CSRC.rglob("*.h")) + list(CSRC.rglob("*.cuh")) + list(INCLUDE.glob("*.h")))


def _obj(src: Path) -> Path:
    rel = src.relative_to(CSRC).with_suffix(".o")
    return BUILD / str(rel).replace(os.sep, "__")


def _extra() -> list[str]:
    """YL_WITH_TRACE=1 in the environment builds the diagnostics variant whose
    decode kernels stamp a timeline (yl_trace_decode_step); the default build
    compiles those stamps out."""
    return ["-DYL_WITH_TRACE=1"] if os.environ.get("YL_WITH_TRACE", "0") == "1" else []


def _compile(src: Path) -> tuple[Path, str]:
    obj = _obj(src)
    cmd = [NVCC, *ARCH, *COMMON, *_extra(), "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [NVCC, *COMMON, *HOST_FLAGS, *_extra(), "-Wno-deprecated-gpu-targets", "-x", "c++", "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src}\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    newest_header = max((h.stat().st_mtime for h in headers()), default=0.0)
    # objects built with other flags (trace on/off) are all stale
    stamp = BUILD / "flags.txt"
    flags = " ".join(_extra())
    same_flags = stamp.exists() and stamp.read_text() == flags
    stale = [s for s in srcs
             if not same_flags or not _obj(s).exists()
             or _obj(s).stat().st_mtime < max(s.stat().st_mtime, newest_header)]
    if stamp.exists() and not same_flags:
        stamp.unlink()  # written again only once every object carries the new flags
    if stale:
        jobs = jobs or min(len(stale), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            for obj, log in ex.map(_compile, stale):
                if verbose and log.strip():
                    print(log)
    stamp.write_text(flags)
    objs = [_obj(s) for s in srcs]
    if stale or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs),
               "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def clean() -> None:
    shutil.rmtree(BUILD, ignore_errors=True)
    if LIB.exists():
        LIB.unlink()


if __name__ == "__main__":
    if "--clean" in sys.argv:
        clean()
    else:
        print(build(verbose="-v" in sys.argv))
