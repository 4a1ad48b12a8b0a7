"""Build recipe for the backend's shared library.

Compiles every ``csrc/*.cu`` for sm_100a (B200) with nvcc and links them into
``yumelayers_b200/libyumecuda.so`` next to this file, so the library travels
with the source tree.  Incremental: a translation unit is rebuilt when it or
any header under ``csrc/`` or ``include/`` is newer than its object file.

    python -m yumelayers_b200.build          # build (or refresh) the library
"""
from __future__ import annotations

import concurrent.futures as cf
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
LIB = PKG / "libyumecuda.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
              "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build")


def _nccl_flags() -> list[str]:
    """Header and library location of NCCL (the system package)."""
    inc = [p for p in ("/usr/include",) if Path(p, "nccl.h").exists()]
    return [f"-I{p}" for p in inc]


def _newest_header() -> float:
    hs = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, obj: Path) -> tuple[Path, str]:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", *_nccl_flags(),
           "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(verbose: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    if not srcs:
        raise RuntimeError(f"no CUDA sources under {CSRC}")
    hdr = _newest_header()
    jobs = []
    for s in srcs:
        o = BUILD / (s.stem + ".o")
        if force or not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, hdr):
            jobs.append((s, o))
    logs = []
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
            for obj, log in ex.map(lambda a: _compile(*a), jobs):
                logs.append((obj, log))
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    newest_obj = max(o.stat().st_mtime for o in objs)
    if force or jobs or not LIB.exists() or LIB.stat().st_mtime < newest_obj:
        tmp = LIB.with_suffix(".so.tmp")
        # cudart is linked statically so the library does not depend on which
        # libcudart.so (torch's or the toolkit's) the process loaded first.
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs),
               "-lnccl", "-Xlinker", "-rpath,$ORIGIN"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        for obj, log in logs:
            keep = [ln for ln in log.splitlines()
                    if "registers" in ln or "spill" in ln or "error" in ln.lower()]
            print(f"[{obj.name}]", *keep, sep="\n  ")
    return LIB


if __name__ == "__main__":
    out = build(verbose="-v" in sys.argv, force="--force" in sys.argv)
    print(out)
