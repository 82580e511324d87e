"""Build recipe for libamp_b200.so (sm_100a only).

Every ``csrc/*.cu`` file is compiled by nvcc for ``sm_100a`` into an object
under ``_build/`` and the objects are linked into ``amp_b200/libamp_b200.so``
(in-tree, so it travels with the working tree).  The CUDA runtime is linked
statically, so the library only needs the driver at run time and can be
``dlopen``-ed by AMP's ``amp_validate_kernel`` (which links no CUDA).

Usage: ``python -m amp_b200.build [-j N] [--force]``.
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
BUILD = ROOT / "_build"
LIB = PKG / "libamp_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-I", str(ROOT / "include"), "-I", str(CSRC),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libamp_b200.so")


def _deps() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted((ROOT / "include").glob("*.h"))


def _stale(out: Path, srcs: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(s.stat().st_mtime > t for s in srcs)


def _compile(src: Path, force: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if force or _stale(obj, [src] + _deps()):
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}\n{r.stdout}")
        if r.stderr.strip():
            sys.stderr.write(r.stderr)
    return obj


def build(jobs: int | None = None, force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    if not sources:
        raise RuntimeError("no CUDA sources found")
    jobs = jobs or min(len(sources), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), sources))
    if force or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        # Driver entry points (cuTensorMapEncodeTiled) are resolved at run time
        # through cudaGetDriverEntryPoint, so libcuda is not a link dependency.
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}\n{r.stdout}")
        os.replace(tmp, LIB)
    build_tools(force)
    check_dropins(force)
    if verbose:
        print(f"built {LIB}")
    return LIB


TOOLS = PKG / "tools"
DROPIN = PKG / "dropin"


def check_dropins(force: bool = False) -> None:
    """Compile the stand-alone kernel files under dropin/ for sm_100a (objects
    only, nothing links them): they are handed to AMP's scripts/amp_check.sh,
    which builds its own wrapper around them."""
    for src in sorted(DROPIN.glob("*.cu")):
        obj = BUILD / ("dropin_" + src.stem + ".o")
        if force or _stale(obj, [src]):
            cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-c", str(src),
                   "-o", str(obj)]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}")


def build_tools(force: bool = False) -> None:
    """Host C++ tools linked against the library (rpath: the package dir)."""
    out_dir = TOOLS / "bin"
    out_dir.mkdir(exist_ok=True)
    for src in sorted(TOOLS.glob("*.cpp")):
        exe = out_dir / ("amp_b200_" + src.stem)
        if force or _stale(exe, [src, LIB] + _deps()):
            cmd = [nvcc(), "-O2", "-std=c++17", "-x", "cu", *ARCH, "-I", str(ROOT / "include"),
                   str(src), "-o", str(exe), "-L", str(PKG), "-lamp_b200",
                   "-Xlinker", "-rpath=$ORIGIN/../.."]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"tool build failed for {src.name}:\n{r.stderr}")


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    build(a.j, a.force, verbose=True)


if __name__ == "__main__":
    main()
