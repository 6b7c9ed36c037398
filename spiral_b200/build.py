"""Build libspiral_b200.so in-tree with nvcc for sm_100a.

Usage: python -m spiral_b200.build [--force] [--verbose]

Every .cu under csrc/ is compiled to an object in csrc/_build/ (in parallel)
and linked into spiral_b200/libspiral_b200.so.  The CUDA runtime is linked
statically so the library depends only on the driver; NCCL is linked
dynamically against the libnccl.so.2 that ships with the torch wheel (a torch
process has already loaded it, so both share one NCCL).
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
CSRC = PKG / "csrc"
BUILD = CSRC / "_build"
LIB = PKG / "libspiral_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-rdc=true",
    "-Xcompiler",
    "-fPIC,-O3,-fvisibility=hidden",
    "-I",
    str(INCLUDE),
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def nccl_dirs() -> tuple[Path | None, Path | None]:
    """Header and library directories of the NCCL that torch loads."""
    try:
        import nvidia.nccl  # type: ignore

        base = Path(list(nvidia.nccl.__path__)[0])
        inc, lib = base / "include", base / "lib"
        if (inc / "nccl.h").exists() and (lib / "libnccl.so.2").exists():
            return inc, lib
    except Exception:
        pass
    return None, None


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    nccl_inc, nccl_lib = nccl_dirs()
    extra = []
    defines = []
    if nccl_inc is not None:
        extra += ["-I", str(nccl_inc)]
        defines += ["-DSPIRAL_HAVE_NCCL=1"]
    objs = []
    jobs = []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers + [Path(__file__)]):
            cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, *defines, "-c", str(src), "-o", str(obj)]
            jobs.append((src, cmd))

    def run(job):
        src, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)
        return src

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            list(ex.map(run, jobs))
    if force or jobs or _stale(LIB, objs):
        link = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs)]
        if nccl_lib is not None:
            link += [f"-L{nccl_lib}", "-l:libnccl.so.2", f"-Xlinker=-rpath,{nccl_lib}"]
        if verbose:
            print(" ".join(link), flush=True)
        r = subprocess.run(link, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args(argv)
    lib = build(force=args.force, verbose=args.verbose)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
