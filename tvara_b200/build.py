"""In-tree build of libtvara_capi.so for sm_100a.

    python -m tvara_b200.build [--force]

Every .cu/.cpp under csrc/ is compiled by nvcc (host compiler /usr/bin/g++)
with ``-gencode arch=compute_100a,code=sm_100a`` into _build/, then linked
into tvara_b200/libtvara_capi.so with the CUDA runtime linked statically.
Objects are rebuilt only when a source or header is newer.
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
BUILD = PKG / "_build"
LIB = PKG / "libtvara_capi.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
HOST_CXX = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise FileNotFoundError("nvcc not found")


def flags() -> list[str]:
    return ARCH + [
        "-O3", "-lineinfo", "-std=c++20", "--expt-relaxed-constexpr", "-ccbin", HOST_CXX,
        "-Xcompiler", "-fPIC,-fvisibility=hidden,-O2", "-I", str(CSRC), "-I", str(INCLUDE),
        "-Xptxas", "-warn-spills",
    ]


def _compile(src: Path, obj: Path, extra: list[str]) -> tuple[Path, str]:
    cmd = [nvcc(), *flags(), *extra, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted([*CSRC.glob("*.cu"), *CSRC.glob("*.cpp")])
    headers = [*CSRC.glob("*.hpp"), *CSRC.glob("*.cuh"), *INCLUDE.glob("*.h")]
    newest_header = max((h.stat().st_mtime for h in headers), default=0)
    jobs = []
    for src in sources:
        obj = BUILD / (src.name + ".o")
        stale = force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header)
        jobs.append((src, obj, stale))
    todo = [(s, o) for s, o, stale in jobs if stale]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as ex:
            for obj, log in ex.map(lambda so: _compile(*so, extra or []), todo):
                if verbose and log.strip():
                    print(log, file=sys.stderr)
    objs = [o for _, o, _ in jobs]
    if todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-ccbin", HOST_CXX, "-o", str(LIB), *map(str, objs),
               "-cudart", "static", "-ldl", "-lpthread", "-lrt", "-Xlinker", "--exclude-libs,ALL"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
