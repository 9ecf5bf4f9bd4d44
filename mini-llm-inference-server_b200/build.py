"""Build the sm_100a shared library `_mlb_paged_kv.so` in-tree with nvcc (no torch headers needed).

    python mini-llm-inference-server_b200/build.py [--force] [--verbose]

Each `csrc/*.cu` is compiled in parallel to an object under `_build/`, then linked with
`-shared` (cudart linked statically, so the library needs only the CUDA driver at run time).
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
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
BUILD = REPO / "_build"
LIB = PKG / "_mlb_paged_kv.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    deps = sources() + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return LIB.stat().st_mtime >= max(p.stat().st_mtime for p in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, flush=True)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    if not force and up_to_date():
        return LIB
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    extra = extra or []
    objs = [BUILD / (src.stem + ".o") for src in sources()]
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(objs), os.cpu_count() or 1))) as ex:
        futs = [ex.submit(_run, [cc, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)], verbose)
                for src, obj in zip(sources(), objs)]
        for f in futs:
            f.result()
    tmp = LIB.with_suffix(".so.tmp")
    _run([cc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs)], verbose)
    os.replace(tmp, LIB)  # atomic: a process that already mapped the old file keeps it
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register / shared-memory use per kernel")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_v else []
    print(build(force=args.force or args.ptxas_v, verbose=args.verbose or args.ptxas_v, extra=extra))


if __name__ == "__main__":
    sys.exit(main())
