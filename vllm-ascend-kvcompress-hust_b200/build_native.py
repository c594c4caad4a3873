"""Build libkvc_b200.so (sm_100a) in-tree with nvcc.

    python build_native.py [--jobs N] [--force]

Each ``csrc/*.cu`` is compiled to an object in ``_build/`` (in parallel, only
when the source or a header changed), then linked into
``vllm_ascend_kvcompress/_native/libkvc_b200.so`` with the CUDA runtime linked
statically, so the library needs only the NVIDIA driver at run time.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
OUT = HERE / "vllm_ascend_kvcompress" / "_native" / "libkvc_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         f"-I{REPO / 'include'}", f"-I{CSRC}"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the sm_100a library cannot be built")
    return cand


def _stale(src: Path, obj: Path, headers: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in headers)


def build(jobs: int | None = None, force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    OUT.parent.mkdir(parents=True, exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted((REPO / "include").glob("*.h"))
    sources = sorted(CSRC.glob("*.cu"))
    objs = [BUILD / (s.stem + ".o") for s in sources]
    todo = [(s, o) for s, o in zip(sources, objs) if force or _stale(s, o, headers)]
    cc = nvcc()

    def compile_one(pair):
        src, obj = pair
        cmd = [cc, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}")
        if verbose and r.stderr:
            print(r.stderr, file=sys.stderr)
        return src.name

    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        list(ex.map(compile_one, todo))
    if todo or not OUT.exists() or any(o.stat().st_mtime > OUT.stat().st_mtime for o in objs):
        tmp = OUT.with_suffix(".so.tmp")
        cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
        os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(args.jobs, args.force, args.verbose))
