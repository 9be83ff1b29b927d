"""Build the CUDA extension ``heimdall_b200/lib/libbifrost_b200.so`` in-tree with nvcc (sm_100a).

    python -m heimdall_b200.build [--force] [--debug]

Each ``csrc/*.cu`` is compiled to an object under ``heimdall_b200/_build/`` (rebuilt when the
source or any header is newer), then linked into one shared library with a plain C ABI
(``include/bifrost_b200.h``).  No torch headers are involved: the library only needs the CUDA
runtime and driver.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lib" / "libbifrost_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def _flags(debug: bool) -> list:
    f = ARCH + ["-std=c++17", "-Xcompiler", "-fPIC", "-lineinfo", f"-I{ROOT / 'include'}", "-Xptxas", "-v",
                "--expt-relaxed-constexpr", "-diag-suppress", "177"]
    f += ["-O0", "-G"] if debug else ["-O3"]
    return f


def _stale(src: Path, obj: Path, headers: list) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in headers)


def build(force: bool = False, debug: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    srcs = sorted(CSRC.glob("*.cu"))
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    todo = [(s, o) for s, o in zip(srcs, objs) if force or _stale(s, o, headers)]
    cc = nvcc()

    def compile_one(so):
        s, o = so
        cmd = [cc, *_flags(debug), "-c", str(s), "-o", str(o)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        log = BUILD / (s.stem + ".log")
        log.write_text(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {s.name}:\n{r.stderr[-6000:]}")
        return s.name

    if todo:
        with ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            for name in ex.map(compile_one, todo):
                if verbose:
                    print("compiled", name)
    if todo or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [cc, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr[-4000:]}")
        if verbose:
            print("linked", LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug", action="store_true")
    a = ap.parse_args(argv)
    print(build(force=a.force, debug=a.debug, verbose=True))


if __name__ == "__main__":
    sys.exit(main())
