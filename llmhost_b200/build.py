"""Build libllmhost_kv.so (the sm_100a kernels + C ABI) in-tree with nvcc.

The library is plain nvcc output: every ``csrc/*.cu`` file is compiled for
``-gencode arch=compute_100a,code=sm_100a`` and linked with the static CUDA
runtime into ``llmhost_b200/_lib/libllmhost_kv.so``.  No torch extension
machinery is involved, so the same .so is what a Rust ``build.rs`` would link.

    python -m llmhost_b200.build [--force] [--ptxas-verbose]
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
BUILD_DIR = PKG / "_build"
LIB_DIR = PKG / "_lib"
LIB_PATH = LIB_DIR / "libllmhost_kv.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3",
              "--expt-relaxed-constexpr", "-I", str(ROOT / "include")]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build llmhost_b200")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def _deps_mtime() -> float:
    files = list(CSRC.glob("*")) + list((ROOT / "include").glob("*.h")) + [Path(__file__)]
    return max(f.stat().st_mtime for f in files if f.is_file())


def _compile(src: Path, ptxas_verbose: bool) -> tuple[Path, str]:
    obj = BUILD_DIR / (src.stem + src.suffix.replace(".", "_") + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = True) -> Path:
    """Compile and link the library if any source is newer than it."""
    if not force and LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= _deps_mtime():
        return LIB_PATH
    BUILD_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, ptxas_verbose), srcs))
    if ptxas_verbose or not quiet:
        for _, log in results:
            if log.strip():
                print(log, file=sys.stderr)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *[str(o) for o, _ in results]]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args()
    path = build(force=args.force or args.ptxas_verbose, ptxas_verbose=args.ptxas_verbose, quiet=False)
    print(path)


if __name__ == "__main__":
    main()
