"""Build libleanb200.so in-tree with nvcc for sm_100a.

``python -m leanstack_b200.build [--force] [--verbose] [--profiling]`` compiles
every ``csrc/*.cu`` into ``leanstack_b200/_lib/libleanb200.so``.
``--profiling`` defines ``LEANB200_PROFILING``, which adds the measurement
hooks (per-CTA timestamp buffers, the NVLink ping-pong probe) to the library;
the default build has none of them.  The library links
the shared CUDA runtime (``libcudart.so.12``), so inside a PyTorch process it
binds to the runtime PyTorch already loaded and sees the same current device
and streams.  No GPU is needed to build.
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
INCLUDE = PKG.parent / "include"
OUT_DIR = PKG / "_lib"
LIB = OUT_DIR / "libleanb200.so"
OBJ_DIR = PKG / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
              "--expt-relaxed-constexpr", "-cudart", "shared"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put /usr/local/cuda/bin on PATH")


def cuda_home() -> Path:
    return Path(nvcc_path()).resolve().parent.parent


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


STAMP = OUT_DIR / "build_flags.txt"


def _compile(src: Path, verbose: bool, ptxas_verbose: bool, defines: list[str]) -> tuple[Path, str]:
    obj = OBJ_DIR / (src.stem + ".o")
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, *defines, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src),
           "-o", str(obj)]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def needs_build(defines: list[str] | None = None) -> bool:
    if not LIB.exists():
        return True
    if not STAMP.exists() or STAMP.read_text().split() != (defines or []):
        return True
    lib_mtime = LIB.stat().st_mtime
    return any(p.stat().st_mtime > lib_mtime for p in [*sources(), *_deps(), Path(__file__)])


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False, profiling: bool = False) -> Path:
    defines = ["-DLEANB200_PROFILING"] if profiling else []
    if not force and not needs_build(defines):
        return LIB
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    for stale in OBJ_DIR.glob("*.o"):  # objects of sources that no longer exist must not be linked
        if not (CSRC / (stale.stem + ".cu")).exists():
            stale.unlink()
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose, ptxas_verbose, defines), srcs))
    if ptxas_verbose:
        for _, log in results:
            if log.strip():
                print(log)
    tmp = LIB.with_suffix(".so.tmp")
    lib64 = cuda_home() / "lib64"
    cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-cudart", "shared", "-o", str(tmp), *[str(o) for o, _ in results],
           "-L", str(lib64), "-Xlinker", f"-rpath,{lib64}"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    STAMP.write_text(" ".join(defines) + "\n")
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers / spills per kernel")
    ap.add_argument("--profiling", action="store_true", help="add the measurement hooks (LEANB200_PROFILING)")
    args = ap.parse_args(argv)
    lib = build(force=args.force, verbose=args.verbose, ptxas_verbose=args.ptxas_verbose, profiling=args.profiling)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
