"""Build ``libtokquay_b200.so`` in-tree with nvcc for sm_100a.

    python -m tokquay_b200.build            # rebuild if a source changed
    python -m tokquay_b200.build --force    # rebuild unconditionally

The library is one CUDA translation unit (``csrc/capi.cu`` includes every
kernel header) plus the host-side planner (``csrc/plan.cpp``).  CUDA's runtime
is linked statically, so the built ``.so`` needs only the driver on the box it
is copied to.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB_NAME = "libtokquay_b200.so"
LIB_PATH = PKG / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-shared",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-cudart", "static",
]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def _inputs() -> list[Path]:
    return sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build libtokquay_b200.so")


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > built for p in _inputs())


def build_library(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None,
                  out: Path | None = None) -> Path:  # fmt: skip
    """Compile the library if it is missing or older than a source; return its path.
    ``out`` builds a variant elsewhere (e.g. with ``-DTQ_ATTN_STAGES=2`` in
    ``extra_flags``) without touching the in-tree library."""
    target = Path(out) if out else LIB_PATH
    if out is None and not force and not is_stale():
        return LIB_PATH
    tmp = target.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, *(extra_flags or []), f"-I{INCLUDE}",
           *map(str, sources()), "-o", str(tmp)]  # fmt: skip
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, file=sys.stderr)
    os.replace(tmp, target)
    return target


HOSTPACK_SRC = CSRC / "hostpack.c"


def hostpack_path() -> Path:
    import sysconfig

    return PKG / ("_hostpack" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_hostpack(force: bool = False, verbose: bool = False) -> Path:
    """Compile the ``_hostpack`` CPython extension (plain C, gcc) in-tree."""
    import sysconfig

    out = hostpack_path()
    if not force and out.exists() and out.stat().st_mtime >= HOSTPACK_SRC.stat().st_mtime:
        return out
    cc = os.environ.get("CC") or shutil.which("gcc") or "cc"
    tmp = out.with_name(out.name + ".tmp")
    cmd = [cc, "-O2", "-shared", "-fPIC", "-Wall", f"-I{sysconfig.get_paths()['include']}",
           str(HOSTPACK_SRC), "-o", str(tmp)]  # fmt: skip
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"{cc} failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, out)
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills per kernel")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_info else None
    path = build_library(force=args.force or args.ptxas_info, verbose=True, extra_flags=extra)
    print(path)
    print(build_hostpack(force=args.force, verbose=True))


if __name__ == "__main__":
    main()
