"""Build the sm_100a CUDA library ``libiq36_b200.so`` in-tree with nvcc.

Every ``csrc/*.cu`` file is compiled for ``sm_100a`` only (no PTX fallback,
no other architecture) and linked into one shared library next to this file.
The C ABI it exports is declared in ``include/iq36_b200.h`` at the repository
root. Rebuilds only when a source or header is newer than the library.
"""

from __future__ import annotations

import concurrent.futures
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
LIB = PKG / "libiq36_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
    "--expt-relaxed-constexpr", f"-I{INCLUDE}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA library cannot be built")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return _sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _deps())


def _compile(src: Path, ptxas_verbose: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = True) -> Path:
    """Compile csrc/*.cu for sm_100a and link libiq36_b200.so; return its path."""
    if not force and not needs_build():
        return LIB
    BUILD.mkdir(exist_ok=True)
    srcs = _sources()
    workers = min(len(srcs), os.cpu_count() or 4)
    logs = []
    with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as ex:
        results = list(ex.map(lambda s: _compile(s, ptxas_verbose), srcs))
    objs = [o for o, _ in results]
    logs = [log for _, log in results]
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    if not quiet or ptxas_verbose:
        for log in logs:
            if log.strip():
                print(log, file=sys.stderr)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, ptxas_verbose="-v" in sys.argv, quiet=False)
    print(LIB)
