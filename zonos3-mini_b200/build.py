"""Build recipe of the C-ABI library ``libzonos3_b200.so`` (all CUDA sources, sm_100a only).

Each ``csrc/*.cu`` compiles to ``_build/<name>.o`` with ``nvcc -gencode arch=compute_100a,code=sm_100a`` and the
objects link into one shared library next to this file. A source recompiles when it or any ``csrc`` header is newer
than its object. nvcc cross-compiles, so this runs on a machine without a GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIBRARY = PKG / "libzonos3_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
]


def nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the zonos3-mini B200 kernels need the CUDA 12.9 toolchain")


def _stale(src: Path, obj: Path, headers: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in headers)


def build(verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile every CUDA source and link the shared library; returns its path."""
    compiler = nvcc()
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h"))
    flags = CFLAGS + list(extra_flags or [])

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        if _stale(src, obj, headers):
            cmd = [compiler, *ARCH, *flags, f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            res = subprocess.run(cmd, capture_output=True, text=True)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
            if verbose and res.stderr:
                print(res.stderr, file=sys.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objects = list(pool.map(compile_one, sources))
    newest = max(o.stat().st_mtime for o in objects)
    if not LIBRARY.exists() or LIBRARY.stat().st_mtime < newest:
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [compiler, *ARCH, "-shared", "-o", str(tmp), *map(str, objects)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
