"""Build ``libldb200.so`` from ``csrc/*.cu`` with nvcc for sm_100a, in-tree.

Each translation unit is compiled in parallel to an object file under
``_build/`` and linked into ``lesiondiffusion_mlx_b200/libldb200.so``.  A unit
is rebuilt only when it or a header under ``csrc/`` or ``include/`` changed.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIBRARY = PACKAGE / "libldb200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-diag-suppress=177",
]


def nvcc() -> str:
    """Path of nvcc (CUDA_HOME, then PATH, then /usr/local/cuda)."""
    for candidate in (
        os.environ.get("CUDA_HOME", "") + "/bin/nvcc",
        shutil.which("nvcc") or "",
        "/usr/local/cuda/bin/nvcc",
    ):
        if candidate and Path(candidate).is_file():
            return candidate
    raise RuntimeError("nvcc not found; set CUDA_HOME")


def _headers_mtime() -> float:
    paths = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((p.stat().st_mtime for p in paths), default=0.0)


def _compile(source: Path, obj: Path, extra: list[str]) -> None:
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(source), "-o", str(obj)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed for {source.name}:\n{result.stdout}\n{result.stderr}")


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile every ``csrc/*.cu`` and link the shared library; return its path."""
    extra = list(extra_flags or [])
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    header_time = _headers_mtime()
    jobs = []
    for source in sources:
        obj = BUILD / (source.stem + ".o")
        stale = force or not obj.exists() or obj.stat().st_mtime < max(source.stat().st_mtime, header_time)
        if stale:
            jobs.append((source, obj))
    if jobs:
        workers = min(len(jobs), os.cpu_count() or 4)
        with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as pool:
            futures = {pool.submit(_compile, s, o, extra): s for s, o in jobs}
            for future in concurrent.futures.as_completed(futures):
                future.result()
                if verbose:
                    print(f"compiled {futures[future].name}", file=sys.stderr)
    objects = [BUILD / (s.stem + ".o") for s in sources]
    newest = max(o.stat().st_mtime for o in objects)
    if force or jobs or not LIBRARY.exists() or LIBRARY.stat().st_mtime < newest:
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", *map(str, objects), "-o", str(tmp),
               "-cudart", "static"]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"link failed:\n{result.stdout}\n{result.stderr}")
        os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
