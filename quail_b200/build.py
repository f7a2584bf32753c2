"""Builds libquailb200.so, the sm_100a kernel library, in-tree.

Each ``csrc/*.cu`` compiles to an object with nvcc for ``sm_100a`` only,
and the objects link into ``quail_b200/libquailb200.so`` with the CUDA
runtime linked statically, so the library carries no dependency on the
runtime version torch bundles. Run as ``python -m quail_b200.build``.
"""

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
INCLUDE = PACKAGE.parent / "include"
LIBRARY = PACKAGE / "libquailb200.so"
BUILD_DIR = PACKAGE.parent / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
                "-Xcompiler", "-fPIC", "-I", str(INCLUDE)]


def nvcc() -> str:
    """Path of nvcc: CUDA_HOME first, then PATH, then /usr/local/cuda."""
    home = os.environ.get("CUDA_HOME")
    if home and (Path(home) / "bin" / "nvcc").exists():
        return str(Path(home) / "bin" / "nvcc")
    found = shutil.which("nvcc")
    if found:
        return found
    return "/usr/local/cuda/bin/nvcc"


def sources() -> list:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _compile(src: Path, verbose_ptxas: bool) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    headers = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    if not _stale(obj, [src, *headers]) and not verbose_ptxas:
        return obj
    cmd = [nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{proc.stdout}\n{proc.stderr}")
    if verbose_ptxas:
        sys.stderr.write(proc.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> Path:
    """Compile every kernel source and link the shared library.

    Returns:
        The path of libquailb200.so.
    """
    BUILD_DIR.mkdir(exist_ok=True)
    srcs = sources()
    if force:
        for obj in BUILD_DIR.glob("*.o"):
            obj.unlink()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as pool:
        objs = list(pool.map(lambda s: _compile(s, verbose_ptxas), srcs))
    if force or _stale(LIBRARY, objs):
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp),
               *map(str, objs), "-lcuda" if False else "-ldl"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
        os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv)
    print(path)
