"""Compiles oracle/tcmodel.c into oracle/libqbmodel.so (test infrastructure).

gcc with -ffp-contract=off, so every fp32 operation rounds where the source
says and fmaf() is the only fused multiply-add.
"""

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "tcmodel.c"
LIBRARY = HERE / "libqbmodel.so"


def build(force: bool = False) -> Path:
    if not force and LIBRARY.exists() and LIBRARY.stat().st_mtime >= SOURCE.stat().st_mtime:
        return LIBRARY
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = ["gcc", "-O3", "-ffp-contract=off", "-fno-math-errno", "-fopenmp", "-shared",
           "-fPIC", "-o", str(tmp), str(SOURCE), "-lm"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"gcc failed on tcmodel.c:\n{proc.stderr}")
    tmp.replace(LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force=True))
