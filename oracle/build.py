"""Build the CPU oracle library (test infrastructure; see bnbq_oracle.c).

Picks a C compiler that accepts -fopenmp; without one, builds single-threaded.
Output: oracle/liboracle_bnbq.so (git-ignored; travels with the tree).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "bnbq_oracle.c"
OUT = HERE / "liboracle_bnbq.so"
BASE_FLAGS = ["-O2", "-std=gnu11", "-fPIC", "-ffp-contract=off", "-fno-fast-math",
              "-mno-fma", "-Wall", "-Wextra", "-shared"]


def _accepts_openmp(cc: str) -> bool:
    with tempfile.TemporaryDirectory() as d:
        src = Path(d) / "t.c"
        src.write_text("#include <omp.h>\nint main(void){return omp_get_max_threads() < 0;}\n")
        r = subprocess.run([cc, "-fopenmp", str(src), "-o", str(Path(d) / "t")],
                           capture_output=True)
        return r.returncode == 0


def build(force: bool = False) -> Path:
    if OUT.exists() and not force and OUT.stat().st_mtime >= SRC.stat().st_mtime:
        return OUT
    candidates = [os.environ.get("OMPCC"), "/usr/bin/gcc", shutil.which("gcc"),
                  os.environ.get("CC"), shutil.which("cc")]
    cc, omp = None, False
    for c in candidates:
        if c and Path(c).exists() and _accepts_openmp(c):
            cc, omp = c, True
            break
    if cc is None:
        cc = next(c for c in candidates if c and Path(c).exists())
    flags = BASE_FLAGS + (["-fopenmp"] if omp else [])
    tmp = OUT.with_suffix(".so.tmp")
    subprocess.run([cc, *flags, "-o", str(tmp), str(SRC), "-lm"], check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force=True))
