"""Build libbnbq.so, the sm_100a kernels behind include/bnbq.h.

    python bitsandbytes-jax_b200/build.py [--force] [-j N]

Each csrc/*.cu is compiled with nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a), with the CUDA runtime linked
statically, then linked into bnb_b200/libbnbq.so next to the Python package
that loads it. Nothing is built at import time and there is no JIT cache:
the .so travels with the source tree. Without --force, sources older than the
library are not rebuilt.

csrc/ffi_xla.cc (the XLA FFI handlers) is compiled into
bnb_b200/libbnbq_xla.so only where jaxlib's FFI headers are found
(jax.ffi.include_dir(), or BNBQ_XLA_FFI_INCLUDE); otherwise it is skipped
(XLA_FFI_STATUS records why).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OUT = HERE / "bnb_b200" / "libbnbq.so"
OUT_XLA = HERE / "bnb_b200" / "libbnbq_xla.so"
BUILD = HERE / "_build"
XLA_FFI_STATUS = "not attempted"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    f"-I{INCLUDE}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return _sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _deps())


def build(force: bool = False, jobs: int = 0, verbose_ptxas: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        cmd = [cc, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose_ptxas:
            print(r.stderr)
        return obj

    jobs = jobs or min(8, os.cpu_count() or 1)
    with ThreadPoolExecutor(jobs) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [cc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "--cudart", "static",
           *map(str, objs), "-o", str(tmp)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, OUT)
    return OUT


def xla_ffi_include() -> Path | None:
    """jaxlib's FFI header root (the directory holding xla/ffi/api/ffi.h)."""
    env = os.environ.get("BNBQ_XLA_FFI_INCLUDE")
    cands = [Path(env)] if env else []
    try:
        import jax.ffi  # noqa: PLC0415 -- optional
        cands.append(Path(jax.ffi.include_dir()))
    except Exception:  # jax absent (as on the development image) or too old
        pass
    for c in cands:
        if (c / "xla" / "ffi" / "api" / "ffi.h").is_file():
            return c
    return None


def build_xla_ffi() -> Path | None:
    """libbnbq_xla.so from csrc/ffi_xla.cc when jaxlib's FFI headers exist;
    None (and XLA_FFI_STATUS says why) otherwise."""
    global XLA_FFI_STATUS
    inc = xla_ffi_include()
    if inc is None:
        XLA_FFI_STATUS = "skipped: jaxlib's XLA FFI headers not found"
        return None
    cuda_inc = Path(nvcc()).resolve().parent.parent / "include"
    cmd = [os.environ.get("CXX", "g++"), "-std=c++17", "-O2", "-shared", "-fPIC", f"-I{INCLUDE}", f"-I{inc}",
           f"-I{cuda_inc}", str(CSRC / "ffi_xla.cc"), f"-L{OUT.parent}", "-lbnbq", "-Wl,-rpath,$ORIGIN",
           "-o", str(OUT_XLA)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"ffi_xla.cc failed to compile:\n{r.stdout}\n{r.stderr}")
    XLA_FFI_STATUS = f"built against {inc}"
    return OUT_XLA


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=0)
    ap.add_argument("--ptxas-v", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, jobs=args.j, verbose_ptxas=args.ptxas_v))
    build_xla_ffi()
    print("XLA FFI handlers:", XLA_FFI_STATUS)
