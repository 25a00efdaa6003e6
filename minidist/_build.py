"""Build the native library ``minidist/_lib/libminidist_cuda.so`` from ``csrc/``.

Every ``csrc/*.cu`` / ``*.cpp`` file is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) into an object under
``minidist/_lib/obj`` and linked into one shared library with ``extern "C"``
entry points that :mod:`minidist.ops._native` loads through ctypes.  The CUDA
runtime is linked statically so the library does not depend on which
``libcudart`` PyTorch happens to ship; kernels, streams and device pointers are
shared with PyTorch through the driver's primary context.

Objects are rebuilt only when their source, a header in ``csrc/`` or the flags
change (tracked by a content hash next to each object), and compile jobs run in
parallel, so ``python -m minidist._build`` is cheap to re-run.
"""

from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "csrc"
LIBDIR = Path(__file__).resolve().parent / "_lib"
OBJDIR = LIBDIR / "obj"
LIBNAME = "libminidist_cuda.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-v",
    "-Wno-deprecated-gpu-targets",
    "-DNDEBUG",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")


def _headers_digest() -> str:
    h = hashlib.sha256()
    for p in sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    return h.hexdigest()


CHECKED_LIBNAME = "libminidist_cuda_checked.so"


def _compile_one(src: Path, flags: list[str], hdr_digest: str, verbose: bool,
                 objdir: Path = OBJDIR) -> tuple[Path, bool, str]:
    obj = objdir / (src.stem + ".o")
    stamp = objdir / (src.stem + ".hash")
    h = hashlib.sha256()
    h.update(src.read_bytes())
    h.update(hdr_digest.encode())
    h.update(" ".join(flags).encode())
    digest = h.hexdigest()
    if obj.exists() and stamp.exists() and stamp.read_text() == digest:
        return obj, False, ""
    cmd = [nvcc_path(), *ARCH_FLAGS, *flags, "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    log = proc.stdout + proc.stderr
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{log}")
    stamp.write_text(digest)
    (objdir / (src.stem + ".ptxas.txt")).write_text(log)
    if verbose:
        print(f"  compiled {src.name}")
    return obj, True, log


def build(verbose: bool = True, jobs: int | None = None, bounds_check: bool = False) -> Path:
    """Compile and link the native library; return its path.

    ``bounds_check=True`` builds the checking variant ``libminidist_cuda_checked.so``
    (``-DMD_BOUNDS_CHECK``: kernels verify data-dependent indices -- token ids, targets,
    table entries -- and on a violation record ``kBadArgument`` with the site and the bad
    value in the status word and skip the access, never trapping).  It is loaded instead
    of the normal library when ``MINIDIST_BOUNDS_CHECK=1``."""
    objdir = OBJDIR / "checked" if bounds_check else OBJDIR
    flags = NVCC_FLAGS + (["-DMD_BOUNDS_CHECK"] if bounds_check else [])
    libname = CHECKED_LIBNAME if bounds_check else LIBNAME
    objdir.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    if not sources:
        raise RuntimeError(f"no sources under {CSRC}")
    hdr = _headers_digest()
    jobs = jobs or min(len(sources), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as pool:
        results = list(pool.map(lambda s: _compile_one(s, flags, hdr, verbose, objdir), sources))
    objs = [r[0] for r in results]
    lib = LIBDIR / libname
    relink = any(r[1] for r in results) or not lib.exists()
    if not relink:
        newest = max(o.stat().st_mtime for o in objs)
        relink = newest > lib.stat().st_mtime
    if relink:
        tmp = LIBDIR / (libname + ".tmp")
        cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-cudart", "static", *map(str, objs), "-o", str(tmp), "-lcuda"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{proc.stdout}{proc.stderr}")
        os.replace(tmp, lib)
        if verbose:
            print(f"  linked {lib.relative_to(ROOT)}")
    return lib


if __name__ == "__main__":
    build(verbose=True, bounds_check="--bounds-check" in sys.argv[1:])
    sys.exit(0)
