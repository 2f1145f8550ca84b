"""Build ``smaq_b200/libsmaq_b200.so`` from ``smaq_b200/csrc/*.cu`` with nvcc for sm_100a.

``python -m smaq_b200.build`` (or ``__graft_entry__.build()``).  Objects are compiled in
parallel into ``smaq_b200/_build/`` and relinked only when a source or header is newer than
the library.  The library is plain C-ABI (include/smaq_b200.h); it does not link against torch.
"""

from __future__ import annotations

import concurrent.futures as cf
import glob
import hashlib
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OUT = os.path.join(PKG, "libsmaq_b200.so")
BUILD = os.path.join(PKG, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", os.path.join(REPO, "include")]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return _sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(REPO, "include", "*.h"))


STAMP = os.path.join(BUILD, "stamp")


def _digest() -> str:
    h = hashlib.sha256()
    for f in sorted(_deps()) + [os.path.abspath(__file__)]:
        h.update(os.path.basename(f).encode())
        with open(f, "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()


def up_to_date() -> bool:
    """Content-hash check (file copies to another machine do not keep mtimes)."""
    if not os.path.exists(OUT) or not os.path.exists(STAMP):
        return False
    with open(STAMP) as fh:
        return fh.read().strip() == _digest()


def _compile(src: str, verbose_ptxas: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, *os.environ.get("SMAQ_NVCC_EXTRA", "").split(), "-c", src, "-o", obj]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose_ptxas:
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), _sources()))
    tmp = OUT + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-lcudart", "-lcuda", "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, OUT)
    with open(STAMP, "w") as fh:
        fh.write(_digest())
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv))
