"""Build the in-tree CUDA library ``liboscar_b200.so`` for sm_100a with nvcc.

    python -m oscar_new_b200.build          # or build() from __graft_entry__

No torch extension machinery: a plain shared library with the C ABI declared in
``include/oscar_b200.h``.  IEEE division/rounding is kept (no fast-math): the INT2
store must stay bit-exact with the reference quantiser.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "liboscar_b200.so"
SOURCES = ["store.cu", "rotate_tc.cu", "attention.cu", "history_f8.cu", "history_mtp.cu", "calibration.cu",
           "noalloc.cu", "metadata.cu", "gram_tc.cu", "sst_tc.cu",
           "prefill.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (cand == "nvcc" or Path(cand).exists()):
            return cand
    raise RuntimeError("nvcc not found")


def build(verbose: bool = False, force: bool = False) -> Path:
    srcs = [CSRC / s for s in SOURCES]
    deps = srcs + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "oscar_b200.h"]
    if not force and LIB.exists() and LIB.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return LIB
    build_dir = ROOT / "_build"
    build_dir.mkdir(exist_ok=True)
    objs = []
    procs = []
    for src in srcs:
        obj = build_dir / (src.stem + ".o")
        cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
               "-I", str(ROOT / "include"), "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        objs.append(obj)
    failed = False
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0 or verbose:
            sys.stderr.write(out)
        failed |= p.returncode != 0
    if failed:
        raise RuntimeError("nvcc failed")
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.check_call([nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"])
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force=True)
    print(LIB)
