"""Build librai_gpu.so (sm_100a) in-tree with nvcc.

    python -m rai_b200.build          # or rai_b200.build.build()

The shared library lands next to this file so it travels with the source
tree; it links the CUDA runtime statically and exports only the C ABI of
include/rai_gpu.h.
"""
from __future__ import annotations

import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "librai_gpu.so")
SOURCES = ["kernels_gemm.cu", "kernels_gemm_tc.cu", "kernels_gemm_tol.cu", "kernels_layers.cu", "kernels_moe.cu", "kernels_sample.cu", "runtime.cu", "convert_host.cpp"]
HEADERS = ["common.cuh", "kernels.h", "layers.h", "moe.h", "quant.cuh", "raimodel_format.h", "tp.cuh"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-Xcompiler", "-ffp-contract=off",
    "--expt-relaxed-constexpr",
    "-I", os.path.join(ROOT, "include"),
]


def _digest() -> str:
    h = hashlib.sha256()
    for f in SOURCES + HEADERS:
        with open(os.path.join(CSRC, f), "rb") as fh:
            h.update(fh.read())
    with open(os.path.join(ROOT, "include", "rai_gpu.h"), "rb") as fh:
        h.update(fh.read())
    h.update(" ".join(FLAGS).encode())
    return h.hexdigest()


EXPF_TABLE = os.path.join(HERE, "expf_exceptions.bin")


def _expf_table_current() -> bool:
    """The table has the versioned layout and was made with this glibc."""
    try:
        with open(EXPF_TABLE, "rb") as f:
            head = f.read(40)
    except OSError:
        return False
    if len(head) < 40 or head[:4] != b"EXP2":
        return False
    made_with = head[8:40].split(b"\0", 1)[0].decode(errors="replace")
    running = os.confstr("CS_GNU_LIBC_VERSION").split()[-1]
    return made_with == running


def build_expf_table(force: bool = False) -> str:
    """Tabulate where the host libm expf differs from correctly rounded exp
    (csrc/gen_expf_table.c); the library loads the table at model load."""
    if os.path.exists(EXPF_TABLE) and not force and _expf_table_current():
        return EXPF_TABLE
    bdir = os.path.join(HERE, "_build")
    os.makedirs(bdir, exist_ok=True)
    exe = os.path.join(bdir, "gen_expf_table")
    subprocess.run(["gcc", "-O2", "-fopenmp", os.path.join(CSRC, "gen_expf_table.c"), "-o", exe, "-lm"],
                   check=True)
    tmp = EXPF_TABLE + ".tmp"
    subprocess.run([exe, tmp], check=True, stdout=subprocess.DEVNULL)
    os.replace(tmp, EXPF_TABLE)
    return EXPF_TABLE


def build(force: bool = False, verbose: bool = False) -> str:
    build_expf_table()
    stamp = LIB + ".sha256"
    digest = _digest()
    if not force and os.path.exists(LIB) and os.path.exists(stamp):
        with open(stamp) as fh:
            if fh.read().strip() == digest:
                return LIB
    objs = []
    bdir = os.path.join(HERE, "_build")
    os.makedirs(bdir, exist_ok=True)
    for src in SOURCES:
        obj = os.path.join(bdir, os.path.splitext(src)[0] + ".o")
        cmd = [NVCC, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB + ".tmp"
    subprocess.run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp, *objs,
                    "-Xcompiler", "-fPIC"], check=True)
    os.replace(tmp, LIB)
    with open(stamp, "w") as fh:
        fh.write(digest)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
