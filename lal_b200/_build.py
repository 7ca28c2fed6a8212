"""Build recipe of liblal_tail.so (sm_100a) -- run by __graft_entry__.build().

Steps:
  1. the glibc-expf fix-up table: compile csrc/gen_expf_fixups.c with the host
     gcc, run it (all 2^31 non-positive floats, a few seconds on 8 cores) and
     keep the result in _gen/expf_fixups.bin; rebuilt only when the generator
     or lal_expf.h change;
  2. nvcc -gencode arch=compute_100a,code=sm_100a for the kernels and the C
     ABI, -fmad=false so that no float multiply-add is contracted;
  3. link lal_b200/liblal_tail.so in-tree, exporting only lal_* (exports.map).
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
GEN = os.path.join(HERE, "_gen")
OBJ = os.path.join(HERE, "_build")
SO = os.path.join(HERE, "liblal_tail.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
HOSTCC = os.environ.get("HOSTCC", "gcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-Xcompiler",
           "-fPIC,-ffp-contract=off", f"-I{INCLUDE}", f"-I{CSRC}"]

CU_SOURCES = ["tail_kernels.cu", "tail_batch.cu", "tail_gpt2.cu", "tail_api.cu",
              "tail_noalloc.cu"]
HEADERS = ["tail_internal.h", "tail_device.cuh", "tail_wide.cuh", "lal_expf.h", "../../include/lal_tail.h",
           "../../include/runtime/lal_q8_kernel.h", "../../include/runtime/lal_sampling.h"]


def _run(cmd, **kw):
    r = subprocess.run(cmd, capture_output=True, text=True, **kw)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} (exit {r.returncode})")
    return r


def _digest(paths):
    h = hashlib.sha256()
    for p in paths:
        with open(p, "rb") as f:
            h.update(f.read())
    return h.hexdigest()[:16]


def build_expf_table(force: bool = False) -> str:
    os.makedirs(GEN, exist_ok=True)
    out = os.path.join(GEN, "expf_fixups.bin")
    stamp = os.path.join(GEN, "expf_fixups.stamp")
    srcs = [os.path.join(CSRC, "gen_expf_fixups.c"), os.path.join(CSRC, "lal_expf.h")]
    dig = _digest(srcs)
    if not force and os.path.exists(out) and os.path.exists(stamp) \
            and open(stamp).read().strip() == dig:
        return out
    exe = os.path.join(GEN, "gen_expf_fixups")
    _run([HOSTCC, "-O2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", f"-I{CSRC}",
          srcs[0], "-o", exe, "-lm"])
    _run([exe, out, str(os.cpu_count() or 4)])
    with open(stamp, "w") as f:
        f.write(dig)
    return out


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every CUDA source for sm_100a and link lal_b200/liblal_tail.so."""
    build_expf_table(force)
    os.makedirs(OBJ, exist_ok=True)
    deps = [os.path.join(CSRC, h) for h in HEADERS]
    objs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src.replace(".cu", ".o"))
        objs.append(o)
        if not force and os.path.exists(o) and \
                os.path.getmtime(o) >= max(os.path.getmtime(x) for x in [s] + deps):
            continue
        r = _run([NVCC, *ARCH, *NVFLAGS, "-Xptxas", "-v", "-c", s, "-o", o])
        if verbose:
            sys.stderr.write(r.stderr)
    blob = os.path.join(OBJ, "expf_blob.o")
    _run([HOSTCC, "-c", os.path.join(CSRC, "expf_blob.S"), f"-Wa,-I,{GEN}", "-o", blob])
    objs.append(blob)
    _run([NVCC, *ARCH, "-shared", "-o", SO, *objs,
          f"-Xlinker=--version-script={os.path.join(CSRC, 'exports.map')}",
          "-Xlinker=-z,noexecstack", "-lpthread", "-ldl", "-lrt"])
    return SO


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
