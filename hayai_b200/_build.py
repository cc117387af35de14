"""Build steps for the native parts of hayai_b200 (called by __graft_entry__.build()).

* ``gen_tables``  -- IQ codebook header from the reference sources (build time only).
* ``build_cuda``  -- libhayai_cuda.so: every .cu under csrc/, sm_100a, static cudart.
* ``build_oracle`` -- the CPU parity oracle (test infrastructure, oracle/_build/).

Builds are incremental: a target is rebuilt when any of its inputs is newer.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
GEN = os.path.join(CSRC, "_gen")
TABLES = os.path.join(GEN, "iq_tables.h")
LIBDIR = os.path.join(PKG, "lib")
CUDA_LIB = os.path.join(LIBDIR, "libhayai_cuda.so")
ORACLE_DIR = os.path.join(ROOT, "oracle")
ORACLE_LIB = os.path.join(ORACLE_DIR, "_build", "liboracle.so")
# the reference checkout (read for its format tables at build time): beside the repository
REFERENCE = os.environ.get("HAYAI_REFERENCE", os.path.join(os.path.dirname(ROOT), "reference"))

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3",
    "-Xptxas", "-O3",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newer(target: str, inputs: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(p) > t for p in inputs if os.path.exists(p))


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ... (exit {r.returncode})")


def gen_tables(force: bool = False) -> str:
    """Generate the IQ codebook header from the reference (needs the reference tree)."""
    script = os.path.join(CSRC, "gen_iq_tables.py")
    srcs = [os.path.join(REFERENCE, "crates/hayai-model/src/iq2.rs"),
            os.path.join(REFERENCE, "crates/hayai-model/src/iq3.rs"),
            os.path.join(REFERENCE, "crates/hayai-model/src/iq4.rs")]
    if all(os.path.exists(s) for s in srcs):
        if force or _newer(TABLES, srcs + [script]):
            _run([sys.executable, script, REFERENCE, TABLES])
    elif not os.path.exists(TABLES):
        missing = [s for s in srcs if not os.path.exists(s)]
        raise RuntimeError(
            "cannot build: the IQ2/IQ3/IQ4 codebooks (GGUF format constants) are generated at build time from "
            f"the reference's sources, and these are missing: {', '.join(missing)}.  Check out aitups/hayai "
            f"v0.2.3 beside this repository (expected at {REFERENCE}) or set HAYAI_REFERENCE to its path; "
            f"the generated header ({TABLES}) is not kept in the repository")
    return TABLES


def build_cuda(force: bool = False) -> str:
    gen_tables()
    cus = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = cus + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + [
        TABLES, os.path.join(ROOT, "include", "hayai_cuda.h"), __file__]
    if not force and not _newer(CUDA_LIB, deps):
        return CUDA_LIB
    os.makedirs(LIBDIR, exist_ok=True)
    objdir = os.path.join(PKG, "_build")
    os.makedirs(objdir, exist_ok=True)
    nvcc = _nvcc()
    objs = []
    procs = []
    for cu in cus:
        obj = os.path.join(objdir, os.path.basename(cu) + ".o")
        objs.append(obj)
        cmd = [nvcc, *NVCC_FLAGS, "-I", CSRC, "-I", os.path.join(ROOT, "include"), "-c", cu, "-o", obj]
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = []
    for cmd, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            failed.append((cmd[-3], out))
    if failed:
        for name, out in failed:
            sys.stderr.write(f"--- {name}\n{out}\n")
        raise RuntimeError(f"nvcc failed for {[os.path.basename(f[0]) for f in failed]}")
    tmp = CUDA_LIB + ".tmp"
    _run([nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static", "-o", tmp, *objs])
    os.replace(tmp, CUDA_LIB)
    return CUDA_LIB


def build_oracle(force: bool = False) -> str:
    gen_tables()
    src = os.path.join(ORACLE_DIR, "hayai_oracle.c")
    if not force and not _newer(ORACLE_LIB, [src, TABLES, __file__]):
        return ORACLE_LIB
    os.makedirs(os.path.dirname(ORACLE_LIB), exist_ok=True)
    tmp = ORACLE_LIB + ".tmp"
    # x86-64-v3 (AVX2) instead of -march=native: the library travels to other hosts.
    _run(["gcc", "-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC",
          "-shared", "-std=c11", "-I", GEN, src, "-o", tmp, "-lm"])
    os.replace(tmp, ORACLE_LIB)
    return ORACLE_LIB


def build_all(force: bool = False) -> None:
    build_oracle(force)
    build_cuda(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print("built", CUDA_LIB, ORACLE_LIB)
