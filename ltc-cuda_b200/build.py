"""Build libltc_sm100.so in-tree with nvcc for sm_100a (B200).

Usage: python build.py [--verbose-ptxas]
The library is written next to this file (``libltc_sm100.so``); it has no
torch dependency (plain C-ABI over the CUDA runtime).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libltc_sm100.so")
SOURCES = ["ltc_capi.cu", "ltc_prep.cu", "ltc_sensory.cu", "ltc_recurrent.cu", "ltc_recurrent_wide.cu",
           "ltc_noalloc.cu", "ltc_recurrent_stream.cu", "ltc_recurrent_sparse.cu", "ltc_recurrent_csparse.cu",
           "ltc_preamble.cu", "ltc_sensory_sparse.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("CUDA_HOME", ""), "/usr/local/cuda"):
        p = os.path.join(cand, "bin", "nvcc") if cand else ""
        if p and os.path.exists(p):
            return p
    p = shutil.which("nvcc")
    if not p:
        raise RuntimeError("nvcc not found (set CUDA_HOME)")
    return p


def sources_newer_than_lib() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(os.path.dirname(HERE), "include", "ltc_sm100.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose_ptxas: bool = False, out: str = LIB, defines=()) -> str:
    if out == LIB and not force and not sources_newer_than_lib():
        return LIB
    cmd = [nvcc_path(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "--expt-relaxed-constexpr", "-o", out + ".tmp"]
    cmd += [f"-D{d}" for d in defines]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    cmd += [os.path.join(CSRC, s) for s in SOURCES]
    cmd += ["-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libltc_sm100.so")
    if verbose_ptxas:
        sys.stderr.write(r.stderr)
    os.replace(out + ".tmp", out)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--out", default=LIB, help="output path (variant builds for tuning)")
    ap.add_argument("-D", dest="defines", action="append", default=[], help="extra preprocessor define")
    ap.add_argument("--checked", action="store_true",
                    help="also build libltc_sm100_checked.so (-DLTC_CHECKED: bounds-checked indices, for tests)")
    a = ap.parse_args()
    print(build(force=a.force or a.verbose_ptxas, verbose_ptxas=a.verbose_ptxas, out=os.path.abspath(a.out),
                defines=a.defines))
    if a.checked:
        print(build(force=True, out=os.path.join(HERE, "libltc_sm100_checked.so"), defines=["LTC_CHECKED"]))
