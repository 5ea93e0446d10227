"""Recipe: stage the reference implementation under ``oracle/_ref/`` (test
infrastructure only; ``oracle/_ref/`` is git-ignored and never part of the product).

Two things are produced, both from the reference checkout named by
``LTC_REFERENCE_DIR`` (or ``--reference``), which must exist where this runs:

1. ``oracle/_ref/ltc.py``, ``ltc_cuda.py``, ``test_ltc_cuda.py`` and
   ``test_ltc_verification.py``: byte copies of the reference's TorchScript model,
   its loader and its acceptance suites, checked against a SHA-256 manifest
   (``oracle/_ref/MANIFEST.sha256``).  They let the GPU box (which carries only this
   repository's tree) run the reference's own TorchScript path as the CPU baseline and
   its acceptance suite against this package's ``ltc_cuda``.
2. ``oracle/_ref/_cuda_build/ltc_cuda_kernels_v2.so``: the reference's CUDA
   extension (``csrc/ltc_kernels.cu``, unmodified) compiled for sm_100a with the
   reference's own flags (``-O3 --use_fast_math``, ``ltc_cuda.py:186``) through
   ``torch.utils.cpp_extension``, compiled from where the source lies.  The staged
   ``ltc_cuda.py`` finds it through its cached-build path (``ltc_cuda.py:112-132``,
   ``:148-163``: with no ``csrc/`` beside it there is no freshness check to trip).
   This is the timing baseline for the reference's own GPU kernels.

Nothing in the product imports ``oracle/_ref``; only ``tests/`` and ``bench.py``'s
reference arms do, and they report the reference as unavailable when it is absent.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
STAGED = ("ltc.py", "ltc_cuda.py", "test_ltc_cuda.py", "test_ltc_verification.py")
EXT_NAME = "ltc_cuda_kernels_v2"  # the reference loader's module name (ltc_cuda.py:25)


def _sha(path: str) -> str:
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def stage_python(ref: str) -> None:
    os.makedirs(OUT, exist_ok=True)
    lines = []
    for name in STAGED:
        src = os.path.join(ref, name)
        dst = os.path.join(OUT, name)
        shutil.copyfile(src, dst)
        assert _sha(dst) == _sha(src), name
        lines.append(f"{_sha(dst)}  {name}\n")
    with open(os.path.join(OUT, "MANIFEST.sha256"), "w") as f:
        f.writelines(lines)


def verify_manifest() -> bool:
    """True when every staged file matches the manifest written at staging time."""
    man = os.path.join(OUT, "MANIFEST.sha256")
    if not os.path.exists(man):
        return False
    with open(man) as f:
        for line in f:
            digest, name = line.split()
            p = os.path.join(OUT, name)
            if not os.path.exists(p) or _sha(p) != digest:
                return False
    return True


def build_cuda(ref: str) -> str:
    src = os.path.join(ref, "csrc", "ltc_kernels.cu")
    bdir = os.path.join(OUT, "_cuda_build")
    so = os.path.join(bdir, EXT_NAME + ".so")
    stamp = os.path.join(bdir, "SOURCE.sha256")
    if os.path.exists(so) and os.path.exists(stamp):
        with open(stamp) as f:
            if f.read().strip() == _sha(src):
                return so
    os.makedirs(bdir, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")  # no GPU here to detect; sm_100a added below
    from torch.utils import cpp_extension
    cpp_extension.load(name=EXT_NAME, sources=[src], build_directory=bdir, verbose=False,
                       extra_cuda_cflags=["-O3", "--use_fast_math", "-gencode", "arch=compute_100a,code=sm_100a"])
    with open(stamp, "w") as f:
        f.write(_sha(src))
    return so


def reference_dir(cli: str | None = None) -> str | None:
    ref = cli or os.environ.get("LTC_REFERENCE_DIR")
    return ref if ref and os.path.exists(os.path.join(ref, "ltc.py")) else None


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="reference checkout (else $LTC_REFERENCE_DIR)")
    ap.add_argument("--no-cuda", action="store_true", help="stage the Python files only")
    a = ap.parse_args(argv)
    ref = reference_dir(a.reference)
    if ref is None:
        print("reference checkout not found: pass --reference or set LTC_REFERENCE_DIR", file=sys.stderr)
        return 1
    stage_python(ref)
    if not a.no_cuda:
        print(build_cuda(ref))
    return 0


if __name__ == "__main__":
    sys.exit(main())
