"""The unchanged reference ltc.py picks up this package's ltc_cuda (CPU check).

Runs only where the reference checkout is available (LTC_REFERENCE_DIR, default the
reference's usual mount); it is skipped elsewhere, e.g. on GPU boxes, which carry
only this repository.
"""
import importlib
import inspect
import os
import subprocess
import sys

import pytest

REF = os.environ.get("LTC_REFERENCE_DIR", "/root/reference")
PKG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "ltc-cuda_b200")


@pytest.mark.skipif(not os.path.exists(os.path.join(REF, "ltc.py")), reason="reference checkout not present")
def test_reference_ltc_imports_this_ltc_cuda():
    code = (
        "import sys; sys.path[:0] = [%r, %r]\n"
        "import ltc, ltc_cuda\n"
        "assert ltc_cuda.__file__.startswith(%r), ltc_cuda.__file__\n"
        "assert ltc.ltc_cuda_forward is ltc_cuda.ltc_cuda_forward\n"
        "import torch\n"
        "assert ltc._HAS_CUDA_KERNELS == torch.cuda.is_available()\n"
        "m = ltc.TrueLiquidTimeConstant(10, 8)\n"
        "out, (h, c) = m(torch.randn(2, 3, 10))\n"  # CPU input: the reference falls back to TorchScript
        "assert out.shape == (2, 3, 8) and h is c\n"
        "print('ok')\n" % (PKG, REF, PKG))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
