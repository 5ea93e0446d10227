"""Drop-in check: the reference's unchanged ``ltc.py`` binds this package's ``ltc_cuda``,
and the reference's own acceptance suites pass through it.

The reference files come from ``oracle/_ref/`` (staged, with a SHA-256 manifest, by
``oracle/build_ref.py``), so they travel with this tree to GPU machines.  Where they
are not staged, the tests are skipped with that reason.

* CPU: the unchanged ``ltc.py`` imports this ``ltc_cuda`` (``ltc.py:12-16``) and runs.
* GPU: ``test_ltc_cuda.py`` (numerical comparison of the CUDA path, ``ltc.py:300-307``,
  against the reference TorchScript path, ``test_ltc_cuda.py:42-336``) and
  ``test_ltc_verification.py`` run as child pytest sessions with this package first
  on ``sys.path``; the child asserts it bound this ``ltc_cuda`` and that the CUDA path
  was taken.
"""
import os
import re
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "ltc-cuda_b200")
sys.path.insert(0, REPO)
from oracle import reference_module as rm  # noqa: E402

REF = rm.REF
WHY = rm.available()


def _env():
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([PKG, REF] + [p for p in env.get("PYTHONPATH", "").split(os.pathsep) if p])
    return env


@pytest.mark.skipif(WHY is not None, reason=str(WHY))
def test_reference_ltc_imports_this_ltc_cuda():
    code = (
        "import ltc, ltc_cuda\n"
        "assert ltc_cuda.__file__.startswith(%r), ltc_cuda.__file__\n"
        "assert ltc.ltc_cuda_forward is ltc_cuda.ltc_cuda_forward\n"
        "import torch\n"
        "assert ltc._HAS_CUDA_KERNELS == torch.cuda.is_available()\n"
        "m = ltc.TrueLiquidTimeConstant(10, 8)\n"
        "out, (h, c) = m(torch.randn(2, 3, 10))\n"  # CPU input: the reference falls back to TorchScript
        "assert out.shape == (2, 3, 8) and h is c\n"
        "print('ok')\n" % (PKG,))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300, env=_env(),
                       cwd=REPO)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr


# plugin for the child session: asserts the binding and counts this library's launches
_CHILD_PLUGIN = '''
import ltc_cuda, pytest
assert ltc_cuda.__file__.startswith(%r), ltc_cuda.__file__
assert ltc_cuda._HAS_CUDA_KERNELS

def pytest_sessionfinish(session, exitstatus):
    print("\\nLTC_LAUNCHES=%%d" %% ltc_cuda.launch_count())
'''


@pytest.mark.gpu
@pytest.mark.skipif(WHY is not None, reason=str(WHY))
@pytest.mark.parametrize("suite", ["test_ltc_cuda.py", "test_ltc_verification.py"])
def test_reference_suite_on_this_ltc_cuda(suite, tmp_path):
    (tmp_path / "ltc_child_plugin.py").write_text(_CHILD_PLUGIN % (PKG,))
    (tmp_path / "pytest.ini").write_text("[pytest]\n")
    env = _env()
    env["PYTHONPATH"] = str(tmp_path) + os.pathsep + env["PYTHONPATH"]
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-s", "-p", "no:cacheprovider",
                        "-p", "ltc_child_plugin", "--rootdir", str(tmp_path), "-c", str(tmp_path / "pytest.ini"),
                        os.path.join(REF, suite)],
                       capture_output=True, text=True, timeout=1200, env=env, cwd=str(tmp_path))
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert " failed" not in out, out[-4000:]
    if suite == "test_ltc_cuda.py":
        # nothing skipped: the CUDA-kernel classes ran, and they ran this library
        assert " skipped" not in out.splitlines()[-1], out[-2000:]
        launches = [int(m) for m in re.findall(r"LTC_LAUNCHES=(\d+)", out)]
        assert launches and launches[-1] > 0, out[-2000:]
