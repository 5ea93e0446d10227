"""Load the reference implementation staged under ``oracle/_ref/`` (TEST
INFRASTRUCTURE, not product; see ``oracle/build_ref.py`` for how it is staged).

Two ways in:

* :func:`import_reference` with ``cuda_kernels="reference"``: the reference's
  ``ltc.py`` (TorchScript solver, ``ltc.py:19-106``) together with the reference's
  own ``ltc_cuda.py`` loader, which picks up the reference CUDA extension compiled
  for sm_100a.  Used by ``bench.py``'s reference arms and its parity check.
* ``cuda_kernels="ours"``: the reference's unchanged ``ltc.py`` importing this
  repository's ``ltc_cuda`` (the drop-in path, ``ltc.py:12-16,293-307``).

Each choice binds the process-wide module name ``ltc_cuda``, so one process can
use only one of them; a second, conflicting request raises.
"""
from __future__ import annotations

import importlib
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")
PKG = os.path.join(os.path.dirname(HERE), "ltc-cuda_b200")


def available(cuda: bool = False) -> str | None:
    """None when the staged reference is usable, else a one-line reason."""
    from oracle import build_ref
    if not os.path.exists(os.path.join(REF, "ltc.py")):
        return "reference not staged (run oracle/build_ref.py where the reference checkout exists)"
    if not build_ref.verify_manifest():
        return "staged reference files do not match their SHA-256 manifest"
    if cuda and not os.path.exists(os.path.join(REF, "_cuda_build", build_ref.EXT_NAME + ".so")):
        return "reference CUDA extension not built (oracle/build_ref.py)"
    return None


def import_reference(cuda_kernels: str = "reference"):
    """Return the reference ``ltc`` module; ``cuda_kernels`` picks whose ``ltc_cuda`` it binds."""
    import torch
    # on a CUDA machine the reference loader would JIT-build its kernels if the
    # prebuilt extension were missing: require it there
    why = available(cuda=cuda_kernels == "reference" and torch.cuda.is_available())
    if why:
        raise RuntimeError(why)
    want = REF if cuda_kernels == "reference" else PKG
    if "ltc_cuda" in sys.modules:
        have = os.path.dirname(os.path.abspath(sys.modules["ltc_cuda"].__file__))
        if have != want:
            raise RuntimeError(f"ltc_cuda already bound to {have}; need {want}")
    for p in (REF, want):
        while p in sys.path:
            sys.path.remove(p)
    # ltc.py is found in REF; ltc_cuda resolves to `want` (placed first)
    sys.path[:0] = [want, REF] if want != REF else [REF]
    ltc = importlib.import_module("ltc")
    import ltc_cuda
    got = os.path.dirname(os.path.abspath(ltc_cuda.__file__))
    if got != want:
        raise RuntimeError(f"ltc_cuda resolved to {got}, expected {want}")
    return ltc


def reference_module(ltc, p, D: int, H: int, dt: float, U: int, density: float, sensory_density: float):
    """The reference ``TrueLiquidTimeConstant`` holding the parameters ``p`` (state-dict names)."""
    m = ltc.TrueLiquidTimeConstant(D, H, dt=dt, ode_unfolds=U, sparsity=density,
                                   sensory_sparsity=sensory_density)
    m.load_state_dict(p)
    return m
