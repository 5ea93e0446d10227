"""The checked build (libltc_sm100_checked.so, -DLTC_CHECKED): every kernel family on
small odd shapes, in a child process bound to that library, must match the oracle and
report no failed index check.

The checked build tests the indices of the table-driven gathers, the shared-memory
slabs of the per-neuron tails and the output writes; a failure is counted (and the
access skipped) rather than faulting the GPU, which stands in for compute-sanitizer,
closed on this pool.  Tolerances are the parity tests' (forward max-abs 1e-3,
gradients rtol 5e-2 / atol 1e-2).
"""
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "ltc-cuda_b200")
CHECKED = os.path.join(PKG, "libltc_sm100_checked.so")


_CHILD = r'''
import ctypes, sys, torch
import ltc_cuda, synth
from ltc_testlib import cuda_solver, oracle_solver, assert_grads_close, FWD_ATOL
from oracle import ltc_oracle as orc

lib = ctypes.CDLL(ltc_cuda.LIB_PATH)
assert lib.ltc_checked_build() > 0, "not the checked build"

def inputs(D, H, B, T, U, dens, sdens, seed):
    p = synth.make_params(D, H, dens, sdens, seed=seed)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, D, generator=g)
    inp = {k: v.detach() for k, v in orc.module_preamble(p, x, 1 / 30, U).items()}
    inp["state"] = torch.randn(B, H, generator=g) * 0.3
    return inp, torch.randn(B, T, H, generator=g), torch.randn(B, H, generator=g)

def skipped_zero(rg, inp, rec, sens):
    rg = {k: v.cpu() for k, v in rg.items()}
    if rec:
        z = (inp["w_pos"] == 0) & (inp["w_erev"] == 0)
        for k in ("w_pos", "w_erev", "mu", "sigma"):
            rg[k] = torch.where(z, torch.zeros_like(rg[k]), rg[k])
    if sens:
        z = inp["sensory_w_pos"] == 0
        for k in ("sensory_w_pos", "sensory_erev", "sensory_mu", "sensory_sigma"):
            rg[k] = torch.where(z, torch.zeros_like(rg[k]), rg[k])
    return rg

# (name, D, H, B, T, U, density, sensory density, mode)
cases = [
    ("dense H17", 7, 17, 5, 3, 2, 0.5, 0.5, "dense"),
    ("dense H64", 12, 64, 9, 4, 3, 0.5, 0.5, "dense"),
    ("cluster H100", 9, 100, 6, 3, 2, 0.5, 0.5, "dense"),
    ("stream H160", 8, 160, 7, 2, 2, 0.5, 0.5, "dense"),
    ("wide H70", 10, 70, 5, 2, 2, 0.5, 0.5, "wide"),
    ("sparse H48", 70, 48, 11, 5, 3, 0.5, 0.5, "skip"),
    ("sparse H33 sensory", 100, 33, 6, 7, 2, 0.4, 0.5, "skip+sens"),
    ("cluster lists H300 sensory", 70, 300, 5, 3, 2, 0.2, 0.3, "skip+sens"),
    ("lean sparse H64", 20, 64, 6, 6, 2, 0.5, 0.5, "skip+lean"),
]
for name, D, H, B, T, U, dens, sdens, mode in cases:
    inp, gout, gh = inputs(D, H, B, T, U, dens, sdens, seed=D * 31 + H)
    ltc_cuda.set_force_wide(mode == "wide")
    ltc_cuda.set_lean_save(mode.endswith("lean"), 2)
    rec = mode.startswith("skip") and not 64 < H <= 128
    with ltc_cuda.skip_zero_synapses(mode.startswith("skip"), sensory="sens" in mode):
        out, h, g = cuda_solver(inp, U, 1e-8, gout=gout, gh=gh)
    ro, rh, rg = oracle_solver(inp, U, 1e-8, gout=gout, gh=gh)
    assert (out.cpu() - ro.cpu()).abs().max().item() < FWD_ATOL, name
    assert (h.cpu() - rh.cpu()).abs().max().item() < FWD_ATOL, name
    assert_grads_close(g, skipped_zero(rg, {k: v.cpu() for k, v in inp.items()}, rec, "sens" in mode), ctx=name)
    count, site = ctypes.c_int(-1), ctypes.c_int(-1)
    assert lib.ltc_check_errors(ctypes.byref(count), ctypes.byref(site)) == 0, name
    assert count.value == 0, f"{name}: {count.value} failed index checks, first at site {site.value}"
    print("checked ok:", name)
ltc_cuda.set_force_wide(False)
ltc_cuda.set_lean_save(False)
print("CHECKED_ALL_OK")
'''


@pytest.mark.gpu
@pytest.mark.skipif(not os.path.exists(CHECKED), reason="checked build not built (ltc-cuda_b200/build.py --checked)")
def test_checked_build_every_family():
    env = dict(os.environ)
    env["LTC_SM100_LIB"] = CHECKED
    env["PYTHONPATH"] = os.pathsep.join([PKG, os.path.join(REPO, "tests"), REPO] +
                                        [p for p in env.get("PYTHONPATH", "").split(os.pathsep) if p])
    r = subprocess.run([sys.executable, "-c", _CHILD], capture_output=True, text=True, timeout=900, env=env,
                       cwd=REPO)
    out = r.stdout + r.stderr
    assert r.returncode == 0 and "CHECKED_ALL_OK" in r.stdout, out[-4000:]


@pytest.mark.skipif(not os.path.exists(CHECKED), reason="checked build not built (ltc-cuda_b200/build.py --checked)")
def test_checked_build_registers_its_checks():
    """No GPU needed: every source file with checks registered its error-word reader in
    the checked build, and the normal build has none."""
    import ctypes
    checked = ctypes.CDLL(CHECKED)
    normal = ctypes.CDLL(os.path.join(PKG, "libltc_sm100.so"))
    assert checked.ltc_checked_build() >= 8  # one per source file that includes the check macros
    assert normal.ltc_checked_build() == 0
