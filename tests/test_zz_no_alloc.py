"""ltc_forward_noalloc: the forward entry point that allocates nothing.

Some callers may not allocate GPU memory where they run the solver -- a plugin in
a serving runtime that owns every allocation under a fixed budget, or a latency-
critical loop where cudaMalloc would synchronise the device.  For them the
library offers ltc_forward_noalloc, whose scratch is a fixed static device array
instead of a caller workspace.  This test calls it through the C-ABI twice in a
row (the second call runs on the scratch the first one left behind) and checks
both results against the CPU oracle and against the regular ltc_forward entry
point, within the forward tolerance of the parity tests, on all three recurrent
kernel families (H <= 64, 64 < H <= 128, and the streamed H > 128 path whose own
scratch region sits at the end of the static array), with and without an initial
state; and that an oversized problem is refused.

The file name sorts last so that a run stopping at the first failure has already
run every other test.
"""
import ctypes

import pytest
import torch

import ltc_cuda
import synth
from ltc_testlib import FWD_ATOL
from oracle import ltc_oracle as orc

pytestmark = pytest.mark.gpu

NOALLOC_BYTES = 16 * 1024 * 1024  # LTC_NOALLOC_SCRATCH_BYTES in include/ltc_sm100.h


def _lib():
    lib = ltc_cuda._require_kernels()
    fn = lib.ltc_forward_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(ltc_cuda.LtcDims), ctypes.POINTER(ltc_cuda.LtcParams), ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return lib


def _problem(cfg_name, B, T, seed, with_h0=True):
    if cfg_name in synth.CONFIGS:
        cfg = synth.CONFIGS[cfg_name]
    else:  # "D<d>H<h>": a small problem on the streamed H > 128 path
        d, h = cfg_name[1:].split("H")
        cfg = synth.LtcConfig(cfg_name, B, T, int(d), int(h), 6, 0.5, 0.5)
    p, x = synth.make_workload(cfg, batch=B, seed=seed)
    inp = {k: v.detach().cuda().contiguous() for k, v in orc.module_preamble(p, x[:, :T], cfg.dt, cfg.U).items()}
    g = torch.Generator().manual_seed(seed)
    h0 = (torch.randn(B, cfg.H, generator=g) * 0.3).cuda() if with_h0 else None
    names = ("w_pos", "w_erev", "mu", "sigma", "sensory_mu", "sensory_sigma", "sensory_erev", "sensory_w_pos",
             "cm_t", "gleak_pos", "vleak")
    params = ltc_cuda.LtcParams(*[inp[n].data_ptr() for n in names])
    dims = ltc_cuda.make_dims(B, T, cfg.D, cfg.H, cfg.U, 1e-8)
    return dims, params, inp, h0


def _oracle_forward(dims, inp, h0):
    cpu = {k: v.cpu() for k, v in inp.items()}
    cpu["state"] = torch.zeros(dims.B, dims.H) if h0 is None else h0.cpu()
    with torch.no_grad():
        return orc.function_forward(cpu, dims.ode_unfolds, 1e-8)


def _regular_forward(lib, dims, params, x, h0):
    pl = ltc_cuda.plan(dims)
    out = torch.empty(dims.B, dims.T, dims.H, device="cuda")
    hT = torch.empty(dims.B, dims.H, device="cuda")
    ws = torch.empty(pl.fwd_workspace_bytes, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.ltc_forward(ctypes.byref(dims), ctypes.byref(params), x.data_ptr(),
                         None if h0 is None else h0.data_ptr(), out.data_ptr(),
                         hT.data_ptr(), None, ws.data_ptr(), pl.fwd_workspace_bytes, st)
    assert rc == 0, lib.ltc_last_error()
    return out, hT


@pytest.mark.parametrize("cfg_name,B,T,with_h0", [
    ("c0", 24, 8, True), ("c2", 5, 3, True), ("D16H160", 8, 4, True), ("D16H160", 8, 4, False), ("c0", 3, 2, False)])
def test_noalloc_matches_oracle_and_regular_forward_twice(cfg_name, B, T, with_h0):
    lib = _lib()
    dims, params, inp, h0 = _problem(cfg_name, B, T, seed=B + T, with_h0=with_h0)
    ref_out, ref_h = _regular_forward(lib, dims, params, inp["x_seq"], h0)
    orc_out, orc_h = _oracle_forward(dims, inp, h0)
    st = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full((B, T, dims.H), float("nan"), device="cuda")
        hT = torch.full((B, dims.H), float("nan"), device="cuda")
        rc = lib.ltc_forward_noalloc(ctypes.byref(dims), ctypes.byref(params), inp["x_seq"].data_ptr(),
                                     None if h0 is None else h0.data_ptr(), out.data_ptr(), hT.data_ptr(), st)
        assert rc == 0, lib.ltc_last_error()
        torch.cuda.synchronize()
        assert (out.cpu() - orc_out).abs().max().item() < FWD_ATOL, f"call {call}: vs oracle"
        assert (hT.cpu() - orc_h).abs().max().item() < FWD_ATOL, f"call {call}: vs oracle"
        assert (out - ref_out).abs().max().item() < FWD_ATOL, f"call {call}: vs ltc_forward"
        assert (hT - ref_h).abs().max().item() < FWD_ATOL, f"call {call}: vs ltc_forward"


def test_noalloc_rejects_oversized_problem():
    lib = _lib()
    B, T, H = 1024, 256, 64  # sensory sums alone: 2*B*T*H*4 bytes = 128 MiB > 16 MiB
    assert 2 * B * T * H * 4 > NOALLOC_BYTES
    dims = ltc_cuda.make_dims(B, T, 8, H, 6, 1e-8)
    dummy = torch.zeros(1, device="cuda")
    params = ltc_cuda.LtcParams(*([dummy.data_ptr()] * 11))
    rc = lib.ltc_forward_noalloc(ctypes.byref(dims), ctypes.byref(params), dummy.data_ptr(), None,
                                 dummy.data_ptr(), dummy.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    assert b"limit" in lib.ltc_last_error()
