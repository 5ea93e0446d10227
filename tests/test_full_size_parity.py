"""Parity at the sizes that are timed: the sm_100a solver against the oracle run on
the GPU, in fp32 (the reference's arithmetic) and in fp64 (to tell kernel error from
fp32 summation-order noise), with the metric's sum loss.

* c2 in full (B=256, T=64, D=256, H=128, U=6);
* c3 on the 512-sample shard each rank runs at 8 GPUs (T=128, full length);
* c4 at full length (T=256, U=12, D=H=512, density 0.2/0.3) on a 4-sample slice,
  the oracle checkpointed per step.

Bars (north star, the reference tests' own): forward max-abs 1e-3 and gradients
``allclose(rtol=5e-2, atol=1e-2)`` against the fp32 oracle.  Each case also prints
its errors against both oracles (run with ``-s`` to see them).
"""
import json

import pytest
import torch

import synth
from golden_io import FN
from ltc_testlib import FWD_ATOL, assert_grads_close, cuda_solver, oracle_solver, rel_err

pytestmark = pytest.mark.gpu


def _inputs(cfg, B, T=None):
    from oracle import ltc_oracle as orc
    p, x = synth.make_workload(cfg, batch=B)
    if T is not None:
        x = x[:, :T].contiguous()
    inp = {k: v.detach() for k, v in orc.module_preamble(p, x, cfg.dt, cfg.U).items()}
    inp["state"] = torch.zeros(x.shape[0], cfg.H)
    return inp


def _errors(out, h, g, ro, rh, rg):
    fwd = max((out.double() - ro.to(out.device).double()).abs().max().item(),
              (h.double() - rh.to(h.device).double()).abs().max().item())
    grel = {k: rel_err(g[k], rg[k]) for k in FN}
    return {"fwd_max_abs": fwd, "grad_max_rel": max(grel.values()),
            "worst_grad": max(grel, key=grel.get)}


@pytest.mark.parametrize("name,B,T,chunk,checkpoint", [
    ("c2", 256, None, 32, False),
    ("c3", 512, None, 64, False),
    ("c4", 4, None, 2, True),
])
def test_timed_size_vs_gpu_oracle(name, B, T, chunk, checkpoint):
    cfg = synth.CONFIGS[name]
    inp = _inputs(cfg, B, T)
    out, h, g = cuda_solver(inp, cfg.U, 1e-8)  # sum loss: grad_out = ones
    ro, rh, rg = oracle_solver(inp, cfg.U, 1e-8, device="cuda", chunk=chunk, checkpoint=checkpoint)
    e32 = _errors(out, h, g, ro, rh, rg)
    rg = {k: v.cpu() for k, v in rg.items()}
    del ro, rh
    torch.cuda.empty_cache()
    ro64, rh64, rg64 = oracle_solver(inp, cfg.U, 1e-8, device="cuda", chunk=chunk, checkpoint=checkpoint,
                                     dtype=torch.float64)
    e64 = _errors(out, h, g, ro64, rh64, rg64)
    print("PARITY " + json.dumps({"config": name, "B": inp["x_seq"].shape[0], "T": inp["x_seq"].shape[1],
                                  "vs_fp32_oracle": e32, "vs_fp64_oracle": e64}))
    assert e32["fwd_max_abs"] < FWD_ATOL, e32
    assert e64["fwd_max_abs"] < FWD_ATOL, e64
    assert_grads_close(g, rg, ctx=f"{name} vs fp32 oracle")
    assert_grads_close(g, rg64, ctx=f"{name} vs fp64 oracle")
