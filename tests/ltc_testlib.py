"""Helpers shared by the parity tests (CUDA product vs oracle / golden fixtures)."""
import torch

import ltc_cuda
from golden_io import FN
from oracle import ltc_oracle as orc

# Parity bar: forward max-abs 1e-3; gradients rtol 5e-2 / atol 1e-2.
FWD_ATOL = 1e-3
GRAD_RTOL, GRAD_ATOL = 5e-2, 1e-2


def cuda_solver(inp, U, eps, gout=None, gh=None, device="cuda", backward=True):
    """Run ltc_cuda_forward on solver inputs; return (out, h, grads dict or None)."""
    leaves = {k: inp[k].detach().to(device=device, dtype=torch.float32).clone().requires_grad_(backward)
              for k in FN}
    with torch.set_grad_enabled(backward):
        out, h = ltc_cuda.ltc_cuda_forward(*[leaves[k] for k in FN], U, eps)
    if not backward:
        return out, h, None
    loss = (out * (torch.ones_like(out) if gout is None else gout.to(device))).sum()
    if gh is not None:
        loss = loss + (h * gh.to(device)).sum()
    g = torch.autograd.grad(loss, [leaves[k] for k in FN])
    return out.detach(), h.detach(), dict(zip(FN, g))


def assert_grads_close(got, ref, keys=FN, rtol=GRAD_RTOL, atol=GRAD_ATOL, ctx=""):
    for k in keys:
        a, b = got[k].detach().cpu().double(), ref[k].detach().cpu().double()
        assert a.shape == b.shape, f"{ctx} {k}: shape {a.shape} vs {b.shape}"
        assert torch.isfinite(a).all(), f"{ctx} {k}: non-finite gradient"
        ok = torch.allclose(a, b, rtol=rtol, atol=atol)
        assert ok, f"{ctx} grad {k}: max abs err {(a - b).abs().max().item():.3e} (ref max {b.abs().max().item():.3e})"


def rel_err(a, b):
    a, b = a.detach().cpu().double(), b.detach().cpu().double()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-12)).item()


def oracle_solver(inp, U, eps, gout=None, gh=None, device="cpu", chunk=None, dtype=torch.float32,
                  checkpoint=False):
    """Oracle outputs and gradients (B-chunked, optionally step-checkpointed, for the
    larger workloads)."""
    moved = {k: v.detach().to(device) for k, v in inp.items()}
    return orc.function_grads(moved, U, eps,
                              grad_out=None if gout is None else gout.to(device),
                              grad_state=None if gh is None else gh.to(device),
                              batch_chunk=chunk, dtype=dtype, checkpoint=checkpoint)
