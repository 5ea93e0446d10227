"""GPU: the fused module preamble (LayerNorm + input affine, ltc.py:259,266) against
the same PyTorch ops in fp64, forward and all five gradients."""
import pytest
import torch
import torch.nn.functional as F

import ltc_cuda

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,D", [(1, 1), (7, 10), (333, 128), (96, 224), (40, 512), (9, 1000)])
def test_preamble_matches_torch(rows, D):
    g = torch.Generator().manual_seed(rows * 7 + D)
    x = (torch.randn(rows, D, generator=g) * 3 + 1).double()
    lw, lb, iw, ib = (torch.randn(D, generator=g).double() for _ in range(4))
    dy = torch.randn(rows, D, generator=g).double()
    leaves = [t.clone().requires_grad_(True) for t in (x, lw, lb, iw, ib)]
    ref = F.layer_norm(leaves[0], (D,), leaves[1], leaves[2], 1e-5) * leaves[3] + leaves[4]
    rg = torch.autograd.grad((ref * dy).sum(), leaves)
    cl = [t.float().cuda().requires_grad_(True) for t in (x, lw, lb, iw, ib)]
    y = ltc_cuda.ltc_preamble(*cl, 1e-5)
    cg = torch.autograd.grad((y * dy.float().cuda()).sum(), cl)
    scale = ref.abs().max().item()
    assert (y.double().cpu() - ref.detach()).abs().max().item() <= 2e-5 * max(1.0, scale)
    for a, b, name in zip(cg, rg, ("x", "ln_w", "ln_b", "in_w", "in_b")):
        err = (a.double().cpu() - b).abs().max().item()
        assert err <= 1e-4 * max(1.0, b.abs().max().item()), f"{name}: {err:.3e}"


def test_preamble_deterministic_and_3d():
    x = torch.randn(4, 33, 128, device="cuda")
    p = [torch.randn(128, device="cuda").requires_grad_(True) for _ in range(4)]
    xs = x.clone().requires_grad_(True)
    outs = []
    for _ in range(2):
        y = ltc_cuda.ltc_preamble(xs, *p, 1e-5)
        outs.append((y.detach().clone(), torch.autograd.grad(y.sum(), [xs, *p])))
    assert y.shape == x.shape
    assert torch.equal(outs[0][0], outs[1][0])
    for a, b in zip(outs[0][1], outs[1][1]):
        assert torch.equal(a, b)
