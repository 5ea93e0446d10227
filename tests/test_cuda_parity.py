"""GPU parity: the sm_100a solver (through ltc_cuda -> C-ABI) against the reference's
golden vectors and against the CPU oracle, on both kernel families (register-resident
"fast" kernels for H <= 64 and the streamed "wide" kernels), plus the reference
test-suite cases (test_ltc_cuda.py) and edge cases.

Tolerances (the reference's own test bar): forward max-abs
1e-3; gradients rtol 5e-2 / atol 1e-2.  Measured errors are ~1e-6 relative.
"""
import pytest
import torch
import torch.nn.functional as F

import ltc_cuda
import ltc_layer
import synth
from golden_io import Case, FN, case_names
from ltc_testlib import (FWD_ATOL, assert_grads_close, cuda_solver, oracle_solver, rel_err)

pytestmark = pytest.mark.gpu

CASES = case_names()


@pytest.fixture(params=["fast", "wide"])
def path(request):
    ltc_cuda.set_force_wide(request.param == "wide")
    yield request.param
    ltc_cuda.set_force_wide(False)


def test_kernels_loaded():
    assert ltc_cuda._HAS_CUDA_KERNELS, "CUDA kernels must load on a GPU box"
    assert torch.cuda.get_device_capability()[0] == 10


@pytest.mark.parametrize("name", CASES)
def test_golden_solver_level(name, path):
    c = Case(name)
    inp = c.solver_inputs
    U, eps = c.meta["U"], c.meta["epsilon"]
    has_bwd = "gout" in c.a
    out, h, g = cuda_solver(inp, U, eps, gout=c.get("gout"), gh=c.get("gh"), backward=has_bwd)
    err = (out.cpu() - c.a["out"]).abs().max().item()
    assert err < FWD_ATOL, f"{name}/{path}: forward max-abs {err:.3e}"
    assert (h.cpu() - c.a["h"]).abs().max().item() < FWD_ATOL
    if has_bwd:
        assert_grads_close(g, c.solver_grads, ctx=f"{name}/{path}")
        # fidelity far inside the bar: normalised error of every gradient <= 1e-3
        for k in FN:
            assert rel_err(g[k], c.solver_grads[k]) < 1e-3, f"{name}/{path} {k}: {rel_err(g[k], c.solver_grads[k]):.2e}"


def _layer_from_case(c):
    m = ltc_layer.TrueLiquidTimeConstant(c.meta["D"], c.meta["H"], dt=c.meta["dt"],
                                         ode_unfolds=c.meta["U"]).cuda()
    m.load_state_dict({k: v.cuda() for k, v in c.params.items()})
    return m


@pytest.mark.parametrize("name", [n for n in CASES if "gm.w" in Case(n).a])
def test_golden_module_level(name):
    """Module (LayerNorm -> affine -> softplus -> solver) against the reference module's grads."""
    c = Case(name)
    m = _layer_from_case(c)
    x = c.a["x"].cuda()
    h0 = c.get("h0")
    out, (h, h2) = m(x, None if h0 is None else (h0.cuda(), h0.cuda()))
    assert h is h2
    assert (out.detach().cpu() - c.a["out"]).abs().max().item() < FWD_ATOL
    loss = F.mse_loss(out, c.a["target"].cuda()) if c.meta["backward"] == "mse" else out.sum()
    loss.backward()
    for k, ref in c.module_grads.items():
        got = dict(m.named_parameters())[k].grad
        assert got is not None, k
        # test_ltc_cuda.py:159-163 and :205-206 tolerances
        assert torch.allclose(got.cpu(), ref, rtol=5e-2, atol=1e-2), \
            f"{name} {k}: max err {(got.cpu() - ref).abs().max().item():.3e}"


# ---- configurations of the benchmark against the oracle (batch/time slices) ----

def _config_inputs(cfg, B, T=None):
    p, x = synth.make_workload(cfg, batch=B)
    if T is not None:
        x = x[:, :T].contiguous()
    from oracle import ltc_oracle as orc
    inp = orc.module_preamble(p, x, cfg.dt, cfg.U)
    inp = {k: v.detach() for k, v in inp.items()}
    inp["state"] = torch.zeros(x.shape[0], cfg.H)
    g = torch.Generator().manual_seed(7)
    gout = torch.randn(x.shape[0], x.shape[1], cfg.H, generator=g)
    gh = torch.randn(x.shape[0], cfg.H, generator=g)
    return inp, gout, gh


@pytest.mark.parametrize("cfg,B,T,device", [
    ("c1", 16, None, "cpu"),
    ("c2", 8, 16, "cpu"),
    ("c3", 24, 32, "cpu"),
    ("c4", 2, 6, "cuda"),
])
def test_config_vs_oracle(cfg, B, T, device, path):
    c = synth.CONFIGS[cfg]
    inp, gout, gh = _config_inputs(c, B, T)
    out, h, g = cuda_solver(inp, c.U, 1e-8, gout=gout, gh=gh)
    ro, rh, rg = oracle_solver(inp, c.U, 1e-8, gout=gout, gh=gh, device=device)
    assert (out.cpu() - ro.cpu()).abs().max().item() < FWD_ATOL
    assert (h.cpu() - rh.cpu()).abs().max().item() < FWD_ATOL
    assert_grads_close(g, rg, ctx=f"{cfg}/{path}")
    for k in FN:
        assert rel_err(g[k], rg[k]) < 2e-3, f"{cfg}/{path} {k}: {rel_err(g[k], rg[k]):.2e}"


# ---- edge cases --------------------------------------------------------------

@pytest.mark.parametrize("B,T,D,H,U", [
    (1, 1, 1, 1, 1), (3, 2, 10, 8, 6), (5, 3, 7, 2, 2), (2, 4, 33, 17, 3), (6, 2, 5, 40, 1),
    (9, 3, 12, 64, 6), (1, 2, 3, 65, 2), (2, 2, 4, 96, 3), (1, 1, 6, 200, 2), (3, 2, 130, 31, 4),
])
def test_edge_shapes_vs_oracle(B, T, D, H, U, path):
    g = torch.Generator().manual_seed(B * 1000 + T * 100 + D * 10 + H + U)
    p = synth.make_params(D, H, 0.5, 0.5, seed=B + H)
    from oracle import ltc_oracle as orc
    x = torch.randn(B, T, D, generator=g)
    inp = {k: v.detach() for k, v in orc.module_preamble(p, x, 1 / 30, U).items()}
    inp["state"] = torch.randn(B, H, generator=g) * 0.3
    gout = torch.randn(B, T, H, generator=g)
    gh = torch.randn(B, H, generator=g)
    out, h, gr = cuda_solver(inp, U, 1e-8, gout=gout, gh=gh)
    ro, rh, rg = oracle_solver(inp, U, 1e-8, gout=gout, gh=gh)
    assert (out.cpu() - ro).abs().max().item() < FWD_ATOL
    assert (h.cpu() - rh).abs().max().item() < FWD_ATOL
    assert_grads_close(gr, rg, ctx=f"edge B{B} T{T} D{D} H{H} U{U}/{path}")


def test_determinism_bitwise(path):
    c = Case("c0_full")
    runs = [cuda_solver(c.solver_inputs, 6, 1e-8, gout=c.a["gout"], gh=c.a["gh"]) for _ in range(3)]
    for o, h, g in runs[1:]:
        assert torch.equal(o, runs[0][0]) and torch.equal(h, runs[0][1])
        for k in FN:
            assert torch.equal(g[k], runs[0][2][k]), f"{k} not bitwise reproducible"


def test_batch_split_forward_bitwise(path):
    """Samples are independent: solving halves of the batch gives bit-identical outputs."""
    c = synth.CONFIGS["c3"]
    inp, _, _ = _config_inputs(c, 600, 8)
    full, hf, _ = cuda_solver(inp, c.U, 1e-8, backward=False)
    for lo, hi in ((0, 300), (300, 600), (17, 18)):
        part = {k: (v[lo:hi] if k in ("x_seq", "state") else v) for k, v in inp.items()}
        o, h, _ = cuda_solver(part, c.U, 1e-8, backward=False)
        assert torch.equal(o, full[lo:hi]) and torch.equal(h, hf[lo:hi])


def test_no_grad_matches_grad_forward(path):
    c = Case("c0_full")
    a = cuda_solver(c.solver_inputs, 6, 1e-8, backward=False)
    b = cuda_solver(c.solver_inputs, 6, 1e-8, gout=c.a["gout"], gh=c.a["gh"])
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_sum_loss_stride_zero_and_state_only():
    """out.sum() gives a stride-0 upstream gradient; h-only losses give grad_outputs=None."""
    c = Case("grad_sum_d32_h16")
    leaves = {k: v.cuda().clone().requires_grad_(True) for k, v in c.solver_inputs.items()}
    out, h = ltc_cuda.ltc_cuda_forward(*[leaves[k] for k in FN], 6, 1e-8)
    g1 = torch.autograd.grad(out.sum(), [leaves[k] for k in FN])
    _, _, g2 = cuda_solver(c.solver_inputs, 6, 1e-8, gout=torch.ones(2, 4, 16))
    for k, a in zip(FN, g1):
        assert torch.equal(a, g2[k]), k
    out, h = ltc_cuda.ltc_cuda_forward(*[leaves[k] for k in FN], 6, 1e-8)
    g3 = torch.autograd.grad((h * 2.0).sum(), [leaves[k] for k in FN])
    _, _, g4 = oracle_solver(c.solver_inputs, 6, 1e-8, gout=torch.zeros(2, 4, 16), gh=torch.full((2, 16), 2.0))
    assert_grads_close(dict(zip(FN, g3)), g4, ctx="state-only")


def test_noncontiguous_inputs_and_side_stream():
    c = Case("c0_full")
    inp = dict(c.solver_inputs)
    x = inp["x_seq"].cuda()
    xt = x.transpose(0, 1).contiguous().transpose(0, 1)  # same values, non-contiguous view
    assert not xt.is_contiguous()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        args = [xt if k == "x_seq" else inp[k].cuda() for k in FN]
        out, h = ltc_cuda.ltc_cuda_forward(*args, 6, 1e-8)
    s.synchronize()
    assert (out.cpu() - c.a["out"]).abs().max().item() < FWD_ATOL


def test_saturated_sigmoids_finite():
    """test_ltc_cuda.py:209-223: sigma = 100 must stay finite."""
    m = ltc_layer.TrueLiquidTimeConstant(32, 16).cuda()
    with torch.no_grad():
        m.sigma.fill_(100.0)
        m.sensory_sigma.fill_(100.0)
    x = torch.randn(2, 4, 32, device="cuda") * 10.0
    out, (h, _) = m(x)
    assert torch.isfinite(out).all() and torch.isfinite(h).all()
    out.sum().backward()
    for n, p in m.named_parameters():
        assert torch.isfinite(p.grad).all(), n


def test_long_rollout_finite():
    """test_ltc_cuda.py:322-336: a 100-step rollout stays finite."""
    m = ltc_layer.TrueLiquidTimeConstant(32, 16).cuda()
    with torch.no_grad():
        out, (h, _) = m(torch.randn(2, 100, 32, device="cuda"))
    assert torch.isfinite(out).all() and torch.isfinite(h).all()


def test_cpu_input_raises():
    m = ltc_layer.TrueLiquidTimeConstant(8, 4)
    with pytest.raises(RuntimeError):
        m(torch.randn(1, 2, 8))


def test_full_c3_gradient_linearity():
    """Size-independent property at the full c3 size: the backward pass is linear in
    the upstream gradient, grads(a*g1 + g2) = a*grads(g1) + grads(g2)."""
    c = synth.CONFIGS["c3"]
    p, x = synth.make_workload(c)
    from oracle import ltc_oracle as orc
    inp = {k: v.detach().cuda() for k, v in orc.module_preamble(p, x, c.dt, c.U).items()}
    inp["state"] = torch.zeros(c.B, c.H, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(3)
    g1 = torch.randn(c.B, c.T, c.H, device="cuda", generator=g)
    g2 = torch.randn(c.B, c.T, c.H, device="cuda", generator=g)
    _, _, a = cuda_solver(inp, c.U, 1e-8, gout=g1)
    _, _, b = cuda_solver(inp, c.U, 1e-8, gout=g2)
    _, _, ab = cuda_solver(inp, c.U, 1e-8, gout=2.0 * g1 + g2)
    for k in FN:
        ref = 2.0 * a[k].double() + b[k].double()
        err = (ab[k].double() - ref).abs().max().item()
        assert err <= 1e-4 * ref.abs().max().item() + 1e-6, f"{k}: {err:.3e}"


def test_streaming_inference_matches_full_sequence():
    """Inference fast path (eval mode, no_grad, cached transforms): feeding the sequence in
    chunks with the carried state (test_ltc_verification.py:126-140 usage) reproduces the
    full-sequence outputs bitwise."""
    torch.manual_seed(5)
    m = ltc_layer.TrueLiquidTimeConstant(48, 64).cuda().eval()
    x = torch.randn(6, 20, 48, device="cuda")
    with torch.no_grad():
        full, (hf, _) = m(x)
        state, outs = None, []
        for t0 in range(0, 20, 7):
            # the preamble normalises each (b, t) row on its own, so chunking is exact
            o, state = m(x[:, t0:t0 + 7], state)
            outs.append(o)
    assert m._cached_transforms is not None
    assert torch.equal(torch.cat(outs, 1), full)
    assert torch.equal(state[0], hf)


@pytest.mark.parametrize("B,H", [(9000, 64), (5000, 128), (1500, 256)])
def test_multi_wave_grid_vs_oracle(B, H):
    """Batches beyond one wave of resident sample groups (the per-CTA sample count is
    capped by shared memory) run as several waves; check them against the oracle."""
    D, T, U = 8, 2, 3
    p = synth.make_params(D, H, 0.5, 0.5, seed=B)
    from oracle import ltc_oracle as orc
    x = torch.randn(B, T, D, generator=torch.Generator().manual_seed(1))
    inp = {k: v.detach() for k, v in orc.module_preamble(p, x, 1 / 30, U).items()}
    inp["state"] = torch.randn(B, H, generator=torch.Generator().manual_seed(2)) * 0.3
    pl = ltc_cuda.plan(ltc_cuda.make_dims(B, T, D, H, U, 1e-8))
    assert pl.fwd_ctas > 148 or pl.bwd_ctas > 148  # really more than one wave
    gout = torch.randn(B, T, H, generator=torch.Generator().manual_seed(3))
    out, h, g = cuda_solver(inp, U, 1e-8, gout=gout)
    ro, rh, rg = oracle_solver(inp, U, 1e-8, gout=gout, device="cuda", chunk=1000)
    assert (out.cpu() - ro.cpu()).abs().max().item() < FWD_ATOL
    assert_grads_close(g, rg, ctx=f"multi-wave B{B} H{H}")
