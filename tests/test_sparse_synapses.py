"""GPU parity of the zero-synapse-skipping path (LTC_FLAG_SKIP_ZERO_SYNAPSES, H <= 64).

With the flag, the solver visits only synapses whose w_pos or w_erev is nonzero.
Every output must match the reference restatement (the oracle, and the golden
fixtures the reference produced) exactly as the dense path does, except the
gradients of w_pos / w_erev at the skipped positions, which are zero by contract
(mu / sigma gradients are zero there in the dense solve as well, since dL/dz = 0).
Module-level gradients -- what training uses -- are unaffected: the module multiplies
those entries by its mask.  Tolerances are the parity tests' (forward max-abs 1e-3,
gradients rtol 5e-2 / atol 1e-2, normalised error < 2e-3).
"""
import pytest
import torch

import ltc_cuda
import ltc_layer
import synth
from golden_io import Case, FN, case_names
from ltc_testlib import FWD_ATOL, assert_grads_close, cuda_solver, oracle_solver, rel_err
from oracle import ltc_oracle as orc

pytestmark = pytest.mark.gpu

SMALL_H = [n for n in case_names() if Case(n).meta["H"] <= 64]


def _sparse_solver(inp, U, eps, gout=None, gh=None, backward=True):
    with ltc_cuda.skip_zero_synapses():
        return cuda_solver(inp, U, eps, gout=gout, gh=gh, backward=backward)


def _expect_masked(ref, inp):
    """Oracle gradients with the skipped positions' w_pos / w_erev entries zeroed."""
    zero = (inp["w_pos"] == 0) & (inp["w_erev"] == 0)
    out = dict(ref)
    for k in ("w_pos", "w_erev"):
        out[k] = torch.where(zero.to(ref[k].device), torch.zeros_like(ref[k]), ref[k])
    for k in ("mu", "sigma"):  # exactly zero in the dense solve too
        assert float(ref[k].to(zero.device)[zero].abs().max().item() if zero.any() else 0.0) < 1e-12, k
    return out


def _check(inp, U, gout, gh, ctx, device="cpu", chunk=None):
    out, h, g = _sparse_solver(inp, U, 1e-8, gout=gout, gh=gh)
    ro, rh, rg = oracle_solver(inp, U, 1e-8, gout=gout, gh=gh, device=device, chunk=chunk)
    assert (out.cpu() - ro.cpu()).abs().max().item() < FWD_ATOL, ctx
    assert (h.cpu() - rh.cpu()).abs().max().item() < FWD_ATOL, ctx
    rg = _expect_masked({k: v.cpu() for k, v in rg.items()}, {k: v.cpu() for k, v in inp.items()})
    assert_grads_close(g, rg, ctx=ctx)
    for k in FN:
        assert rel_err(g[k], rg[k]) < 2e-3, f"{ctx} {k}: {rel_err(g[k], rg[k]):.2e}"
    return out, h, g


def test_plan_uses_sparse_kernels():
    dims = ltc_cuda.make_dims(64, 4, 16, 64, 6, 1e-8, ltc_cuda.LTC_FLAG_SKIP_ZERO_SYNAPSES)
    assert ltc_cuda.plan(dims).bwd_workspace_bytes > ltc_cuda.plan(ltc_cuda.make_dims(64, 4, 16, 64, 6, 1e-8)).bwd_workspace_bytes


@pytest.mark.parametrize("name", SMALL_H)
def test_golden_solver_level_sparse(name):
    c = Case(name)
    if "gout" not in c.a:
        out, h, _ = _sparse_solver(c.solver_inputs, c.meta["U"], c.meta["epsilon"], backward=False)
        assert (out.cpu() - c.a["out"]).abs().max().item() < FWD_ATOL
        return
    out, h, g = _sparse_solver(c.solver_inputs, c.meta["U"], c.meta["epsilon"], gout=c.get("gout"), gh=c.get("gh"))
    assert (out.cpu() - c.a["out"]).abs().max().item() < FWD_ATOL
    assert (h.cpu() - c.a["h"]).abs().max().item() < FWD_ATOL
    ref = _expect_masked(c.solver_grads, c.solver_inputs)
    assert_grads_close(g, ref, ctx=name)
    for k in FN:
        assert rel_err(g[k], ref[k]) < 1e-3, f"{name} {k}: {rel_err(g[k], ref[k]):.2e}"


def _inputs(D, H, B, T, U, density, seed, mask=None):
    p = synth.make_params(D, H, density, 0.5, seed=seed)
    if mask is not None:
        p["sparsity_mask"] = mask
        p["erev"] = p["erev"].abs().clamp_min(1.0) * torch.where(torch.rand(H, H) < 0.5, 1.0, -1.0) * mask
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, D, generator=g)
    inp = {k: v.detach() for k, v in orc.module_preamble(p, x, 1 / 30, U).items()}
    inp["state"] = torch.randn(B, H, generator=g) * 0.3
    return inp, torch.randn(B, T, H, generator=g), torch.randn(B, H, generator=g)


@pytest.mark.parametrize("H,density", [(64, 0.5), (64, 0.2), (48, 0.5), (33, 0.5), (32, 0.5), (32, 1.0),
                                       (17, 0.3), (8, 0.5), (1, 1.0)])
def test_densities_vs_oracle(H, density):
    inp, gout, gh = _inputs(12, H, 9, 5, 4, density, seed=H * 7 + int(density * 10))
    _check(inp, 4, gout, gh, f"H{H} d{density}")


def test_capacity_boundary_48_per_neuron():
    """Every row and column at exactly the capacity (48 of 64): a circulant band."""
    H = 64
    idx = torch.arange(H)
    mask = (((idx[None, :] - idx[:, None]) % H) < ltc_cuda.SKIP_MAX_SYNAPSES_PER_NEURON).float()
    assert ltc_cuda.skip_zero_synapses_fits(mask)
    inp, gout, gh = _inputs(10, H, 7, 4, 3, 0.5, seed=17, mask=mask)
    _check(inp, 3, gout, gh, "capacity")


def test_over_capacity_gives_nan_and_module_falls_back():
    """A mask beyond the capacity poisons the outputs with NaN (a loud failure, not a
    wrong number); the module checks the mask and runs the dense kernels instead."""
    H = 64
    mask = (torch.rand(H, H, generator=torch.Generator().manual_seed(9)) < 0.5).float()
    mask[3, :50] = 1.0
    assert not ltc_cuda.skip_zero_synapses_fits(mask)
    inp, gout, gh = _inputs(10, H, 5, 3, 3, 0.5, seed=19, mask=mask)
    out, h, g = _sparse_solver(inp, 3, 1e-8, gout=gout, gh=gh)
    assert torch.isnan(out).all() and torch.isnan(h).all()
    assert all(torch.isnan(g[k]).any() for k in ("x_seq", "w_pos", "mu", "cm_t"))
    torch.manual_seed(8)
    m = ltc_layer.TrueLiquidTimeConstant(16, H, sparsity=0.9).cuda()
    assert not ltc_cuda.skip_zero_synapses_fits(m.sparsity_mask)
    out, (hh, _) = m(torch.randn(3, 4, 16, device="cuda"))
    out.sum().backward()
    assert torch.isfinite(out).all() and all(torch.isfinite(q.grad).all() for q in m.parameters())


def test_empty_rows_and_columns():
    """Neurons with no outgoing (rows) or incoming (columns) synapses, and an all-zero block."""
    H = 64
    mask = (torch.rand(H, H, generator=torch.Generator().manual_seed(3)) < 0.5).float()
    mask[5] = 0.0
    mask[:, 9] = 0.0
    mask[40:, :] = 0.0
    inp, gout, gh = _inputs(8, H, 6, 4, 3, 0.5, seed=11, mask=mask)
    _check(inp, 3, gout, gh, "empty rows/cols")
    inp0, gout0, gh0 = _inputs(8, H, 6, 4, 3, 0.5, seed=12, mask=torch.zeros(H, H))
    _check(inp0, 3, gout0, gh0, "all-zero mask")


@pytest.mark.parametrize("cfg,B,T", [("c1", 16, None), ("c3", 64, 32)])
def test_configs_vs_oracle(cfg, B, T):
    c = synth.CONFIGS[cfg]
    p, x = synth.make_workload(c, batch=B)
    if T is not None:
        x = x[:, :T].contiguous()
    inp = {k: v.detach() for k, v in orc.module_preamble(p, x, c.dt, c.U).items()}
    inp["state"] = torch.zeros(x.shape[0], c.H)
    g = torch.Generator().manual_seed(7)
    _check(inp, c.U, torch.randn(x.shape[0], x.shape[1], c.H, generator=g), None, cfg)


def test_multi_wave_and_odd_batch():
    inp, gout, gh = _inputs(8, 64, 6001, 2, 3, 0.5, seed=5)
    _check(inp, 3, gout, gh, "B6001", device="cuda", chunk=1500)


def test_determinism_and_batch_split():
    inp, gout, gh = _inputs(16, 64, 300, 6, 6, 0.5, seed=21)
    runs = [_sparse_solver(inp, 6, 1e-8, gout=gout, gh=gh) for _ in range(2)]
    assert torch.equal(runs[0][0], runs[1][0])
    for k in FN:
        assert torch.equal(runs[0][2][k], runs[1][2][k]), k
    part = {k: (v[100:200] if k in ("x_seq", "state") else v) for k, v in inp.items()}
    o, h, _ = _sparse_solver(part, 6, 1e-8, backward=False)
    assert torch.equal(o, runs[0][0][100:200])


def test_lean_save_with_sparse():
    inp, gout, gh = _inputs(16, 64, 40, 9, 3, 0.5, seed=31)
    ref = _sparse_solver(inp, 3, 1e-8, gout=gout, gh=gh)
    ltc_cuda.set_lean_save(True, chunk_steps=4)
    try:
        got = _sparse_solver(inp, 3, 1e-8, gout=gout, gh=gh)
    finally:
        ltc_cuda.set_lean_save(False)
    assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1])
    for k in FN:
        assert rel_err(got[2][k], ref[2][k]) < 1e-5, k


def test_module_grads_match_dense_path():
    """Module level: the skipping path gives the same parameter gradients as the dense one."""
    torch.manual_seed(4)
    m = ltc_layer.TrueLiquidTimeConstant(40, 64, sparsity=0.4).cuda()
    assert m.skip_zero_synapses
    x = torch.randn(128, 40, 40, device="cuda")  # B*T above ltc_layer.SKIP_MIN_ROWS
    grads = []
    for skip in (True, False):
        m.skip_zero_synapses = skip
        m.zero_grad()
        out, (h, _) = m(x)
        (out.sum() + h.square().sum()).backward()
        grads.append({n: q.grad.clone() for n, q in m.named_parameters()})
    for n in grads[0]:
        a, b = grads[0][n], grads[1][n]
        assert rel_err(a, b) < 1e-5, f"{n}: {rel_err(a, b):.3e}"  # summation order only


# ---- 128 < H <= 512: cluster kernels with resident synapse lists ----------------------

@pytest.mark.parametrize("H,density,B,T,U", [(160, 0.3, 9, 5, 3), (256, 0.4, 13, 3, 4), (512, 0.2, 10, 3, 3),
                                             (300, 0.2, 70, 2, 2), (512, 0.2, 33, 2, 12)])
def test_wide_densities_vs_oracle(H, density, B, T, U):
    inp, gout, gh = _inputs(24, H, B, T, U, density, seed=H + B)
    assert ltc_cuda.skip_zero_synapses_fits(inp["w_pos"])
    _check(inp, U, gout, gh, f"wide H{H} d{density} B{B}", device="cuda")


def test_wide_plan_and_capacity():
    H = 512
    mask = (torch.rand(H, H, generator=torch.Generator().manual_seed(2)) < 0.2).float()
    assert ltc_cuda.skip_zero_synapses_fits(mask)
    over = mask.clone()
    over[7, :300] = 1.0  # 300 nonzero synapses leave neuron 7: beyond what a lane pair holds
    assert not ltc_cuda.skip_zero_synapses_fits(over)
    inp, gout, gh = _inputs(8, H, 5, 2, 2, 0.2, seed=3, mask=over)
    out, h, g = _sparse_solver(inp, 2, 1e-8, gout=gout, gh=gh)
    assert torch.isnan(out).all() and torch.isnan(g["w_pos"]).any()


def test_wide_c4_slice_vs_oracle():
    c = synth.CONFIGS["c4"]
    p, x = synth.make_workload(c, batch=4)
    x = x[:, :16].contiguous()
    inp = {k: v.detach() for k, v in orc.module_preamble(p, x, c.dt, c.U).items()}
    inp["state"] = torch.zeros(4, c.H)
    _check(inp, c.U, None, None, "c4 slice", device="cuda")


def test_wide_determinism_and_lean():
    inp, gout, gh = _inputs(16, 384, 40, 5, 3, 0.2, seed=41)
    a = _sparse_solver(inp, 3, 1e-8, gout=gout, gh=gh)
    b = _sparse_solver(inp, 3, 1e-8, gout=gout, gh=gh)
    assert torch.equal(a[0], b[0])
    for k in FN:
        assert torch.equal(a[2][k], b[2][k]), k
    ltc_cuda.set_lean_save(True, chunk_steps=2)
    try:
        c = _sparse_solver(inp, 3, 1e-8, gout=gout, gh=gh)
    finally:
        ltc_cuda.set_lean_save(False)
    assert torch.equal(c[0], a[0])
    for k in FN:
        assert rel_err(c[2][k], a[2][k]) < 1e-5, k


@pytest.mark.parametrize("D", [40, 300, 600, 700])
def test_sensory_lists_vs_oracle(D):
    """Skipped sensory synapses: empty and full columns, every shared-memory geometry of
    the sensory list pass (double- and single-buffered tiles of 4 rows per lane, 2 rows
    per lane) and, at D = 700, the dense fallback."""
    H = 64
    p = synth.make_params(D, H, 0.5, 0.3, seed=D)
    smask = p["sensory_sparsity_mask"].clone()
    smask[:, 3] = 0.0       # a column with no input
    smask[:, 5] = 1.0       # a column with every input
    smask[D // 2, :] = 0.0  # an input feeding nothing
    p["sensory_sparsity_mask"] = smask
    g = torch.Generator().manual_seed(D)
    x = torch.randn(7, 6, D, generator=g)
    inp = {k: v.detach() for k, v in orc.module_preamble(p, x, 1 / 30, 3).items()}
    inp["state"] = torch.randn(7, H, generator=g) * 0.3
    _check(inp, 3, torch.randn(7, 6, H, generator=g), torch.randn(7, H, generator=g), f"D{D}")


# ---- sensory backward over the nonzero sensory synapses (LTC_FLAG_SKIP_ZERO_SENSORY) --

def _check_sensory(inp, U, gout, gh, ctx):
    with ltc_cuda.skip_zero_synapses(sensory=True):
        out, h, g = cuda_solver(inp, U, 1e-8, gout=gout, gh=gh)
    ro, rh, rg = oracle_solver(inp, U, 1e-8, gout=gout, gh=gh)
    assert (out.cpu() - ro.cpu()).abs().max().item() < FWD_ATOL, ctx
    rg = {k: v.cpu() for k, v in rg.items()}
    H = inp["w_pos"].shape[0]
    if not 64 < H <= 128:  # 64 < H <= 128 keeps the dense recurrent kernels
        rg = _expect_masked(rg, {k: v.cpu() for k, v in inp.items()})
    zs = inp["sensory_w_pos"].cpu() == 0
    for k in ("sensory_w_pos", "sensory_erev", "sensory_mu", "sensory_sigma"):
        rg[k] = torch.where(zs, torch.zeros_like(rg[k]), rg[k])
        assert float(g[k].cpu()[zs].abs().max().item() if zs.any() else 0.0) == 0.0, f"{ctx} {k} skipped != 0"
    assert_grads_close(g, rg, ctx=ctx)
    for k in FN:
        assert rel_err(g[k], rg[k]) < 2e-3, f"{ctx} {k}: {rel_err(g[k], rg[k]):.2e}"


@pytest.mark.parametrize("D,H,sdens,B,T", [(128, 64, 0.5, 9, 70), (40, 64, 0.3, 5, 20), (100, 48, 0.5, 3, 33),
                                           (70, 32, 1.0, 4, 40), (16, 17, 0.5, 6, 9), (100, 160, 0.3, 5, 14),
                                           (70, 300, 0.3, 6, 11), (130, 512, 0.3, 3, 9), (90, 128, 0.5, 4, 12),
                                           (60, 100, 0.4, 5, 7)])
def test_sensory_backward_vs_oracle(D, H, sdens, B, T):
    """Ragged input chunks (D not a multiple of 64), rows not a multiple of the tile,
    H <= 32 (any pattern), a dense sensory mask at H = 32, H > 64 (several column blocks,
    dx partials summed in the finish kernel), and 64 < H <= 128, where the recurrent
    kernels stay dense."""
    p = synth.make_params(D, H, 0.5 if H <= 64 else 0.2, sdens, seed=D + H)
    g = torch.Generator().manual_seed(D * H)
    x = torch.randn(B, T, D, generator=g)
    inp = {k: v.detach() for k, v in orc.module_preamble(p, x, 1 / 30, 3).items()}
    inp["state"] = torch.randn(B, H, generator=g) * 0.3
    assert ltc_cuda.skip_zero_sensory_fits(p["sensory_sparsity_mask"])
    _check_sensory(inp, 3, torch.randn(B, T, H, generator=g), torch.randn(B, H, generator=g), f"D{D} H{H}")


def test_sensory_capacity_and_module():
    """The fits check mirrors the kernel's capacity; the module turns the sensory path on
    only where it fits, and its gradients then equal the dense path's."""
    d, q = torch.arange(128)[:, None], torch.arange(64)[None, :]
    m = (((q - d) % 64) < 48).float()  # every input feeds 48 columns, every column gets 48 per chunk
    assert ltc_cuda.skip_zero_sensory_fits(m)
    m[3, (3 + 48) % 64] = 1.0  # input 3 feeds 49 columns
    assert not ltc_cuda.skip_zero_sensory_fits(m)
    torch.manual_seed(5)
    mod = ltc_layer.TrueLiquidTimeConstant(72, 64, sparsity=0.4, sensory_sparsity=0.5).cuda()
    assert mod._skip_sensory_fits()
    x = torch.randn(128, 40, 72, device="cuda")
    grads = []
    for skip in (True, False):
        mod.skip_zero_synapses = skip
        mod.zero_grad()
        out, (h, _) = mod(x)
        (out.sum() + h.square().sum()).backward()
        grads.append({n: q.grad.clone() for n, q in mod.named_parameters()})
    for n in grads[0]:
        a, b = grads[0][n], grads[1][n]
        assert rel_err(a, b) < 1e-5, f"{n}: {rel_err(a, b):.3e}"
