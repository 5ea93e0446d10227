"""GPU: memory-lean training (LTC_FLAG_LEAN_SAVE).  The forward keeps only the state at
each step boundary and the backward recomputes the unfolds segment by segment; the
results must equal the full-save path (forward bitwise, gradients up to the order of
the cross-segment partial sums) on every kernel family, and match the oracle."""
import pytest
import torch

import ltc_cuda
import synth
from golden_io import FN
from ltc_testlib import FWD_ATOL, assert_grads_close, cuda_solver, oracle_solver
from oracle import ltc_oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def restore_modes():
    yield
    ltc_cuda.set_lean_save(False)
    ltc_cuda.set_force_wide(False)


def _inputs(B, T, D, H, U, seed):
    p = synth.make_params(D, H, 0.5, 0.5, seed=seed)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, D, generator=g)
    inp = {k: v.detach() for k, v in orc.module_preamble(p, x, 1 / 30, U).items()}
    inp["state"] = torch.randn(B, H, generator=g) * 0.3
    gout = torch.randn(B, T, H, generator=g)
    gh = torch.randn(B, H, generator=g)
    return inp, gout, gh


CASES = [  # (B, T, D, H, U, wide, chunk): register-resident, cluster, streamed, forced wide
    (64, 9, 16, 64, 3, False, 2),
    (40, 7, 8, 128, 2, False, 3),
    (24, 5, 8, 256, 2, False, 2),
    (16, 4, 8, 512, 2, False, 3),
    (48, 6, 16, 40, 3, True, 4),
    (33, 8, 12, 17, 4, False, 0),   # library-sized segments (one segment here)
    (20, 11, 10, 64, 2, False, 1),  # one step per segment
]


@pytest.mark.parametrize("B,T,D,H,U,wide,chunk", CASES)
def test_lean_matches_full_save(B, T, D, H, U, wide, chunk):
    inp, gout, gh = _inputs(B, T, D, H, U, seed=B + 3 * T + H)
    ltc_cuda.set_force_wide(wide)
    out_f, h_f, g_f = cuda_solver(inp, U, 1e-8, gout=gout, gh=gh)
    ltc_cuda.set_lean_save(True, chunk)
    out_l, h_l, g_l = cuda_solver(inp, U, 1e-8, gout=gout, gh=gh)
    assert torch.equal(out_f, out_l) and torch.equal(h_f, h_l)
    for k in FN:
        a, b = g_l[k].double(), g_f[k].double()
        err = (a - b).abs().max().item() / max(b.abs().max().item(), 1e-12)
        assert err < 1e-5, f"lean vs full {k}: rel err {err:.2e}"
    ro, rh, rg = oracle_solver(inp, U, 1e-8, gout=gout, gh=gh)
    assert (out_l.cpu() - ro).abs().max().item() < FWD_ATOL
    assert_grads_close(g_l, rg, ctx=f"lean B{B} T{T} H{H}")


def test_lean_plan_saves_step_states_only():
    B, T, D, H, U = 256, 64, 32, 128, 6
    full = ltc_cuda.plan(ltc_cuda.make_dims(B, T, D, H, U, 1e-8))
    lean = ltc_cuda.plan(ltc_cuda.make_dims(B, T, D, H, U, 1e-8, ltc_cuda.LTC_FLAG_LEAN_SAVE))
    assert lean.saved_bytes == (T + 1) * B * H * 4 + 256
    assert full.saved_bytes == (2 * T * U + 1) * B * H * 4 + 256
    assert 1 <= lean.lean_chunk_steps <= T and full.lean_chunk_steps == 0
    fixed = ltc_cuda.plan(ltc_cuda.make_dims(B, T, D, H, U, 1e-8,
                                             ltc_cuda.LTC_FLAG_LEAN_SAVE | (5 << ltc_cuda.LTC_LEAN_CHUNK_SHIFT)))
    assert fixed.lean_chunk_steps == 5


def test_lean_mode_is_remembered_by_the_backward():
    """A forward run in lean mode is differentiated in lean mode even if the switch
    changed in between (and the other way round)."""
    B, T, D, H, U = 12, 6, 8, 64, 2
    inp, gout, _ = _inputs(B, T, D, H, U, seed=5)
    _, _, ref = cuda_solver(inp, U, 1e-8, gout=gout)
    for first in (True, False):
        ltc_cuda.set_lean_save(first, 2)
        leaves = {k: inp[k].cuda().clone().requires_grad_(True) for k in FN}
        out, _ = ltc_cuda.ltc_cuda_forward(*[leaves[k] for k in FN], U, 1e-8)
        ltc_cuda.set_lean_save(not first, 2)
        g = torch.autograd.grad((out * gout.cuda()).sum(), [leaves[k] for k in FN])
        for k, a in zip(FN, g):
            b = ref[k]
            assert (a - b).abs().max().item() <= 1e-5 * max(b.abs().max().item(), 1e-12), k


def test_lean_zero_initial_state():
    """Zero initial state through the lean path."""
    B, T, D, H, U = 10, 5, 8, 64, 3
    inp, gout, _ = _inputs(B, T, D, H, U, seed=9)
    inp["state"] = torch.zeros(B, H)
    _, _, ref = cuda_solver(inp, U, 1e-8, gout=gout)
    ltc_cuda.set_lean_save(True, 2)
    _, _, got = cuda_solver(inp, U, 1e-8, gout=gout)
    for k in FN:
        assert (got[k] - ref[k]).abs().max().item() <= 1e-5 * max(ref[k].abs().max().item(), 1e-12), k
