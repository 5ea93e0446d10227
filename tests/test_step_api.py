"""GPU: the step-level calls with the reference's names (ltc_sensory_fwd, ltc_ode_unfold_fwd,
ltc_sensory_bwd, ltc_ode_unfold_bwd; reference csrc/ltc_kernels.cu:675-950) against the oracle,
on the register-resident (H<=64), cluster (H=128) and streamed (H>128) kernel families."""
import pytest
import torch

import ltc_cuda
import synth
from ltc_testlib import FWD_ATOL, GRAD_ATOL, GRAD_RTOL
from oracle import ltc_oracle as orc

pytestmark = pytest.mark.gpu
M = ltc_cuda._cuda_module


def _setup(B, D, H, U, seed):
    p = synth.make_params(D, H, 0.5, 0.5, seed)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, 1, D, generator=g)
    inp = {k: v.detach() for k, v in orc.module_preamble(p, x, 1 / 30, U).items()}
    inp["x_seq"] = inp["x_seq"][:, 0]
    state = torch.randn(B, H, generator=g) * 0.3
    return inp, state, g


def _close(a, b, rtol=GRAD_RTOL, atol=GRAD_ATOL, what=""):
    a, b = a.detach().cpu().double(), b.detach().cpu().double()
    assert torch.allclose(a, b, rtol=rtol, atol=atol), f"{what}: max err {(a - b).abs().max().item():.3e}"


@pytest.mark.parametrize("B,D,H,U", [(5, 12, 16, 6), (9, 40, 64, 3), (3, 20, 96, 2), (2, 16, 200, 2)])
def test_step_calls_match_oracle(B, D, H, U):
    inp, state, g = _setup(B, D, H, U, seed=B * 7 + H)
    sens = [inp[k] for k in ("sensory_sigma", "sensory_mu", "sensory_w_pos", "sensory_erev")]
    rec = [inp[k] for k in ("w_pos", "w_erev", "mu", "sigma")]
    neu = [inp[k] for k in ("cm_t", "gleak_pos", "vleak")]
    cu = lambda ts: [t.cuda() for t in ts]

    # sensory forward
    wn, wd = M.ltc_sensory_fwd(inp["x_seq"].cuda(), *cu(sens))
    rn, rd = orc.sensory_drive(inp["x_seq"], inp["sensory_mu"], inp["sensory_sigma"], inp["sensory_erev"],
                               inp["sensory_w_pos"])
    assert (wn.cpu() - rn).abs().max() < FWD_ATOL and (wd.cpu() - rd).abs().max() < FWD_ATOL

    # unfold forward (state and the input of every unfold)
    out, vbuf = M.ltc_ode_unfold_fwd(state.cuda(), *cu(rec), rn.cuda(), rd.cuda(), *cu(neu), U, 1e-8, True)
    rv, rins = orc.unfold_loop(state, *rec, rn, rd, *neu, U, 1e-8)
    assert (out.cpu() - rv).abs().max() < FWD_ATOL
    assert (vbuf.cpu() - torch.stack(rins)).abs().max() < FWD_ATOL

    # unfold backward against autograd through the oracle unfolds
    go = torch.randn(B, H, generator=g)
    got = M.ltc_ode_unfold_bwd(vbuf, *cu(rec), rn.cuda(), rd.cuda(), *cu(neu), go.cuda(), U, 1e-8)
    leaves = [t.clone().requires_grad_(True) for t in [state, rn, rd] + rec + neu]
    v, _ = orc.unfold_loop(leaves[0], *leaves[3:7], leaves[1], leaves[2], *leaves[7:], U, 1e-8)
    ref = torch.autograd.grad((v * go).sum(), leaves)
    names = ["state", "w_num", "w_den", "w_pos", "w_erev", "mu", "sigma", "cm_t", "gleak", "vleak"]
    for a, b, n in zip(got, ref, names):
        _close(a, b, what=f"unfold bwd {n}")

    # sensory backward against autograd through the oracle sensory drive
    gwn, gwd = torch.randn(B, H, generator=g), torch.randn(B, H, generator=g)
    got = M.ltc_sensory_bwd(gwn.cuda(), gwd.cuda(), inp["x_seq"].cuda(), *cu(sens))
    leaves = [t.clone().requires_grad_(True) for t in [inp["x_seq"]] + sens]
    n_, d_ = orc.sensory_drive(leaves[0], leaves[2], leaves[1], leaves[4], leaves[3])
    ref = torch.autograd.grad((n_ * gwn).sum() + (d_ * gwd).sum(), leaves)
    for a, b, n in zip(got, ref, ["inputs", "sensory_sigma", "sensory_mu", "sensory_w_pos", "sensory_erev"]):
        _close(a, b, what=f"sensory bwd {n}")


def test_stepwise_loop_equals_full_sequence():
    """Driving the time loop with the step calls reproduces ltc_full_forward."""
    B, T, D, H, U = 4, 5, 24, 32, 6
    p = synth.make_params(D, H, 0.5, 0.5, 3)
    x = torch.randn(B, T, D, generator=torch.Generator().manual_seed(4))
    inp = {k: v.detach().cuda() for k, v in orc.module_preamble(p, x, 1 / 30, U).items()}
    h0 = torch.zeros(B, H, device="cuda")
    sens = [inp[k] for k in ("sensory_sigma", "sensory_mu", "sensory_w_pos", "sensory_erev")]
    rec = [inp[k] for k in ("w_pos", "w_erev", "mu", "sigma")]
    neu = [inp[k] for k in ("cm_t", "gleak_pos", "vleak")]
    full = M.ltc_full_forward(inp["x_seq"], h0, *rec, inp["sensory_mu"], inp["sensory_sigma"],
                              inp["sensory_erev"], inp["sensory_w_pos"], *neu, U, 1e-8, False)[0]
    v = h0
    for t in range(T):
        wn, wd = M.ltc_sensory_fwd(inp["x_seq"][:, t].contiguous(), *sens)
        v, _ = M.ltc_ode_unfold_fwd(v, *rec, wn, wd, *neu, U, 1e-8, False)
        assert torch.equal(v, full[:, t]), f"step {t}"
