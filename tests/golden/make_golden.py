"""Generate the golden fixtures from the reference implementation itself.

Run in a checkout that has the reference project available (its directory is
given by ``--reference``); it imports the reference's ``ltc.py`` and runs its
TorchScript solver on CPU.  Each case is written to ``<case>.npz`` beside this
script with:

* ``meta``     -- JSON (shape, dt, ode_unfolds, epsilon, loss kind)
* ``p.<name>`` -- the module state dict used
* ``x``, ``h0`` (optional), ``target`` (optional, MSE loss)
* ``out``, ``h`` -- module forward results
* ``gm.<name>`` -- module parameter gradients (if the case has a backward)
* ``f.<name>``  -- the 13 solver inputs after the module preamble
* ``gout``, ``gh`` -- upstream gradients used at solver level
* ``gf.<name>`` -- the reference's solver-level gradients for
  loss = <gout, out> + <gh, h>, from ``_ltc_forward_loop_jit`` (``ltc.py:68``)

The reference tests' own shapes (``test_ltc_cuda.py``, ``test_ltc_verification.py``)
and the configuration c0 of the benchmark are covered.  Nothing at test time
reads the reference: only these files.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "ltc-cuda_b200"))

# solver inputs that equal a module parameter and so are not stored twice
DERIVED = {"mu": "mu", "sigma": "sigma", "sensory_mu": "sensory_mu",
           "sensory_sigma": "sensory_sigma", "sensory_erev": "sensory_erev", "vleak": "vleak"}

FN = ("x_seq", "state", "w_pos", "w_erev", "mu", "sigma", "sensory_mu", "sensory_sigma",
      "sensory_erev", "sensory_w_pos", "cm_t", "gleak_pos", "vleak")


def build(ltc_mod, D, H, dt, U, dens, sdens, seed, params=None):
    torch.manual_seed(seed)
    m = ltc_mod.TrueLiquidTimeConstant(D, H, dt=dt, ode_unfolds=U, sparsity=dens,
                                       sensory_sparsity=sdens, input_mapping="affine")
    if params is not None:
        m.load_state_dict(params)
    m._force_torchscript = True
    return m


def solver_inputs(m, x, h0):
    xn = m.input_norm(x) * m.input_w + m.input_b
    w_pos = F.softplus(m.w) * m.sparsity_mask
    return {
        "x_seq": xn, "state": h0, "w_pos": w_pos, "w_erev": w_pos * m.erev,
        "mu": m.mu, "sigma": m.sigma, "sensory_mu": m.sensory_mu,
        "sensory_sigma": m.sensory_sigma, "sensory_erev": m.sensory_erev,
        "sensory_w_pos": F.softplus(m.sensory_w) * m.sensory_sparsity_mask,
        "cm_t": F.softplus(m.cm) / (m.dt / m.ode_unfolds),
        "gleak_pos": F.softplus(m.gleak), "vleak": m.vleak,
    }


def case(ltc_mod, name, D, H, B, T, *, dt=1 / 30, U=6, dens=0.5, sdens=0.5, seed=42,
         xseed=123, h0=False, backward="sum", params=None, xscale=1.0, edit=None):
    m = build(ltc_mod, D, H, dt, U, dens, sdens, seed, params)
    if edit is not None:
        edit(m)
    g = torch.Generator().manual_seed(xseed)
    x = torch.randn(B, T, D, generator=g) * xscale
    hs = torch.randn(B, H, generator=g) if h0 else None
    rec = {"x": x}
    if hs is not None:
        rec["h0"] = hs
    target = None
    if backward == "mse":
        target = torch.randn(B, T, H, generator=g) * xscale
        rec["target"] = target
    m.zero_grad(set_to_none=True)
    out, (h, _) = m(x, (hs, hs) if hs is not None else None)
    if backward == "sum":
        out.sum().backward()
    elif backward == "mse":
        F.mse_loss(out, target).backward()
    rec["out"], rec["h"] = out.detach(), h.detach()
    for k, v in m.state_dict().items():
        rec["p." + k] = v.detach().clone()
    if backward != "none":
        for k, v in m.named_parameters():
            if v.grad is not None:
                rec["gm." + k] = v.grad.detach().clone()
    # solver-level inputs and the reference's solver gradients
    state0 = hs if hs is not None else torch.zeros(B, H)
    with torch.no_grad():
        fin = solver_inputs(m, x, state0)
    for k in FN:
        if k in DERIVED:  # identical to a module parameter; the loader restores it
            continue
        rec["f." + k] = fin[k].detach().clone()
    if backward != "none":
        leaves = {k: fin[k].detach().clone().requires_grad_(True) for k in FN}
        fo, fh = ltc_mod._ltc_forward_loop_jit(*[leaves[k] for k in FN], m.ode_unfolds, m.epsilon)
        gout = torch.randn(B, T, H, generator=g)
        gh = torch.randn(B, H, generator=g)
        ((fo * gout).sum() + (fh * gh).sum()).backward()
        rec["gout"], rec["gh"] = gout, gh
        for k in FN:
            rec["gf." + k] = leaves[k].grad.detach().clone()
    meta = dict(name=name, B=B, T=T, D=D, H=H, U=m.ode_unfolds, dt=m.dt, epsilon=m.epsilon,
                backward=backward, h0=bool(h0))
    arrays = {k: v.numpy().astype(np.float32) for k, v in rec.items()}
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrays)
    print(f"{name}: {sum(a.nbytes for a in arrays.values()) / 1e3:.0f} kB")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="directory holding the reference ltc.py")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import ltc as ltc_mod  # the reference module
    assert os.path.dirname(os.path.abspath(ltc_mod.__file__)) == os.path.abspath(args.reference)
    import synth

    # shapes of the reference parity tests (test_ltc_cuda.py)
    case(ltc_mod, "fwd_h0_d32_h16", 32, 16, 4, 8, h0=True, backward="none")
    case(ltc_mod, "single_t_d32_h16", 32, 16, 2, 1, xseed=456, backward="none")
    case(ltc_mod, "zero_state_d32_h16", 32, 16, 4, 4, xseed=789, backward="none")
    case(ltc_mod, "fwd_d224_h64", 224, 64, 24, 8, xseed=101, backward="none")
    case(ltc_mod, "grad_sum_d32_h16", 32, 16, 2, 4, xseed=202)
    for s in (11, 23, 47):
        for sc in (0.1, 1.0, 5.0):
            case(ltc_mod, f"grad_mse_s{s}_x{sc:g}", 48, 24, 3, 6, seed=s, xseed=s, backward="mse",
                 xscale=sc)
    case(ltc_mod, "saturated_d32_h16", 32, 16, 2, 4, xseed=303, xscale=10.0,
         edit=lambda m: (m.sigma.data.fill_(100.0), m.sensory_sigma.data.fill_(100.0)))
    for H in (17, 33, 63, 65):
        case(ltc_mod, f"odd_h{H}", 32, H, 4, 4, xseed=808, backward="sum" if H in (33, 63) else "none")
    # module-spec shapes (test_ltc_verification.py): dt=0.1, tiny, and ode_unfolds=1
    case(ltc_mod, "verif_d10_h8", 10, 8, 3, 5, dt=0.1, xseed=5)
    case(ltc_mod, "unfold1_d10_h8", 10, 8, 1, 3, dt=1 / 30, U=1, xseed=6)
    # benchmark configuration c0, full, with the synthetic generator's parameters
    c0 = synth.CONFIGS["c0"]
    p0, x0 = synth.make_workload(c0)
    case(ltc_mod, "c0_full", c0.D, c0.H, c0.B, c0.T, params=p0, xseed=1000)
    # large-H shapes on tiny batches (c2 and c4 parameter distributions)
    c2 = synth.CONFIGS["c2"]
    p2 = synth.make_params(16, 128, c2.density, c2.sensory_density, 1002)
    case(ltc_mod, "h128_d16", 16, 128, 2, 3, params=p2, xseed=1002)
    p4 = synth.make_params(16, 160, 0.2, 0.3, 1004)
    case(ltc_mod, "h160_d16_u12", 16, 160, 1, 2, U=12, dens=0.2, sdens=0.3, params=p4, xseed=1004)


if __name__ == "__main__":
    main()
