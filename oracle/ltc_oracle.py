"""CPU oracle for the LTC ODE-solver hot path (TEST INFRASTRUCTURE, not product).

This module restates, in plain PyTorch tensor arithmetic, the algorithm of the
reference's TorchScript solver so that the CUDA product can be checked against
it.  Gradients come from PyTorch autograd over this restatement, exactly as
the reference obtains its TorchScript gradients.  It is imported only by
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs.

Pinning: ``tests/test_oracle_golden.py`` checks this restatement against golden
vectors produced by the reference itself (``ltc.py`` imported from the
reference checkout, fixtures and generating script under ``tests/golden/``).

Reference map (paths inside the reference project):

* :func:`sensory_drive`   -- ``ltc.py:44-47``  (state-independent sensory term)
* :func:`ode_step`        -- ``ltc.py:19-65``  (one timestep, U implicit-Euler unfolds)
* :func:`unfold_loop`     -- ``ltc.py:50-63``  (the unfolds of one step, given its sensory sums)
* :func:`forward_loop`    -- ``ltc.py:68-106`` (outer loop over T)
* :func:`module_preamble` -- ``ltc.py:249-288`` (LayerNorm, affine map, softplus transforms)
"""
from __future__ import annotations

from typing import Dict, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

# Order of the 13 tensor inputs of the solver (and of its 13 gradients), as in
# ``ltc_cuda.py:249-267`` / ``ltc_cuda.py:342-359`` of the reference.
FUNCTION_INPUTS: Tuple[str, ...] = (
    "x_seq", "state", "w_pos", "w_erev", "mu", "sigma",
    "sensory_mu", "sensory_sigma", "sensory_erev", "sensory_w_pos",
    "cm_t", "gleak_pos", "vleak",
)


def sensory_drive(inputs, sensory_mu, sensory_sigma, sensory_erev, sensory_w_pos):
    """Sensory numerator/denominator contributions for one timestep.

    ``inputs`` is (B, D); parameters are (D, H).  Returns ((B,H), (B,H)).
    Follows ``ltc.py:44-47``: sigmoid(sigma*(x - mu)) weighted by w and reduced over D.
    """
    act = torch.sigmoid(sensory_sigma * (inputs.unsqueeze(-1) - sensory_mu))
    w_act = sensory_w_pos * act
    return (w_act * sensory_erev).sum(dim=1), w_act.sum(dim=1)


def ode_step(inputs, state, w_pos, w_erev, mu, sigma,
             sensory_mu, sensory_sigma, sensory_erev, sensory_w_pos,
             cm_t, gleak_pos, vleak, ode_unfolds: int, epsilon: float):
    """One timestep of the fused implicit-Euler solver (``ltc.py:19-65``).

    Recurrent matrices are indexed [pre, post]; the reduction runs over the
    presynaptic axis (dim 1 of the (B, H_pre, H_post) broadcast).
    """
    num_s, den_s = sensory_drive(inputs, sensory_mu, sensory_sigma, sensory_erev, sensory_w_pos)
    return unfold_loop(state, w_pos, w_erev, mu, sigma, num_s, den_s, cm_t, gleak_pos, vleak,
                       ode_unfolds, epsilon)[0]


def unfold_loop(state, w_pos, w_erev, mu, sigma, num_s, den_s, cm_t, gleak_pos, vleak,
                ode_unfolds: int, epsilon: float):
    """The U implicit-Euler unfolds of one step given its sensory sums (``ltc.py:50-63``).

    Returns (final state, [input state of every unfold]).
    """
    v = state
    inputs_of_unfolds = []
    for _ in range(ode_unfolds):
        inputs_of_unfolds.append(v)
        act = torch.sigmoid(sigma * (v.unsqueeze(-1) - mu))
        w_num = (act * w_erev).sum(dim=1) + num_s
        w_den = (w_pos * act).sum(dim=1) + den_s
        numerator = cm_t * v + gleak_pos * vleak + w_num
        denominator = cm_t + gleak_pos + w_den
        v = numerator / (denominator + epsilon)
    return v, inputs_of_unfolds


def forward_loop(x_seq, state, w_pos, w_erev, mu, sigma,
                 sensory_mu, sensory_sigma, sensory_erev, sensory_w_pos,
                 cm_t, gleak_pos, vleak, ode_unfolds: int, epsilon: float,
                 checkpoint: bool = False):
    """Outer time loop (``ltc.py:68-106``).  Returns (outputs (B,T,H), final state (B,H)).

    ``checkpoint=True`` recomputes each timestep in the backward pass
    (``torch.utils.checkpoint``) so that large batches fit in host memory; the
    arithmetic is unchanged.
    """
    B, T, _ = x_seq.shape
    outs = []
    params = (w_pos, w_erev, mu, sigma, sensory_mu, sensory_sigma, sensory_erev,
              sensory_w_pos, cm_t, gleak_pos, vleak)
    for t in range(T):
        if checkpoint:
            state = torch.utils.checkpoint.checkpoint(
                ode_step, x_seq[:, t, :], state, *params, ode_unfolds, epsilon,
                use_reentrant=False)
        else:
            state = ode_step(x_seq[:, t, :], state, *params, ode_unfolds, epsilon)
        outs.append(state)
    return torch.stack(outs, dim=1), state


def module_preamble(p: Dict[str, torch.Tensor], x_seq: torch.Tensor, dt: float,
                    ode_unfolds: int, eps_ln: float = 1e-5):
    """Module-level transforms in front of the solver (``ltc.py:249-288``).

    ``p`` holds the module parameters by their state-dict names.  Returns the
    13 solver inputs except ``state`` as a dict keyed like :data:`FUNCTION_INPUTS`.
    """
    D = x_seq.shape[-1]
    x = F.layer_norm(x_seq, (D,), p["input_norm.weight"], p["input_norm.bias"], eps_ln)
    x = x * p["input_w"] + p["input_b"]
    w_pos = F.softplus(p["w"]) * p["sparsity_mask"]
    return {
        "x_seq": x,
        "w_pos": w_pos,
        "w_erev": w_pos * p["erev"],
        "mu": p["mu"],
        "sigma": p["sigma"],
        "sensory_mu": p["sensory_mu"],
        "sensory_sigma": p["sensory_sigma"],
        "sensory_erev": p["sensory_erev"],
        "sensory_w_pos": F.softplus(p["sensory_w"]) * p["sensory_sparsity_mask"],
        "cm_t": F.softplus(p["cm"]) / (dt / ode_unfolds),
        "gleak_pos": F.softplus(p["gleak"]),
        "vleak": p["vleak"],
    }


def function_forward(inp: Dict[str, torch.Tensor], ode_unfolds: int, epsilon: float,
                     checkpoint: bool = False):
    """Solver forward on a dict of the 13 inputs (names of :data:`FUNCTION_INPUTS`)."""
    return forward_loop(*[inp[k] for k in FUNCTION_INPUTS], ode_unfolds, epsilon,
                        checkpoint=checkpoint)


def function_grads(inp: Dict[str, torch.Tensor], ode_unfolds: int, epsilon: float,
                   grad_out: Optional[torch.Tensor] = None,
                   grad_state: Optional[torch.Tensor] = None,
                   dtype: torch.dtype = torch.float32,
                   checkpoint: bool = False,
                   batch_chunk: Optional[int] = None):
    """Outputs and the 13 solver-input gradients for loss = <grad_out, out> + <grad_state, h>.

    ``grad_out=None`` means the sum loss of the metric (all ones).  Because that
    loss is a sum over samples, gradients are additive over batch chunks;
    ``batch_chunk`` runs the batch in slices and adds their gradients (the large
    configurations would not fit in memory otherwise).  Returns
    (outputs, final_state, {name: grad}).
    """
    B = inp["x_seq"].shape[0]
    chunk = batch_chunk or B
    per_sample = ("x_seq", "state")
    grads: Dict[str, torch.Tensor] = {}
    outs, finals = [], []
    for b0 in range(0, B, chunk):
        b1 = min(B, b0 + chunk)
        leaf = {}
        for k in FUNCTION_INPUTS:
            t = inp[k][b0:b1] if k in per_sample else inp[k]
            leaf[k] = t.detach().to(dtype).clone().requires_grad_(True)
        out, h = function_forward(leaf, ode_unfolds, epsilon, checkpoint=checkpoint)
        go = torch.ones_like(out) if grad_out is None else grad_out[b0:b1].to(dtype)
        loss = (out * go).sum()
        if grad_state is not None:
            loss = loss + (h * grad_state[b0:b1].to(dtype)).sum()
        g = torch.autograd.grad(loss, [leaf[k] for k in FUNCTION_INPUTS])
        for k, gk in zip(FUNCTION_INPUTS, g):
            if k in per_sample:
                grads.setdefault(k, []).append(gk.detach())
            else:
                grads[k] = gk.detach() if k not in grads else grads[k] + gk.detach()
        outs.append(out.detach())
        finals.append(h.detach())
    for k in per_sample:
        grads[k] = torch.cat(grads[k], 0)
    return torch.cat(outs, 0), torch.cat(finals, 0), grads


def module_forward(p: Dict[str, torch.Tensor], x_seq, h0, dt: float, ode_unfolds: int,
                   epsilon: float = 1e-8):
    """Whole module forward (``ltc.py:233-326``) on the TorchScript-equivalent path."""
    B = x_seq.shape[0]
    H = p["w"].shape[0]
    state = torch.zeros(B, H, dtype=x_seq.dtype, device=x_seq.device) if h0 is None else h0
    inp = module_preamble(p, x_seq, dt, ode_unfolds)
    inp["state"] = state
    out, h = function_forward(inp, ode_unfolds, epsilon)
    return out, (h, h)


def parameter_names() -> Sequence[str]:
    """Trainable module parameters, in module registration order (``ltc.py:150-186``)."""
    return ("w", "mu", "sigma", "erev", "sensory_w", "sensory_mu", "sensory_sigma",
            "sensory_erev", "gleak", "vleak", "cm", "input_w", "input_b",
            "input_norm.weight", "input_norm.bias")
