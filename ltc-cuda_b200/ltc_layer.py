"""``TrueLiquidTimeConstant`` with the reference module's constructor and forward contract.

Constructor ``(input_dim, hidden_dim=64, dt=1/30, ode_unfolds=6, sparsity=0.5,
sensory_sparsity=0.5, input_mapping="affine", epsilon=1e-8)`` and
``forward(x_seq, h0=None) -> (outputs (B,T,H), (h, h))`` follow ``ltc.py:128-326``
of the reference; parameter and buffer names match its state dict, so a
reference checkpoint loads unchanged.  The module preamble (LayerNorm, input
affine map, softplus/mask transforms, eval-mode cache) runs in PyTorch; the
solver runs in ``ltc_cuda`` on the GPU.  Unlike the reference there is no
TorchScript fallback: a CPU or non-fp32 input raises.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

import ltc_cuda

# Solver used by forward(); tests may swap in a CPU restatement to exercise the
# host logic (e.g. multi-process data parallel) on machines without a GPU.
_solver: Callable = ltc_cuda.ltc_cuda_forward

# B*T below which the module keeps the dense recurrent kernels even when it may skip
# masked synapses: the per-call slot-table build (tens of microseconds) outweighs the
# saving there (measured on B200: c0/c1, B*T = 192/512, are faster dense)
SKIP_MIN_ROWS = 4096


def set_solver(fn: Optional[Callable]) -> None:
    global _solver
    _solver = ltc_cuda.ltc_cuda_forward if fn is None else fn


def _wiring(rows: int, cols: int, density: float, excitatory: float = 0.8):
    """Bernoulli(density) mask with >= 1 input per neuron and +-1 reversal potentials
    (~80% excitatory), zeroed off the mask (``ltc.py:193-230``)."""
    if density >= 1.0:
        mask = torch.ones(rows, cols)
    else:
        mask = (torch.rand(rows, cols) < density).float()
        for c in range(cols):
            if not bool(mask[:, c].any()):
                mask[int(torch.randint(0, rows, (1,))), c] = 1.0
    erev = torch.where(torch.rand(rows, cols) < excitatory, 1.0, -1.0) * mask
    return mask, erev


class TrueLiquidTimeConstant(nn.Module):
    def __init__(self, input_dim: int, hidden_dim: int = 64, dt: float = 1.0 / 30.0, ode_unfolds: int = 6,
                 sparsity: float = 0.5, sensory_sparsity: float = 0.5, input_mapping: str = "affine",
                 epsilon: float = 1e-8):
        super().__init__()
        self.input_dim = input_dim
        self.hidden_dim = hidden_dim
        self.dt = float(dt)
        self.ode_unfolds = int(max(1, ode_unfolds))
        self.sparsity = sparsity
        self.sensory_sparsity = sensory_sparsity
        self.input_mapping = input_mapping
        self.epsilon = epsilon
        # let the solver skip masked synapses (their solver-level gradients are discarded
        # by the mask); a plain attribute, not part of the state dict
        self.skip_zero_synapses = sparsity < 1.0
        H, D = hidden_dim, input_dim

        self.w = nn.Parameter(torch.empty(H, H).uniform_(0.001, 1.0))
        self.mu = nn.Parameter(torch.empty(H, H).uniform_(0.3, 0.8))
        self.sigma = nn.Parameter(torch.empty(H, H).uniform_(3.0, 8.0))
        mask, erev = _wiring(H, H, sparsity)
        self.register_buffer("sparsity_mask", mask)
        self.erev = nn.Parameter(erev)

        self.sensory_w = nn.Parameter(torch.empty(D, H).uniform_(0.001, 1.0))
        self.sensory_mu = nn.Parameter(torch.empty(D, H).uniform_(0.3, 0.8))
        self.sensory_sigma = nn.Parameter(torch.empty(D, H).uniform_(3.0, 8.0))
        smask, serev = _wiring(D, H, sensory_sparsity)
        self.register_buffer("sensory_sparsity_mask", smask)
        self.sensory_erev = nn.Parameter(serev)

        self.gleak = nn.Parameter(torch.empty(H).uniform_(0.001, 1.0))
        self.vleak = nn.Parameter(torch.empty(H).uniform_(-0.2, 0.2))
        self.cm = nn.Parameter(torch.empty(H).uniform_(0.4, 0.6))

        if input_mapping == "affine":
            self.input_w = nn.Parameter(torch.ones(D))
            self.input_b = nn.Parameter(torch.zeros(D))
        elif input_mapping == "linear":
            self.input_w = nn.Parameter(torch.ones(D))
            self.register_buffer("input_b", torch.zeros(D))
        else:
            self.register_buffer("input_w", torch.ones(D))
            self.register_buffer("input_b", torch.zeros(D))
        self.input_norm = nn.LayerNorm(D)
        self._cached_transforms: Optional[dict] = None

    def _transforms(self):
        if not self.training and self._cached_transforms is not None:
            c = self._cached_transforms
            return c["w_pos"], c["w_erev"], c["cm_t"], c["gleak_pos"], c["sensory_w_pos"]
        w_pos = F.softplus(self.w) * self.sparsity_mask
        w_erev = w_pos * self.erev
        cm_t = F.softplus(self.cm) / (self.dt / self.ode_unfolds)
        gleak_pos = F.softplus(self.gleak)
        sensory_w_pos = F.softplus(self.sensory_w) * self.sensory_sparsity_mask
        if not self.training:
            self._cached_transforms = {"w_pos": w_pos, "w_erev": w_erev, "cm_t": cm_t,
                                       "gleak_pos": gleak_pos, "sensory_w_pos": sensory_w_pos}
        return w_pos, w_erev, cm_t, gleak_pos, sensory_w_pos

    def forward(self, x_seq: torch.Tensor, h0: Optional[Tuple[torch.Tensor, torch.Tensor]] = None):
        B, T, D = x_seq.shape
        state = torch.zeros(B, self.hidden_dim, device=x_seq.device, dtype=x_seq.dtype)
        if h0 is not None:
            state = h0[0]
        if (_solver is ltc_cuda.ltc_cuda_forward and x_seq.is_cuda and x_seq.dtype == torch.float32
                and D <= ltc_cuda.PREAMBLE_MAX_D):
            # LayerNorm + affine map fused in one kernel each way (same arithmetic as below)
            x = ltc_cuda.ltc_preamble(x_seq, self.input_norm.weight, self.input_norm.bias, self.input_w,
                                      self.input_b, self.input_norm.eps)
        else:
            x = self.input_norm(x_seq)
            x = x * self.input_w + self.input_b
        if state.dtype != x.dtype:
            state = state.to(x.dtype)
        w_pos, w_erev, cm_t, gleak_pos, sensory_w_pos = self._transforms()
        if _solver is ltc_cuda.ltc_cuda_forward and not (x.is_cuda and x.dtype == torch.float32):
            raise RuntimeError(f"TrueLiquidTimeConstant: the sm_100a solver needs fp32 CUDA input "
                               f"(got {x.dtype} on {x.device}); there is no CPU fallback")
        # w_pos = softplus(w) * mask: the solver's gradients at masked synapses are
        # multiplied by zero on the way to w and erev, so the solver may skip them
        # (small problems stay dense: rebuilding the slot tables costs more than it saves)
        skip = self.skip_zero_synapses and B * T >= SKIP_MIN_ROWS and self._skip_fits()
        # sensory_w_pos = softplus(sensory_w) * mask: the same holds for the sensory synapses
        with ltc_cuda.skip_zero_synapses(skip, sensory=skip and self._skip_sensory_fits()):
            outputs, state = _solver(x, state, w_pos, w_erev, self.mu, self.sigma, self.sensory_mu,
                                     self.sensory_sigma, self.sensory_erev, sensory_w_pos, cm_t, gleak_pos,
                                     self.vleak, self.ode_unfolds, self.epsilon)
        return outputs, (state, state)

    def _skip_fits(self) -> bool:
        """Whether the solver's synapse-skipping kernels can hold this mask (checked
        once per mask version; one device sync the first time)."""
        m = self.sparsity_mask
        key = (m.data_ptr(), m._version, tuple(m.shape))
        if getattr(self, "_skip_key", None) != key:
            self._skip_ok = ltc_cuda.skip_zero_synapses_fits(m)
            self._skip_key = key
        return self._skip_ok

    def _skip_sensory_fits(self) -> bool:
        """Whether the sensory backward's skipping kernel can hold the sensory mask
        (checked once per mask version)."""
        m = self.sensory_sparsity_mask
        key = (m.data_ptr(), m._version, tuple(m.shape))
        if getattr(self, "_sskip_key", None) != key:
            self._sskip_ok = bool((m == 0).any().item()) and ltc_cuda.skip_zero_sensory_fits(m)
            self._sskip_key = key
        return self._sskip_ok

    def train(self, mode: bool = True):
        if mode:
            self._cached_transforms = None
        return super().train(mode)

    @property
    def W_rec(self) -> nn.Parameter:
        return self.w


TemporalLTC = TrueLiquidTimeConstant
