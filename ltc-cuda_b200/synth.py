"""Seeded synthetic workloads for the LTC solver (the benchmark configurations).

The reference measures on no public dataset; these generators produce inputs
and module parameters with the distributions the benchmark configurations
name: x ~ N(0,1); sigma ~ U(3,8); mu ~ U(0.3,0.8); w ~ U(0.001,1);
gleak ~ U(0.001,1); vleak ~ U(-0.2,0.2); cm ~ U(0.4,0.6); sensory parameters
drawn the same way; masks Bernoulli(density) with at least one input per
neuron (as the reference wiring does, ``ltc.py:193-203``); reversal potentials
uniform in {-1,+1} times the mask; LayerNorm and input affine at their
defaults (weight 1, bias 0).  A CPU ``torch.Generator`` seeded with
``1000 + config index`` makes every run reproduce the same tensors.
"""
from __future__ import annotations

import dataclasses
from typing import Dict, Optional

import torch


@dataclasses.dataclass(frozen=True)
class LtcConfig:
    name: str
    B: int
    T: int
    D: int
    H: int
    U: int
    density: float
    sensory_density: float
    dt: float = 1.0 / 30.0
    training_step: bool = False  # includes the optimizer step in the timed step

    @property
    def synapses_per_step(self) -> int:
        """Synapse visits per (sample, timestep): D*H sensory + U*H*H recurrent."""
        return self.D * self.H + self.U * self.H * self.H


CONFIGS = {
    "c0": LtcConfig("c0", 24, 8, 128, 64, 6, 0.5, 0.5),
    "c1": LtcConfig("c1", 16, 32, 128, 64, 6, 0.5, 0.5),
    "c2": LtcConfig("c2", 256, 64, 256, 128, 6, 0.5, 0.5),
    "c3": LtcConfig("c3", 4096, 128, 128, 64, 6, 0.5, 0.5, training_step=True),
    "c4": LtcConfig("c4", 1024, 256, 512, 512, 12, 0.2, 0.3),
}


def _mask(g: torch.Generator, rows: int, cols: int, density: float) -> torch.Tensor:
    if density >= 1.0:
        return torch.ones(rows, cols)
    m = (torch.rand(rows, cols, generator=g) < density).float()
    for c in range(cols):
        if not bool(m[:, c].any()):
            m[int(torch.randint(0, rows, (1,), generator=g)), c] = 1.0
    return m


def _u(g, shape, lo, hi):
    return torch.empty(*shape).uniform_(lo, hi, generator=g)


def make_params(D: int, H: int, density: float, sensory_density: float,
                seed: int) -> Dict[str, torch.Tensor]:
    """Module state dict (names as the reference module registers them)."""
    g = torch.Generator().manual_seed(seed)
    mask = _mask(g, H, H, density)
    smask = _mask(g, D, H, sensory_density)
    erev = torch.where(torch.rand(H, H, generator=g) < 0.5, 1.0, -1.0) * mask
    serev = torch.where(torch.rand(D, H, generator=g) < 0.5, 1.0, -1.0) * smask
    return {
        "w": _u(g, (H, H), 0.001, 1.0),
        "mu": _u(g, (H, H), 0.3, 0.8),
        "sigma": _u(g, (H, H), 3.0, 8.0),
        "erev": erev,
        "sparsity_mask": mask,
        "sensory_w": _u(g, (D, H), 0.001, 1.0),
        "sensory_mu": _u(g, (D, H), 0.3, 0.8),
        "sensory_sigma": _u(g, (D, H), 3.0, 8.0),
        "sensory_erev": serev,
        "sensory_sparsity_mask": smask,
        "gleak": _u(g, (H,), 0.001, 1.0),
        "vleak": _u(g, (H,), -0.2, 0.2),
        "cm": _u(g, (H,), 0.4, 0.6),
        "input_w": torch.ones(D),
        "input_b": torch.zeros(D),
        "input_norm.weight": torch.ones(D),
        "input_norm.bias": torch.zeros(D),
    }


def make_inputs(B: int, T: int, D: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed + 7919)
    return torch.randn(B, T, D, generator=g)


def make_workload(cfg: LtcConfig, seed: Optional[int] = None, batch: Optional[int] = None):
    """(params, x) for a configuration; ``batch`` truncates B (same leading samples)."""
    idx = int(cfg.name[1:]) if cfg.name[1:].isdigit() else 0
    s = 1000 + idx if seed is None else seed
    p = make_params(cfg.D, cfg.H, cfg.density, cfg.sensory_density, s)
    x = make_inputs(cfg.B, cfg.T, cfg.D, s)
    if batch is not None and batch < cfg.B:
        x = x[:batch].contiguous()
    return p, x
