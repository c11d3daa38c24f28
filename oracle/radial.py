"""Radial basis restatement (test infrastructure only, see ``oracle/__init__``).

The reference calls ``e3nn.math.soft_one_hot_linspace(x, start, end, number,
basis=..., cutoff=True)`` (``models/pure_cartesian_ictd_layers_full.py:464,
930-937``; ``models/pure_cartesian_sparse_layers.py:319-321, 410-412``;
``models/pure_cartesian_ictd_layers_o3.py:524, 953-955``) and multiplies the
result by ``sqrt(number)``.  e3nn (pinned ``e3nn>=0.4.4,<0.6.0``,
``setup.py:81``) is neither vendored nor installed.  This module restates the
published e3nn definition of the basis families:

* grid: ``number`` centres on ``linspace(start, end, number + 2)[1:-1]`` when
  ``cutoff`` (``linspace(start, end, number)`` otherwise), spacing ``step``;
  ``d = (x - centre) / step``;
* ``gaussian``: ``exp(-d^2) / 1.12``;
* ``cosine``: ``cos(pi/2 d)`` on ``|d| < 1``;
* ``smooth_finite``: ``1.14136 e^2 u(d + 1) u(1 - d)`` with the soft unit step
  ``u(t) = exp(-1/t)`` for ``t > 0``;
* ``fourier``: ``sin(pi i y) / sqrt(0.25 + number/2)`` on ``0 < y < 1`` with
  ``y = (x - start)/(end - start)``, ``i = 1..number`` (cutoff form);
* ``bessel``: ``sqrt(2/c) sin(pi i (x - start)/c) / (x - start)`` on
  ``0 < (x - start)/c < 1``, ``c = end - start``, ``i = 1..number``
  (the DimeNet radial Bessel basis, Klicpera et al. 2020).
"""

from __future__ import annotations

import math

import torch


def _soft_unit_step(t: torch.Tensor) -> torch.Tensor:
    z = torch.zeros_like(t)
    safe = torch.where(t > 0, t, torch.ones_like(t))
    return torch.where(t > 0, torch.exp(-1.0 / safe), z)


def soft_one_hot_linspace(x: torch.Tensor, start: float, end: float, number: int,
                          basis: str = "gaussian", cutoff: bool = True) -> torch.Tensor:
    """Restated e3nn ``soft_one_hot_linspace``; returns ``x.shape + (number,)``."""
    if cutoff not in (True, False):
        raise ValueError("cutoff must be specified")
    if cutoff:
        grid = torch.linspace(start, end, number + 2, dtype=x.dtype, device=x.device)
        step = grid[1] - grid[0]
        centres = grid[1:-1]
    else:
        centres = torch.linspace(start, end, number, dtype=x.dtype, device=x.device)
        step = centres[1] - centres[0]
    d = (x[..., None] - centres) / step

    if basis == "gaussian":
        return torch.exp(-d.pow(2)) / 1.12
    if basis == "cosine":
        return torch.cos(math.pi / 2 * d) * (d < 1) * (-1 < d)
    if basis == "smooth_finite":
        return 1.14136 * math.exp(2.0) * _soft_unit_step(d + 1) * _soft_unit_step(1 - d)
    if basis == "fourier":
        y = (x[..., None] - start) / (end - start)
        if not cutoff:
            i = torch.arange(0, number, dtype=x.dtype, device=x.device)
            return torch.cos(math.pi * i * y) / math.sqrt(0.25 + number / 2)
        i = torch.arange(1, number + 1, dtype=x.dtype, device=x.device)
        return torch.sin(math.pi * i * y) / math.sqrt(0.25 + number / 2) * (0 < y) * (y < 1)
    if basis == "bessel":
        xs = x[..., None] - start
        c = end - start
        roots = torch.arange(1, number + 1, dtype=x.dtype, device=x.device) * math.pi
        out = math.sqrt(2 / c) * torch.sin(roots * xs / c) / xs
        if not cutoff:
            return out
        return out * ((xs / c) < 1) * (0 < xs)
    raise ValueError(f'basis="{basis}" is not a valid entry')
