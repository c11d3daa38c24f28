"""Deterministic seeded parameters for synthetic benchmarks and parity fixtures.

A freshly constructed reference model predicts E = 0 exactly because its
``RobustScalarWeightedSum`` starts at zero (``models/mlp.py:126-127``), so every
benchmark and parity case sets all parameters from a seeded generator instead.
``seeded_state_dict`` maps a ``{name: shape}`` dict (the reference state_dict
layout) to tensors drawn in sorted-name order from one ``torch.Generator``; the
scale of each family keeps features O(1) through all layers.
"""

from __future__ import annotations

from typing import Dict, Tuple

import torch


def seeded_state_dict(shapes: Dict[str, Tuple[int, ...]], seed: int,
                      dtype: torch.dtype = torch.float64) -> Dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(int(seed))
    out = {}
    for name in sorted(shapes):
        shape = tuple(shapes[name])
        r = torch.randn(shape, generator=g, dtype=torch.float64)
        leaf = name.rsplit(".", 1)[-1]
        if "tp2" in name and leaf == "weight" and len(shape) == 4:
            t = r / (shape[2] * shape[3]) ** 0.5            # path weights (P, o, i, j)
        elif name.startswith("W_read"):
            t = r * 0.05
        elif name == "weighted_sum.weights":
            t = r * 0.3
        elif ("layer_norms" in name or "input_norm" in name) and leaf == "weight":
            t = 1.0 + 0.1 * r
        elif leaf == "bias":
            t = 0.1 * r
        elif "embedding" in name:
            t = r
        elif len(shape) == 2:
            t = r * (2.0 / shape[1]) ** 0.5                # Kaiming-like for Linear (out, in)
        else:
            t = r * 0.1
        out[name] = t.to(dtype)
    return out
