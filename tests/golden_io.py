"""Helpers to load the golden fixtures under ``tests/golden``."""

from __future__ import annotations

import os

import numpy as np
import torch

from fsctep_b200.weights import seeded_state_dict

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLDEN, name), allow_pickle=False)


def model_case(tag, dtype=torch.float64, prefix="ictd_model"):
    z = load(f"{prefix}_{tag}.npz")
    shapes = {k[len("sdshape/"):]: tuple(int(x) for x in z[k]) for k in z.files if k.startswith("sdshape/")}
    sd = seeded_state_dict(shapes, int(z["sd_seed"]), torch.float64)
    close = lambda a, b: abs(a - b) <= 1e-9 * max(1.0, abs(b))  # noqa: E731
    for k in list(sd):
        want = float(z[f"sdsum/{k}"])
        if close(float(sd[k].sum()), want):
            continue
        # a module registered under two names (pure_cartesian_sparse_layers.py: e3_conv_emb is
        # e3_conv_layers[0]) shares its tensors: the key loaded last wins
        alias = [k2 for k2, v2 in sd.items() if k2 != k and tuple(v2.shape) == tuple(sd[k].shape)
                 and close(float(v2.sum()), want)]
        if not alias:
            raise AssertionError(f"seeded state_dict mismatch for {k}: {float(sd[k].sum())} vs {want}")
        sd[k] = sd[alias[0]]
    sd = {k: v.to(dtype) for k, v in sd.items()}
    cfg = {k[4:]: z[k].item() for k in z.files if k.startswith("cfg_")}
    case = {k: z[k] for k in z.files if not (k.startswith("sd") or k.startswith("cfg_"))}
    return cfg, sd, case


def o3_case(tag, dtype=torch.float64):
    """(cfg, state_dict, case) of an ``ictd_o3_<tag>.npz`` fixture."""
    return model_case(tag, dtype, prefix="ictd_o3")


def sparse_case(tag, dtype=torch.float64):
    """(cfg, state_dict, case) of a ``sparse_<tag>.npz`` fixture."""
    return model_case(tag, dtype, prefix="sparse")
