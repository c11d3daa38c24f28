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
    for k, v in sd.items():
        want = float(z[f"sdsum/{k}"])
        got = float(v.sum())
        if abs(got - want) > 1e-9 * max(1.0, abs(want)):
            raise AssertionError(f"seeded state_dict mismatch for {k}: {got} vs {want}")
    sd = {k: v.to(dtype) for k, v in sd.items()}
    cfg = {k[4:]: z[k].item() for k in z.files if k.startswith("cfg_")}
    case = {k: z[k] for k in z.files if not (k.startswith("sd") or k.startswith("cfg_"))}
    return cfg, sd, case


def o3_case(tag, dtype=torch.float64):
    """(cfg, state_dict, case) of an ``ictd_o3_<tag>.npz`` fixture."""
    return model_case(tag, dtype, prefix="ictd_o3")
