"""Shared helpers of the GPU parity tests."""

import numpy as np
import pytest
import torch

import golden_io
from fsctep_b200.ictd import ICTDConfig, ICTDEngine, GraphCSR

needs_gpu = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")

# Tolerances of the north star: energies relative 1e-5, forces and stress relative 1e-4 (fp32).
E_RTOL = 1e-5
F_RTOL = 1e-4
S_RTOL = 1e-4


def rel_max(a, b):
    a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


def golden_engine(tag):
    cfg, sd, c = golden_io.model_case(tag)
    icfg = ICTDConfig(channels=int(cfg["channels"]), lmax=int(cfg["lmax"]),
                      num_interaction=int(cfg["num_interaction"]), number_of_basis=int(cfg["number_of_basis"]),
                      max_radius=float(cfg["max_radius"]), function_type=str(cfg["function_type"]),
                      max_atomvalue=int(cfg["max_atomvalue"]))
    eng = ICTDEngine(sd, icfg, "cuda")
    dev = torch.device("cuda")
    g = GraphCSR.from_edges(torch.tensor(c["edge_src"], device=dev).long(),
                            torch.tensor(c["edge_dst"], device=dev).long(),
                            torch.tensor(c["edge_shifts"], device=dev).float(), int(c["pos"].shape[0]))
    inputs = (torch.tensor(c["pos"], device=dev), torch.tensor(c["Z"], device=dev),
              torch.tensor(c["batch"], device=dev), torch.tensor(c["cell"], device=dev))
    return eng, g, inputs, c, icfg, sd
