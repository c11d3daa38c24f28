"""Parity of pure-cartesian-sparse at the channel widths of BASELINE configs 2 (C 64, lmax 2) and
5 (C 128, lmax 3), against the reference's own outputs (fixtures ``sparse_c`` / ``sparse_d``), on
both aggregation paths (tensor cores and their CUDA-core twins).  At these widths a 128-row tile
of the tensor-core kernels holds 2 or 1 feature rows and conv1's backward runs its 2- and
4-channel-per-lane variants; fixtures ``sparse_a`` / ``sparse_b`` are C 32."""

import numpy as np
import pytest
import torch

import golden_io
import gpu_util as U
from fsctep_b200 import _native as NAT
from fsctep_b200.ictd import GraphCSR
from fsctep_b200.sparse import SparseConfig, SparseEngine

pytestmark = [pytest.mark.gpu, U.needs_gpu]


@pytest.mark.parametrize("gemm_path", [0, 1])
@pytest.mark.parametrize("tag", ["c", "d"])
def test_sparse_config_widths_match_reference(tag, gemm_path):
    cfg, sd, c = golden_io.sparse_case(tag)
    scfg = SparseConfig(channels=int(cfg["channels"]), lmax=int(cfg["lmax"]),
                        num_interaction=int(cfg["num_interaction"]), number_of_basis=int(cfg["number_of_basis"]),
                        max_radius=float(cfg["max_radius"]), function_type=str(cfg["function_type"]),
                        max_atomvalue=int(cfg["max_atomvalue"]))
    dev = torch.device("cuda")
    g = GraphCSR.from_edges(torch.tensor(c["edge_src"], device=dev).long(), torch.tensor(c["edge_dst"], device=dev).long(),
                            torch.tensor(c["edge_shifts"], device=dev).float(), int(c["pos"].shape[0]))
    NAT.lib().fsc_ictd_set_gemm_path(gemm_path)
    try:
        eng = SparseEngine(sd, scfg, "cuda")
        out = eng.energy_forces(torch.tensor(c["pos"], device=dev), torch.tensor(c["Z"], device=dev),
                                torch.tensor(c["batch"], device=dev), torch.tensor(c["cell"], device=dev), g)
        torch.cuda.synchronize()
        assert eng.status() == 0
    finally:
        NAT.lib().fsc_ictd_set_gemm_path(0)
    E = out["energy"].double().cpu().numpy()
    assert np.all(np.abs(E - c["ref64_energy"]) <= U.E_RTOL * np.abs(c["ref64_energy"])), (E, c["ref64_energy"])
    assert U.rel_max(out["forces"].cpu().numpy(), c["ref64_forces"]) <= U.F_RTOL, \
        U.rel_max(out["forces"].cpu().numpy(), c["ref64_forces"])
    assert U.rel_max(out["stress"].cpu().numpy(), c["ref64_stress"]) <= U.S_RTOL
