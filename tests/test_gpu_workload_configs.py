"""Parity of pure-cartesian-sparse at the channel counts of BASELINE configs 2 (C 64, lmax 2) and
5 (C 128, lmax 3), against the fp64 oracle, on both aggregation paths (tensor cores and their
CUDA-core twins).  At these widths a 128-row tile of the tensor-core kernels holds 2 or 1
feature rows and conv1's backward runs its 2- and 4-channel-per-lane variants; the fixtures are
C 32."""

import numpy as np
import pytest
import torch

import gpu_util as U
from fsctep_b200 import _native as NAT
from fsctep_b200 import systems
from fsctep_b200.ictd import GraphCSR
from fsctep_b200.models import PureCartesianSparseTransformerLayer
from fsctep_b200.sparse import SparseConfig, SparseEngine
from fsctep_b200.weights import seeded_state_dict

pytestmark = [pytest.mark.gpu, U.needs_gpu]


@pytest.mark.parametrize("C,lmax", [(64, 2), (128, 3)])
def test_sparse_config_widths_match_oracle(C, lmax):
    from oracle import neighbors as ON
    from oracle import sparse_model as SP
    from oracle.ictd_model import ICTDConfig as OCfg

    with torch.device("meta"):
        m = PureCartesianSparseTransformerLayer(max_embed_radius=5.0, main_max_radius=5.0, main_number_of_basis=8,
                                                hidden_dim_conv=C, lmax=lmax, num_interaction=3, max_atomvalue=30)
    sd = seeded_state_dict({k: tuple(v.shape) for k, v in m.state_dict().items()}, 77)
    s = systems.fcc_crystal(n_cells=(2, 2, 2), seed=5)  # 32 atoms, ~44 neighbours each
    src, dst, S = ON.neighbor_list(s["pos"], s["cell"][0], 5.0)
    ocfg = OCfg(channels=C, lmax=lmax, num_interaction=3, number_of_basis=8, function_type="gaussian",
                max_atomvalue=30)
    ref = SP.sparse_energy_forces_stress(sd, ocfg, torch.tensor(s["pos"]), torch.tensor(s["Z"]),
                                         torch.tensor(s["batch"]).long(), torch.tensor(src), torch.tensor(dst),
                                         torch.tensor(S, dtype=torch.float64), torch.tensor(s["cell"]))
    scfg = SparseConfig(channels=C, lmax=lmax, num_interaction=3, number_of_basis=8, max_radius=5.0,
                        function_type="gaussian", max_atomvalue=30)
    dev = torch.device("cuda")
    g = GraphCSR.from_edges(torch.tensor(src, device=dev), torch.tensor(dst, device=dev),
                            torch.tensor(S, device=dev).float(), len(s["pos"]))
    pos, cell = torch.tensor(s["pos"], device=dev), torch.tensor(s["cell"], device=dev)
    Z = torch.tensor(s["Z"], device=dev)
    batch = torch.zeros(len(s["pos"]), dtype=torch.int64, device=dev)
    E_ref, F_ref, S_ref = ref["energy"].numpy(), ref["forces"].numpy(), ref["stress"].numpy()
    for path in (0, 1):
        NAT.lib().fsc_ictd_set_gemm_path(path)
        try:
            eng = SparseEngine(sd, scfg, "cuda")
            out = eng.energy_forces(pos, Z, batch, cell, g)
            torch.cuda.synchronize()
            assert eng.status() == 0
        finally:
            NAT.lib().fsc_ictd_set_gemm_path(0)
        E = out["energy"].double().cpu().numpy()
        assert np.all(np.abs(E - E_ref) <= U.E_RTOL * np.abs(E_ref)), (path, E, E_ref)
        assert U.rel_max(out["forces"].cpu().numpy(), F_ref) <= U.F_RTOL, (path, U.rel_max(out["forces"].cpu().numpy(), F_ref))
        assert U.rel_max(out["stress"].cpu().numpy(), S_ref) <= U.S_RTOL, path
