"""The O3 oracle restatement against the reference's own outputs (golden fixtures)."""

import numpy as np
import pytest
import torch

import golden_io
from oracle import ictd_o3 as O3
from oracle.ictd_model import ICTDConfig


@pytest.mark.parametrize("tag", ["a", "b", "e"])
def test_o3_oracle_matches_reference(tag):
    cfg, sd, c = golden_io.o3_case(tag)
    ocfg = ICTDConfig(channels=int(cfg["channels"]), num_interaction=int(cfg["num_interaction"]),
                      number_of_basis=int(cfg["number_of_basis"]), function_type=str(cfg["function_type"]),
                      max_atomvalue=int(cfg["max_atomvalue"]))
    r = O3.o3_energy_forces(sd, ocfg, torch.tensor(c["pos"]), torch.tensor(c["Z"]), torch.tensor(c["batch"]),
                            torch.tensor(c["edge_src"]).long(), torch.tensor(c["edge_dst"]).long(),
                            torch.tensor(c["edge_shifts"]).double(), torch.tensor(c["cell"]),
                            torch.tensor(c["field"]))
    np.testing.assert_allclose(r["energy"].numpy(), c["ref64_energy"], rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(r["forces"].numpy(), c["ref64_forces"], rtol=1e-8, atol=1e-10)
    np.testing.assert_allclose(r["dipole"].numpy(), c["ref64_dipole"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(r["polar0"].numpy(), c["ref64_polar0"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(r["polar2"].numpy(), c["ref64_polar2"], rtol=1e-10, atol=1e-12)


def test_o3_paths_and_closure():
    paths = O3.o3_paths(O3.ACTIVE)
    assert len(paths) == 17
    # the canonical-parity blocks {0e, 1o, 2e} are closed under products with Y, and give the
    # 11 SO(3) paths; 1e only couples to itself
    even = [p for p in paths if p[1] == (-1) ** p[0] and p[3] == (-1) ** p[2]]
    assert [(p[0], p[2], p[4]) for p in even] == [(0, 0, 0), (0, 1, 1), (0, 2, 2), (1, 0, 1), (1, 1, 0), (1, 1, 2),
                                                  (1, 2, 1), (2, 0, 2), (2, 1, 1), (2, 2, 0), (2, 2, 2)]
