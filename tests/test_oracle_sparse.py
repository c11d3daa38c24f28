"""The pure-cartesian-sparse oracle restatement against the reference's own outputs."""

import numpy as np
import pytest
import torch

import golden_io
from oracle import sparse_model as SP
from oracle.ictd_model import ICTDConfig


def _cfg(cfg):
    return ICTDConfig(channels=int(cfg["channels"]), lmax=int(cfg["lmax"]), num_interaction=int(cfg["num_interaction"]),
                      number_of_basis=int(cfg["number_of_basis"]), function_type=str(cfg["function_type"]),
                      max_atomvalue=int(cfg["max_atomvalue"]))


@pytest.mark.parametrize("tag", ["a", "b", "c", "d", "e", "z"])
def test_sparse_oracle_matches_reference(tag):
    cfg, sd, c = golden_io.sparse_case(tag)
    r = SP.sparse_energy_forces_stress(sd, _cfg(cfg), torch.tensor(c["pos"]), torch.tensor(c["Z"]),
                                       torch.tensor(c["batch"]), torch.tensor(c["edge_src"]).long(),
                                       torch.tensor(c["edge_dst"]).long(), torch.tensor(c["edge_shifts"]).double(),
                                       torch.tensor(c["cell"]))
    np.testing.assert_allclose(r["energy"].numpy(), c["ref64_energy"], rtol=1e-10)
    np.testing.assert_allclose(r["forces"].numpy(), c["ref64_forces"], rtol=1e-8, atol=1e-10)
    np.testing.assert_allclose(r["stress"].numpy(), c["ref64_stress"], rtol=1e-8, atol=1e-10)


def test_sparse_paths():
    assert SP.sparse_paths(2) == [(0, 0, 0), (0, 1, 1), (0, 2, 2), (1, 0, 1), (1, 1, 2), (2, 0, 2)]
    assert len(SP.sparse_paths(3)) == 10
