"""sync_after_scatter through the drop-in modules (stepwise native engine) against the reference.

The fixtures ``ictd_hook`` / ``ictd_o3_hook`` hold the reference's energies and forces with a
seeded differentiable hook (per-node scale, then "ghost" rows overwritten by "owner" rows; see
``tests/golden/make_golden.py``).  The reference calls the hook after conv1 and after every conv2
scatter (``pure_cartesian_ictd_layers_full.py:923-953``, ``pure_cartesian_ictd_layers_o3.py:947-972``).
"""

import numpy as np
import pytest
import torch

import golden_io
import gpu_util as U
from fsctep_b200.models import PureCartesianICTDTransformerLayer

pytestmark = [pytest.mark.gpu, U.needs_gpu]


def _hook(c, dev):
    scale = torch.tensor(c["hook_scale"], device=dev)
    ghosts = torch.tensor(c["hook_ghosts"], device=dev)
    owners = torch.tensor(c["hook_owners"], device=dev)
    calls = []

    def hook(x):
        calls.append(tuple(x.shape))
        y = x * scale.to(x.dtype).unsqueeze(1)
        return y.index_copy(0, ghosts, y[owners])

    return hook, calls


def _model(kind):
    if kind == "ictd":
        cfg, sd, c = golden_io.model_case("hook", prefix="ictd")
        m = PureCartesianICTDTransformerLayer(max_embed_radius=5.0, main_max_radius=5.0, main_number_of_basis=8,
                                              hidden_dim_conv=int(cfg["channels"]),
                                              num_interaction=int(cfg["num_interaction"]),
                                              function_type_main=str(cfg["function_type"]),
                                              max_atomvalue=int(cfg["max_atomvalue"]))
    else:
        from test_models_cpu import _o3_module

        cfg, sd, c = golden_io.model_case("hook", prefix="ictd_o3")
        m = _o3_module(cfg, device="cpu", heads=False)
    m.load_state_dict({k: v.float() for k, v in sd.items()})
    return m.cuda(), c, cfg


def _args(c, dev):
    return (torch.tensor(c["Z"], device=dev), torch.tensor(c["batch"], device=dev),
            torch.tensor(c["edge_src"], device=dev), torch.tensor(c["edge_dst"], device=dev),
            torch.tensor(c["edge_shifts"], device=dev).float(), torch.tensor(c["cell"], device=dev).float())


@pytest.mark.parametrize("kind", ["ictd", "o3"])
def test_hook_matches_reference(kind):
    m, c, cfg = _model(kind)
    dev = torch.device("cuda")
    hook, calls = _hook(c, dev)
    pos = torch.tensor(c["pos"], device=dev, dtype=torch.float32).requires_grad_(True)
    kw = {"sync_after_scatter": hook}
    if kind == "o3":
        kw["external_tensor"] = torch.tensor(c["field"], device=dev)
    e = m(pos, *_args(c, dev), **kw)
    b = torch.tensor(c["batch"], device=dev)
    Eg = torch.zeros(c["cell"].shape[0], device=dev).index_add(0, b, e.view(-1))
    (gp,) = torch.autograd.grad(Eg.sum(), [pos])
    nint = int(cfg["num_interaction"])
    width = int(cfg["channels"]) * (12 if kind == "o3" else 9)
    assert calls == [(c["pos"].shape[0], width)] * nint
    E, ref = Eg.detach().double().cpu().numpy(), c["ref64_energy"]
    assert np.all(np.abs(E - ref) <= U.E_RTOL * np.abs(ref).max()), (E, ref)
    assert U.rel_max(-gp.cpu().numpy(), c["ref64_forces"]) <= U.F_RTOL


def test_identity_hook_is_the_plain_path():
    """The stepwise evaluation with an identity hook gives the same energies and forces, bit for
    bit, as the one-call path, also through precomputed edge vectors."""
    m, c, _ = _model("ictd")
    dev = torch.device("cuda")
    outs = []
    for hook in (None, lambda x: x):
        pos = torch.tensor(c["pos"], device=dev, dtype=torch.float32).requires_grad_(True)
        e = m(pos, *_args(c, dev), sync_after_scatter=hook)
        (g,) = torch.autograd.grad(e.sum(), [pos])
        outs.append((e.detach(), g))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
