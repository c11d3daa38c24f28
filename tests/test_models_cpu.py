"""Host-side checks of the drop-in module (no GPU): state_dict layout identical to the reference."""

import pytest
import torch

import golden_io
from fsctep_b200.ictd import ICTDConfig
from fsctep_b200.models import PureCartesianICTDTransformerLayer, reference_state_dict_shapes


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_state_dict_keys_and_shapes_match_reference(tag):
    z = golden_io.load(f"ictd_model_{tag}.npz")
    ref = {k[len("sdshape/"):]: tuple(int(x) for x in z[k]) for k in z.files if k.startswith("sdshape/")}
    cfg = ICTDConfig(channels=int(z["cfg_channels"]), num_interaction=int(z["cfg_num_interaction"]),
                     function_type=str(z["cfg_function_type"]), max_atomvalue=int(z["cfg_max_atomvalue"]))
    assert reference_state_dict_shapes(cfg) == ref


def test_loads_reference_state_dict():
    cfg, sd, _ = golden_io.model_case("a")
    m = PureCartesianICTDTransformerLayer(max_embed_radius=5.0, main_max_radius=5.0, main_number_of_basis=8,
                                          hidden_dim_conv=32, num_interaction=2, function_type_main="bessel")
    m.load_state_dict({k: v.float() for k, v in sd.items()})


def test_unsupported_options_raise():
    with pytest.raises(NotImplementedError):
        PureCartesianICTDTransformerLayer(5.0, 5.0, 8, 32, external_tensor_rank=1)
    with pytest.raises(NotImplementedError):
        PureCartesianICTDTransformerLayer(5.0, 5.0, 8, 32, function_type_main="fourier")
    m = PureCartesianICTDTransformerLayer(5.0, 5.0, 8, 32)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.zeros(2, 3), torch.ones(2).long(), torch.zeros(2).long(), torch.zeros(1).long(),
          torch.ones(1).long(), torch.zeros(1, 3), torch.eye(3)[None])


def _o3_module(cfg, device="meta", heads=True):
    from fsctep_b200.models import PureCartesianICTDO3TransformerLayer

    heads = {"dipole": {"irreps": ["1o"], "reduce": "sum"}, "polarizability": {"ls": [0, 2], "reduce": "sum"}} \
        if heads else None
    with torch.device(device):
        return PureCartesianICTDO3TransformerLayer(
            max_embed_radius=float(cfg["max_radius"]), main_max_radius=float(cfg["max_radius"]),
            main_number_of_basis=int(cfg["number_of_basis"]), hidden_dim_conv=int(cfg["channels"]),
            hidden_dim_sh=32, hidden_dim=64, lmax=2, num_interaction=int(cfg["num_interaction"]),
            function_type_main=str(cfg["function_type"]), max_atomvalue=int(cfg["max_atomvalue"]),
            external_tensor_rank=1, external_tensor_irrep="1o", physical_tensor_outputs=heads,
            o3_active_irreps=["0e", "1e", "1o", "2e"])


@pytest.mark.parametrize("tag", ["a", "b"])
def test_o3_module_state_dict_matches_reference(tag):
    z = golden_io.load(f"ictd_o3_{tag}.npz")
    ref = {k[len("sdshape/"):]: tuple(int(x) for x in z[k]) for k in z.files if k.startswith("sdshape/")}
    cfg = {k[4:]: z[k].item() for k in z.files if k.startswith("cfg_")}
    m = _o3_module(cfg)
    mine = {k: tuple(v.shape) for k, v in m.state_dict().items()}
    assert mine == ref


def test_o3_module_rejects_uncovered_options():
    from fsctep_b200.models import PureCartesianICTDO3TransformerLayer

    with pytest.raises(NotImplementedError):
        PureCartesianICTDO3TransformerLayer(5.0, 5.0, 8, 32, o3_irrep_preset="full")
    with pytest.raises(NotImplementedError):
        PureCartesianICTDO3TransformerLayer(5.0, 5.0, 8, 32, external_tensor_rank=2)


def _sparse_module(cfg, device="meta"):
    from fsctep_b200.models import PureCartesianSparseTransformerLayer

    with torch.device(device):
        return PureCartesianSparseTransformerLayer(
            max_embed_radius=float(cfg["max_radius"]), main_max_radius=float(cfg["max_radius"]),
            main_number_of_basis=int(cfg["number_of_basis"]), hidden_dim_conv=int(cfg["channels"]),
            hidden_dim_sh=32, hidden_dim=64, lmax=int(cfg["lmax"]), num_interaction=int(cfg["num_interaction"]),
            function_type_main=str(cfg["function_type"]), max_atomvalue=int(cfg["max_atomvalue"]))


@pytest.mark.parametrize("tag", ["a", "b"])
def test_sparse_module_state_dict_matches_reference(tag):
    z = golden_io.load(f"sparse_{tag}.npz")
    ref = {k[len("sdshape/"):]: tuple(int(x) for x in z[k]) for k in z.files if k.startswith("sdshape/")}
    cfg = {k[4:]: z[k].item() for k in z.files if k.startswith("cfg_")}
    mine = {k: tuple(v.shape) for k, v in _sparse_module(cfg).state_dict().items()}
    assert mine == ref


def test_feature_layout_maps_to_the_reference_merge():
    """Native rows (l^2 + m, channel innermost) <-> the reference's flat node layout (per irrep
    block channel-major (C, 2l + 1), pure_cartesian_ictd_layers_full.py _merge_irreps); the o3
    model's 1e block has no native storage and maps to zeros."""
    from fsctep_b200.models import _native_to_ref, _ref_to_native

    n, C = 5, 4
    feats = torch.randn(n, 9, C, dtype=torch.float64)
    blocks = [(0, 1), (1, 3), (4, 5)]
    flat = _native_to_ref(feats, blocks)
    ref = torch.cat([feats[:, l * l:(l + 1) ** 2, :].transpose(1, 2).reshape(n, -1) for l in range(3)], dim=-1)
    assert torch.equal(flat, ref)
    back = torch.zeros_like(feats)
    _ref_to_native(flat, blocks, back)
    assert torch.equal(back, feats)
    o3 = [(0, 1), (None, 3), (1, 3), (4, 5)]
    flat3 = _native_to_ref(feats, o3)
    assert flat3.shape == (n, 12 * C) and torch.count_nonzero(flat3[:, C:4 * C]) == 0
    assert torch.equal(flat3[:, 4 * C:7 * C], ref[:, C:4 * C])
