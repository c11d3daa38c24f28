"""Generate the golden fixtures in this directory from the unmodified reference.

Run where the reference source tree is available, with ``FSCTEP_REFERENCE_ROOT`` naming it;
the outputs are committed and the tests read only them, so nothing at test time needs the
reference.

    FSCTEP_REFERENCE_ROOT=<reference tree> python tests/golden/make_golden.py

Fixtures:

* ``ictd_tables.npz`` -- harmonic bases, normalised CG tensors, packed U_g per
  (l1,l2) group, direction projectors and product_5 factors for lmax 2 and 3,
  taken from the reference's own functions (``models/ictd_irreps.py``).
* ``ictd_model_{a,b}.npz`` -- seeded inputs, a seed-perturbed state_dict (fresh
  models output E = 0, ``mlp.py:126-127``) and the reference's per-graph energy,
  forces and stress (float64, and float32 for the tolerance budget), computed with
  ``PureCartesianICTDTransformerLayer`` (``pure_cartesian_ictd_layers_full.py``)
  and the calculator/trainer conventions (F = -dE/dpos, sigma = (1/V) dE/d eps).
* ``ictd_o3_{a,b}.npz`` -- the same for ``PureCartesianICTDO3TransformerLayer``
  (``pure_cartesian_ictd_layers_o3.py``) with active irreps 0e,1e,1o,2e, an external 1o field
  drawn from N(0, 0.05) per graph and dipole (1o) + polarizability (0e, 2e) heads on batches
  of non-periodic molecules: energies, forces, per-atom energies and the heads' outputs.
* ``sparse_{a,b}.npz`` -- the same for ``PureCartesianSparseTransformerLayer``
  (``pure_cartesian_sparse_layers.py``; max_rank_other 1, k_policy k0): a config-2-like water box
  (Lmax 2) and a config-5-like FCC crystal (Lmax 3, with stress); ``sparse_{c,d}.npz`` the same
  at configs 2 and 5's channel widths (C 64 / Lmax 2, C 128 / Lmax 3).
* ``ictd_hook.npz`` / ``ictd_o3_hook.npz`` -- an ictd and an o3 model evaluated with a seeded,
  differentiable ``sync_after_scatter`` (per-node scale, then ghost rows overwritten by owner
  rows): energies and forces.
* ``ictd_model_e.npz`` / ``ictd_o3_e.npz`` / ``sparse_e.npz`` -- the three models on frames with a
  receiver that has no neighbours (a bonded chain plus one atom 30 A away, a lone-atom frame, a
  dimer); ``ictd_model_z.npz`` / ``sparse_z.npz`` -- a system with no edges at all.  The reference
  clamps the neighbour count at 1 (``pure_cartesian_ictd_layers_full.py:471,929``,
  ``pure_cartesian_sparse_layers.py:328``) and averages E/N over the whole system
  (``pure_cartesian_sparse_layers.py:419``).
* ``tp_ops.npz`` -- the ``_C_ictd_tp`` operator family evaluated by the reference's
  einsum references (``models/ictd_irreps_cuda.py:169-311``) on the shapes of
  ``test/test_ictd_tp_backend.py``.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import ref_import  # noqa: E402

if "FSCTEP_REFERENCE_ROOT" not in os.environ:
    raise SystemExit("set FSCTEP_REFERENCE_ROOT to the reference source tree")
ref_import.install(os.environ["FSCTEP_REFERENCE_ROOT"])

from fsctep_b200 import systems  # noqa: E402
from fsctep_b200.weights import seeded_state_dict  # noqa: E402
from oracle import neighbors  # noqa: E402


def tables():
    from molecular_force_field.models import ictd_irreps as R

    out = {}
    for L in range(0, 5):
        out[f"basis_{L}"] = R._harmonic_basis_cpu_f64(L).numpy()
    for lmax in (2, 3):
        tp = R.HarmonicFullyConnectedTensorProduct(4, 1, 4, lmax, internal_compute_dtype=torch.float64)
        cg = tp._get_cg_list(torch.device("cpu"), torch.float64)
        for p, (l1, l2, l3) in enumerate(tp.paths):
            out[f"L{lmax}_cg_{l1}{l2}{l3}"] = cg[p].numpy()
        U = tp._get_proj_group_list(torch.device("cpu"), torch.float64)
        for g, u in zip(tp._groups, U):
            out[f"L{lmax}_U_{g['l1']}{g['l2']}"] = u.numpy()
        out[f"L{lmax}_paths"] = np.array(tp.paths, dtype=np.int64)
        ew = R.HarmonicElementwiseProduct(lmax=lmax, mul=4, irreps_out="0e")
        out[f"L{lmax}_p5_factors"] = np.array(ew._0e_factors, dtype=np.float64)
    for l in range(0, 5):
        out[f"dirproj_{l}"] = R._dir_proj_cpu_f64(l).numpy()
    g = torch.Generator().manual_seed(7)
    n = torch.randn(64, 3, generator=g, dtype=torch.float64)
    n = n / n.norm(dim=1, keepdim=True)
    out["dir_n"] = n.numpy()
    for l in range(0, 5):
        out[f"dir_Y_{l}"] = R.direction_harmonics_fast(n, l).numpy()
    np.savez_compressed(os.path.join(HERE, "ictd_tables.npz"), **out)


def _perturb(model, seed):
    """Overwrite every parameter from ``fsctep_b200.weights.seeded_state_dict``; the
    tests rebuild the same tensors from the seed, so only a checksum is stored."""
    shapes = {k: tuple(v.shape) for k, v in model.state_dict().items()}
    sd = seeded_state_dict(shapes, seed, torch.float64)
    model.load_state_dict(sd)
    return shapes


def _ref_efs(model, pos, Z, batch, src, dst, shifts, cell, dtype):
    model = model.to(dtype)
    pos = torch.tensor(pos, dtype=dtype, requires_grad=True)
    cell_t = torch.tensor(cell, dtype=dtype)
    b = torch.tensor(batch)
    nb = cell_t.shape[0]
    strain = torch.zeros(nb, 3, 3, dtype=dtype, requires_grad=True)
    D = torch.eye(3, dtype=dtype) + 0.5 * (strain + strain.transpose(-1, -2))
    pos_in = torch.einsum("ni,nij->nj", pos, D[b])
    cell_in = torch.bmm(cell_t, D)
    e = model(pos_in, torch.tensor(Z), b, torch.tensor(src), torch.tensor(dst),
              torch.tensor(shifts, dtype=dtype), cell_in)
    Eg = torch.zeros(nb, dtype=dtype).index_add(0, b, e.squeeze(-1))
    gp, gs = torch.autograd.grad(Eg.sum(), [pos, strain])
    vol = torch.abs(torch.det(cell_t))
    return {"energy": Eg.detach().numpy(), "forces": (-gp).numpy(),
            "stress": (gs / vol.view(-1, 1, 1)).numpy(), "atom_energy": e.detach().squeeze(-1).numpy()}


def model_case(tag, system, cfg, seed):
    from molecular_force_field.models.pure_cartesian_ictd_layers_full import PureCartesianICTDTransformerLayer

    torch.set_default_dtype(torch.float64)
    model = PureCartesianICTDTransformerLayer(
        max_embed_radius=cfg["max_radius"], main_max_radius=cfg["max_radius"],
        main_number_of_basis=cfg["number_of_basis"], hidden_dim_conv=cfg["channels"], hidden_dim_sh=32,
        hidden_dim=64, lmax=cfg["lmax"], num_interaction=cfg["num_interaction"],
        function_type_main=cfg["function_type"], max_atomvalue=cfg["max_atomvalue"],
        internal_compute_dtype=torch.float64, device=torch.device("cpu"))
    shapes = _perturb(model, seed)
    src, dst, S = neighbors.batched_neighbor_list(system["pos"], system["batch"], system["cell"],
                                                  cfg["max_radius"], system["pbc"])
    args = (system["pos"], system["Z"], system["batch"], src, dst, S.astype(np.float64), system["cell"])
    r64 = _ref_efs(model, *args, torch.float64)
    sd64 = {k: v.detach().clone() for k, v in model.state_dict().items()}
    model.internal_compute_dtype = torch.float32
    for mod in model.modules():
        if hasattr(mod, "internal_compute_dtype"):
            mod.internal_compute_dtype = torch.float32
    torch.set_default_dtype(torch.float32)
    r32 = _ref_efs(model, *args, torch.float32)
    torch.set_default_dtype(torch.float64)
    out = {"pos": system["pos"], "Z": system["Z"], "batch": system["batch"], "cell": system["cell"],
           "pbc": np.array(system["pbc"]), "edge_src": src.astype(np.int32), "edge_dst": dst.astype(np.int32),
           "edge_shifts": S.astype(np.int8)}
    for k, v in cfg.items():
        out[f"cfg_{k}"] = np.array(v)
    out["sd_seed"] = np.array(seed)
    for k, v in sd64.items():
        out[f"sdshape/{k}"] = np.array(shapes[k], dtype=np.int64)
        out[f"sdsum/{k}"] = np.array(float(v.double().sum()))
    for k, v in r64.items():
        out[f"ref64_{k}"] = v
    for k, v in r32.items():
        out[f"ref32_{k}"] = v
    np.savez_compressed(os.path.join(HERE, f"ictd_model_{tag}.npz"), **out)
    print(tag, "atoms", system["pos"].shape[0], "edges", src.shape[0], "E", r64["energy"],
          "max|dE| fp32", np.abs(r64["energy"] - r32["energy"]).max(),
          "max|dF| fp32", np.abs(r64["forces"] - r32["forces"]).max(), "max|F|", np.abs(r64["forces"]).max())


O3_HEADS = {"dipole": {"irreps": ["1o"], "reduce": "sum"}, "polarizability": {"ls": [0, 2], "reduce": "sum"}}


def o3_case(tag, system, cfg, seed, field_seed):
    from molecular_force_field.models.pure_cartesian_ictd_layers_o3 import PureCartesianICTDO3TransformerLayer

    torch.set_default_dtype(torch.float64)
    model = PureCartesianICTDO3TransformerLayer(
        max_embed_radius=cfg["max_radius"], main_max_radius=cfg["max_radius"],
        main_number_of_basis=cfg["number_of_basis"], hidden_dim_conv=cfg["channels"], hidden_dim_sh=32,
        hidden_dim=64, lmax=cfg["lmax"], num_interaction=cfg["num_interaction"],
        function_type_main=cfg["function_type"], max_atomvalue=cfg["max_atomvalue"],
        internal_compute_dtype=torch.float64, device=torch.device("cpu"),
        external_tensor_rank=1, external_tensor_irrep="1o", physical_tensor_outputs=O3_HEADS,
        o3_active_irreps=["0e", "1e", "1o", "2e"])
    shapes = _perturb(model, seed)
    B = system["cell"].shape[0]
    field = np.random.default_rng(field_seed).normal(scale=0.05, size=(B, 3))
    src, dst, S = neighbors.batched_neighbor_list(system["pos"], system["batch"], system["cell"],
                                                  cfg["max_radius"], system["pbc"])
    pos = torch.tensor(system["pos"], requires_grad=True)
    b = torch.tensor(system["batch"])
    e, phys = model(pos, torch.tensor(system["Z"]), b, torch.tensor(src), torch.tensor(dst),
                    torch.tensor(S.astype(np.float64)), torch.tensor(system["cell"]),
                    external_tensor=torch.tensor(field), return_physical_tensors=True)
    Eg = torch.zeros(B, dtype=torch.float64).index_add(0, b, e.squeeze(-1))
    (gp,) = torch.autograd.grad(Eg.sum(), [pos])
    out = {"pos": system["pos"], "Z": system["Z"], "batch": system["batch"], "cell": system["cell"],
           "pbc": np.array(system["pbc"]), "edge_src": src.astype(np.int32), "edge_dst": dst.astype(np.int32),
           "edge_shifts": S.astype(np.int8), "field": field}
    for k, v in cfg.items():
        out[f"cfg_{k}"] = np.array(v)
    out["sd_seed"] = np.array(seed)
    for k, v in model.state_dict().items():
        out[f"sdshape/{k}"] = np.array(shapes[k], dtype=np.int64)
        out[f"sdsum/{k}"] = np.array(float(v.double().sum()))
    out["ref64_energy"] = Eg.detach().numpy()
    out["ref64_forces"] = (-gp).numpy()
    out["ref64_atom_energy"] = e.detach().squeeze(-1).numpy()
    out["ref64_dipole"] = phys["dipole"][1].detach().numpy()
    out["ref64_polar0"] = phys["polarizability"][0].detach().numpy()
    out["ref64_polar2"] = phys["polarizability"][2].detach().numpy()
    np.savez_compressed(os.path.join(HERE, f"ictd_o3_{tag}.npz"), **out)
    print("o3", tag, "atoms", system["pos"].shape[0], "edges", src.shape[0], "E", out["ref64_energy"][:3],
          "dipole", out["ref64_dipole"].reshape(B, -1)[0])


def sparse_case(tag, system, cfg, seed):
    from molecular_force_field.models.pure_cartesian_sparse_layers import PureCartesianSparseTransformerLayer

    torch.set_default_dtype(torch.float64)
    model = PureCartesianSparseTransformerLayer(
        max_embed_radius=cfg["max_radius"], main_max_radius=cfg["max_radius"],
        main_number_of_basis=cfg["number_of_basis"], hidden_dim_conv=cfg["channels"], hidden_dim_sh=32,
        hidden_dim=64, lmax=cfg["lmax"], num_interaction=cfg["num_interaction"],
        function_type_main=cfg["function_type"], max_atomvalue=cfg["max_atomvalue"], device=torch.device("cpu"))
    shapes = _perturb(model, seed)
    src, dst, S = neighbors.batched_neighbor_list(system["pos"], system["batch"], system["cell"],
                                                  cfg["max_radius"], system["pbc"])
    args = (system["pos"], system["Z"], system["batch"], src, dst, S.astype(np.float64), system["cell"])
    r64 = _ref_efs(model, *args, torch.float64)
    out = {"pos": system["pos"], "Z": system["Z"], "batch": system["batch"], "cell": system["cell"],
           "pbc": np.array(system["pbc"]), "edge_src": src.astype(np.int32), "edge_dst": dst.astype(np.int32),
           "edge_shifts": S.astype(np.int8)}
    for k, v in cfg.items():
        out[f"cfg_{k}"] = np.array(v)
    out["sd_seed"] = np.array(seed)
    for k, v in model.state_dict().items():
        out[f"sdshape/{k}"] = np.array(shapes[k], dtype=np.int64)
        out[f"sdsum/{k}"] = np.array(float(v.double().sum()))
    for k, v in r64.items():
        out[f"ref64_{k}"] = v
    np.savez_compressed(os.path.join(HERE, f"sparse_{tag}.npz"), **out)
    print("sparse", tag, "atoms", system["pos"].shape[0], "edges", src.shape[0], "E", r64["energy"],
          "max|F|", np.abs(r64["forces"]).max())


def sparse():
    cfg2 = dict(channels=32, lmax=2, num_interaction=3, number_of_basis=8, max_radius=5.0,
                function_type="gaussian", max_atomvalue=10)
    sparse_case("a", systems.water_box(n_side=4, box=12.4, seed=18), cfg2, seed=6)
    cfg5 = dict(channels=32, lmax=3, num_interaction=3, number_of_basis=8, max_radius=5.0,
                function_type="gaussian", max_atomvalue=30)
    sparse_case("b", systems.fcc_crystal(n_cells=(3, 3, 3), seed=19), cfg5, seed=7)


def sparse_widths():
    """Configs 2 and 5's channel widths (the fixtures above are C 32): C 64 / Lmax 2 on a small
    water box and C 128 / Lmax 3 on a 32-atom FCC crystal."""
    cfg2 = dict(channels=64, lmax=2, num_interaction=3, number_of_basis=8, max_radius=5.0,
                function_type="gaussian", max_atomvalue=10)
    sparse_case("c", systems.water_box(n_side=3, box=9.3, seed=20), cfg2, seed=8)
    cfg5 = dict(channels=128, lmax=3, num_interaction=3, number_of_basis=8, max_radius=5.0,
                function_type="gaussian", max_atomvalue=30)
    sparse_case("d", systems.fcc_crystal(n_cells=(2, 2, 2), seed=21), cfg5, seed=9)


def isolated_frames(seed):
    """Three non-periodic frames: a 12-atom bonded chain with one O atom 30 A from its centre, a
    lone C atom, and an H-O dimer at 1.2 A."""
    m = systems.organic_molecules(n_mol=1, min_atoms=12, max_atoms=12, seed=seed)
    far = m["pos"].mean(axis=0) + np.array([30.0, 0.0, 0.0])
    pos = np.vstack([m["pos"], far, [[50.0, 50.0, 50.0]], [[50.0, 50.0, 50.0], [51.2, 50.1, 49.9]]])
    Z = np.concatenate([m["Z"], [8, 6, 1, 8]])
    batch = np.concatenate([np.zeros(13, dtype=np.int64), [1, 2, 2]])
    cells = np.stack([np.eye(3) * 100.0] * 3)
    return systems._system(pos, Z, batch, cells, pbc=(False, False, False))


def no_edge_frames():
    """Two non-periodic frames of three atoms each, 8 A apart: no pair within the 5 A cutoff."""
    pos = np.array([[10.0, 10.0, 10.0], [18.0, 10.0, 10.0], [10.0, 18.0, 10.0],
                    [10.0, 10.0, 10.0], [10.0, 10.0, 18.0], [18.0, 18.0, 18.0]])
    return systems._system(pos, [1, 6, 8, 8, 7, 1], [0, 0, 0, 1, 1, 1], np.stack([np.eye(3) * 40.0] * 2),
                           pbc=(False, False, False))


def edge_cases():
    cfg = dict(channels=32, lmax=2, num_interaction=3, number_of_basis=8, max_radius=5.0,
               function_type="gaussian", max_atomvalue=10)
    model_case("e", isolated_frames(seed=30), cfg, seed=31)
    o3_case("e", isolated_frames(seed=30), cfg, seed=32, field_seed=33)
    sparse_case("e", isolated_frames(seed=30), cfg, seed=34)
    model_case("z", no_edge_frames(), cfg, seed=35)
    sparse_case("z", no_edge_frames(), cfg, seed=36)


def tp_ops():
    from molecular_force_field.models import ictd_irreps_cuda as RC

    out = {}
    g = torch.Generator().manual_seed(100)
    B, I, m1, m2, P, K, O = 4, 3, 3, 3, 2, 3, 4
    a = torch.randn(B, I, m1, generator=g, dtype=torch.float64)
    b = torch.randn(B, 1, m2, generator=g, dtype=torch.float64)
    U = torch.randn(m1 * m2, P * K, generator=g, dtype=torch.float64)
    w = torch.randn(P, O, I, generator=g, dtype=torch.float64)
    gates = torch.randn(B, P, generator=g, dtype=torch.float64)
    y = RC._project_forward_reference(a, b, U, P)
    gy = torch.randn(y.shape, generator=g, dtype=torch.float64)
    ga, gb, gu = RC._project_transpose_reference(gy, a, b, U, need_a=True, need_b=True, need_u=True)
    mo, _ = RC._mix_forward_reference(y, w, gates)
    go = torch.randn(mo.shape, generator=g, dtype=torch.float64)
    my, mw, mg = RC._mix_transpose_reference(go, y, w, gates, need_y=True, need_w=True, need_g=True)
    for k, v in dict(a=a, b=b, U=U, w=w, gates=gates, y=y, gy=gy, ga=ga, gb=gb, gu=gu, mo=mo, go=go,
                     my=my, mw=mw, mg=mg).items():
        out[k] = v.numpy()
    np.savez_compressed(os.path.join(HERE, "tp_ops.npz"), **out)


def layer_hook(n, seed):
    """A deterministic, differentiable sync_after_scatter stand-in: every node's features scaled by
    a seeded factor, then the rows of n // 8 "ghost" nodes replaced by copies of other ("owner")
    nodes' rows, the shape of a halo exchange (cli/inference_ddp.py:143-340)."""
    rng = np.random.default_rng(seed)
    scale = rng.uniform(0.8, 1.2, n)
    perm = rng.permutation(n)
    ghosts, owners = perm[: n // 8], perm[n // 8: 2 * (n // 8)]

    def hook(x):
        y = x * torch.tensor(scale, dtype=x.dtype).unsqueeze(1)
        return y.index_copy(0, torch.tensor(ghosts), y[torch.tensor(owners)])

    return hook, {"hook_scale": scale, "hook_ghosts": ghosts.astype(np.int64), "hook_owners": owners.astype(np.int64)}


def hook_cases():
    """ictd (C 32, 3 layers) and o3 (0e, 1e, 1o, 2e, field) with the layer_hook stand-in as
    sync_after_scatter: per-graph energies and forces of the reference, float64."""
    from molecular_force_field.models.pure_cartesian_ictd_layers_full import PureCartesianICTDTransformerLayer
    from molecular_force_field.models.pure_cartesian_ictd_layers_o3 import PureCartesianICTDO3TransformerLayer

    torch.set_default_dtype(torch.float64)
    cases = [("ictd_hook", systems.diamond_crystal(n_cells=(2, 2, 2), seed=22),
              dict(channels=32, lmax=2, num_interaction=3, number_of_basis=8, max_radius=5.0,
                   function_type="gaussian", max_atomvalue=16), 31, None),
             ("ictd_o3_hook", systems.organic_molecules(n_mol=4, seed=23),
              dict(channels=32, lmax=2, num_interaction=3, number_of_basis=8, max_radius=5.0,
                   function_type="gaussian", max_atomvalue=10), 32, 33)]
    for name, system, cfg, seed, field_seed in cases:
        kw = dict(max_embed_radius=cfg["max_radius"], main_max_radius=cfg["max_radius"],
                  main_number_of_basis=cfg["number_of_basis"], hidden_dim_conv=cfg["channels"], hidden_dim_sh=32,
                  hidden_dim=64, lmax=cfg["lmax"], num_interaction=cfg["num_interaction"],
                  function_type_main=cfg["function_type"], max_atomvalue=cfg["max_atomvalue"],
                  internal_compute_dtype=torch.float64, device=torch.device("cpu"))
        if field_seed is None:
            model = PureCartesianICTDTransformerLayer(**kw)
        else:
            model = PureCartesianICTDO3TransformerLayer(external_tensor_rank=1, external_tensor_irrep="1o",
                                                        o3_active_irreps=["0e", "1e", "1o", "2e"], **kw)
        shapes = _perturb(model, seed)
        n = system["pos"].shape[0]
        B = system["cell"].shape[0]
        hook, hook_data = layer_hook(n, seed + 100)
        src, dst, S = neighbors.batched_neighbor_list(system["pos"], system["batch"], system["cell"],
                                                      cfg["max_radius"], system["pbc"])
        pos = torch.tensor(system["pos"], requires_grad=True)
        b = torch.tensor(system["batch"])
        extra = {}
        if field_seed is not None:
            field = np.random.default_rng(field_seed).normal(scale=0.05, size=(B, 3))
            extra = {"external_tensor": torch.tensor(field)}
        e = model(pos, torch.tensor(system["Z"]), b, torch.tensor(src), torch.tensor(dst),
                  torch.tensor(S.astype(np.float64)), torch.tensor(system["cell"]), sync_after_scatter=hook, **extra)
        Eg = torch.zeros(B, dtype=torch.float64).index_add(0, b, e.squeeze(-1))
        (gp,) = torch.autograd.grad(Eg.sum(), [pos])
        out = {"pos": system["pos"], "Z": system["Z"], "batch": system["batch"], "cell": system["cell"],
               "pbc": np.array(system["pbc"]), "edge_src": src.astype(np.int32), "edge_dst": dst.astype(np.int32),
               "edge_shifts": S.astype(np.int8), **hook_data}
        if field_seed is not None:
            out["field"] = field
        for k, v in cfg.items():
            out[f"cfg_{k}"] = np.array(v)
        out["sd_seed"] = np.array(seed)
        for k, v in model.state_dict().items():
            out[f"sdshape/{k}"] = np.array(shapes[k], dtype=np.int64)
            out[f"sdsum/{k}"] = np.array(float(v.double().sum()))
        out["ref64_energy"] = Eg.detach().numpy()
        out["ref64_forces"] = (-gp).numpy()
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
        print(name, "atoms", n, "edges", src.shape[0], "E", out["ref64_energy"][:3])


def main():
    tables()
    tp_ops()
    cfg_a = dict(channels=32, lmax=2, num_interaction=2, number_of_basis=8, max_radius=5.0,
                 function_type="bessel", max_atomvalue=10)
    model_case("a", systems.random_frames(n_frames=2, n_atoms=96, box=10.0, seed=11), cfg_a, seed=1)
    cfg_b = dict(channels=32, lmax=2, num_interaction=3, number_of_basis=8, max_radius=5.0,
                 function_type="gaussian", max_atomvalue=16)
    model_case("b", systems.diamond_crystal(n_cells=(2, 2, 2), seed=12), cfg_b, seed=2)
    cfg_c = dict(channels=64, lmax=2, num_interaction=3, number_of_basis=8, max_radius=5.0,
                 function_type="gaussian", max_atomvalue=16)
    model_case("c", systems.diamond_crystal(n_cells=(2, 2, 2), seed=13, sigma=0.15), cfg_c, seed=3)
    o3()
    sparse()
    sparse_widths()
    hook_cases()
    edge_cases()


def o3():
    cfg = dict(channels=32, lmax=2, num_interaction=3, number_of_basis=8, max_radius=5.0,
               function_type="gaussian", max_atomvalue=10)
    o3_case("a", systems.organic_molecules(n_mol=6, seed=14), cfg, seed=4, field_seed=15)
    cfg64 = dict(cfg, channels=64, function_type="bessel")
    o3_case("b", systems.organic_molecules(n_mol=4, seed=16), cfg64, seed=5, field_seed=17)


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "o3":
        o3()
    elif len(sys.argv) > 1 and sys.argv[1] == "sparse":
        sparse()
    elif len(sys.argv) > 1 and sys.argv[1] == "sparse_widths":
        sparse_widths()
    elif len(sys.argv) > 1 and sys.argv[1] == "hooks":
        hook_cases()
    elif len(sys.argv) > 1 and sys.argv[1] == "edge_cases":
        edge_cases()
    else:
        main()
