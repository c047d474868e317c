"""Write the committed golden fixtures under tests/golden/ from the reference's own code and data.

Run once in a container where the reference checkout is available:

    python tests/golden/make_golden.py <reference_root>

It writes two kinds of fixture (all fp32, npz):

* ``ref_golden_tiny.npz`` / ``ref_golden_bulk.npz`` -- the reference's committed fairchem goldens
  (tests/data/golden_tiny.npz: ethanol, 9 atoms, 72 edges, aperiodic; golden_bulk_tiny.npz: Si
  diamond x(2,1,1), 4 atoms, 112 edges, periodic), reduced to config, weights, tables, inputs,
  the gamma-independent host terms and the outputs (energy, forces, node embedding).
* ``ref_run_*.npz`` -- this framework's seeded inputs and random-init weights evaluated by the
  reference's OWN CPU path: ``tt_atom.geometry.radius_graph`` + ``HostGeometry`` +
  ``tests/mirror.py`` + torch autograd, with the strain leaf of tt_atom/forces.py:515-524 for the
  virial. These pin the neighbour list (edge_index, shifts: bit-exact) and E/F/virial.
* ``ref_orb_geometry.npz`` / ``ref_orb_host_terms.npz`` -- the reference's Orb edge features and
  their VJP, its host ZBL pair repulsion (energy, forces, stress), its normalisers and its
  charge / spin conditioning, on seeded inputs.
* ``ref_run_orb.npz`` -- the reference's own Orb backbone forward and reverse pass (energy,
  forces, virial) on seeded inputs and random-init weights, run on the CPU through
  ``ttnn_cpu.py`` (an fp32 torch stand-in for the ttnn calls).
* ``ref_run_spectral.npz`` -- the reference's spectral feed-forward (uma-s-1's) on seeded node
  features, through the same stand-in.

Nothing at test time reads the reference; the tests read only these files.
"""
import json
import pathlib
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parents[1]


def _reduce_fairchem(ref_root, name, out):
    z = np.load(ref_root / "tests" / "data" / name)
    zt = np.load(ref_root / "tests" / "data" / "golden_tiny.npz")   # tables shared by both
    keep = {"config": z["config"]}
    for k in z.files:
        if k.startswith("w@") or k.startswith("in@") or k.startswith("out@"):
            keep[k] = z[k]
    for k in ("x_edge", "edge_envelope", "x_message_init", "sys_node_embedding", "edge_distance",
              "to_m", "gauss_offset", "gauss_coeff", "to_grid_mat", "from_grid_mat"):
        src = z if f"host@{k}" in z.files else zt
        if f"host@{k}" in src.files:
            keep[f"host@{k}"] = src[f"host@{k}"]
    np.savez_compressed(HERE / out, **keep)
    print("wrote", out, len(keep), "arrays")


def _run_reference(ref_root, out, cfg, w, tables, sysd, compute_stress):
    # this framework's package is also called tt_atom: drop it so the reference's is imported
    for mod in [m for m in sys.modules if m == "tt_atom" or m.startswith("tt_atom.")]:
        del sys.modules[mod]
    sys.path[:] = [p for p in sys.path if not p.endswith("tt-atom_b200")]
    sys.path.insert(0, str(ref_root))
    sys.path.insert(0, str(ref_root / "tests"))
    import mirror                                           # noqa: E402 (reference)
    from tt_atom.geometry import HostGeometry, csd_embedding, radius_graph   # noqa: E402

    pos = torch.from_numpy(sysd["pos"]).float()
    Z = torch.from_numpy(sysd["Z"]).long()
    cell = torch.from_numpy(sysd["cell"]).float() if sysd["pbc"] else None
    pbc = [True] * 3 if sysd["pbc"] else None
    ei, shift = radius_graph(pos, cfg["cutoff"], cell=cell, pbc=pbc)
    C = cfg["sphere_channels"]
    se = csd_embedding(w, torch.tensor([0.0]), torch.tensor([0.0]), C, dataset=cfg["task"])
    se = se[torch.zeros(Z.shape[0], dtype=torch.long)]
    geo = HostGeometry(w, cfg, tables["to_m"], tables["gauss_offset"], tables["gauss_coeff"])
    p = pos.clone().requires_grad_(True)
    strain, edge_vec = None, None
    if compute_stress:
        strain = torch.zeros(3, 3, requires_grad=True)
        ev = p[ei[0]] - p[ei[1]] + shift
        edge_vec = ev + ev @ (0.5 * (strain + strain.T))
    t = geo(p, Z, ei, se, edge_vec=edge_vec, edge_cell_shift=shift if sysd["pbc"] else None)
    ne = mirror.backbone(w, cfg, t["x_init"], t["wigner"], t["wigner_inv"], t["x_edge"],
                         t["edge_envelope"], se, ei, tables["to_grid_mat"], tables["from_grid_mat"])
    E = mirror.energy(ne, w)
    ins = [p] if strain is None else [p, strain]
    g = torch.autograd.grad(E, ins)
    arrs = {"config": np.frombuffer(json.dumps(cfg).encode(), dtype=np.uint8),
            "in@pos": sysd["pos"], "in@Z": sysd["Z"],
            "in@cell": sysd["cell"] if sysd["pbc"] else np.zeros((3, 3), np.float32),
            "in@pbc": np.array(sysd["pbc"]),
            "out@edge_index": ei.numpy(), "out@shift": shift.numpy().astype(np.float32),
            "out@sys_emb": se[0].detach().numpy(),
            "out@energy": np.array([E.item()], np.float32),
            "out@forces": (-g[0]).numpy(), "out@node_embedding": ne.detach().numpy()}
    if compute_stress:
        arrs["out@virial"] = g[1].numpy()
    arrs.update({f"w@{k}": v.numpy() for k, v in w.items()})
    for k in ("to_m", "gauss_offset", "gauss_coeff", "to_grid_mat", "from_grid_mat"):
        arrs[f"host@{k}"] = tables[k].numpy()
    np.savez_compressed(HERE / out, **arrs)
    print("wrote", out, "N", len(sysd["Z"]), "E", ei.shape[1], "energy", E.item())


def _orb_geometry(ref_root, out):
    """Reference Orb edge features (tt_atom/orb_geometry.py:65-97) and their closed-form VJP
    (:100-139) on a seeded periodic cell, from the reference's own code."""
    for mod in [m for m in sys.modules if m == "tt_atom" or m.startswith("tt_atom.")]:
        del sys.modules[mod]
    sys.path[:] = [p for p in sys.path if not p.endswith("tt-atom_b200")]
    sys.path.insert(0, str(ref_root))
    from tt_atom.geometry import radius_graph
    from tt_atom.orb_geometry import host_edge_features, host_edge_features_vjp
    g = torch.Generator().manual_seed(5)
    pos = torch.rand(40, 3, generator=g) * 7.0
    cell = torch.diag(torch.tensor([7.0, 7.5, 8.0]))
    ei, shift = radius_graph(pos, 4.0, cell=cell, pbc=[True] * 3)
    senders, receivers = ei[1], ei[0]
    feat, cut, vec = host_edge_features(pos, senders, receivers, shift, r_max=4.0, num_bases=8)
    g_feat = torch.randn(feat.shape, generator=g)
    g_cut = torch.randn(cut.shape, generator=g)
    forces = host_edge_features_vjp(vec, senders, receivers, 40, g_feat, g_cut, r_max=4.0,
                                    num_bases=8)
    np.savez_compressed(HERE / out, pos=pos.numpy(), cell=cell.numpy(), edge_index=ei.numpy(),
                        shift=shift.numpy(), feat=feat.numpy(), cut=cut.numpy(),
                        g_feat=g_feat.numpy(), g_cut=g_cut.numpy(), forces=forces.numpy())
    print("wrote", out, "E", ei.shape[1])


def _orb_host_terms(ref_root, out, covalent_radii):
    """The reference's host-side Orb terms on seeded inputs: the ZBL pair repulsion
    (tt_atom/orb_model.py:491-587: energy with per-node mean and sum aggregation, forces through
    its own autograd, Voigt stress) and the energy head's normaliser ``host_energy_denormalize``
    (:590-600). They read ``ase.data.covalent_radii``; ASE is not installed here, so a stand-in
    module carries this framework's covalent-radius table (the table itself stays unpinned;
    the ZBL formula, the Z + 1 indexing convention, the envelope and the aggregation are what
    this pins)."""
    import types
    ase = types.ModuleType("ase")
    ase.data = types.ModuleType("ase.data")
    ase.data.covalent_radii = np.asarray(covalent_radii, dtype=np.float64)
    sys.modules["ase"], sys.modules["ase.data"] = ase, ase.data
    for mod in [m for m in sys.modules if m == "tt_atom" or m.startswith("tt_atom.")]:
        del sys.modules[mod]
    sys.path[:] = [p for p in sys.path if not p.endswith("tt-atom_b200")]
    sys.path.insert(0, str(ref_root))
    from tt_atom.geometry import radius_graph
    from tt_atom.orb_model import (host_energy_denormalize, host_zbl_energy, host_zbl_forces,
                                   host_zbl_stress)
    g = torch.Generator().manual_seed(9)
    arrays = {}
    # a compressed periodic SiO2-like cell (many pairs inside the covalent-radius sums) and an
    # aperiodic cluster with short contacts
    n = 48
    cell = torch.diag(torch.tensor([7.2, 7.6, 8.0]))
    pos_p = torch.rand(n, 3, generator=g) @ cell
    Z_p = torch.where(torch.rand(n, generator=g) < 1 / 3, 14, 8).long()
    pos_m = torch.rand(24, 3, generator=g) * 5.0
    Z_m = torch.tensor([1, 6, 7, 8, 9, 16] * 4).long()
    for tag, pos, Z, c in (("p", pos_p, Z_p, cell), ("m", pos_m, Z_m, None)):
        ei, shift = radius_graph(pos, 5.0, cell=c, pbc=[True] * 3 if c is not None else None)
        senders, receivers = ei[1], ei[0]
        vec = pos[receivers].double() - pos[senders].double()
        if c is not None:
            vec = vec + shift.double()
        arrays[f"{tag}_pos"], arrays[f"{tag}_Z"] = pos.numpy(), Z.numpy()
        arrays[f"{tag}_edge_index"], arrays[f"{tag}_shift"] = ei.numpy(), shift.numpy()
        for agg in ("mean", "sum"):
            e = host_zbl_energy(Z, senders, receivers, vec, node_aggregation=agg)
            f = host_zbl_forces(Z, senders, receivers, pos,
                                shift.double() if c is not None else None, node_aggregation=agg)
            arrays[f"{tag}_zbl_energy_{agg}"] = np.float64(e)
            arrays[f"{tag}_zbl_forces_{agg}"] = f.numpy()
            if c is not None:
                st = host_zbl_stress(Z, senders, receivers, vec, c, node_aggregation=agg)
                arrays[f"{tag}_zbl_stress_{agg}"] = st.numpy()
        if c is not None:
            arrays["p_cell"] = c.numpy()
    raw = torch.randn(3, generator=g, dtype=torch.float64)
    mean = torch.randn(1, generator=g, dtype=torch.float64)
    var = torch.rand(1, generator=g, dtype=torch.float64) + 0.5
    refw = torch.randn(118, generator=g, dtype=torch.float64)
    arrays.update(denorm_raw=raw.numpy(), denorm_mean=mean.numpy(), denorm_var=var.numpy(),
                  denorm_ref=refw.numpy())
    arrays["denorm_out"] = np.array([
        float(host_energy_denormalize(raw[k], Z_p, len(Z_p), running_mean=mean,
                                      running_var=var, ref_weight=refw)) for k in range(3)])
    # the other host-side normalisers and the OrbMol conditioning vector
    from tt_atom.orb_model import (host_charge_spin_embedding, host_conservative_force_denormalize,
                                   host_conservative_stress, host_force_denormalize,
                                   host_stress_denormalize)
    fmean, fvar = torch.randn(1, generator=g, dtype=torch.float64), torch.rand(1, generator=g,
                                                                               dtype=torch.float64) + 0.5
    raw_f = torch.randn(7, 3, generator=g, dtype=torch.float64)
    st = [torch.randn(1, generator=g, dtype=torch.float64) for _ in range(2)]
    sv = [torch.rand(1, generator=g, dtype=torch.float64) + 0.5 for _ in range(2)]
    raw_s = torch.randn(6, generator=g, dtype=torch.float64)
    vir = torch.randn(3, 3, generator=g, dtype=torch.float64)
    arrays.update(fnorm_mean=fmean.numpy(), fnorm_var=fvar.numpy(), fnorm_raw=raw_f.numpy(),
                  fnorm_out=host_force_denormalize(raw_f, running_mean=fmean,
                                                   running_var=fvar).numpy(),
                  snorm_dmean=st[0].numpy(), snorm_omean=st[1].numpy(),
                  snorm_dvar=sv[0].numpy(), snorm_ovar=sv[1].numpy(), snorm_raw=raw_s.numpy(),
                  snorm_out=host_stress_denormalize(raw_s, diag_mean=st[0], diag_var=sv[0],
                                                    offdiag_mean=st[1],
                                                    offdiag_var=sv[1]).numpy(),
                  cons_forces=host_conservative_force_denormalize(raw_f, 48,
                                                                  running_var=var).numpy(),
                  cons_virial=vir.numpy(),
                  cons_stress=host_conservative_stress(vir, 48, cell, running_var=var).numpy())
    W_c = torch.randn(128, generator=g, dtype=torch.float64)
    W_s = torch.randn(128, generator=g, dtype=torch.float64)
    cw = {"conditioner.charge_embedding.W": W_c, "conditioner.spin_embedding.W": W_s}
    arrays.update(cs_Wc=W_c.numpy(), cs_Ws=W_s.numpy())
    for tag, (q, sp) in {"a": (-1.0, 2.0), "b": (0.0, 0.0), "c": (2.0, 1.0)}.items():
        arrays[f"cs_{tag}"] = np.array([q, sp])
        arrays[f"cs_out_{tag}"] = host_charge_spin_embedding(cw, q, sp, 2, 512)[0].numpy()
    np.savez_compressed(HERE / out, **arrays)
    del sys.modules["ase"], sys.modules["ase.data"]
    print("wrote", out, {k: np.shape(v) for k, v in arrays.items() if k.endswith("edge_index")})


def _orb_reference_run(ref_root, out, cases):
    """The reference's own Orb forward and reverse pass (tt_atom/orb_model.py:92-338 and
    tt_atom/orb_forces.py:307-372: encoder, attention interaction layers, energy head, the
    hand-written VJP and the host autograd finish through tt_atom/orb_geometry.py), run on the
    CPU through ``ttnn_cpu`` (an fp32 torch stand-in for the ttnn calls), on this framework's
    seeded inputs and random-init weights. ``cases``: name -> (cfg, weights, system, charge,
    spin). Writes raw (normalised-space) energy, forces and, for periodic cells, the virial,
    with the inputs and the (uncapped) edge list."""
    import os
    sys.path.insert(0, str(HERE))
    import ttnn_cpu
    ttnn_cpu.install()
    os.environ["TT_ATOM_ORB_FUSED_SILU_BW"] = "0"
    os.environ["TT_ATOM_ORB_MINIMAL_MATMUL"] = "0"
    for mod in [m for m in sys.modules if m == "tt_atom" or m.startswith("tt_atom.")]:
        del sys.modules[mod]
    sys.path[:] = [p for p in sys.path if not p.endswith("tt-atom_b200")]
    sys.path.insert(0, str(ref_root))
    from tt_atom.geometry import radius_graph
    from tt_atom.orb_forces import energy_and_forces
    from tt_atom.orb_model import (AttentionInteractionLayer, Encoder, EnergyHead,
                                   host_charge_spin_embedding, host_node_features)
    arrays = {}
    for name, (cfg, w, sysd, charge, spin) in cases.items():
        w = {k: v.float() for k, v in w.items()}
        C, Hd = cfg["latent_dim"], cfg["hidden_dim"]
        enc = Encoder(w, None, node_in=cfg["node_embed_size"], edge_in=cfg["edge_embed_size"],
                      latent_dim=C, hidden_dim=Hd)
        layers = [AttentionInteractionLayer(w, f"gnn_stacks.{i}", None, latent_dim=C,
                                            hidden_dim=Hd)
                  for i in range(cfg["num_message_passing_steps"])]
        head = EnergyHead(w, None, latent_dim=C, hidden_dim=Hd)
        pos = torch.from_numpy(sysd["pos"]).float()
        Z = torch.from_numpy(sysd["Z"]).long()
        periodic = bool(sysd["pbc"])
        cell = torch.from_numpy(sysd["cell"]).float() if periodic else None
        ei, shift = radius_graph(pos, cfg["cutoff"], cell=cell, pbc=[True] * 3 if periodic else None)
        cond = None
        if "conditioner.charge_embedding.W" in w:
            cond = host_charge_spin_embedding(w, charge, spin, len(Z), C)
        res = energy_and_forces(enc, layers, head, None, pos=pos, senders=ei[1], receivers=ei[0],
                                atomic_numbers=Z, node_feat=host_node_features(w, Z),
                                cell_shift=shift if periodic else None, r_max=cfg["cutoff"],
                                num_bases=cfg["num_bases"], compute_stress=periodic,
                                cond_nodes=cond)
        arrays.update({f"{name}@pos": pos.numpy(), f"{name}@Z": Z.numpy(),
                       f"{name}@edge_index": ei.numpy(), f"{name}@shift": shift.numpy(),
                       f"{name}@energy": np.float64(res[0]), f"{name}@forces": res[1].numpy(),
                       f"{name}@charge_spin": np.array([charge, spin])})
        if periodic:
            arrays[f"{name}@cell"] = cell.numpy()
            arrays[f"{name}@virial"] = res[2].numpy()
        print(" ", name, "N", len(Z), "E", ei.shape[1], "energy", float(res[0]))
    np.savez_compressed(HERE / out, **arrays)
    print("wrote", out)


def _spectral_reference_run(ref_root, out, cases):
    """The reference's spectral feed-forward (tt_atom/spectral.py:41-188, ``SpectralAtomwise``,
    both its flat block-diagonal path and its per-degree path) on seeded node features, through
    ``ttnn_cpu``. ``cases``: name -> (cfg, weights, prefix, N)."""
    import os
    sys.path.insert(0, str(HERE))
    import ttnn_cpu
    ttnn_cpu.install()
    arrays = {}
    for fused in ("1", "0"):
        os.environ["TT_ATOM_SPECTRAL_FUSED"] = fused
        for mod in [m for m in sys.modules if m == "tt_atom" or m.startswith("tt_atom.")]:
            del sys.modules[mod]
        sys.path[:] = [p for p in sys.path if not p.endswith("tt-atom_b200")]
        if str(ref_root) not in sys.path:
            sys.path.insert(0, str(ref_root))
        from tt_atom.spectral import SpectralAtomwise
        for name, (cfg, w, prefix, N) in cases.items():
            g = torch.Generator().manual_seed(21)
            x = torch.randn(N, 9, cfg["sphere_channels"], generator=g)
            ff = SpectralAtomwise({k: v.float() for k, v in w.items()}, prefix, None,
                                  sphere_channels=cfg["sphere_channels"],
                                  hidden_channels=cfg["hidden_channels"], lmax=2, mmax=2)
            arrays[f"{name}@x"] = x.numpy()
            arrays[f"{name}@out_fused{fused}"] = ff(x).numpy()
            print(" ", name, "fused", fused, "N", N)
    np.savez_compressed(HERE / out, **arrays)
    print("wrote", out)


def main(ref_root):
    ref_root = pathlib.Path(ref_root)
    _reduce_fairchem(ref_root, "golden_tiny.npz", "ref_golden_tiny.npz")
    _reduce_fairchem(ref_root, "golden_bulk_tiny.npz", "ref_golden_bulk.npz")
    sys.path.insert(0, str(REPO / "tt-atom_b200"))
    from tt_atom import configs                              # seeded inputs and weights
    from tt_atom.orb import COVALENT_RADII
    cfg = configs.model_config("tiny")
    w = configs.random_weights(cfg, seed=0)
    t = configs.lmax2_tables()
    off, coeff = configs.gaussian_basis(cfg)
    tables = dict(t, gauss_offset=off, gauss_coeff=coeff)
    mol = configs.tiny_molecule(seed=0)
    fcc = configs.fcc_alloy(reps=(2, 2, 2), seed=1)
    _run_reference(ref_root, "ref_run_tiny_molecule.npz", cfg, w, tables, mol, False)
    _run_reference(ref_root, "ref_run_tiny_fcc.npz", cfg, w, tables, fcc, True)
    _orb_geometry(ref_root, "ref_orb_geometry.npz")
    _orb_host_terms(ref_root, "ref_orb_host_terms.npz", COVALENT_RADII)
    tiny, v3 = configs.orb_config("orb-tiny"), configs.orb_config("orb-v3")
    cases = {
        "tiny_sio2": (tiny, configs.orb_random_weights(tiny, seed=0),
                      configs.amorphous_sio2(n_si=20, n_o=40, seed=2), 0.0, 0.0),
        "tiny_mol": (tiny, configs.orb_random_weights(tiny, seed=0), configs.tiny_molecule(seed=0),
                     0.0, 0.0),
        "tiny_omol": (tiny, configs.orb_random_weights(tiny, seed=3, cond=True),
                      configs.tiny_molecule(seed=1), 1.0, 2.0),
        "v3_sio2": (v3, configs.orb_random_weights(v3, seed=0),
                    configs.amorphous_sio2(n_si=16, n_o=32, seed=5), 0.0, 0.0),
    }
    _orb_reference_run(ref_root, "ref_run_orb.npz", cases)
    sp_tiny = configs.model_config("tiny", ff_type="spectral")
    sp_s1 = configs.model_config("uma-s-1", ff_type="spectral")
    _spectral_reference_run(ref_root, "ref_run_spectral.npz", {
        "tiny": (sp_tiny, configs.random_weights(sp_tiny, seed=0), "blocks.1.atom_wise", 40),
        "uma_s1": (sp_s1, configs.random_weights(sp_s1, seed=0), "blocks.3.atom_wise", 40)})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference_root>")
    main(sys.argv[1])
