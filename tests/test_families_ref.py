"""Model families against the reference framework's own implementations: the same state dict
gives the same energies, forces and stress (float64)."""
import pytest
import torch

from ref_oracle import batch, compare, load_same_weights, ref_module


@pytest.fixture(autouse=True)
def _f64():
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    yield
    torch.set_default_dtype(old)


def _pair(mod_name, ref_cls, mine_cls, seed=0, **kw):
    mod = ref_module(mod_name)
    torch.manual_seed(seed)
    ref = getattr(mod, ref_cls)(**kw).double()
    mine = mine_cls(**kw).double()
    load_same_weights(mine, ref)
    return mine, ref


@pytest.mark.parametrize("readout", ["mlp", "gated"])
@pytest.mark.parametrize("periodic", [False, True])
def test_tensornet(readout, periodic):
    from xnn_b200.models.tensornet import TensorNet
    mine, ref = _pair("xnn.gnn.models.tensornet", "TensorNet", TensorNet, n_features=8, n_interactions=2, n_rbf=8,
                      cutoff=5.0, readout=readout)
    compare(mine, ref, batch(periodic), periodic)


@pytest.mark.parametrize("hardness", ["element", "environment"])
@pytest.mark.parametrize("periodic", [False, True])
def test_qet(hardness, periodic):
    from xnn_b200.models.qet import QET
    mine, ref = _pair("xnn.gnn.models.qet", "QET", QET, n_features=8, n_interactions=2, n_rbf=8, cutoff=5.0,
                      hardness=hardness)
    b = batch(periodic)
    extra = {"total_charge": torch.tensor([1.0, -1.0] + ([0.0] if not periodic else []))}
    compare(mine, ref, b, periodic, keys=("charges",), **extra)


def _properties(mine, ref, b, train, **extra):
    from ref_oracle import ref_graph
    mine.train(train)
    ref.train(train)
    g = b.clone()
    for k, v in extra.items():
        setattr(g, k, v)
    o, o_ref = mine(g), ref(ref_graph(b, **extra))
    torch.testing.assert_close(o["properties"], o_ref["properties"], rtol=1e-10, atol=1e-11)
    torch.testing.assert_close(o["structure_features"], o_ref["structure_features"], rtol=1e-10, atol=1e-11)


@pytest.mark.parametrize("train", [False, True])
@pytest.mark.parametrize("classification", [False, True])
def test_cgcnn(train, classification):
    from xnn_b200.models.cgcnn import CGCNN
    mine, ref = _pair("xnn.gnn.models.cgcnn", "CGCNN", CGCNN, n_features=8, n_interactions=2, n_rbf=12,
                      cutoff=5.0, max_neighbors=6, atom_features="onehot", classification=classification,
                      dropout=0.0)
    with torch.no_grad():   # non-trivial batch-norm statistics and affine parameters
        for mod in list(ref.modules()):
            if isinstance(mod, torch.nn.BatchNorm1d):
                mod.running_mean.uniform_(-0.5, 0.5); mod.running_var.uniform_(0.5, 2.0)
                mod.weight.uniform_(0.5, 1.5); mod.bias.uniform_(-0.3, 0.3)
    load_same_weights(mine, ref)
    _properties(mine, ref, batch(False, cutoff=5.0), train)


@pytest.mark.parametrize("states", [None, 3])
def test_megnet(states):
    from xnn_b200.models.megnet import MEGNet
    mine, ref = _pair("xnn.gnn.models.megnet", "MEGNet", MEGNet, n_features=8, n_interactions=2, n_rbf=10,
                      cutoff=4.0, n_state_types=states)
    extra = {"state": torch.tensor([0, 2, 1])} if states else {}
    _properties(mine, ref, batch(False, cutoff=4.0), False, **extra)


@pytest.mark.parametrize("preset", ["ani1x", "ani2x", "ani1"])
def test_ani(preset):
    from xnn_b200.models.ani import ANI
    mod = ref_module("xnn.dnn.models.ani")
    torch.manual_seed(0)
    ref = getattr(mod.ANI, preset)().double()
    mine = getattr(ANI, preset)().double()
    load_same_weights(mine, ref)
    sp = [1, 6, 7, 8, 16, 9, 17] if preset == "ani2x" else [1, 6, 7, 8]
    compare(mine, ref, batch(False, cutoff=mine.cutoff, species=sp), rtol=1e-9, atol=1e-9)
    compare(mine, ref, batch(True, cutoff=mine.cutoff), True, rtol=1e-9, atol=1e-9)


_CUTS = [{"kind": "cosine", "r_cut": 5.0}, {"kind": "tanh", "r_cut": 4.0, "r_inner": 0.5},
         {"kind": "polynomial", "r_cut": 4.5, "exponent": 3}]


def _functions(species):
    f = []
    for zc in species:
        for zn in species:
            f.append({"element": zc, "type": 2, "neighbors": [zn], "eta": 0.3, "rs": 1.0, "cutoff": 1})
            f.append({"element": zc, "type": 1, "neighbors": [zn], "n_features": 2, "cutoff": 2})
        for a in species:
            for b in species:
                if a <= b:
                    f.append({"element": zc, "type": 3, "neighbors": [a, b], "eta": 0.02, "lambda": -1.0,
                              "zeta": 2.0})
                    f.append({"element": zc, "type": 9, "neighbors": [b, a], "eta": 0.01, "lambda": 1.0,
                              "zeta": 4.0, "cutoff": 1})
                    f.append({"element": zc, "type": 8, "neighbors": [a, b], "eta": 0.001, "theta_s": 100.0})
    return f


@pytest.mark.parametrize("generation,periodic", [(2, False), (2, True), (3, False), (4, False), (4, True)])
def test_hdnnp(generation, periodic):
    from xnn_b200.featurizers.acsf import AtomCenteredSymmetryFunctions
    from xnn_b200.models.hdnnp import HDNNP
    sp = [6, 8] if not periodic else [8]
    refm = ref_module("xnn.dnn.models.hdnnp")
    reff = ref_module("xnn.dnn.featurizers.acsf")
    torch.manual_seed(0)
    kw = dict(generation=generation, hidden=(6, 5), atomic_energies=[-1.0 * z for z in sp],
              screening={"kind": "cosine", "r_cut": 3.0} if generation >= 3 else None)
    ref = refm.HDNNP(sp, reff.AtomCenteredSymmetryFunctions(sp, _CUTS, _functions(sp), mode="center_scale"),
                     **kw).double()
    mine = HDNNP(sp, AtomCenteredSymmetryFunctions(sp, _CUTS, _functions(sp), mode="center_scale"), **kw).double()
    b = batch(periodic, cutoff=5.0, species=sp)
    with torch.no_grad():
        ref.featurizer.stat_min.uniform_(-0.1, 0.1); ref.featurizer.stat_max.uniform_(1.0, 2.0)
        ref.featurizer.stat_avg.uniform_(0.0, 0.5)
    load_same_weights(mine, ref)
    keys = ("charges",) if generation >= 3 else ()
    extra = {"total_charge": torch.tensor([1.0, 0.0] + ([] if periodic else [-1.0]))} if generation >= 3 else {}
    compare(mine, ref, b, periodic, rtol=1e-9, atol=1e-9, keys=keys, **extra)


@pytest.mark.parametrize("symmetrize", [False, True])
def test_nnp1g(symmetrize):
    from xnn_b200.data import collate, structure_to_graph
    from xnn_b200.models.hdnnp import NNP1G
    mine, ref = _pair("xnn.dnn.models.hdnnp", "NNP1G", NNP1G, species=[8, 1, 1], hidden=(7,),
                      coordinates="exponential", symmetrize=symmetrize)
    torch.manual_seed(3)
    ss = [{"pos": torch.randn(3, 3), "atomic_numbers": torch.tensor([8, 1, 1])} for _ in range(2)]
    compare(mine, ref, collate([structure_to_graph(s, 1.0) for s in ss]), rtol=1e-10, atol=1e-10)


@pytest.mark.parametrize("lr_cutoff,dispersion", [(None, False), (8.0, False), (None, True), (8.0, True)])
def test_physnet(lr_cutoff, dispersion):
    from xnn_b200.models.physnet import PhysNet
    mine, ref = _pair("xnn.dnn.models.physnet", "PhysNet", PhysNet, cutoff=5.0, lr_cutoff=lr_cutoff, n_features=8,
                      n_rbf=6, num_blocks=2, use_dispersion=dispersion)
    with torch.no_grad():   # the zero-initialised heads would hide most of the network
        for name, p in ref.named_parameters():
            if "k2f" in name or "output_blocks" in name:
                p.uniform_(-0.3, 0.3)
    load_same_weights(mine, ref)
    if dispersion:   # the same radii tables (the reference keeps float32 roundings of them)
        for name in ("_d3_rcov", "_d3_r2r4", "_d3_c6ab"):
            getattr(mine, name).copy_(getattr(ref, name))
    b = batch(False, cutoff=lr_cutoff or 5.0)
    compare(mine, ref, b, rtol=1e-10, atol=1e-10, keys=("charges", "nh_loss"),
            total_charge=torch.tensor([1.0, 0.0, -2.0]))


@pytest.mark.parametrize("charge_model", ["recursive", "qeq"])
def test_qrnn(charge_model):
    from xnn_b200.models.qrnn import QRNN
    mine, ref = _pair("xnn.dnn.models.qrnn", "QRNN", QRNN, hidden=(8, 6), charge_model=charge_model)
    b = batch(False, cutoff=mine.cutoff, species=[1, 6, 7, 8, 16, 17])
    compare(mine, ref, b, rtol=1e-9, atol=1e-9, keys=("charges",), total_charge=torch.tensor([1.0, 0.0, -1.0]))


@pytest.mark.parametrize("energy_constraint,symmetric", [(False, False), (True, False), (False, True)])
def test_sgdml_fit_and_predict(energy_constraint, symmetric):
    """Both frameworks fit the same training set; the fitted models agree on new structures."""
    from xnn_b200.data import collate, structure_to_graph
    from xnn_b200.models.sgdml import SGDML
    refm = ref_module("xnn.krnn.models.sgdml")
    z = torch.tensor([8, 1, 1, 6])
    torch.manual_seed(4)
    base = torch.tensor([[0.0, 0.0, 0.0], [0.95, 0.1, 0.0], [-0.3, 0.9, 0.1], [0.2, -0.4, 1.4]])

    def structs(k):
        out = []
        for _ in range(k):
            p = base + 0.05 * torch.randn(4, 3)
            d = torch.cdist(p, p) + torch.eye(4)
            e = (1.0 / d).triu(1).sum()
            f = -torch.autograd.functional.jacobian(lambda q: (1.0 / (torch.cdist(q, q) + torch.eye(4))).triu(1).sum(), p)
            out.append({"pos": p, "atomic_numbers": z, "energy": e.reshape(1), "forces": f})
        return [structure_to_graph(s, 1.0) for s in out]

    train, test = structs(6), structs(3)
    perms = [[0, 1, 2, 3], [0, 2, 1, 3]] if symmetric else None
    mine = SGDML([8, 1, 1, 6], sigma=2.0, use_symmetries=False)
    ref = refm.SGDML([8, 1, 1, 6], sigma=2.0, use_symmetries=False)
    mine.fit(train, energy_constraint=energy_constraint, perms=perms)
    ref.fit(train, energy_constraint=energy_constraint, perms=perms, solver="analytic")
    b = collate(test)
    compare(mine, ref, b, rtol=1e-7, atol=1e-8)


@pytest.mark.parametrize("coulomb,channels,periodic", [("simple", 1, False), ("simple", 2, False), ("dsf", 1, True),
                                                      ("ewald", 1, True), (None, 1, False)])
def test_aimnet2(coulomb, channels, periodic):
    from xnn_b200.models.aimnet2 import AIMNet2
    sp = [1, 6, 7, 8] if not periodic else [8]
    kw = dict(species=sp, cutoff=4.0, n_features=4, n_rbf=6, hidden=[[12, 10], [12, 10], [12, 10, 8]],
              n_vector_combinations=3, aim_size=8, readout_hidden=(6,), charge_channels=channels, coulomb=coulomb,
              lr_cutoff=6.0, atomic_energies=[-0.5 * z for z in sp])
    mine, ref = _pair("xnn.gnn.models.aimnet2", "AIMNet2", AIMNet2, **kw)
    b = batch(periodic, cutoff=mine.cutoff, species=sp if not periodic else None)
    tq = torch.tensor([1.0, 0.0] + ([] if periodic else [-1.0]))
    extra = {"total_charge": tq}
    if channels == 2:
        extra["spin_multiplicity"] = torch.tensor([2.0, 1.0, 2.0])
    compare(mine, ref, b, periodic, rtol=1e-9, atol=1e-9, keys=("charges",), **extra)


@pytest.mark.parametrize("max_nu,passes,receiver", [(2, 1, False), (3, 2, True), (4, 1, False)])
def test_cace(max_nu, passes, receiver):
    from xnn_b200.models.cace import CACE
    mine, ref = _pair("xnn.gnn.models.cace", "CACE", CACE, species=[1, 6, 7, 8], cutoff=4.5, n_atom_basis=2,
                      n_rbf=4, max_l=3, max_nu=max_nu, num_message_passing=passes, embed_receiver_nodes=receiver,
                      readout_hidden=[8], atomic_energies=[-0.5, -1.0, -1.5, -2.0])
    compare(mine, ref, batch(False, cutoff=4.5, species=[1, 6, 7, 8]), rtol=1e-9, atol=1e-9)
    compare(mine, ref, batch(True, cutoff=4.5, species=[8]), True, rtol=1e-9, atol=1e-9)


@pytest.mark.parametrize("cls_name,gate,ref_basis", [("DimeNet", "kj", False), ("DimeNet", "ji", True),
                                                     ("DimeNetPP", "kj", False), ("DimeNetPP", "ji", False)])
def test_dimenet(cls_name, gate, ref_basis):
    from xnn_b200.models import dimenet as M
    kw = dict(n_features=8, n_interactions=2, n_rbf=4, n_spherical=3, cutoff=4.5, radial_gate=gate,
              reference_basis=ref_basis, n_output_layers=1, species=[1, 6, 7, 8], atomic_energies=[-1.0, -2, -3, -4])
    kw.update(dict(n_bilinear=3) if cls_name == "DimeNet" else dict(n_triplet_features=6, n_basis_features=3,
                                                                     n_output_features=10))
    mine, ref = _pair("xnn.gnn.models.dimenet", cls_name, getattr(M, cls_name), **kw)
    compare(mine, ref, batch(False, cutoff=4.5), rtol=1e-9, atol=1e-9)
    compare(mine, ref, batch(True, cutoff=4.5), True, rtol=1e-9, atol=1e-9)


@pytest.mark.parametrize("quadruplets,direct", [(False, False), (True, False), (False, True)])
def test_gemnet(quadruplets, direct):
    from xnn_b200.models.gemnet import GemNet
    kw = dict(n_features=6, n_edge_features=8, n_interactions=1, n_rbf=3, n_spherical=3, cutoff=3.5, int_cutoff=4.0,
              n_triplet_features=4, n_quadruplet_features=4, n_rbf_features=3, n_cbf_features=3, n_sbf_features=4,
              n_bilinear_triplet=5, n_bilinear_quadruplet=4, quadruplets=quadruplets, direct_forces=direct,
              forces_coupled=direct, species=[1, 6, 7, 8], atomic_energies=[-1.0, -2, -3, -4])
    mine, ref = _pair("xnn.gnn.models.gemnet", "GemNet", GemNet, **kw)
    with torch.no_grad():
        for fac in ref.scale_factors().values():
            fac.scale_factor.uniform_(0.5, 1.5)
    load_same_weights(mine, ref)
    ref.set_use_fast(False)
    b = batch(False, cutoff=mine.cutoff)
    compare(mine, ref, b, rtol=1e-9, atol=1e-9)
    if not direct:
        compare(mine, ref, batch(True, cutoff=mine.cutoff), True, rtol=1e-9, atol=1e-9)
    from ref_oracle import ref_graph
    fitted, fitted_ref = mine.fit_scaling_factors([b.clone()]), ref.fit_scaling_factors([ref_graph(b)])
    assert fitted.keys() == fitted_ref.keys()
    for k in fitted:
        assert abs(fitted[k] - fitted_ref[k]) < 1e-9 * abs(fitted_ref[k]), k


@pytest.mark.parametrize("influence,vector_cutoff,nb", [("both", True, True), ("keys", False, False),
                                                        ("values", True, True), ("none", False, True)])
def test_et(influence, vector_cutoff, nb):
    from xnn_b200.models.et import EquivariantTransformer
    mine, ref = _pair("xnn.trfnn.models.et", "EquivariantTransformer", EquivariantTransformer, n_features=8,
                      n_interactions=2, n_rbf=6, cutoff=4.5, num_heads=2, distance_influence=influence,
                      vector_cutoff=vector_cutoff, neighbor_embedding=nb, species=[1, 6, 7, 8],
                      atomic_energies=[-1.0, -2, -3, -4])
    ref.set_use_fast(False)
    compare(mine, ref, batch(False, cutoff=4.5), rtol=1e-9, atol=1e-9)
    compare(mine, ref, batch(True, cutoff=4.5), True, rtol=1e-9, atol=1e-9)


@pytest.mark.parametrize("elec,disp,layers", [(True, False, 3), (False, True, 2), (True, True, 4)])
def test_bamboo(elec, disp, layers):
    from xnn_b200.models.bamboo import BAMBOO
    mine, ref = _pair("xnn.hybnn.models.bamboo", "BAMBOO", BAMBOO, dim=8, num_rbf=6, cutoff=5.0, n_layers=layers,
                      num_heads=2, use_electrostatics=elec, use_dispersion=disp, disp_cutoff=5.0)
    ref.set_use_fast(False)
    if disp:   # the same radii tables (the reference keeps float32 roundings of them)
        for name in ("_rcov", "_r2r4", "_c6ab"):
            getattr(mine.dispersion, name).copy_(getattr(ref.dispersion, name))
    compare(mine, ref, batch(False, cutoff=5.0), rtol=1e-9, atol=1e-9, keys=("charges",),
            total_charge=torch.tensor([0.0, 1.0, -1.0]))


@pytest.mark.parametrize("norm,blocks", [(None, 3), ("batch", 2)])
def test_cnn3d(norm, blocks):
    from xnn_b200.models.cnn3d import CNN3D
    mine, ref = _pair("xnn.cnn.models.cnn3d", "CNN3D", CNN3D, species=[1, 6, 7, 8], cutoff=3.5, grid_size=7,
                      n_features=8, n_blocks=blocks, kernel_size=3, normalization=norm,
                      atomic_energies=[-1.0, -2, -3, -4])
    with torch.no_grad():
        ref.readout[-1].weight.uniform_(-0.5, 0.5)
    load_same_weights(mine, ref)
    ref.set_use_fast(False)
    compare(mine, ref, batch(False, cutoff=3.5, species=[1, 6, 7, 8]), rtol=1e-9, atol=1e-9)


@pytest.mark.parametrize("opts,periodic", [(dict(charge_solve=True), False),
                                           (dict(charge_solve=True, hardness="features"), True),
                                           (dict(charge_solve=True, fragments=True), False),
                                           (dict(method="pme", constrain_charge=True), True),
                                           (dict(constrain_charge=True, charge_weights="learned", dielectric=2.0),
                                            False)])
def test_latent_ewald_options(opts, periodic):
    from xnn_b200.models.les import LatentEwald
    from xnn_b200.models.schnet import SchNet
    les_ref = ref_module("xnn.common.models.les")
    schnet_ref = ref_module("xnn.gnn.models.schnet")
    torch.manual_seed(0)
    kw = dict(n_features=8, n_interactions=2, n_rbf=6, cutoff=5.0)
    ref = les_ref.LatentEwald(schnet_ref.SchNet(**kw), n_channels=2, **opts).double()
    mine = LatentEwald(SchNet(**kw), n_channels=2, **opts).double()
    load_same_weights(mine, ref)
    if periodic:
        b = batch(True, cutoff=5.0)
        extra = {"total_charge": torch.tensor([0.0, 1.0])}
    else:
        b = batch(False, cutoff=5.0, species=[11, 17, 6, 8, 1, 1] if opts.get("fragments") else None)
        extra = {"total_charge": torch.tensor([0.0, 0.0, 0.0] if opts.get("fragments") else [1.0, 0.0, -1.0])}
    keys = ("les_charges", "energy_lr") + (("energy_charge",) if opts.get("charge_solve") else ())
    compare(mine, ref, b, periodic, rtol=1e-8, atol=1e-8, keys=keys, **extra)


@pytest.mark.parametrize("opts,periodic", [
    (dict(), False),
    (dict(attention="exact", n_residual=2), False),
    (dict(lr_cutoff=6.0), True),
    (dict(lr_cutoff=6.0, ewald=True, spin_embedding=False, exp_weighting=True), True),
    (dict(nonlocal_interactions=False, zbl_repulsion=False, d4_dispersion=False), False),
])
def test_spookynet(opts, periodic):
    from xnn_b200.models.spookynet import SpookyNet
    mine, ref = _pair("xnn.hybnn.models.spookynet", "SpookyNet", SpookyNet, n_features=8, n_interactions=2, n_rbf=6,
                      cutoff=4.0, seed=3, **opts)
    ref.set_use_fast(False)
    with torch.no_grad():   # the zero-initialised output layers and biases carry values
        for p_ref in ref.parameters():
            p_ref.add_(0.05 * torch.randn_like(p_ref))
    load_same_weights(mine, ref)
    b = batch(periodic, cutoff=6.0 if periodic else 4.0)
    ng = 2 if periodic else 3
    extra = {"total_charge": torch.tensor([1.0, -1.0, 0.0][:ng]), "spin_multiplicity": torch.tensor([2.0, 1.0, 3.0][:ng])}
    compare(mine, ref, b, periodic, rtol=1e-9, atol=1e-9, keys=("charges", "dipole", "energy_dispersion"), **extra)


# the reference's e3nn-based models run on this framework's o3 (see ref_oracle): their model logic
# against these implementations with one state dict
@pytest.mark.parametrize("kw", [dict(), dict(l_max=1, n_layers=2, num_features=8, resnet=True)])
@pytest.mark.parametrize("periodic", [False, True])
def test_nequip(kw, periodic):
    from xnn_b200.models.nequip import NequIP
    mine, ref = _pair("xnn.gnn.models.nequip", "NequIP", NequIP, species=[1, 6, 7, 8], cutoff=4.0, **kw)
    compare(mine, ref, batch(periodic, cutoff=4.0, species=[1, 6, 7, 8]), periodic, rtol=1e-9, atol=1e-9)


@pytest.mark.parametrize("kw", [dict(), dict(hidden_irreps="16x0e+16x1o", max_ell=2, correlation=2, num_interactions=2)])
@pytest.mark.parametrize("periodic", [False, True])
def test_mace(kw, periodic):
    from xnn_b200.models.mace import MACE
    mine, ref = _pair("xnn.gnn.models.mace", "MACE", MACE, species=[1, 6, 7, 8], cutoff=4.0, **kw)
    if hasattr(ref, "set_use_fast"):
        ref.set_use_fast(False)
    compare(mine, ref, batch(periodic, cutoff=4.0, species=[1, 6, 7, 8]), periodic, rtol=1e-9, atol=1e-9)


@pytest.mark.parametrize("kw", [dict(), dict(l_max=2, num_layers=3, num_tensor_features=8, parity="o3_restricted",
                                             avg_num_neighbors=6.0, two_body_latent=[16, 32], latent=[32],
                                             env_embed=[16], edge_eng=[16]),
                                dict(parity="so3", latent_resnet=False, num_tensor_features=4)])
@pytest.mark.parametrize("periodic", [False, True])
def test_allegro(kw, periodic):
    from xnn_b200.models.allegro import Allegro
    mine, ref = _pair("xnn.gnn.models.allegro", "Allegro", Allegro, species=[1, 6, 7, 8], cutoff=4.0, **kw)
    if hasattr(ref, "set_use_fast"):
        ref.set_use_fast(False)
    with torch.no_grad():
        ref._resnet_params.copy_(torch.linspace(-0.5, 0.5, ref._resnet_params.numel()))
    load_same_weights(mine, ref)
    compare(mine, ref, batch(periodic, cutoff=4.0, species=[1, 6, 7, 8]), periodic, rtol=1e-9, atol=1e-9)


_SMALL_EQUIFORMER = dict(irreps_node_embedding="16x0e+8x1e+4x2e", irreps_head="8x0e+4x1e+2x2e", num_heads=2,
                         irreps_mlp_mid="24x0e+12x1e+6x2e", irreps_feature="32x0e", n_rbf=8, radial_hidden=[16],
                         n_interactions=2, cutoff=4.0)


@pytest.mark.parametrize("kw", [dict(), dict(attention="dot_product", radial_basis="gaussian", rescale_degree=True),
                                dict(nonlinear_message=False, radial_basis="bessel", smooth_cutoff=True),
                                dict(irreps_node_embedding="16x0e+4x0o+4x1e+4x1o", irreps_head="8x0e+2x0o+2x1e+2x1o",
                                     irreps_mlp_mid="24x0e+6x0o+6x1e+6x1o")])
@pytest.mark.parametrize("periodic", [False, True])
def test_equiformer(kw, periodic):
    from xnn_b200.models.equiformer import Equiformer
    mine, ref = _pair("xnn.trfnn.models.equiformer", "Equiformer", Equiformer, **{**_SMALL_EQUIFORMER, **kw})
    if hasattr(ref, "set_use_fast"):
        ref.set_use_fast(False)
    compare(mine, ref, batch(periodic, cutoff=4.0), periodic, rtol=1e-9, atol=1e-9)


@pytest.mark.parametrize("kw", [dict(), dict(normalization="batch", fields=[[4, 2, 1], [3, 2], [6]], strides=[1, 2, 1],
                                             bandlimit="conservative", activation="relu")])
@pytest.mark.parametrize("train", [False, True])
def test_se3cnn(kw, train):
    from xnn_b200.models.se3cnn import SteerableCNN
    mine, ref = _pair("xnn.cnn.models.steerable", "SteerableCNN", SteerableCNN, species=[1, 6, 7, 8], cutoff=3.5,
                      grid_size=9, n_features=6, n_blocks=3, l_max=2, kernel_size=3, atomic_energies=[-1.0, -2, -3, -4],
                      **kw)
    with torch.no_grad():
        ref.readout[-1].weight.uniform_(-0.5, 0.5)
    load_same_weights(mine, ref)
    if hasattr(ref, "set_use_fast"):
        ref.set_use_fast(False)
    mine.train(train)
    ref.train(train)
    compare(mine, ref, batch(False, cutoff=3.5, species=[1, 6, 7, 8]), rtol=1e-9, atol=1e-9)


@pytest.mark.parametrize("kw", [dict(), dict(normalization=None, set_readout=[6, 4, 6], cutoff_fn="cosine", exponent=2.0)])
@pytest.mark.parametrize("train", [False, True])
def test_s2cnn(kw, train):
    from xnn_b200.models.s2cnn import SphericalCNN
    mine, ref = _pair("xnn.cnn.models.spherical", "SphericalCNN", SphericalCNN, species=[1, 6, 7, 8], cutoff=3.5,
                      bandwidth=4, features=[3, 5], bandwidths=[4, 2], n_beta=1, n_gamma=2,
                      atomic_energies=[-1.0, -2, -3, -4], **kw)
    with torch.no_grad():
        for m in (ref.readout, ref.set_readout["psi"] if ref.set_readout is not None else ref.readout):
            m[-1].weight.uniform_(-0.5, 0.5)
    load_same_weights(mine, ref)
    if hasattr(ref, "set_use_fast"):
        ref.set_use_fast(False)
    mine.train(train)
    ref.train(train)
    compare(mine, ref, batch(False, cutoff=3.5, species=[1, 6, 7, 8]), rtol=1e-8, atol=1e-9)


_SMALL_EQV2 = dict(n_features=8, n_interactions=2, cutoff=4.0, n_rbf=8, l_max=2, m_max=2, num_heads=2,
                   attn_hidden_channels=6, attn_alpha_channels=4, attn_value_channels=3, ffn_hidden_channels=8,
                   edge_channels=8, grid_resolution=8, species=[1, 6, 7, 8], atomic_energies=[-1.0, -2, -3, -4])


@pytest.mark.parametrize("kw", [dict(), dict(activation="gate", norm_type="layer_norm", use_grid_mlp=False),
                                dict(l_max=3, m_max=1, activation="s2", norm_type="rms_norm_sh", grid_resolution=None,
                                     use_m_share_rad=True, use_attn_renorm=False),
                                dict(share_atom_edge_embedding=True, smooth_cutoff=True, activation="sep_s2",
                                     use_grid_mlp=False),
                                dict(direct_forces=True, m_max=1)])
@pytest.mark.parametrize("periodic", [False, True])
def test_equiformer_v2(kw, periodic):
    from xnn_b200.models.equiformer_v2 import EquiformerV2
    cfg = {**_SMALL_EQV2, **kw}
    mine, ref = _pair("xnn.trfnn.models.equiformer_v2", "EquiformerV2", EquiformerV2, **cfg)
    if hasattr(ref, "set_use_fast"):
        ref.set_use_fast(False)
    compare(mine, ref, batch(periodic and not cfg.get("direct_forces"), cutoff=4.0, species=[1, 6, 7, 8]),
            periodic and not cfg.get("direct_forces"), rtol=1e-9, atol=1e-9)


@pytest.mark.parametrize("periodic", [False, True])
def test_acsf_fit_scaling_matches_reference(periodic):
    from xnn_b200.featurizers.acsf import AtomCenteredSymmetryFunctions
    reff = ref_module("xnn.dnn.featurizers.acsf")
    sp = [6, 8] if not periodic else [8]
    mine = AtomCenteredSymmetryFunctions(sp, _CUTS, _functions(sp), mode="center_scale").double()
    ref = reff.AtomCenteredSymmetryFunctions(sp, _CUTS, _functions(sp), mode="center_scale").double()
    graphs = [batch(periodic, cutoff=5.0, species=sp, seed=s) for s in (2, 5)]
    mine.fit_scaling([g.clone() for g in graphs])
    from ref_oracle import ref_graph
    ref.fit_scaling([ref_graph(g) for g in graphs])
    for name in ("stat_min", "stat_max", "stat_avg"):
        torch.testing.assert_close(getattr(mine, name), getattr(ref, name), rtol=1e-12, atol=1e-12, msg=name)
