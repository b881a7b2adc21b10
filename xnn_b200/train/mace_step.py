"""One MACE training step written out by hand: energies, forces, the loss and every parameter
gradient, with no autograd graph over the model.

A force-matching loss ``L(E, F)`` with ``F = -dE/dx`` needs ``dL/dtheta``. Writing
``a_s = dL/dE_s`` and ``g_i = dL/dF_i`` (both evaluated at the current forces),

    dL/dtheta = d/dtheta [ sum_s a_s E_s  -  E_dot ],     E_dot = sum_i g_i . dE/dx_i ,

where ``E_dot`` is the directional derivative of the energy when every atom moves along
``g_i`` and ``a``, ``g`` are held fixed. So the step is

1. the energy forward pass (every intermediate kept);
2. the force pass: the reverse sweep of ``E`` towards the positions only;
3. the loss, ``a`` and ``g``;
4. a tangent (forward-mode) sweep along ``x_dot = g`` that carries ``X_dot`` next to every
   intermediate ``X``: ``v_dot = g_dst - g_src`` per edge, ``r_dot`` and ``Y_dot`` from the edge
   geometry, ``R_dot = R'(r) r_dot`` from the radial network (whose forward pass already carries
   ``R' = dR/dr`` in stacked rows), and the product rule through the convolution, the linears
   and the symmetric contraction;
5. the reverse sweep of ``Phi = a . E - E_dot`` towards the parameters, which moves a pair of
   cotangents ``(X_bar, X_dot_bar)`` through every stage. Cotangents of quantities that depend
   on the positions only (``Y``, ``r``, their tangents) are never formed.

Each linear stage handles primal and tangent rows with the same matrix, so its weight gradient
is one reduction over both, ``W_bar = X^T X_bar + X_dot^T X_dot_bar``; the symmetric contraction
needs its gradient, its Hessian-vector product and the gradient of its invariants; the
convolution (a trilinear form in features, radial weights and harmonics) needs only the
contractions it already has (``csrc/conv.cu``).

This replaces, for MACE with scalar hidden features, the reference's energy-and-force
training step: ``Trainer`` computes the energy, the forces by ``torch.autograd.grad(...,
create_graph=True)`` and back-propagates the loss through that graph
(``src/xnn/common/train/trainer.py:1117``, ``src/xnn/common/models/outputs.py:209``). The
gradients are the same numbers (checked against autograd in float64), reached with a fixed
schedule of kernels and without the autograd engine's bookkeeping.

On the CPU every stage runs as PyTorch operations (the checking path); on CUDA the stages are
the package's kernels.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch
from torch import Tensor
from torch.nn import functional as F

from ..ops import gemm
from ..ops import mace_ops as K
from ..ops import node_gemm as NG
from ..ops import radial as RAD
from ..ops.scatter import structure_sum


# ----------------------------------------------------------------------------- eligibility
def supports(potential, optim) -> Tuple[bool, str]:
    """Whether the hand-written step covers this model and loss (else the autograd step runs)."""
    from ..models.mace import MACE, LinearReadout, NonLinearReadout
    m = getattr(potential, "model", None)
    if not isinstance(m, MACE):
        return False, "not a MACE model"
    if type(potential).__name__ != "ForceStressOutput" or getattr(potential, "compute_stress", False):
        return False, "needs a ForceStressOutput without stress"
    if not m.fast_eligible():
        return False, "architecture outside the fused path"
    if any(not blk.residual for blk in m.interactions):
        return False, "non-residual interaction blocks"
    if any(not p.use_sc for p in m.products):
        return False, "product without self-connection"
    for k, ro in enumerate(m.readouts):
        last = k == len(m.readouts) - 1
        if not isinstance(ro, NonLinearReadout if last else LinearReadout):
            return False, "readout layout"
    if isinstance(m.readouts[-1], NonLinearReadout):
        act = m.readouts[-1].non_linearity.act
        if act is None or getattr(act, "f", None) is not F.silu:
            return False, "readout activation is not SiLU"
    if m.edge_feat.rbf.freqs.requires_grad:
        return False, "trainable radial basis"
    if optim.stress_weight > 0 or optim.dipole_weight > 0 or optim.polarizability_weight > 0 \
            or optim.charge_weight > 0 or optim.property_weight > 0:
        return False, "loss terms beyond energy and forces"
    if optim.huber_delta or optim.huber_delta_energy or optim.huber_delta_forces:
        return False, "Huber loss"
    if optim.reaction_weight > 0:
        return False, "reaction-energy term"
    return True, ""


def _silu_parts(q: Tensor):
    s = torch.sigmoid(q)
    f = q * s
    f1 = s * (1.0 + q * (1.0 - s))
    f2 = s * (1.0 - s) * (2.0 + q * (1.0 - 2.0 * s))
    return f, f1, f2


# ----------------------------------------------------------------------------- operations
class _Ops:
    """Convolution, symmetric contraction and edge geometry, as kernels (CUDA) or PyTorch (CPU)."""

    def __init__(self, cuda: bool, lmax: int, corr: int, ef):
        self.cuda = cuda
        self.lmax, self.P, self.D = lmax, lmax + 1, (lmax + 1) ** 2
        self.corr = corr
        self.ef = ef
        self.lidx = torch.repeat_interleave(torch.arange(self.P), torch.tensor([2 * l + 1 for l in range(self.P)]))

    # ---------------------------------------------------------------- geometry
    def geometry(self, vec: Tensor):
        ef = self.ef
        Y, _ = K.edge_features_torch(vec, self.lmax, ef.rbf.freqs.to(vec), ef.rbf.norm, ef.cutoff, ef.envelope.p) \
            if not self.cuda else K._C().edge_geometry_fwd(vec.contiguous(), self.lmax, ef.rbf.freqs.to(vec),
                                                          float(ef.rbf.norm), float(ef.cutoff), int(ef.envelope.p))
        return Y, torch.linalg.norm(vec, dim=-1)

    def geometry_vjp(self, vec: Tensor, gY: Tensor) -> Tensor:
        ef = self.ef
        if self.cuda:
            return K._C().edge_geometry_bwd(vec.contiguous(), self.lmax, ef.rbf.freqs.to(vec), float(ef.rbf.norm),
                                            float(ef.cutoff), int(ef.envelope.p), gY.contiguous(), None)
        with torch.enable_grad():
            v = vec.detach().requires_grad_(True)
            Y, _ = K.edge_features_torch(v, self.lmax, ef.rbf.freqs.to(v), ef.rbf.norm, ef.cutoff, ef.envelope.p)
            (g,) = torch.autograd.grad(Y, v, gY)
        return g

    def geometry_jvp(self, vec: Tensor, u: Tensor) -> Tensor:
        ef = self.ef
        if self.cuda:
            dY, _ = K._C().edge_geometry_jvp(vec.contiguous(), self.lmax, ef.rbf.freqs.to(vec), float(ef.rbf.norm),
                                              float(ef.cutoff), int(ef.envelope.p), u.contiguous(), True, False)
            return dY
        fn = lambda v: K.edge_features_torch(v, self.lmax, ef.rbf.freqs.to(v), ef.rbf.norm, ef.cutoff,  # noqa: E731
                                             ef.envelope.p)[0]
        return torch.func.jvp(fn, (vec,), (u,))[1]

    # ---------------------------------------------------------------- convolution
    def gather(self, plan: K.EdgePlan, terms) -> Tensor:
        """``A = sum_terms conv(x, R, Y)`` (D, N, C)."""
        if self.cuda:
            xs, Rs, Ys = zip(*terms)
            N, C = plan.n_nodes, xs[0].shape[1]
            return K._C().conv_gather(N, C, self.P, plan.dst_ptr, plan.src32, plan.dst_perm,
                                      [x.contiguous() for x in xs], [R.contiguous() for R in Rs],
                                      [Y.contiguous() for Y in Ys])
        return K._gather_torch(plan, self.P, terms)

    def tee(self, plan: K.EdgePlan, G: Tensor, Y: Tensor) -> Tensor:
        """``T[e, l, c] = sum_m G[lm, dst_e, c] Y[e, lm]`` (E, P, C)."""
        Gd = G.index_select(1, plan.dst)                       # (D, E, C)
        prod = Gd * Y.t()[:, :, None]
        out = torch.zeros(self.P, Y.shape[0], G.shape[2], dtype=G.dtype, device=G.device)
        out.index_add_(0, self.lidx.to(G.device), prod)
        return out.transpose(0, 1)

    def scatter(self, plan: K.EdgePlan, pairs) -> Tensor:
        """``x_bar[s] = sum_{e out of s} sum_l a[e, l] b[e, l]`` over the (a, b) pairs (N, C)."""
        if self.cuda:
            a, b = zip(*pairs)
            return K._C().conv_scatter(plan.n_senders, a[0].shape[2], self.P, plan.src_ptr, plan.src_perm,
                                       [x.contiguous() for x in a], [y.contiguous() for y in b])
        acc = sum((a * b).sum(1) for a, b in pairs)
        return torch.zeros(plan.n_senders, acc.shape[1], dtype=acc.dtype, device=acc.device).index_add_(0, plan.src, acc)

    def edge_force(self, plan: K.EdgePlan, G: Tensor, Y: Tensor, u: Tensor, R: Tensor, Rd: Tensor,
                   sender: bool = True):
        """Force pass of one convolution with cotangent ``G``: ``(r_bar, Y_bar, u_bar)`` where
        ``r_bar[e] = sum u[s] T R'``, ``Y_bar[e, lm] = sum_c G R u[s]`` and (with ``sender``)
        ``u_bar[s] = sum_{e out of s} sum_l T R`` with ``T = tee(G, Y)``; each edge's term of
        ``u_bar`` is an ``(E, C)`` row of the edge kernel, summed per sender."""
        if self.cuda:
            N, C = plan.n_nodes, u.shape[1]
            g_r, gY, _, _, v = K._C().conv_edge(N, C, self.P, plan.n_edges, plan.dst_ptr, plan.src32,
                                                plan.dst_perm, G.contiguous(), [Y], [u], [False], True, [u], [R],
                                                Rd.contiguous(), R.contiguous() if sender else None)
            ub = K._C().conv_sender_sum(plan.n_senders, plan.src_ptr, plan.src_perm, v) if sender else None
            return g_r, gY, ub
        T = self.tee(plan, G, Y)
        us = u.index_select(0, plan.src)[:, None, :]
        g_r = (us * T * Rd).sum((1, 2))
        Gd = G.index_select(1, plan.dst)                       # (D, E, C)
        gY = (Gd * (R[:, self.lidx.to(R.device), :] * us).transpose(0, 1)).sum(-1).t()
        ub = self.scatter(plan, [(R, T)]) if sender else None
        return g_r, gY, ub

    def edge_terms(self, plan: K.EdgePlan, G: Tensor, Ys, xs) -> Tuple[Optional[Tensor], List[Tensor]]:
        """``gR = sum_k x_k[s] * tee(G, Y_k)`` and every ``tee(G, Y_k)``."""
        if self.cuda:
            N, C = plan.n_nodes, G.shape[2]
            gR, _, T0, T1, _ = K._C().conv_edge(N, C, self.P, plan.n_edges, plan.dst_ptr, plan.src32, plan.dst_perm,
                                             G.contiguous(), [y.contiguous() for y in Ys],
                                             [x.contiguous() if x is not None else None for x in xs],
                                             [True] * len(Ys), any(x is not None for x in xs), [], [], None)
            return gR, [T0, T1][:len(Ys)]
        Ts = [self.tee(plan, G, y) for y in Ys]
        gR = None
        for x, T in zip(xs, Ts):
            if x is not None:
                part = x.index_select(0, plan.src)[:, None, :] * T
                gR = part if gR is None else gR + part
        return gR, Ts

    def dual_reverse(self, plan: K.EdgePlan, G: Tensor, Gd: Tensor, Y: Tensor, Yd: Tensor, rdot: Tensor,
                     u: Tensor, ud: Optional[Tensor], R: Tensor, Rd: Tensor):
        """Reverse of the tangent-carrying convolution for cotangents ``(G, G_dot)``:
        ``(R_bar, R'_bar, u_bar, u_dot_bar)`` (the last ``None`` without ``u_dot``), see
        ``csrc/mace_dual.cu``."""
        if self.cuda and plan.dst_perm is None:
            Rb, Rdb, ub, ubd = K._C().mace_dual_reverse(plan.dst_ptr, plan.src32, plan.src_ptr, plan.src_perm,
                                                         G.contiguous(), Gd.contiguous(), Y.contiguous(),
                                                         Yd.contiguous(), rdot.contiguous(), u.contiguous(),
                                                         None if ud is None else ud.contiguous(), R.contiguous(),
                                                         Rd.contiguous())
            return Rb, Rdb, ub, (ubd if ud is not None else None)
        gR_a, (T1,) = self.edge_terms(plan, G, [Y], [u])
        gR_b, (T2, T4) = self.edge_terms(plan, Gd, [Y, Yd], [ud, u])
        T2r = T2 * rdot[:, None, None]
        Rdbar = u.index_select(0, plan.src)[:, None, :] * T2r
        ub = self.scatter(plan, [(R, T1 + T4), (Rd, T2r)])
        ubd = self.scatter(plan, [(R, T2)]) if ud is not None else None
        return gR_a + gR_b, Rdbar, ub, ubd

    # ---------------------------------------------------------------- symmetric contraction
    def symcon(self, A: Tensor, z: Tensor, W: Tensor) -> Tensor:
        if self.cuda:
            return K._C().symcon_fwd(A.contiguous(), z, W.contiguous(), self.lmax, self.corr)
        return K.symmetric_contraction_torch(A, W, z, self.lmax, self.corr)

    def symcon_vjp(self, A: Tensor, z: Tensor, W: Tensor, g: Tensor) -> Tensor:
        if self.cuda:
            gA, _ = K._C().symcon_bwd(A.contiguous(), z, W.contiguous(), g.contiguous(), self.lmax, self.corr,
                                      True, False)
            return gA
        with torch.enable_grad():
            a = A.detach().requires_grad_(True)
            (gA,) = torch.autograd.grad(K.symmetric_contraction_torch(a, W, z, self.lmax, self.corr), a, g)
        return gA

    def symcon_jvp(self, A: Tensor, z: Tensor, W: Tensor, dA: Tensor) -> Tensor:
        if self.cuda:
            cg, _, _ = K._C().symcon_bwd2(A.contiguous(), z, W.contiguous(), A.new_zeros(A.shape[1:]),
                                          dA.contiguous(), None, self.lmax, self.corr, True, False, False)
            return cg
        fn = lambda a: K.symmetric_contraction_torch(a, W, z, self.lmax, self.corr)  # noqa: E731
        return torch.func.jvp(fn, (A,), (dA,))[1]

    def symcon_dual_reverse(self, A: Tensor, z: Tensor, W: Tensor, dA: Tensor, gB: Tensor, gBd: Tensor):
        """Reverse of ``(B, B_dot) = (S(A), dS(A) . dA)`` for cotangents ``(gB, gBd)``:
        ``(A_bar, dA_bar, Wa_bar)`` with the weight cotangent per atom (N, K, C)."""
        if self.cuda:
            C = K._C()
            gA1, gW1 = C.symcon_bwd(A.contiguous(), z, W.contiguous(), gB.contiguous(), self.lmax, self.corr,
                                    True, True)
            _, cA, cW = C.symcon_bwd2(A.contiguous(), z, W.contiguous(), gBd.contiguous(), dA.contiguous(), None,
                                      self.lmax, self.corr, False, True, True)
            gdA, _ = C.symcon_bwd(A.contiguous(), z, W.contiguous(), gBd.contiguous(), self.lmax, self.corr,
                                  True, False)
            return gA1 + cA, gdA, gW1 + cW
        with torch.enable_grad():
            a = A.detach().requires_grad_(True)
            da = dA.detach().requires_grad_(True)
            Wa = W.index_select(0, z).detach().requires_grad_(True)       # (N, K, C) per-atom weights
            I = K.invariants_torch(a, self.lmax, self.corr)               # (K, N, C)
            B = (Wa * I.transpose(0, 1)).sum(1)
            (dB,) = torch.autograd.grad(B, a, gBd, create_graph=True)    # gBd . dS/dA
            phi = (gB * B).sum() + (dB * da).sum()
            gA, gdA, gWa = torch.autograd.grad(phi, (a, da, Wa))
        return gA, gdA, gWa


# ----------------------------------------------------------------------------- weights
@dataclass
class _Weights:
    """Effective matrices of one step (scaled views of the parameters, detached)."""

    emb: Tensor                      # (n_el, C)
    up: List[Tensor]                 # (C, C)
    sc: List[Tensor]                 # (n_el, C, C)
    radial: List[List[Tensor]]       # effective radial layers
    spec: List[RAD.RadialSpec]
    lin: List[List[Tensor]]          # per degree (C, C), divided by avg_num_neighbors
    sym: List[Tensor]                # (n_el, K, C)
    prod: List[Tensor]               # (C, C)
    ro_lin: List[Tensor]             # (C, 1) for the linear readouts
    ro_w1: Tensor                    # (C, H)
    ro_w2: Tensor                    # (H, 1)
    ro_c: float                      # SiLU normalisation constant


@dataclass
class _Entry:
    """One effective matrix: ``view(param) * scalar`` (times ``col`` per column when given)."""

    param: torch.nn.Parameter
    offset: int
    shape: Tuple[int, ...]
    permute: Optional[Tuple[int, ...]]
    scalar: float
    col: Optional[Tensor] = None

    def base(self, t: Tensor) -> Tensor:
        """The entry's block of ``t`` (a parameter or its gradient) in the parameter's layout."""
        return t.reshape(-1).narrow(0, self.offset, math.prod(self.shape)).view(self.shape)

    def view(self, t: Tensor) -> Tensor:
        v = self.base(t)
        return v.permute(*self.permute) if self.permute is not None else v


class _WeightMap:
    """The effective matrices of a MACE model as scaled views of its parameters.

    Every matrix the step multiplies with is a parameter (or a slice of one) times a constant --
    the e3nn path normalisations, ``1 / avg_num_neighbors``, the radial layers' factors and the
    tensor-product path coefficients per column. So the step builds them with one multi-tensor
    multiply and returns their gradients the same way (scaled and added into the parameters'
    gradient buffers), with no autograd graph over the weights."""

    def __init__(self, m, like: Tensor):
        from ..models.mace_fast import _conv_path_scale
        from ..o3 import wigner_3j
        n_el = len(m.species)
        ef = m.edge_feat
        self.order: Dict[str, object] = {}

        def lin_entries(lin, extra: float = 1.0) -> List[_Entry]:
            out, off = [], 0
            for ins in lin.instructions:
                shp = tuple(int(x) for x in ins.path_shape)
                out.append(_Entry(lin.weight, off, shp, None, float(ins.path_weight) * extra))
                off += math.prod(shp)
            return out

        def species_entry(tp) -> _Entry:
            ins = tp.instructions[0]
            c_in, ne, c_out = (int(x) for x in ins.path_shape)
            l = tp.irreps_out[ins.i_out].ir.l
            cg = float(wigner_3j(l, 0, l, dtype=torch.float64)[0, 0, 0])
            return _Entry(tp.weight, 0, (c_in, ne, c_out), (1, 0, 2), float(ins.path_weight) * cg)

        self.emb = lin_entries(m.node_embedding)[0]
        self.up, self.sc, self.radial, self.spec, self.lin, self.sym, self.prod = [], [], [], [], [], [], []
        for blk, pr in zip(m.interactions, m.products):
            self.up.append(lin_entries(blk.linear_up)[0])
            self.sc.append(species_entry(blk.skip_tp))
            spec = RAD.RadialSpec(blk.conv_tp_weights, _conv_path_scale(blk, like), ef.rbf.freqs, ef.rbf.norm,
                                  ef.cutoff, ef.envelope.p)
            self.spec.append(spec)
            layers = [layer.weight for layer in blk.conv_tp_weights]
            rad = [_Entry(w, 0, tuple(w.shape), None, f) for w, f in zip(layers, spec.factors)]
            rad[-1].col = spec.col_scale
            self.radial.append(rad)
            self.lin.append(lin_entries(blk.linear, 1.0 / float(blk.avg_num_neighbors)))
            con = pr.symmetric_contractions.contractions[0]
            self.sym.append([_Entry(w, 0, tuple(w.shape), None, 1.0) for w in con.weights])
            self.prod.append(lin_entries(pr.linear)[0])
        self.ro_lin = [lin_entries(ro.linear)[0] for ro in m.readouts[:-1]]
        last = m.readouts[-1]
        self.w1 = lin_entries(last.linear_1)[0]
        self.w2 = lin_entries(last.linear_2)[0]
        act = last.non_linearity.act
        self.c = 1.0 if act._is_id else float(act.cst)

    def _flat(self) -> List[_Entry]:
        out = [self.emb] + self.up + self.sc + [e for es in self.radial for e in es] + \
            [e for es in self.lin for e in es] + [e for es in self.sym for e in es] + self.prod + self.ro_lin + \
            [self.w1, self.w2]
        return out

    def build(self) -> _Weights:
        ents = self._flat()
        # one multi-tensor multiply over blocks in the parameters' own (contiguous) layout; the
        # permutations are views of its outputs
        scaled = torch._foreach_mul([e.base(e.param.detach()) for e in ents], [e.scalar for e in ents])
        eff = {}
        for e, v in zip(ents, scaled):
            if e.permute is not None:
                v = v.permute(*e.permute)
            eff[id(e)] = v * e.col.to(v) if e.col is not None else v
        g = lambda e: eff[id(e)]  # noqa: E731
        return _Weights(g(self.emb), [g(e) for e in self.up], [g(e) for e in self.sc],
                        [[g(e) for e in es] for es in self.radial], self.spec,
                        [[g(e) for e in es] for es in self.lin],
                        [torch.cat([g(e) for e in es], dim=1) for es in self.sym],
                        [g(e) for e in self.prod], [g(e) for e in self.ro_lin], g(self.w1), g(self.w2), self.c)

    def interaction_pairs(self, t: int, up, sc, radial, lin, sym, prod, ro=None) -> List[Tuple[_Entry, Tensor]]:
        """(entry, gradient) pairs of interaction ``t`` (its block, product and readout)."""
        pairs: List[Tuple[_Entry, Tensor]] = [(self.up[t], up), (self.sc[t], sc), (self.prod[t], prod)]
        pairs += list(zip(self.radial[t], radial)) + list(zip(self.lin[t], lin))
        k0 = 0
        for e in self.sym[t]:
            k = e.shape[1]
            pairs.append((e, sym[:, k0:k0 + k]))
            k0 += k
        if t < len(self.ro_lin):
            pairs.append((self.ro_lin[t], ro))
        else:
            pairs += [(self.w1, ro[0]), (self.w2, ro[1])]
        return pairs

    def add_grads(self, pairs: Sequence[Tuple[_Entry, Tensor]]) -> None:
        """Add effective-matrix gradients to the parameters' ``.grad`` (created as zeros where
        missing): scaled back by each entry's constants, one multi-tensor add."""
        live = [(e, g) for e, g in pairs if e.param.requires_grad]
        if not live:
            return
        src, dst = [], []
        for e, g in live:
            if e.param.grad is None:
                e.param.grad = torch.zeros_like(e.param)
            if e.col is not None:
                g = g * e.col.to(g)
            if e.permute is not None:
                g = g.permute(*[e.permute.index(k) for k in range(len(e.permute))])
            # both lists contiguous in the parameters' layout, so the multi-tensor kernels take
            # them all in one launch each (mixed strides send every tensor to its own launch)
            src.append(g.contiguous())
            dst.append(e.base(e.param.grad))
        torch._foreach_add_(dst, torch._foreach_mul(src, [e.scalar for e, _ in live]))


# ----------------------------------------------------------------------------- the step
def _per_degree_problems(A: Tensor, Y: Tensor, mats: List[Tensor], packed: Optional[List[Tensor]],
                         accumulate: bool = False) -> List[NG.MM]:
    """Row products ``Y[l-block] = A[l-block] @ mats[l]`` of the component-major ``(D, N, C)``
    tensors, one problem per degree."""
    out = []
    C = A.shape[-1]
    for l, Wl in enumerate(mats):
        sl = slice(l * l, (l + 1) * (l + 1))
        out.append(NG.MM(A[sl].reshape(-1, C), Wl, Y[sl].reshape(-1, Wl.shape[1]),
                         None if packed is None else packed[l], accumulate=accumulate))
    return out


class MACEStep:
    """Loss and parameter gradients of one energy + force training step of a MACE potential.

    ``__call__(batch)`` returns ``(loss, logs, out)`` and accumulates every parameter's gradient
    into its ``.grad``; the loss and logs are the ones of
    :func:`~xnn_b200.train.losses.weighted_loss` for the energy and force terms.

    The node-level products run as a few batched launches (``ops/node_gemm.py``): per stage one
    table of problems, the primal and tangent rows of a product as two problems of one launch,
    the per-element self-connection as one problem per element over the atoms of that element
    (a stable sort by element gives the row permutation and segments). Every weight is packed
    into the tensor-core operand layout once per step.
    """

    def __init__(self, potential, energy_weight: float, force_weight: float):
        self.pot = potential
        self.m = potential.model
        self.we, self.wf = float(energy_weight), float(force_weight)
        self.corr = int(self.m.correlation[0])
        if any(int(c) != self.corr for c in self.m.correlation[:len(self.m.interactions)]):
            raise NotImplementedError("one correlation order for every interaction")
        # constants read once (a captured step may not read device memory from the host)
        self.scale = float(self.m.scale_shift.scale)
        self.shift = float(self.m.scale_shift.shift)
        self._maps: Dict[tuple, _WeightMap] = {}

    def bucket_params(self) -> List[List[torch.nn.Parameter]]:
        """Parameter groups in the order the reverse sweep finishes them: interaction ``T - 1``
        (block, product, readout) first, down to interaction 0; every other parameter (node
        embedding, reference energies) is final only at the end."""
        m = self.m
        groups = []
        for t in range(len(m.interactions) - 1, -1, -1):
            mods = (m.interactions[t], m.products[t], m.readouts[t])
            groups.append([p for mod in mods for p in mod.parameters()])
        return groups

    def __call__(self, b, bucket_hook: Optional[Callable[[int], None]] = None
                 ) -> Tuple[Tensor, Dict[str, Tensor], Dict[str, Tensor]]:
        """``bucket_hook(i)`` is called as soon as the gradients of group ``i`` of
        :meth:`bucket_params` are final (a data-parallel reduction may start there)."""
        m = self.m
        mdt = m.atom_ref.weight.dtype
        if b.compute_dtype is None and b.pos.dtype != mdt:
            b.compute_dtype = mdt          # float64 geometry driving a float32 model, as the module path does
        vec = b.edge_vectors().detach()
        dev, dt = vec.device, vec.dtype
        ops = _Ops(vec.is_cuda, m.max_ell, self.corr, m.edge_feat)
        key = (vec.device, vec.dtype)
        if self._maps.get(key) is None:
            self._maps[key] = _WeightMap(m, vec)
        wmap = self._maps[key]
        Wt = wmap.build()
        n_el, C, T = len(m.species), m.num_features, len(m.interactions)
        P, D = ops.P, ops.D
        N, E = b.num_nodes, vec.shape[0]
        Z = b.atomic_numbers
        z = m.z_to_index[Z].clamp(min=0)
        if b.edge_plan is not None and b.edge_order == "dst":
            plan = K.EdgePlan.from_packed(b.edge_index, N, b.edge_plan)
        else:
            plan = K.EdgePlan.build(b.edge_index, N, assume_dst_sorted=b.edge_order == "dst")
        scale, shift = self.scale, self.shift
        perm, seg = NG.species_sort(z, n_el)
        emb = Wt.emb.detach()
        up = [w.detach() for w in Wt.up]
        scw = [w.detach() for w in Wt.sc]
        lin = [[w.detach() for w in ws] for ws in Wt.lin]
        symw = [w.detach() for w in Wt.sym]
        prod = [w.detach() for w in Wt.prod]
        rol = [w.detach() for w in Wt.ro_lin]
        w1, w2, c_ro = Wt.ro_w1.detach(), Wt.ro_w2.detach(), Wt.ro_c
        radial_w = [[w.detach() for w in ws] for ws in Wt.radial]
        # the matrices of every node product, forward and transposed (reverse) forms
        mats: Dict[str, List[Tensor]] = {"up": [], "sc": [], "rev": [], "lin": [], "linT": [], "prod": [],
                                          "prodT": []}
        for t in range(T):
            mats["up"].append(up[t])
            mats["sc"] += [scw[t][k] for k in range(n_el)]
            mats["rev"] += [(up[t].t(), scw[t][k].t()) for k in range(n_el)]     # stacked rows, packed as is
            mats["lin"] += lin[t]
            mats["linT"] += [w.t() for w in lin[t]]
            mats["prod"].append(prod[t])
            mats["prodT"].append(prod[t].t())
        mats["w1"], mats["w1T"] = [w1], [w1.t()]
        Pk: Dict[str, List[Optional[Tensor]]] = {}
        if NG.kernels(vec):
            flat = [w for key in mats for w in mats[key]]                  # any strides: the pack reads them
            packed = iter(NG.pack(flat))
            Pk = {key: [next(packed) for _ in mats[key]] for key in mats}
        else:
            Pk = {key: [None] * len(mats[key]) for key in mats}

        def sc_problems(t: int, X: Tensor, Y: Tensor) -> List[NG.MM]:
            return [NG.MM(X, scw[t][k], Y, Pk["sc"][t * n_el + k], perm=perm, seg=seg[k:k + 2], rows=N)
                    for k in range(n_el)]

        def rev_problems(t: int, ub: Tensor, Hb: Tensor, Y: Tensor) -> List[NG.MM]:
            """``Y += [u_bar | H_bar] @ [W_up^T ; W_sc[z]^T]`` per element."""
            return [NG.MM(ub, mats["rev"][t * n_el + k], Y, Pk["rev"][t * n_el + k], X1=Hb, perm=perm,
                          seg=seg[k:k + 2], rows=N, accumulate=True) for k in range(n_el)]

        def empty_nc():
            return torch.empty(N, C, dtype=dt, device=dev)

        # ---------------------------------------------------------------- 1. energy forward
        Y, r = ops.geometry(vec)
        Rs, Rds, acts, H0s = [], [], [], []
        for t in range(T):
            R, Rd, a, H0 = RAD._forward(r, radial_w[t], Wt.spec[t])
            Rs.append(R.view(E, P, C))
            Rds.append(Rd.view(E, P, C))
            acts.append(a)
            H0s.append(H0)
        h = [emb.index_select(0, z)]
        u, A, A2, Bs = [], [], [], []
        for t in range(T):
            u.append(empty_nc())
            hn = empty_nc()                                            # sc now, h_{t+1} after the product
            NG.mm([NG.MM(h[t], up[t], u[t], Pk["up"][t])] + sc_problems(t, h[t], hn))
            A.append(ops.gather(plan, [(u[t], Rs[t], Y)]))
            A2.append(torch.empty_like(A[t]))
            NG.mm(_per_degree_problems(A[t], A2[t], lin[t], Pk["lin"][P * t:P * t + P]))
            Bs.append(ops.symcon(A2[t], z, symw[t]))
            NG.mm([NG.MM(Bs[t], prod[t], hn, Pk["prod"][t], accumulate=True)])
            h.append(hn)
        q = torch.empty(N, w1.shape[1], dtype=dt, device=dev)
        NG.mm([NG.MM(h[T], w1, q, Pk["w1"][0])])
        f0, f1, f2 = _silu_parts(q)
        inter = (c_ro * f0) @ w2
        for t in range(T - 1):
            inter = inter + h[t + 1] @ rol[t]
        e0 = m.atom_ref.weight.detach()[Z, 0]
        node_e = e0 + scale * inter.squeeze(-1) + shift
        energy = structure_sum(node_e, b.batch, b.num_graphs)

        # ---------------------------------------------------------------- 2. force pass
        hb = [None] * (T + 1)
        qb = (scale * c_ro) * f1 * w2.t()                             # d(node_e)/dq
        hb[T] = empty_nc()
        NG.mm([NG.MM(qb, w1.t(), hb[T], Pk["w1T"][0])])
        for t in range(T - 1):
            hb[t + 1] = (scale * rol[t].t()).expand(N, C).contiguous()
        g_r = None
        gY = None
        for t in range(T - 1, -1, -1):
            Bb = empty_nc()
            NG.mm([NG.MM(hb[t + 1], prod[t].t(), Bb, Pk["prodT"][t])])
            A2b = ops.symcon_vjp(A2[t], z, symw[t], Bb)
            Ab = torch.empty_like(A2b)
            NG.mm(_per_degree_problems(A2b, Ab, [w.t() for w in lin[t]], Pk["linT"][P * t:P * t + P]))
            gr_t, gY_t, ub = ops.edge_force(plan, Ab, Y, u[t], Rs[t], Rds[t], sender=t > 0)
            g_r = gr_t if g_r is None else g_r + gr_t
            gY = gY_t if gY is None else gY + gY_t
            if t > 0:
                NG.mm(rev_problems(t, ub, hb[t + 1], hb[t]))
        rhat = vec / r.clamp_min(1e-30)[:, None]
        vbar = ops.geometry_vjp(vec, gY) + g_r[:, None] * rhat
        fdt = b.pos.dtype
        src, dst = plan.src, plan.dst
        forces = NG.edge_forces(plan, vbar, fdt)

        # ---------------------------------------------------------------- 3. loss
        loss, logs, a_s, g = self._loss(b, energy, forces)

        # ---------------------------------------------------------------- 4. tangent sweep along x_dot = g
        gg = g.to(dt)
        vdot = gg.index_select(0, dst) - gg.index_select(0, src)
        rdot = (rhat * vdot).sum(-1)
        Ydot = ops.geometry_jvp(vec, vdot)
        Yr = Y * rdot[:, None]
        hd = [torch.zeros_like(h[0])]
        ud, Ad, A2d, Bd = [None], [], [], []
        for t in range(T):
            hdn = empty_nc()
            if t > 0:
                ud.append(empty_nc())
                NG.mm([NG.MM(hd[t], up[t], ud[t], Pk["up"][t])] + sc_problems(t, hd[t], hdn))
            terms = [(u[t], Rds[t], Yr), (u[t], Rs[t], Ydot)]
            if t > 0:
                terms.insert(0, (ud[t], Rs[t], Y))
            Ad.append(ops.gather(plan, terms))
            A2d.append(torch.empty_like(Ad[t]))
            NG.mm(_per_degree_problems(Ad[t], A2d[t], lin[t], Pk["lin"][P * t:P * t + P]))
            Bd.append(ops.symcon_jvp(A2[t], z, symw[t], A2d[t]))
            NG.mm([NG.MM(Bd[t], prod[t], hdn, Pk["prod"][t], accumulate=t > 0)])
            hd.append(hdn)
        qd = torch.empty_like(q)
        NG.mm([NG.MM(hd[T], w1, qd, Pk["w1"][0])])

        # ---------------------------------------------------------------- 5. reverse sweep of a.E - E_dot
        ob = (scale * a_s.to(dt)).index_select(0, b.batch)[:, None]   # cotangent of the primal readouts
        obd = torch.full((N, 1), -scale, dtype=dt, device=dev)        # cotangent of the tangent readouts
        pb = ob @ w2.t()
        pbd = obd @ w2.t()
        p_ = c_ro * f0
        pd_ = c_ro * f1 * qd
        gw2 = p_.t() @ ob + pd_.t() @ obd
        qbar = c_ro * (f1 * pb + f2 * qd * pbd)
        qbard = c_ro * f1 * pbd
        gw1 = torch.empty(w1.shape, dtype=w1.dtype, device=w1.device)
        red = [NG.MMT(h[T], qbar, gw1, X1=hd[T], D1=qbard)]     # reductions of the current interaction
        hb = [None] * (T + 1)
        hbd = [None] * (T + 1)
        hb[T], hbd[T] = empty_nc(), empty_nc()
        NG.mm([NG.MM(qbar, w1.t(), hb[T], Pk["w1T"][0]), NG.MM(qbard, w1.t(), hbd[T], Pk["w1T"][0])])
        g_rol = []
        for t in range(T - 1):
            hb[t + 1] = (ob * rol[t].t()).contiguous()
            hbd[t + 1] = (obd * rol[t].t()).contiguous()
            g_rol.append(h[t + 1].t() @ ob + hd[t + 1].t() @ obd)
        # gradient outputs of the reductions: contiguous (the weights may be permuted views)
        fresh = lambda w: torch.empty(w.shape, dtype=w.dtype, device=w.device)  # noqa: E731
        g_up = [fresh(w) for w in up]
        g_sc = [fresh(w) for w in scw]
        g_lin = [[fresh(w) for w in ws] for ws in lin]
        g_prod = [fresh(w) for w in prod]
        g_rad, g_sym = [None] * T, [None] * T
        for t in range(T - 1, -1, -1):
            Hb, Hbd = hb[t + 1], hbd[t + 1]
            red.append(NG.MMT(Bs[t], Hb, g_prod[t], X1=Bd[t], D1=Hbd))
            Bb, Bbd = empty_nc(), empty_nc()
            NG.mm([NG.MM(Hb, prod[t].t(), Bb, Pk["prodT"][t]), NG.MM(Hbd, prod[t].t(), Bbd, Pk["prodT"][t])])
            A2b, A2bd, gWa = ops.symcon_dual_reverse(A2[t], z, symw[t], A2d[t], Bb, Bbd)
            g_sym[t] = NG.segment_sum(gWa, perm, seg, z, n_el)
            for l in range(P):
                sl = slice(l * l, (l + 1) * (l + 1))
                red.append(NG.MMT(A[t][sl].reshape(-1, C), A2b[sl].reshape(-1, C), g_lin[t][l],
                                  X1=Ad[t][sl].reshape(-1, C), D1=A2bd[sl].reshape(-1, C)))
            Ab, Abd = torch.empty_like(A2b), torch.empty_like(A2bd)
            linT = [w.t() for w in lin[t]]
            NG.mm(_per_degree_problems(A2b, Ab, linT, Pk["linT"][P * t:P * t + P])
                  + _per_degree_problems(A2bd, Abd, linT, Pk["linT"][P * t:P * t + P]))
            Rbar, Rdbar, ub, ubd = ops.dual_reverse(plan, Ab, Abd, Y, Ydot, rdot, u[t], ud[t] if t > 0 else None,
                                                    Rs[t], Rds[t])
            if ubd is None:
                ubd = torch.zeros_like(ub)
            g_rad[t] = RAD._reverse(E, radial_w[t], Wt.spec[t], acts[t], H0s[t],
                                    Rbar.reshape(E, P * C), Rdbar.reshape(E, P * C))
            red.append(NG.MMT(h[t], ub, g_up[t], X1=hd[t], D1=ubd))
            red += [NG.MMT(h[t], Hb, g_sc[t][k], X1=hd[t], D1=Hbd, perm=perm, seg=seg[k:k + 2], rows0=N, rows1=N)
                    for k in range(n_el)]
            if hb[t] is None:
                hb[t] = torch.zeros(N, C, dtype=dt, device=dev)
                hbd[t] = torch.zeros(N, C, dtype=dt, device=dev)
            probs = rev_problems(t, ub, Hb, hb[t])
            if t > 0:
                probs += rev_problems(t, ubd, Hbd, hbd[t])
            NG.mm(probs)
            # interaction t is done: its weight gradients, then its bucket may be reduced
            NG.mmT(red)
            red = []
            ro = (gw1, gw2) if t == T - 1 else g_rol[t]
            wmap.add_grads(wmap.interaction_pairs(t, g_up[t], g_sc[t], g_rad[t], g_lin[t], g_sym[t], g_prod[t], ro))
            if bucket_hook is not None:
                bucket_hook(T - 1 - t)
        g_emb = NG.segment_sum(hb[0], perm, seg, z, n_el)
        wmap.add_grads([(wmap.emb, g_emb)])
        ar = m.atom_ref.weight
        if ar.requires_grad and self.we > 0:
            gar = torch.zeros_like(ar).index_add_(0, Z, a_s.to(ar.dtype).index_select(0, b.batch)[:, None])
            if ar.grad is None:
                ar.grad = gar
            else:
                ar.grad.add_(gar)
        out = {"energy": energy.detach(), "forces": forces.detach(), "node_energy": node_e.detach()}
        return loss, logs, out

    # ------------------------------------------------------------------ loss
    def _loss(self, b, energy: Tensor, forces: Tensor):
        """Energy and force terms of ``weighted_loss`` and their cotangents ``a = dL/dE``,
        ``g = dL/dF``."""
        logs: Dict[str, Tensor] = {}
        has_e, has_f = self.we > 0 and b.energy is not None, self.wf > 0 and b.forces is not None
        if energy.is_cuda and forces.dtype in (torch.float32, torch.float64) and hasattr(K._C(), "mace_loss"):
            # one kernel: both terms, their sums and the cotangents
            f64 = lambda t: None if t is None else t.to(torch.float64).contiguous()  # noqa: E731
            msk = lambda t: None if t is None else t.to(torch.bool).contiguous()  # noqa: E731
            out, a, g = K._C().mace_loss(
                energy.to(torch.float64).contiguous(), f64(b.energy) if has_e else None, b.n_atoms.long().contiguous(),
                f64(b.weight), f64(b.energy_weight), msk(b.energy_mask), forces.contiguous(),
                f64(b.forces) if has_f else None, b.batch.long().contiguous(), f64(b.force_weight),
                msk(b.forces_mask), f64(b.atom_force_weight), float(self.we), float(self.wf))
            if has_e:
                logs["energy"] = out[1]
            if has_f:
                logs["forces"] = out[2]
            return out[0], logs, a, g
        total = torch.zeros((), dtype=torch.float64, device=energy.device)
        a = torch.zeros_like(energy)
        g = torch.zeros_like(forces)

        def struct_w(mask, extra):
            w = b.weight
            if extra is not None:
                w = extra if w is None else w * extra
            if mask is not None:
                mm = mask.to(torch.float64)
                w = mm if w is None else w * mm
            return w

        if self.we > 0 and b.energy is not None:
            n = b.n_atoms.to(torch.float64)
            res = (energy.to(torch.float64) - b.energy.to(torch.float64)) / n
            w = struct_w(b.energy_mask, b.energy_weight)
            w = torch.ones_like(res) if w is None else w.to(res.dtype)
            den = w.sum().clamp_min(1e-12)
            term = (w * res * res).sum() / den
            logs["energy"] = term.detach()
            total = total + self.we * term
            a = (self.we * 2.0) * w * res / n / den
        if self.wf > 0 and b.forces is not None:
            res = forces - b.forces.to(forces.dtype)
            w = struct_w(b.forces_mask, b.force_weight)
            wa = None if w is None else w.index_select(0, b.batch)
            if b.atom_force_weight is not None:
                wa = b.atom_force_weight if wa is None else wa * b.atom_force_weight
            sq = (res * res).sum(-1) / 3.0
            if wa is None:
                wa = torch.ones_like(sq)
            wa = wa.to(sq.dtype)
            den = wa.sum().clamp_min(1e-12)
            term = (sq * wa).sum() / den
            logs["forces"] = term.detach()
            total = total + self.wf * term
            g = (self.wf * 2.0 / 3.0) * (wa / den)[:, None] * res
        return total, logs, a, g
