"""Spatial domain decomposition: one large structure evaluated by several processes.

Behaviour follows the reference's ``DomainParallel`` (``src/xnn/common/deploy/domain.py:266-719``):
the box (a periodic cell, or the bounding box of a molecule) is cut into a grid of sub-domains,
one per process; a process owns the atoms whose fractional coordinates fall in its sub-domain
and evaluates them together with a shell of ghost atoms, keeping only the energies of its owned
atoms. The shell is one cutoff thick with ghost features refreshed from their owners before
every layer that reads neighbours (``halo="layer"``), or the whole receptive field with no
exchange inside the model (``halo="field"``). Ghost positions come from their owners through
the same exchange, so the derivative of a process's energy with respect to its ghosts flows back
to their owners: each process ends with the forces on its own atoms, and only the energy and
virial are summed. A plan is built with a ``skin`` and stays valid while atoms moved less than
the skin allows (``holds``), so an MD loop rebuilds it only occasionally (``reshard``).

Device-side design: plans are built where the positions live (the native CUDA cell list on a
GPU), ghost rows move either through ``all_to_all_single`` of the process group (NCCL, or Gloo
on the CPU) or, with ``exchange="p2p"``, through one kernel per direction that packs the rows
and stores them straight into the receiving GPUs' ghost buffers over NVLink
(:mod:`xnn_b200.parallel.halo`).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist
from torch import Tensor, nn
from torch.autograd import Function

from ..data.atomic_graph import AtomicGraph
from ..data.neighborlist import build_neighbor_list
from ..ops.modes import force_pass
from ..ops.scatter import domain_hooks, structure_sum

#: added to the ghost shell and the neighbour-list reach so rounding never drops an atom on an edge
HALO_MARGIN = 1e-6
HALOS = ("auto", "layer", "field")
EXCHANGES = ("collective", "p2p")


def _process(group) -> tuple:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


# --------------------------------------------------------------------------- collectives
class _AllToAllRows(Function):
    """Rows ``x[send_rows]`` sent to every process; the rows received, concatenated by source.

    The backward sends the gradient rows back to their owners and accumulates them into the
    owned rows they were copied from.
    """

    @staticmethod
    def forward(ctx, x: Tensor, plan: "DomainPlan", group, exchanger):
        ctx.plan, ctx.group, ctx.exchanger, ctx.n = plan, group, exchanger, x.shape[0]
        if exchanger is not None:
            return exchanger.forward(x, plan)
        send = x.index_select(0, plan.send_rows).contiguous()
        out = send.new_empty((plan.n_ghost,) + tuple(send.shape[1:]))
        dist.all_to_all_single(out, send, plan.recv_counts, plan.send_counts, group=group)
        return out

    @staticmethod
    def backward(ctx, g: Tensor):
        plan = ctx.plan
        if ctx.exchanger is not None:
            return ctx.exchanger.backward(g.contiguous(), plan, ctx.n), None, None, None
        back = g.new_empty((int(plan.send_rows.shape[0]),) + tuple(g.shape[1:]))
        dist.all_to_all_single(back, g.contiguous(), plan.send_counts, plan.recv_counts, group=ctx.group)
        gx = g.new_zeros((ctx.n,) + tuple(g.shape[1:]))
        gx.index_add_(0, plan.send_rows, back)
        return gx, None, None, None


class _AllReduceSum(Function):
    @staticmethod
    def forward(ctx, x: Tensor, group):
        ctx.group = group
        y = x.clone()
        dist.all_reduce(y, group=group)
        return y

    @staticmethod
    def backward(ctx, g: Tensor):
        g = g.clone()
        dist.all_reduce(g, group=ctx.group)
        return g, None


def _tie(x: Tensor) -> Tensor:
    """An exact float64 zero that depends on ``x``.

    Each collective of an evaluation adds the tie of the previous collective's output to its
    input, and the energy adds the ties of all of them, so the backward pass of every process
    runs the adjoint collectives in exactly the reverse order of the forward ones whatever the
    shape of its own graph (the same device of the reference, ``domain.py:255-263``)."""
    return x.reshape(-1)[:0].sum(dtype=torch.float64)


# --------------------------------------------------------------------------- plan
def _rows3(x: Tensor, m: Tensor) -> Tensor:
    """``x @ m`` for ``x (n, 3)`` and ``m (3, 3)`` as one broadcast product and sum: a library
    GEMM with an inner size of 3 wastes a launch configuration meant for large ``K``."""
    return (x.unsqueeze(-1) * m.to(x.dtype)).sum(1)


@dataclass
class DomainPlan:
    """What one process evaluates: owned atoms, ghosts, exchanges, neighbour list.

    Field names and meanings are those of the reference's ``DomainPlan``
    (``domain.py:109-204``) so MD drivers written against it port unchanged. Local atoms are the
    owned atoms (ascending atom index) followed by the ghosts (grouped by owner).
    """

    grid: tuple
    rank: int
    world: int
    owned: Tensor
    ghosts: Tensor
    ghost_shifts: Optional[Tensor]
    send_rows: Tensor
    send_counts: list
    recv_counts: list
    edge_index: Tensor
    cell_shifts: Tensor
    pbc: Optional[Tensor]
    atomic_numbers: Tensor
    total_charge: Optional[Tensor]
    spin_multiplicity: Optional[Tensor]
    reference: Tensor
    cell: Optional[Tensor]
    counts: list
    order: Tensor
    need: float
    skin: float
    #: peer-memory exchange: first row of this process's rows in every receiver's ghost list,
    #: first row of its ghosts in every owner's send list, and the largest ghost or send count
    #: of any process (sizes the shared receive buffers)
    remote_offsets: Optional[list] = None
    remote_send_offsets: Optional[list] = None
    max_rows: int = 0
    #: float64 inverse of ``cell`` (reused while the cell stays the plan's)
    inv_cell: Optional[Tensor] = None

    @property
    def n_owned(self) -> int:
        return int(self.owned.shape[0])

    @property
    def n_ghost(self) -> int:
        return int(self.ghosts.shape[0])

    @property
    def n_local(self) -> int:
        return self.n_owned + self.n_ghost

    @property
    def n_atoms(self) -> int:
        return int(self.atomic_numbers.shape[0])

    @property
    def index(self) -> Tensor:
        """Atom of the structure behind every local atom ``(n_local,)``."""
        return torch.cat([self.owned, self.ghosts])


def choose_grid(n_domains: int, widths: Sequence[float], halo: float) -> tuple:
    """The factorisation ``gx * gy * gz = n_domains`` that evaluates the fewest ghosts.

    Cutting an axis of width ``w`` into ``g`` slabs adds a shell ``halo`` thick on both sides
    of each slab, multiplying the evaluated volume by ``1 + 2 halo g / w``; the grid with the
    smallest product is returned (ties keep the first in lexicographic order).
    """
    best, best_cost = None, math.inf
    for gx in range(1, n_domains + 1):
        if n_domains % gx:
            continue
        rest = n_domains // gx
        for gy in range(1, rest + 1):
            if rest % gy:
                continue
            grid = (gx, gy, rest // gy)
            cost = 1.0
            for g, w in zip(grid, widths):
                if g > 1:
                    cost *= 1.0 + 2.0 * halo * g / max(float(w), 1e-12)
            if cost < best_cost - 1e-12:
                best, best_cost = grid, cost
    return best


def _model_dtype(model: nn.Module) -> Optional[torch.dtype]:
    for t in list(model.parameters()) + list(model.buffers()):
        if t.is_floating_point():
            return t.dtype
    return None


class _Hooks:
    """The object the model's ``refresh_ghosts`` / ``whole_structure_sum`` calls go to."""

    def __init__(self, dp: "DomainParallel", plan: DomainPlan, ties: List[Tensor]):
        self.dp, self.plan, self.ties = dp, plan, ties

    def refresh(self, x: Tensor) -> Tensor:
        plan = self.plan
        rows = max(plan.n_local, 1)
        if not self.dp.layer:
            return x
        if x.shape[0] != rows:
            raise ValueError(f"refresh_ghosts got {x.shape[0]} rows for {rows} local atoms")
        fresh = self.dp._exchange(plan, x[:plan.n_owned], self.ties)
        return torch.cat([x[:plan.n_owned], fresh, x[plan.n_local:]])

    def whole_sum(self, values: Tensor, batch: Tensor, num_graphs: int) -> Tensor:
        n = self.plan.n_owned
        part = structure_sum(values[:n], batch[:n], num_graphs)
        if self.plan.world > 1:
            part = part + _tie(self.ties[-1]).to(part.dtype) if self.ties else part
            part = _AllReduceSum.apply(part, self.dp.group)
            self.ties.append(part)
        return part


# --------------------------------------------------------------------------- module
class DomainParallel(nn.Module):
    """Evaluate one structure split over the processes of a distributed launch.

    Every method is collective (all processes call it together). ``model`` is an
    :class:`~xnn_b200.models.base.InteratomicPotential` (or a ``ForceStressOutput`` around one)
    with a bounded receptive field. ``exchange`` selects how ghost rows move: ``"collective"``
    (``all_to_all_single`` of the process group) or ``"p2p"`` (peer-memory kernels, CUDA only).
    Evaluation only: no second derivatives.
    """

    def __init__(self, model: nn.Module, grid: Optional[Sequence[int]] = None,
                 receptive_field: Optional[float] = None, compute_stress: bool = True, group=None,
                 halo: str = "auto", skin: float = 0.0, exchange: str = "collective"):
        super().__init__()
        inner = getattr(model, "model", None)
        if inner is not None and hasattr(model, "compute_forces"):
            model = inner
        if receptive_field is None:
            field = getattr(model, "receptive_field", None)
            receptive_field = field() if callable(field) else None
        if receptive_field is None:
            raise ValueError(f"{type(model).__name__} has no bounded receptive field; pass "
                             "receptive_field= to decompose it anyway")
        if halo not in HALOS:
            raise ValueError(f"halo={halo!r} is not supported; options: {list(HALOS)}")
        refreshes = bool(getattr(model, "refreshes_ghosts", False))
        if halo == "layer" and not refreshes:
            raise ValueError(f"{type(model).__name__} does not refresh its ghosts between layers; "
                             "use halo='field'")
        if skin < 0:
            raise ValueError(f"skin must not be negative, got {skin}")
        if exchange not in EXCHANGES:
            raise ValueError(f"exchange={exchange!r} is not supported; options: {list(EXCHANGES)}")
        self.model = model
        self.cutoff = float(model.cutoff)
        self.receptive_field = float(receptive_field)
        self.layer = halo == "layer" or (halo == "auto" and refreshes)
        self.need = self.cutoff if self.layer else self.receptive_field
        self.skin = float(skin)
        self.grid = tuple(int(g) for g in grid) if grid is not None else None
        self.compute_stress = compute_stress
        self.group = group
        self.exchange = exchange
        self._exchanger = None
        self._plan: Optional[DomainPlan] = None

    @property
    def halo(self) -> str:
        return "layer" if self.layer else "field"

    # ---------------------------------------------------------------- planning
    @torch.no_grad()
    def plan(self, data: AtomicGraph) -> DomainPlan:
        """Partition ``data`` (one structure, the same on every process) and build this
        process's ghosts and neighbour list."""
        if data.num_graphs != 1:
            raise ValueError("DomainParallel evaluates one structure, not a batch")
        periodic = data.cell is not None and data.pbc is not None and bool(data.pbc.any())
        if periodic and not bool(data.pbc.all()):
            raise ValueError("DomainParallel takes structures periodic along all axes or none")
        return self._build(data.pos, data.atomic_numbers, data.cell[0] if periodic else None,
                           data.total_charge, data.spin_multiplicity)

    def _build(self, positions: Tensor, atomic_numbers: Tensor, cell: Optional[Tensor],
               total_charge: Optional[Tensor], spin_multiplicity: Optional[Tensor]) -> DomainPlan:
        rank, world = _process(self.group)
        pos = positions.detach().to(torch.float64)
        device, n = pos.device, int(pos.shape[0])
        halo = self.need + self.skin + HALO_MARGIN
        periodic = cell is not None
        if periodic:
            cell = cell.detach().to(device=device, dtype=torch.float64)
            inv = torch.linalg.inv(cell)
            raw = _rows3(pos, inv)
            frac = raw - torch.floor(raw)
            widths_t = 1.0 / torch.linalg.norm(inv, dim=0)      # plane spacings of the cell
        else:
            low = pos.min(0).values if n else pos.new_zeros(3)
            widths_t = (pos.max(0).values - low if n else pos.new_zeros(3)) + 1e-6
            frac = (pos - low) / widths_t
        widths = [float(w) for w in widths_t.cpu()]
        grid = self.grid if self.grid is not None else choose_grid(world, widths, halo)
        if len(grid) != 3 or math.prod(grid) != world:
            raise ValueError(f"grid {tuple(grid)} does not hold {world} processes")
        coords = (rank // (grid[1] * grid[2]), (rank // grid[2]) % grid[1], rank % grid[2])

        g = torch.tensor(grid, device=device)
        cells = torch.minimum(torch.floor(frac * g).long().clamp(min=0), g - 1)
        owner = (cells[:, 0] * grid[1] + cells[:, 1]) * grid[2] + cells[:, 2]
        owned = (owner == rank).nonzero().flatten()
        counts = torch.bincount(owner, minlength=world).tolist()
        order = torch.sort(owner, stable=True).indices

        # ghost shell: atoms (or their periodic images along cut axes) within `halo` of the slab
        masks, steps = [], []
        for a in range(3):
            if grid[a] == 1:
                masks.append(torch.ones(n, 1, dtype=torch.bool, device=device))
                steps.append(torch.zeros(1, dtype=torch.long, device=device))
                continue
            shell = halo / widths[a]
            lo, hi = coords[a] / grid[a] - shell, (coords[a] + 1) / grid[a] + shell
            m = math.floor(shell) + 1 if periodic else 0
            image = torch.arange(-m, m + 1, device=device)
            x = frac[:, a, None] + image.to(torch.float64)
            masks.append((x >= lo) & (x < hi))
            steps.append(image)
        mask = masks[0][:, :, None, None] & masks[1][:, None, :, None] & masks[2][:, None, None, :]
        atom, i0, i1, i2 = mask.nonzero(as_tuple=True)
        image = torch.stack([steps[0][i0], steps[1][i1], steps[2][i2]], dim=1)
        keep = ~((owner[atom] == rank) & (image == 0).all(1))
        atom, image = atom[keep], image[keep]
        by_owner = torch.sort(owner[atom], stable=True).indices
        ghosts, ghost_image = atom[by_owner], image[by_owner]
        recv_counts_t = torch.bincount(owner[ghosts], minlength=world)

        remote_offsets = None
        if world > 1:
            # every process asks the owners of its ghosts for them
            send_counts_t = torch.empty_like(recv_counts_t)
            dist.all_to_all_single(send_counts_t, recv_counts_t, group=self.group)
            send_counts = send_counts_t.tolist()
            recv_counts = recv_counts_t.tolist()
            requested = ghosts.new_empty(int(sum(send_counts)))
            dist.all_to_all_single(requested, ghosts, send_counts, recv_counts, group=self.group)
            # where this process's rows start inside every receiver's ghost list, and where its
            # ghosts start inside every owner's send list
            starts = torch.stack([torch.cumsum(recv_counts_t, 0) - recv_counts_t,
                                  torch.cumsum(send_counts_t, 0) - send_counts_t], 1).contiguous()
            remote = torch.empty_like(starts)
            dist.all_to_all_single(remote, starts, group=self.group)
            remote_offsets, remote_send_offsets = remote[:, 0].tolist(), remote[:, 1].tolist()
            most = torch.tensor([max(len(ghosts), len(requested))], dtype=torch.long, device=device)
            dist.all_reduce(most, op=dist.ReduceOp.MAX, group=self.group)
            max_rows = int(most[0])
        else:
            send_counts, requested = recv_counts_t.tolist(), ghosts
            recv_counts = recv_counts_t.tolist()
            remote_offsets, remote_send_offsets, max_rows = [0], [0], len(ghosts)
        send_rows = torch.searchsorted(owned, requested)
        if len(requested) and not (len(owned) and bool(
                (owned[send_rows.clamp(max=len(owned) - 1)] == requested).all())):
            raise RuntimeError("the processes disagree on the owners of the atoms")

        if periodic:
            local = _rows3(torch.cat([frac[owned], frac[ghosts] + ghost_image.to(torch.float64)]), cell)
            reference = frac[owned]
        else:
            local = torch.cat([pos[owned], pos[ghosts]])
            reference = pos[owned]
        reach = self.cutoff + self.skin + HALO_MARGIN
        native = [periodic and grid[a] == 1 for a in range(3)]
        if not len(local):
            edge_index = torch.zeros((2, 0), dtype=torch.long, device=device)
            cell_shifts = torch.zeros((0, 3), dtype=torch.long, device=device)
            pbc = torch.tensor(native) if any(native) else None
        elif any(native):
            # stretch the cut axes far beyond the shell so only the explicit images are
            # neighbours along them, while the uncut axes keep the box's periodicity
            search = cell.clone()
            for a in range(3):
                if not native[a]:
                    search[a] *= 1.0 + 1.0 / grid[a] + 2.0 * (halo + reach) / widths[a]
            edge_index, cell_shifts = build_neighbor_list(local, reach, search,
                                                          torch.ones(3, dtype=torch.bool))
            cut = torch.tensor([not x for x in native], device=cell_shifts.device)
            if bool((cell_shifts[:, cut] != 0).any()):
                raise RuntimeError("a neighbour across a cut axis was found through the box's periodicity")
            pbc = torch.tensor(native)
        else:
            edge_index, cell_shifts = build_neighbor_list(local, reach)
            pbc = None
        if self.layer:
            # ghost features are replaced by their owners' before they are read: no messages
            # into ghosts are needed
            keep = edge_index[1] < len(owned)
            edge_index, cell_shifts = edge_index[:, keep], cell_shifts[keep.to(cell_shifts.device)]
        return DomainPlan(
            grid=tuple(grid), rank=rank, world=world, owned=owned, ghosts=ghosts,
            ghost_shifts=ghost_image if periodic else None, send_rows=send_rows,
            send_counts=send_counts, recv_counts=recv_counts, edge_index=edge_index.to(device),
            cell_shifts=cell_shifts.to(device), pbc=pbc, atomic_numbers=atomic_numbers,
            total_charge=total_charge, spin_multiplicity=spin_multiplicity, reference=reference,
            cell=cell, counts=counts, order=order, need=self.need, skin=self.skin,
            remote_offsets=remote_offsets, remote_send_offsets=remote_send_offsets, max_rows=max_rows,
            inv_cell=inv if periodic else None)

    def _cell(self, plan: DomainPlan, cell: Optional[Tensor]) -> Optional[Tensor]:
        if plan.cell is None:
            return None
        if cell is None:
            return plan.cell
        return cell[0] if cell.dim() == 3 else cell

    @torch.no_grad()
    def holds(self, plan: DomainPlan, pos: Tensor, cell: Optional[Tensor] = None) -> bool:
        """Whether the plan is valid for new owned positions (and cell): it holds while
        ``need + 2 d <= (1 - e)(need + skin)`` with ``d`` the largest displacement since the
        plan was built and ``e`` the relative strain of the cell. The same on every process."""
        cell = self._cell(plan, cell)
        strain = 0.0
        if cell is None:
            moved = pos.detach().to(torch.float64) - plan.reference
        else:
            cell = cell.detach().to(torch.float64)
            same = plan.inv_cell is not None and (cell is plan.cell or bool(torch.equal(cell, plan.cell)))
            inv = plan.inv_cell if same else torch.linalg.inv(cell)
            frac = _rows3(pos.detach().to(torch.float64), inv) - plan.reference
            moved = _rows3(frac - torch.round(frac), cell)
            if not same:
                strain = float(torch.linalg.matrix_norm(torch.linalg.inv(plan.cell) @ (cell - plan.cell), ord=2))
        largest = moved.norm(dim=-1).max() if len(moved) else moved.new_zeros(())
        if plan.world > 1:
            largest = largest.reshape(1).clone()
            dist.all_reduce(largest, op=dist.ReduceOp.MAX, group=self.group)
            largest = largest[0]
        need = plan.need
        return need + 2.0 * float(largest) <= (1.0 - strain) * (need + plan.skin + HALO_MARGIN)

    @torch.no_grad()
    def reshard(self, plan: DomainPlan, pos: Tensor, *fields: Tensor, cell: Optional[Tensor] = None) -> tuple:
        """A new plan for the current positions, with ``pos`` and every per-atom field moved
        to the atoms' new owners. Returns ``(plan, pos, *fields)``."""
        cell = self._cell(plan, cell)
        whole = [self._gather(plan, x) for x in (pos,) + fields]
        new = self._build(whole[0], plan.atomic_numbers, cell, plan.total_charge, plan.spin_multiplicity)
        return (new,) + tuple(x[new.owned] for x in whole)

    def _gather(self, plan: DomainPlan, rows: Tensor) -> Tensor:
        """Rows of every process's owned atoms, in the atom order of the structure."""
        whole = rows.new_empty((plan.n_atoms,) + tuple(rows.shape[1:]))
        if plan.world == 1:
            whole[plan.owned] = rows
            return whole
        size = max(plan.counts)
        padded = rows.new_zeros((size,) + tuple(rows.shape[1:]))
        padded[:len(rows)] = rows
        parts = [torch.empty_like(padded) for _ in range(plan.world)]
        dist.all_gather(parts, padded.contiguous(), group=self.group)
        whole[plan.order] = torch.cat([p[:c] for p, c in zip(parts, plan.counts)])
        return whole

    # ---------------------------------------------------------------- exchange
    def _get_exchanger(self, plan: DomainPlan, like: Tensor):
        if self.exchange != "p2p" or plan.world == 1 or not like.is_cuda:
            return None
        if self._exchanger is None:
            from .halo import PeerHaloExchange
            self._exchanger = PeerHaloExchange(like.device, self.group)
        return self._exchanger

    def _exchange(self, plan: DomainPlan, rows: Tensor, ties: List[Tensor]) -> Tensor:
        """Rows of the ghosts, sent by their owners from ``rows`` (the owned atoms)."""
        if plan.world == 1:
            return rows.index_select(0, plan.send_rows)
        if ties:
            rows = rows + _tie(ties[-1]).to(rows.dtype)
        out = _AllToAllRows.apply(rows, plan, self.group, self._get_exchanger(plan, rows))
        ties.append(out)
        return out

    # ---------------------------------------------------------------- evaluation
    def evaluate(self, plan: DomainPlan, pos: Tensor, cell: Optional[Tensor] = None) -> dict:
        """Energy (whole structure, float64 ``(1,)``), forces on the owned atoms and, for a
        periodic structure with ``compute_stress``, the stress ``(1, 3, 3)``."""
        if pos.shape[0] != plan.n_owned:
            raise ValueError(f"{pos.shape[0]} positions for the {plan.n_owned} atoms of the plan")
        cell = self._cell(plan, cell)
        p = pos.detach().requires_grad_(True)
        dtype, device = p.dtype, p.device
        strain, volume, own = None, None, p
        if cell is not None:
            c64 = cell.detach().to(torch.float64)
            same = plan.inv_cell is not None and (cell is plan.cell or bool(torch.equal(c64, plan.cell)))
            inv = plan.inv_cell if same else torch.linalg.inv(c64)
            cell = cell.detach().to(dtype)
            volume = torch.linalg.det(c64).abs().reshape(1)
            jumps = torch.round(_rows3(p.detach().to(torch.float64), inv) - plan.reference).to(dtype)
            if self.compute_stress:
                strain = torch.zeros((3, 3), dtype=dtype, device=device, requires_grad=True)
                sym = 0.5 * (strain + strain.transpose(0, 1))
                own = own + own @ sym
                cell = cell + cell @ sym
            # owned atoms brought back next to where the plan saw them
            own = own - _rows3(jumps, cell)
        ties: List[Tensor] = []
        ghosts = self._exchange(plan, own, ties)
        if cell is not None:
            ghosts = ghosts + _rows3(plan.ghost_shifts.to(dtype), cell)
        local = torch.cat([own, ghosts])
        numbers = plan.atomic_numbers[plan.index]
        if plan.n_local == 0:
            # an empty sub-domain evaluates one isolated stand-in (energy dropped) so that it
            # takes part in every exchange of the others
            local = local.new_zeros((1, 3))
            numbers = plan.atomic_numbers[:1]
        edge_index, cell_shifts = plan.edge_index, plan.cell_shifts
        with torch.no_grad():
            vec = local[edge_index[1]] - local[edge_index[0]]
            if plan.pbc is not None:
                vec = vec + _rows3(cell_shifts.to(dtype), cell)
            keep = (vec * vec).sum(-1) < self.cutoff ** 2
        edge_index, cell_shifts = edge_index[:, keep], cell_shifts[keep]
        model_dtype = _model_dtype(self.model)
        n_local = int(local.shape[0])
        graph = AtomicGraph(
            pos=local, atomic_numbers=numbers, edge_index=edge_index, cell_shifts=cell_shifts,
            batch=torch.zeros(n_local, dtype=torch.long, device=device),
            n_atoms=torch.tensor([n_local], dtype=torch.long, device=device),
            cell=cell[None] if plan.pbc is not None else None,
            pbc=plan.pbc[None].to(device) if plan.pbc is not None else None,
            total_charge=plan.total_charge, spin_multiplicity=plan.spin_multiplicity,
            compute_dtype=model_dtype if model_dtype is not None and model_dtype != dtype else None)
        graph.edge_order = "dst"
        with domain_hooks(_Hooks(self, plan, ties)):
            out = self.model(graph)
        energy = out["node_energy"][:plan.n_owned].to(torch.float64).sum()
        for t in ties:
            energy = energy + _tie(t)
        inputs = [p] + ([strain] if strain is not None else [])
        grads = [None] * len(inputs)
        if energy.requires_grad:
            # only position / strain derivatives: the fused ops skip their weight gradients
            with force_pass():
                grads = list(torch.autograd.grad([energy], inputs, allow_unused=True))
        g_pos = grads[0] if grads[0] is not None else torch.zeros_like(p)
        g_strain = (grads[1] if strain is not None and grads[1] is not None
                    else torch.zeros((3, 3), dtype=torch.float64, device=device))
        total = torch.cat([energy.detach().reshape(1), g_strain.to(torch.float64).reshape(9)])
        if plan.world > 1:
            dist.all_reduce(total, group=self.group)
        if self._exchanger is not None:
            self._exchanger.check()
        result = {"energy": total[:1], "forces": -g_pos.to(dtype)}
        if strain is not None:
            result["stress"] = (total[1:10].view(1, 3, 3) / volume).to(dtype)
        return result

    def forward(self, data: AtomicGraph) -> dict:
        """Energy, forces (all atoms, gathered) and stress of ``data``, given on every
        process; the plan of the previous call is reused while it holds."""
        periodic = data.cell is not None and data.pbc is not None and bool(data.pbc.any())
        cell = data.cell[0] if periodic else None
        plan = self._plan
        if (plan is None or plan.n_atoms != data.num_nodes or (plan.cell is None) == periodic
                or not torch.equal(plan.atomic_numbers, data.atomic_numbers)
                or not self.holds(plan, data.pos[plan.owned], cell)):
            plan = self._plan = self.plan(data)
        plan.total_charge, plan.spin_multiplicity = data.total_charge, data.spin_multiplicity
        out = self.evaluate(plan, data.pos[plan.owned], cell)
        out["forces"] = self._gather(plan, out["forces"])
        return out

    def close(self) -> None:
        if self._exchanger is not None:
            self._exchanger.close()
            self._exchanger = None
