"""Spatial domain decomposition: one large structure evaluated by several processes.

The behaviour is that of the reference's ``DomainParallel``
(``src/xnn/common/deploy/domain.py:266-719``): the box (a periodic cell, or the bounding box of
a molecule) is cut into a grid of sub-domains, one per process. A process owns the atoms whose
fractional coordinates fall in its sub-domain and evaluates them together with a shell of
ghosts, keeping the energies of its owned atoms only. The shell is one cutoff thick with ghost
features refreshed from their owners before every layer that reads neighbours
(``halo="layer"``), or the whole receptive field with no exchange inside the model
(``halo="field"``). Ghost positions come from their owners through the same exchange, so the
derivative of a process's energy with respect to its ghosts flows back to the owners: each
process ends with the forces on its own atoms, and only energy and virial are summed. A plan is
built with a ``skin`` and stays valid while the atoms moved less than the skin allows
(:meth:`DomainParallel.holds`), so an MD loop rebuilds it only now and then
(:meth:`DomainParallel.reshard`).

How a plan is built here:

* ownership: the sub-domain cell of every atom's fractional coordinates (row-major rank order);
* ghosts: for every atom and every cut axis, the integer image range ``k`` with
  ``lo <= f + k < hi`` (the slab widened by the shell) is computed directly, and the atom's
  images are the mixed-radix enumeration of the per-axis ranges -- no fixed image window, so
  cells thinner than the shell need no special case;
* the handshake: one exchange of ghost counts, one of the requested atom ids and one of a small
  table per peer (where my rows start in its ghost list, where its rows start in my send list,
  my largest row count) -- the last replaces a separate reduction for the buffer size;
* validation is collective: every consistency check (counts against lists, requested atoms
  against ownership) is agreed by a reduction before anyone raises, so a rank that finds a
  problem makes every rank raise instead of leaving the others waiting in the next collective;
* the local neighbour list is built with the box periodic along the uncut axes only (open
  along the cut ones, where the ghosts are explicit images).

Ghost rows move through ``all_to_all_single`` of the process group (NCCL, or Gloo on the CPU)
or, with ``exchange="p2p"``, through one kernel per direction that stores the rows straight
into the receiving GPUs' buffers over NVLink (:mod:`xnn_b200.parallel.halo`).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

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


class PlanError(RuntimeError):
    """The processes built inconsistent plans (raised on every process together)."""


def _process(group) -> Tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def _agree(ok: bool, world: int, group, device) -> bool:
    """Whether ``ok`` holds on every process (a MIN reduction; every process calls it)."""
    if world == 1:
        return ok
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return bool(flag.item())


# --------------------------------------------------------------------------- collectives
class _RowExchange(Function):
    """Ghost rows from their owners (``x[send_rows]`` to every process, received by source);
    the backward returns the ghost cotangents to the owners and adds them to the owned rows."""

    @staticmethod
    def forward(ctx, x: Tensor, plan: "DomainPlan", group, exchanger):
        ctx.plan, ctx.group, ctx.exchanger, ctx.rows = plan, group, exchanger, x.shape[0]
        if exchanger is not None:
            return exchanger.forward(x, plan)
        outgoing = x.index_select(0, plan.send_rows).contiguous()
        incoming = outgoing.new_empty((plan.n_ghost,) + tuple(outgoing.shape[1:]))
        dist.all_to_all_single(incoming, outgoing, plan.recv_counts, plan.send_counts, group=group)
        return incoming

    @staticmethod
    def backward(ctx, g: Tensor):
        plan = ctx.plan
        if ctx.exchanger is not None:
            return ctx.exchanger.backward(g.contiguous(), plan, ctx.rows), None, None, None
        returned = g.new_empty((plan.send_rows.shape[0],) + tuple(g.shape[1:]))
        dist.all_to_all_single(returned, g.contiguous(), plan.send_counts, plan.recv_counts, group=ctx.group)
        grad = g.new_zeros((ctx.rows,) + tuple(g.shape[1:]))
        return grad.index_add_(0, plan.send_rows, returned), None, None, None


class _SumOverRanks(Function):
    @staticmethod
    def forward(ctx, x: Tensor, group):
        ctx.group = group
        total = x.clone()
        dist.all_reduce(total, group=group)
        return total

    @staticmethod
    def backward(ctx, g: Tensor):
        total = g.clone()
        dist.all_reduce(total, group=ctx.group)
        return total, None


def _order_link(x: Tensor) -> Tensor:
    """An exact float64 zero that depends on ``x`` (an empty slice of it, summed).

    Adding the link of the previous collective's output to the next collective's input (and the
    links of all of them to the energy) chains the collectives in the autograd graph, so every
    process runs the adjoint collectives in the reverse order of the forward ones whatever the
    shape of its own graph."""
    return x.reshape(-1).narrow(0, 0, 0).sum(dtype=torch.float64)


def _apply3(rows: Tensor, m: Tensor) -> Tensor:
    """``rows @ m`` for ``rows (n, 3)`` and a 3 x 3 ``m``, as three scaled rows summed (a library
    GEMM with an inner size of 3 runs a launch configuration meant for large matrices)."""
    m = m.to(rows.dtype)
    return rows[:, 0:1] * m[0] + rows[:, 1:2] * m[1] + rows[:, 2:3] * m[2]


# --------------------------------------------------------------------------- plan
@dataclass
class DomainPlan:
    """What one process evaluates: owned atoms, ghosts, exchanges, neighbour list.

    Field names and meanings are the reference's ``DomainPlan`` (``domain.py:109-204``), so MD
    drivers written against it port unchanged. Local atoms are the owned atoms (ascending atom
    index) followed by the ghosts (grouped by owner).
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

    Cutting an axis of width ``w`` into ``g`` slabs adds a shell ``halo`` thick on both sides of
    each slab, multiplying the evaluated volume by ``1 + 2 halo g / w``; the grid with the
    smallest product wins (ties keep the first in lexicographic order)."""
    def cost(grid):
        c = 1.0
        for g, w in zip(grid, widths):
            if g > 1:
                c *= 1.0 + 2.0 * halo * g / max(float(w), 1e-12)
        return c

    grids = [(a, b, n_domains // (a * b)) for a in range(1, n_domains + 1) if n_domains % a == 0
             for b in range(1, n_domains // a + 1) if (n_domains // a) % b == 0]
    best = grids[0]
    for g in grids[1:]:
        if cost(g) < cost(best) - 1e-12:
            best = g
    return best


def _model_dtype(model: nn.Module) -> Optional[torch.dtype]:
    for t in list(model.parameters()) + list(model.buffers()):
        if t.is_floating_point():
            return t.dtype
    return None


def _frame(pos: Tensor, cell: Optional[Tensor]):
    """Fractional coordinates in [0, 1) per axis, the slab widths and the inverse cell."""
    if cell is not None:
        inv = torch.linalg.inv(cell)
        f = _apply3(pos, inv)
        return f - torch.floor(f), 1.0 / torch.linalg.norm(inv, dim=0), inv
    if pos.shape[0] == 0:
        return pos.new_zeros((0, 3)), pos.new_full((3,), 1e-6), None
    low = pos.min(0).values
    width = pos.max(0).values - low + 1e-6
    return (pos - low) / width, width, None


def _owners(frac: Tensor, grid: Sequence[int]) -> Tensor:
    g = torch.tensor(list(grid), device=frac.device)
    cell = torch.floor(frac * g.to(frac.dtype)).long()
    cell = torch.maximum(torch.minimum(cell, g - 1), torch.zeros_like(cell))
    return (cell[:, 0] * grid[1] + cell[:, 1]) * grid[2] + cell[:, 2]


def _halo_members(frac: Tensor, owner: Tensor, rank: int, coords, grid, widths: List[float], halo: float,
                  periodic: bool) -> Tuple[Tensor, Tensor]:
    """``(atom, image)`` of every ghost: atoms (and periodic images along cut axes) inside this
    process's slab widened by ``halo``, the process's own atoms at image 0 excluded; ordered by
    atom, then image."""
    n, device = frac.shape[0], frac.device
    kmin, span = [], []
    for a in range(3):
        if grid[a] == 1:
            kmin.append(torch.zeros(n, dtype=torch.long, device=device))
            span.append(torch.ones(n, dtype=torch.long, device=device))
            continue
        shell = halo / widths[a]
        lo = coords[a] / grid[a] - shell
        hi = (coords[a] + 1) / grid[a] + shell
        f = frac[:, a]
        k0 = torch.ceil(lo - f).long()
        k1 = torch.ceil(hi - f).long() - 1              # lo <= f + k < hi  <=>  k0 <= k <= k1
        if not periodic:
            k0 = torch.clamp(k0, min=0)
            k1 = torch.clamp(k1, max=0)
        kmin.append(k0)
        span.append((k1 - k0 + 1).clamp(min=0))
    per_atom = span[0] * span[1] * span[2]
    atom = torch.repeat_interleave(torch.arange(n, device=device), per_atom)
    first = torch.cumsum(per_atom, 0) - per_atom
    j = torch.arange(atom.shape[0], device=device) - first[atom]
    s0, s1 = span[0][atom], span[1][atom]
    image = torch.stack([kmin[0][atom] + j % s0, kmin[1][atom] + (j // s0) % s1, kmin[2][atom] + j // (s0 * s1)], 1)
    own_copy = (owner[atom] == rank) & (image == 0).all(1)
    return atom[~own_copy], image[~own_copy]


def _ghost_counts(ghost_owner: Tensor, world: int) -> Tensor:
    return torch.bincount(ghost_owner, minlength=world)


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
        if hasattr(model, "compute_forces") and getattr(model, "model", None) is not None:
            model = model.model
        if receptive_field is None:
            rf = getattr(model, "receptive_field", None)
            receptive_field = rf() if callable(rf) else None
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
        self.grid = None if grid is None else tuple(int(g) for g in grid)
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

    def _handshake(self, owned: Tensor, ghosts: Tensor, ghost_owner: Tensor, rank: int, world: int):
        """Send lists and peer offsets; raises :class:`PlanError` on every process together."""
        device = ghosts.device
        recv_t = _ghost_counts(ghost_owner, world)
        if world == 1:
            ok = int(recv_t.sum()) == int(ghosts.shape[0])
            send_rows = torch.searchsorted(owned, ghosts)
            ok = ok and bool((owned[send_rows.clamp(max=max(len(owned) - 1, 0))] == ghosts).all()) \
                if len(ghosts) else ok
            if not ok:
                raise PlanError("inconsistent halo plan: ghost counts or owners")
            counts = recv_t.tolist()
            return send_rows, counts, counts, [0], [0], int(ghosts.shape[0])
        send_t = torch.empty_like(recv_t)
        dist.all_to_all_single(send_t, recv_t, group=self.group)
        consistent = int(recv_t.sum()) == int(ghosts.shape[0]) and bool((send_t >= 0).all())
        if not _agree(consistent, world, self.group, device):
            raise PlanError("inconsistent halo plan: a process's ghost counts do not match its ghost list")
        send_counts, recv_counts = send_t.tolist(), recv_t.tolist()
        requested = ghosts.new_empty(int(send_t.sum()))
        dist.all_to_all_single(requested, ghosts, send_counts, recv_counts, group=self.group)
        send_rows = torch.searchsorted(owned, requested)
        mine = True
        if len(requested):
            mine = len(owned) > 0 and bool((owned[send_rows.clamp(max=len(owned) - 1)] == requested).all())
        if not _agree(mine, world, self.group, device):
            raise PlanError("inconsistent halo plan: the processes disagree on the owners of the atoms")
        # per peer: where its rows start in my ghost list, where my rows for it start in my send
        # list, my largest row count; received back, the first two columns are where my rows
        # start in the peer's lists
        table = torch.stack([torch.cumsum(recv_t, 0) - recv_t, torch.cumsum(send_t, 0) - send_t,
                             torch.full_like(recv_t, max(len(ghosts), len(requested)))], 1).contiguous()
        back = torch.empty_like(table)
        dist.all_to_all_single(back, table, group=self.group)
        return (send_rows, send_counts, recv_counts, back[:, 0].tolist(), back[:, 1].tolist(),
                int(back[:, 2].max()))

    def _local_edges(self, local: Tensor, cell: Optional[Tensor], grid, device):
        reach = self.cutoff + self.skin + HALO_MARGIN
        if not len(local):
            return (torch.zeros((2, 0), dtype=torch.long, device=device),
                    torch.zeros((0, 3), dtype=torch.long, device=device), None)
        if cell is None:
            ei, sh = build_neighbor_list(local, reach)
            return ei, sh, None
        # periodic along the uncut axes only; the cut axes carry explicit ghost images
        uncut = torch.tensor([g == 1 for g in grid])
        if not bool(uncut.any()):
            ei, sh = build_neighbor_list(local, reach)
            return ei, sh, None
        ei, sh = build_neighbor_list(local, reach, cell, uncut)
        return ei, sh, uncut

    def _build(self, positions: Tensor, atomic_numbers: Tensor, cell: Optional[Tensor],
               total_charge: Optional[Tensor], spin_multiplicity: Optional[Tensor]) -> DomainPlan:
        rank, world = _process(self.group)
        pos = positions.detach().to(torch.float64)
        device = pos.device
        halo = self.need + self.skin + HALO_MARGIN
        periodic = cell is not None
        if periodic:
            cell = cell.detach().to(device=device, dtype=torch.float64)
        frac, widths_t, inv = _frame(pos, cell)
        widths = widths_t.tolist()
        grid = self.grid if self.grid is not None else choose_grid(world, widths, halo)
        if len(grid) != 3 or math.prod(grid) != world:
            raise ValueError(f"grid {tuple(grid)} does not hold {world} processes")
        coords = (rank // (grid[1] * grid[2]), (rank // grid[2]) % grid[1], rank % grid[2])
        owner = _owners(frac, grid)
        owned = torch.nonzero(owner == rank).flatten()
        counts = torch.bincount(owner, minlength=world).tolist()
        order = torch.argsort(owner, stable=True)
        atom, image = _halo_members(frac, owner, rank, coords, grid, widths, halo, periodic)
        by_owner = torch.argsort(owner[atom], stable=True)
        ghosts, ghost_image = atom[by_owner], image[by_owner]
        send_rows, send_counts, recv_counts, r_off, r_send_off, max_rows = self._handshake(
            owned, ghosts, owner[ghosts], rank, world)
        if periodic:
            local = _apply3(torch.cat([frac[owned], frac[ghosts] + ghost_image.to(torch.float64)]), cell)
            reference = frac[owned]
        else:
            local = torch.cat([pos[owned], pos[ghosts]])
            reference = pos[owned]
        edge_index, cell_shifts, pbc = self._local_edges(local, cell, grid, device)
        if self.layer:
            # ghost features are replaced by their owners' before they are read: no messages
            # into ghosts are needed
            into_owned = edge_index[1] < len(owned)
            edge_index = edge_index[:, into_owned]
            cell_shifts = cell_shifts[into_owned.to(cell_shifts.device)]
        return DomainPlan(
            grid=tuple(grid), rank=rank, world=world, owned=owned, ghosts=ghosts,
            ghost_shifts=ghost_image if periodic else None, send_rows=send_rows,
            send_counts=send_counts, recv_counts=recv_counts, edge_index=edge_index.to(device),
            cell_shifts=cell_shifts.to(device), pbc=pbc, atomic_numbers=atomic_numbers,
            total_charge=total_charge, spin_multiplicity=spin_multiplicity, reference=reference,
            cell=cell, counts=counts, order=order, need=self.need, skin=self.skin,
            remote_offsets=r_off, remote_send_offsets=r_send_off, max_rows=max_rows, inv_cell=inv)

    def _plan_cell(self, plan: DomainPlan, cell: Optional[Tensor]) -> Optional[Tensor]:
        """The cell to evaluate with: the given one (``(3, 3)`` or ``(1, 3, 3)``), else the plan's."""
        if plan.cell is None or cell is None:
            return plan.cell
        return cell.reshape(3, 3)

    def _inverse(self, plan: DomainPlan, cell64: Tensor) -> Tuple[Tensor, bool]:
        unchanged = plan.inv_cell is not None and (cell64 is plan.cell or bool(torch.equal(cell64, plan.cell)))
        return (plan.inv_cell if unchanged else torch.linalg.inv(cell64)), unchanged

    @torch.no_grad()
    def holds(self, plan: DomainPlan, pos: Tensor, cell: Optional[Tensor] = None) -> bool:
        """Whether the plan is still valid for new owned positions (and cell).

        The ghost shell stays complete while ``need + 2 d <= (1 - e)(need + skin)`` with ``d``
        the largest displacement since the plan was built (minimum image) and ``e`` the
        relative strain of the cell (spectral norm of ``h0^-1 (h - h0)``); ``d`` is agreed over
        the processes, so every process gets the same answer."""
        cell = self._plan_cell(plan, cell)
        p64 = pos.detach().to(torch.float64)
        strain = 0.0
        if cell is None:
            moved = p64 - plan.reference
        else:
            c64 = cell.detach().to(torch.float64)
            inv, unchanged = self._inverse(plan, c64)
            df = _apply3(p64, inv) - plan.reference
            moved = _apply3(df - torch.round(df), c64)
            if not unchanged:
                strain = float(torch.linalg.matrix_norm(torch.linalg.solve(plan.cell, c64 - plan.cell), ord=2))
        worst = moved.norm(dim=-1).max().reshape(1) if len(moved) else moved.new_zeros(1)
        if plan.world > 1:
            dist.all_reduce(worst, op=dist.ReduceOp.MAX, group=self.group)
        budget = (1.0 - strain) * (plan.need + plan.skin + HALO_MARGIN)
        return plan.need + 2.0 * float(worst[0]) <= budget

    @torch.no_grad()
    def reshard(self, plan: DomainPlan, pos: Tensor, *fields: Tensor, cell: Optional[Tensor] = None) -> tuple:
        """A new plan for the current positions, with ``pos`` and every per-atom field moved
        to the atoms' new owners. Returns ``(plan, pos, *fields)``."""
        cell = self._plan_cell(plan, cell)
        full = [self._gather(plan, x) for x in (pos,) + fields]
        new = self._build(full[0], plan.atomic_numbers, cell, plan.total_charge, plan.spin_multiplicity)
        return (new,) + tuple(x.index_select(0, new.owned) for x in full)

    def _gather(self, plan: DomainPlan, rows: Tensor) -> Tensor:
        """Rows of every process's owned atoms, in the atom order of the structure."""
        out = rows.new_empty((plan.n_atoms,) + tuple(rows.shape[1:]))
        if plan.world == 1:
            out[plan.owned] = rows
            return out
        width = max(plan.counts)
        mine = rows.new_zeros((width,) + tuple(rows.shape[1:]))
        mine[:rows.shape[0]] = rows
        parts = [torch.empty_like(mine) for _ in range(plan.world)]
        dist.all_gather(parts, mine.contiguous(), group=self.group)
        out[plan.order] = torch.cat([part[:c] for part, c in zip(parts, plan.counts)])
        return out

    # ---------------------------------------------------------------- exchange
    def _get_exchanger(self, plan: DomainPlan, like: Tensor):
        if self.exchange != "p2p" or plan.world == 1 or not like.is_cuda:
            return None
        if self._exchanger is None:
            from .halo import PeerHaloExchange
            self._exchanger = PeerHaloExchange(like.device, self.group)
        return self._exchanger

    def _exchange(self, plan: DomainPlan, rows: Tensor, links: List[Tensor]) -> Tensor:
        """Rows of the ghosts, sent by their owners from ``rows`` (the owned atoms)."""
        if plan.world == 1:
            return rows.index_select(0, plan.send_rows)
        if links:
            rows = rows + _order_link(links[-1]).to(rows.dtype)
        out = _RowExchange.apply(rows, plan, self.group, self._get_exchanger(plan, rows))
        links.append(out)
        return out

    # ---------------------------------------------------------------- evaluation
    def evaluate(self, plan: DomainPlan, pos: Tensor, cell: Optional[Tensor] = None) -> dict:
        """Energy (whole structure, float64 ``(1,)``), forces on the owned atoms and, for a
        periodic structure with ``compute_stress``, the stress ``(1, 3, 3)``."""
        if pos.shape[0] != plan.n_owned:
            raise ValueError(f"{pos.shape[0]} positions for the {plan.n_owned} atoms of the plan")
        cell = self._plan_cell(plan, cell)
        x = pos.detach().requires_grad_(True)
        dtype, device = x.dtype, x.device
        strain, volume, own = None, None, x
        if cell is not None:
            c64 = cell.detach().to(torch.float64)
            inv, _ = self._inverse(plan, c64)
            volume = torch.linalg.det(c64).abs().reshape(1)
            # whole cells each owned atom moved since the plan (to bring it back next to its ghosts)
            wraps = torch.round(_apply3(x.detach().to(torch.float64), inv) - plan.reference).to(dtype)
            cell = cell.detach().to(dtype)
            if self.compute_stress:
                strain = torch.zeros((3, 3), dtype=dtype, device=device, requires_grad=True)
                sym = 0.5 * (strain + strain.t())
                own = own + own @ sym
                cell = cell + cell @ sym
            own = own - _apply3(wraps, cell)
        links: List[Tensor] = []
        ghost_pos = self._exchange(plan, own, links)
        if cell is not None:
            ghost_pos = ghost_pos + _apply3(plan.ghost_shifts.to(dtype), cell)
        local = torch.cat([own, ghost_pos])
        numbers = plan.atomic_numbers.index_select(0, plan.index)
        if plan.n_local == 0:
            # an empty sub-domain evaluates one isolated stand-in (energy dropped) so that it
            # takes part in every exchange of the others
            local = local.new_zeros((1, 3))
            numbers = plan.atomic_numbers[:1]
        with torch.no_grad():
            d = local.index_select(0, plan.edge_index[1]) - local.index_select(0, plan.edge_index[0])
            if plan.pbc is not None:
                d = d + _apply3(plan.cell_shifts.to(dtype), cell)
            inside = (d * d).sum(-1) < self.cutoff ** 2
        edge_index, cell_shifts = plan.edge_index[:, inside], plan.cell_shifts[inside]
        mdt = _model_dtype(self.model)
        n_local = int(local.shape[0])
        graph = AtomicGraph(
            pos=local, atomic_numbers=numbers, edge_index=edge_index, cell_shifts=cell_shifts,
            batch=torch.zeros(n_local, dtype=torch.long, device=device),
            n_atoms=torch.tensor([n_local], dtype=torch.long, device=device),
            cell=cell[None] if plan.pbc is not None else None,
            pbc=plan.pbc[None].to(device) if plan.pbc is not None else None,
            total_charge=plan.total_charge, spin_multiplicity=plan.spin_multiplicity,
            compute_dtype=mdt if mdt is not None and mdt != dtype else None)
        graph.edge_order = "dst"
        with domain_hooks(_Hooks(self, plan, links)):
            out = self.model(graph)
        energy = out["node_energy"][:plan.n_owned].to(torch.float64).sum()
        for t in links:
            energy = energy + _order_link(t)
        wrt = [x] + ([strain] if strain is not None else [])
        grads: List[Optional[Tensor]] = [None] * len(wrt)
        if energy.requires_grad:
            # only position / strain derivatives: the fused ops skip their weight gradients
            with force_pass():
                grads = list(torch.autograd.grad([energy], wrt, allow_unused=True))
        g_pos = grads[0] if grads[0] is not None else torch.zeros_like(x)
        g_strain = grads[1] if strain is not None and grads[1] is not None else \
            torch.zeros((3, 3), dtype=torch.float64, device=device)
        summed = torch.cat([energy.detach().reshape(1), g_strain.to(torch.float64).reshape(9)])
        if plan.world > 1:
            dist.all_reduce(summed, group=self.group)
        if self._exchanger is not None:
            self._exchanger.check()
        result = {"energy": summed[:1], "forces": -g_pos.to(dtype)}
        if strain is not None:
            result["stress"] = (summed[1:].view(1, 3, 3) / volume).to(dtype)
        return result

    def forward(self, data: AtomicGraph) -> dict:
        """Energy, forces (all atoms, gathered) and stress of ``data``, given on every process;
        the plan of the previous call is reused while it holds."""
        periodic = data.cell is not None and data.pbc is not None and bool(data.pbc.any())
        cell = data.cell[0] if periodic else None
        plan = self._plan
        reusable = (plan is not None and plan.n_atoms == data.num_nodes and (plan.cell is not None) == periodic
                    and torch.equal(plan.atomic_numbers, data.atomic_numbers))
        if not (reusable and self.holds(plan, data.pos.index_select(0, plan.owned), cell)):
            plan = self._plan = self.plan(data)
        plan.total_charge, plan.spin_multiplicity = data.total_charge, data.spin_multiplicity
        out = self.evaluate(plan, data.pos.index_select(0, plan.owned), cell)
        out["forces"] = self._gather(plan, out["forces"])
        return out

    def close(self) -> None:
        if self._exchanger is not None:
            self._exchanger.close()
            self._exchanger = None


class _Hooks:
    """The object the model's ``refresh_ghosts`` / ``whole_structure_sum`` calls go to."""

    def __init__(self, dp: DomainParallel, plan: DomainPlan, links: List[Tensor]):
        self.dp, self.plan, self.links = dp, plan, links

    def refresh(self, x: Tensor) -> Tensor:
        plan = self.plan
        if not self.dp.layer:
            return x
        rows = max(plan.n_local, 1)
        if x.shape[0] != rows:
            raise ValueError(f"refresh_ghosts got {x.shape[0]} rows for {rows} local atoms")
        fresh = self.dp._exchange(plan, x[:plan.n_owned], self.links)
        return torch.cat([x[:plan.n_owned], fresh, x[plan.n_local:]])

    def whole_sum(self, values: Tensor, batch: Tensor, num_graphs: int) -> Tensor:
        n = self.plan.n_owned
        part = structure_sum(values[:n], batch[:n], num_graphs)
        if self.plan.world > 1:
            if self.links:
                part = part + _order_link(self.links[-1]).to(part.dtype)
            part = _SumOverRanks.apply(part, self.dp.group)
            self.links.append(part)
        return part
