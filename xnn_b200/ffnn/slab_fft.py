"""Reciprocal-space PME over a mesh split into z-slabs across processes (distributed 3D FFT).

Every process holds all sites (positions and multipoles are replicated, as in a replicated-data
MD step) and owns the planes ``[z0, z1)`` of the ``K1 x K2 x K3`` mesh:

1. spread: each process applies the multipole operator to the B-spline stencils of the sites
   whose stencils reach its planes and accumulates only into its planes (no ghost planes to
   exchange);
2. forward transform: a real FFT along x and a complex FFT along y of the local planes, then a
   transpose that gives each process all ``K3`` planes of its share of the ``K1 // 2 + 1``
   x-frequencies (an all-to-all of ``(kx, ky)`` lines), then the FFT along z;
3. energy: ``(1/2) sum infl(m) |F(m)|^2`` over the local frequencies (a partial energy: the
   caller sums the processes' parts).

Everything is differentiable: the transpose is an autograd function whose adjoint is the
reverse transpose, so ``d E_local / d positions`` is each process's share of the reciprocal
forces and fields. The transpose goes through ``all_to_all_single`` of the process group, or,
with ``exchange="p2p"`` on CUDA, through the peer-memory exchange kernel of
:mod:`xnn_b200.parallel.halo` (pack, NVLink stores and unpack in one launch per direction).
"""
from __future__ import annotations

import math
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist
from torch import Tensor
from torch.autograd import Function

from .multipoles import bspline_moduli, spread, _freq


def split_range(n: int, parts: int, k: int) -> Tuple[int, int]:
    base, extra = divmod(n, parts)
    lo = k * base + min(k, extra)
    return lo, lo + base + (1 if k < extra else 0)


class _Transpose(Function):
    """``(nkx, K2, nz_r)`` planes of every process -> ``(nkx_r, K2, K3)`` lines of this one."""

    @staticmethod
    def forward(ctx, x: Tensor, fft: "SlabFFT"):
        ctx.fft = fft
        return fft._to_lines(x)

    @staticmethod
    def backward(ctx, g: Tensor):
        return ctx.fft._to_planes(g.contiguous()), None


class SlabFFT:
    def __init__(self, mesh: List[int], group=None, exchange: str = "collective"):
        self.mesh = [int(m) for m in mesh]
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        K1, K2, K3 = self.mesh
        self.nkx = K1 // 2 + 1
        self.z = [split_range(K3, self.world, r) for r in range(self.world)]
        self.x = [split_range(self.nkx, self.world, r) for r in range(self.world)]
        self.exchange = exchange
        self._peer = None
        self._infl = None

    # ---------------------------------------------------------------- transposes
    def _peer_exchange(self, like: Tensor):
        if self.exchange != "p2p" or self.world == 1 or not like.is_cuda:
            return None
        if self._peer is None:
            from ..parallel.halo import PeerHaloExchange
            self._peer = PeerHaloExchange(like.device, self.group)
        return self._peer

    def _a2a(self, send: List[Tensor], recv_shapes: List[Tuple[int, ...]], like: Tensor) -> List[Tensor]:
        """Send ``send[p]`` to process ``p``; returns what every process sent here."""
        flat = torch.cat([t.reshape(-1) for t in send])
        in_counts = [t.numel() for t in send]
        out_counts = [math.prod(s) for s in recv_shapes]
        peer = self._peer_exchange(like)
        if peer is not None:
            # rows of 8 bytes (one complex64 value): the exchange kernel moves any row size
            src = torch.view_as_real(flat).contiguous()
            out = torch.empty(sum(out_counts), 2, dtype=src.dtype, device=src.device)
            offs = self._remote_offsets(tuple(out_counts))
            peer.reserve(self._max_rows() * 8)
            peer.launch([src.view(-1, 2)], [None], [in_counts], [offs], [out], 8)
            res = torch.view_as_complex(out)
        else:
            res = torch.empty(sum(out_counts), dtype=flat.dtype, device=flat.device)
            dist.all_to_all_single(res, flat, out_counts, in_counts, group=self.group)
        parts, o = [], 0
        for s in recv_shapes:
            n = math.prod(s)
            parts.append(res[o:o + n].view(*s))
            o += n
        return parts

    def _max_rows(self) -> int:
        """Largest receive of any process in either direction (the same on every process)."""
        K1, K2, K3 = self.mesh
        lines = max((x1 - x0) * K2 * K3 for x0, x1 in self.x)
        planes = max(self.nkx * K2 * (z1 - z0) for z0, z1 in self.z)
        return max(lines, planes)

    def _remote_offsets(self, my_recv_counts: Tuple[int, ...]) -> List[int]:
        """Where this process's rows land in every receiver's buffer (an all-to-all of starts,
        cached per direction)."""
        cache = self.__dict__.setdefault("_offs", {})
        if my_recv_counts not in cache:
            starts = torch.tensor([sum(my_recv_counts[:p]) for p in range(self.world)], dtype=torch.long)
            dev = torch.device("cuda", torch.cuda.current_device())
            s = starts.to(dev)
            out = torch.empty_like(s)
            dist.all_to_all_single(out, s, group=self.group)
            cache[my_recv_counts] = out.tolist()
        return cache[my_recv_counts]

    def check(self) -> None:
        if self._peer is not None:
            self._peer.check()

    def _to_lines(self, planes: Tensor) -> Tensor:
        K1, K2, K3 = self.mesh
        if self.world == 1:
            return planes
        send = [planes[x0:x1].contiguous() for x0, x1 in self.x]
        x0, x1 = self.x[self.rank]
        parts = self._a2a(send, [(x1 - x0, K2, z1 - z0) for z0, z1 in self.z], planes)
        return torch.cat(parts, dim=2)

    def _to_planes(self, lines: Tensor) -> Tensor:
        K1, K2, K3 = self.mesh
        if self.world == 1:
            return lines
        send = [lines[:, :, z0:z1].contiguous() for z0, z1 in self.z]
        z0, z1 = self.z[self.rank]
        parts = self._a2a(send, [(x1 - x0, K2, z1 - z0) for x0, x1 in self.x], lines)
        return torch.cat(parts, dim=0)

    # ---------------------------------------------------------------- influence
    def influence(self, cell: Tensor, alpha: float, order: int, dtype) -> Tensor:
        key = (tuple(cell.detach().reshape(-1).tolist()), alpha, order)
        if self._infl is not None and self._infl[0] == key:
            return self._infl[1]
        K1, K2, K3 = self.mesh
        dev = cell.device
        x0, x1 = self.x[self.rank]
        rec = torch.linalg.inv(cell.detach()).t().to(torch.float64)
        f1 = torch.arange(x0, x1, device=dev, dtype=torch.float64)
        f2, f3 = _freq(K2, dev).double(), _freq(K3, dev).double()
        m = f1[:, None, None, None] * rec[0] + f2[None, :, None, None] * rec[1] + f3[None, None, :, None] * rec[2]
        m2 = (m * m).sum(-1)
        vol = torch.det(cell.detach().to(torch.float64)).abs()
        B = (bspline_moduli(K1, order, torch.float64, dev)[x0:x1, None, None]
             * bspline_moduli(K2, order, torch.float64, dev)[None, :, None]
             * bspline_moduli(K3, order, torch.float64, dev)[None, None, :])
        safe = torch.where(m2 > 0, m2, torch.ones_like(m2))
        val = torch.where(m2 > 0, torch.exp(-math.pi ** 2 * m2 / alpha ** 2) / (math.pi * vol * safe) * B,
                          torch.zeros_like(m2))
        w = torch.full((x1 - x0,), 2.0, dtype=torch.float64, device=dev)
        w[(f1 == 0)] = 1.0
        if K1 % 2 == 0:
            w[(f1 == K1 // 2)] = 1.0
        out = (val * w[:, None, None]).to(dtype)
        self._infl = (key, out)
        return out

    # ---------------------------------------------------------------- energy
    def energy(self, pos: Tensor, cell: Tensor, q, d, Q, setup) -> Tensor:
        """This process's share of the reciprocal energy (Coulomb units)."""
        K1, K2, K3 = self.mesh
        p = setup.order
        z0, z1 = self.z[self.rank]
        if self.world > 1:
            # only the sites whose stencil (planes base - p + 1 .. base) reaches this slab
            with torch.no_grad():
                uz = (pos.detach() @ torch.linalg.inv(cell.detach()))[:, 2] * K3
                base = torch.floor(uz).long()
                keep = torch.nonzero(((base - z0) % K3) < (z1 - z0) + p - 1).flatten()
            pos, q = pos.index_select(0, keep), q.index_select(0, keep) if q is not None else None
            d = d.index_select(0, keep) if d is not None else None
            Q = Q.index_select(0, keep) if Q is not None else None
        planes = spread(pos, cell, q, d, Q, self.mesh, p, z_range=(z0, z1), out_dtype=setup.fft_dtype).to(
            setup.fft_dtype)
        F = torch.fft.rfft(planes, dim=0)                 # (K1//2+1, K2, nz)
        F = torch.fft.fft(F, dim=1)
        F = _Transpose.apply(F, self)                      # (nkx_r, K2, K3)
        F = torch.fft.fft(F, dim=2)
        infl = self.influence(cell, setup.alpha, p, setup.fft_dtype)
        return (0.5 * (infl * (F.real * F.real + F.imag * F.imag)).sum()).to(pos.dtype)

    def _slab_sites(self, pos: Tensor, cell: Tensor, p: int) -> Tensor:
        """Indices of the sites whose stencil (planes base - p + 1 .. base) reaches this slab."""
        K3 = self.mesh[2]
        z0, z1 = self.z[self.rank]
        with torch.no_grad():
            uz = (pos.detach() @ torch.linalg.inv(cell.detach()))[:, 2] * K3
            base = torch.floor(uz).long()
            return torch.nonzero(((base - z0) % K3) < (z1 - z0) + p - 1).flatten()

    def dipole_field(self, pos: Tensor, cell: Tensor, d: Tensor, setup) -> Tensor:
        """This process's share of the reciprocal field ``-dE/dd`` of dipoles ``d`` (Coulomb
        units, ``(n, 3)``; the caller sums the shares), without an energy graph: spread onto this
        slab, forward transform and transpose, influence, the inverse pipeline (the adjoint of the
        forward one) back to the slab's mesh potential ``dE/dgrid``, and the gather of its stencil
        derivatives at the sites that reach the slab."""
        from .multipoles import gather_dipole_gradient
        K1, K2, K3 = self.mesh
        p = setup.order
        z0, z1 = self.z[self.rank]
        keep = self._slab_sites(pos, cell, p) if self.world > 1 else None
        pk = pos if keep is None else pos.index_select(0, keep)
        dk = d if keep is None else d.index_select(0, keep)
        planes = spread(pk, cell, None, dk, None, self.mesh, p, z_range=(z0, z1),
                        out_dtype=setup.fft_dtype).to(setup.fft_dtype)
        F = torch.fft.fft(torch.fft.rfft(planes, dim=0), dim=1)
        F = torch.fft.fft(self._to_lines(F), dim=2)
        infl = self.influence(cell, setup.alpha, p, setup.fft_dtype)
        x0, x1 = self.x[self.rank]
        w = torch.full((x1 - x0,), 2.0, dtype=infl.dtype, device=infl.device)
        f1 = torch.arange(x0, x1, device=infl.device)
        w[f1 == 0] = 1.0
        if K1 % 2 == 0:
            w[f1 == K1 // 2] = 1.0
        # the unweighted influence (the inverse real transform restores the conjugate half) times
        # the mesh size (the unnormalised inverse)
        G = torch.fft.ifft(F * (infl / w[:, None, None] * float(K1 * K2 * K3)), dim=2)
        G = torch.fft.ifft(self._to_planes(G.contiguous()), dim=1)
        phi = torch.fft.irfft(G, n=K1, dim=0).contiguous()
        gk = gather_dipole_gradient(pk, cell, dk, self.mesh, p, (z0, z1), phi)
        if keep is None:
            return -gk
        return torch.zeros_like(d).index_add_(0, keep, -gk)

    def close(self) -> None:
        if self._peer is not None:
            self._peer.close()
            self._peer = None
