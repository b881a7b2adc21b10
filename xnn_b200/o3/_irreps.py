"""Irreducible representations of O(3) and direct sums of them.

The string forms (``"16x0e+16x1o"``), the ordering of irreps and the layout of a
feature vector (each ``mul x ir`` block stored multiplicity-major, ``(mul, 2l+1)``)
follow the conventions of e3nn, which the reference's checkpoints depend on
(``src/xnn/gnn/models/blocks.py:40-115`` builds every irreps it uses through them).
"""
from __future__ import annotations

import re
from typing import Iterator, List, NamedTuple, Tuple, Union


class Irrep(tuple):
    """An irreducible representation ``(l, p)`` of O(3); ``p = +1`` (even) or ``-1`` (odd)."""

    def __new__(cls, l: Union[int, str, "Irrep", tuple], p: int | None = None):
        if isinstance(l, Irrep):
            return l
        if isinstance(l, str):
            s = l.strip()
            m = re.fullmatch(r"(\d+)([eoy])", s)
            if m is None:
                raise ValueError(f"cannot parse irrep {l!r}")
            lv = int(m.group(1))
            ch = m.group(2)
            pv = {"e": 1, "o": -1, "y": (-1) ** lv}[ch]
            return super().__new__(cls, (lv, pv))
        if isinstance(l, tuple):
            l, p = l
        if p not in (1, -1) or int(l) < 0:
            raise ValueError(f"invalid irrep l={l} p={p}")
        return super().__new__(cls, (int(l), int(p)))

    @property
    def l(self) -> int:  # noqa: E743
        return self[0]

    @property
    def p(self) -> int:
        return self[1]

    @property
    def dim(self) -> int:
        return 2 * self[0] + 1

    def __repr__(self) -> str:
        return f"{self[0]}{'e' if self[1] == 1 else 'o'}"

    __str__ = __repr__

    def __mul__(self, other: "Irrep") -> Iterator["Irrep"]:
        """The irreps of the tensor product ``self x other`` in increasing ``l``."""
        other = Irrep(other)
        p = self.p * other.p
        for l in range(abs(self.l - other.l), self.l + other.l + 1):
            yield Irrep(l, p)

    def __rmul__(self, mul: int) -> "Irreps":
        return Irreps([(int(mul), self)])

    def is_scalar(self) -> bool:
        return self == (0, 1)


class MulIr(NamedTuple):
    mul: int
    ir: Irrep

    @property
    def dim(self) -> int:
        return self.mul * self.ir.dim

    def __repr__(self) -> str:
        return f"{self.mul}x{self.ir}"


class Irreps(tuple):
    """A direct sum of irreps with multiplicities, e.g. ``Irreps("32x0e+16x1o")``."""

    def __new__(cls, irreps=None):
        if isinstance(irreps, Irreps):
            return irreps
        out: List[MulIr] = []
        if irreps is None:
            pass
        elif isinstance(irreps, Irrep):
            out.append(MulIr(1, irreps))
        elif isinstance(irreps, str):
            s = irreps.strip()
            if s:
                for term in s.split("+"):
                    term = term.strip()
                    if "x" in term:
                        mul, ir = term.split("x")
                        out.append(MulIr(int(mul), Irrep(ir)))
                    else:
                        out.append(MulIr(1, Irrep(term)))
        else:
            for item in irreps:
                if isinstance(item, MulIr):
                    out.append(item)
                elif isinstance(item, (str, Irrep)):
                    out.append(MulIr(1, Irrep(item)))
                elif isinstance(item, tuple) and len(item) == 2:
                    mul, ir = item
                    if isinstance(mul, int) and not isinstance(ir, int):
                        out.append(MulIr(int(mul), Irrep(ir)))
                    else:  # a bare (l, p) pair
                        out.append(MulIr(1, Irrep(mul, ir)))
                else:
                    raise ValueError(f"cannot parse irreps entry {item!r}")
        return super().__new__(cls, out)

    @staticmethod
    def spherical_harmonics(lmax: int, p: int = -1) -> "Irreps":
        """``1x0e + 1x1o + ... + 1x lmax`` with parity ``p**l`` (the SH series)."""
        return Irreps([(1, Irrep(l, p ** l)) for l in range(lmax + 1)])

    @property
    def dim(self) -> int:
        return sum(m.dim for m in self)

    @property
    def num_irreps(self) -> int:
        return sum(m.mul for m in self)

    @property
    def lmax(self) -> int:
        if len(self) == 0:
            raise ValueError("empty irreps have no lmax")
        return max(m.ir.l for m in self)

    @property
    def ls(self) -> List[int]:
        return [m.ir.l for m in self for _ in range(m.mul)]

    def count(self, ir) -> int:  # type: ignore[override]
        ir = Irrep(ir)
        return sum(m.mul for m in self if m.ir == ir)

    def __contains__(self, ir) -> bool:  # type: ignore[override]
        ir = Irrep(ir)
        return any(m.ir == ir for m in self)

    def slices(self) -> List[slice]:
        out, i = [], 0
        for m in self:
            out.append(slice(i, i + m.dim))
            i += m.dim
        return out

    def sort(self) -> "SortedIrreps":
        """Sorted irreps, the permutation ``p`` (old -> new position) and its inverse, as a named
        tuple ``(irreps, p, inv)``."""
        keyed = sorted((m.ir, i, m.mul) for i, m in enumerate(self))
        inv = tuple(i for _, i, _ in keyed)
        p = [0] * len(inv)
        for new, old in enumerate(inv):
            p[old] = new
        return SortedIrreps(Irreps([(mul, ir) for ir, _, mul in keyed]), tuple(p), inv)

    def simplify(self) -> "Irreps":
        out: List[Tuple[int, Irrep]] = []
        for m in self:
            if out and out[-1][1] == m.ir:
                out[-1] = (out[-1][0] + m.mul, m.ir)
            elif m.mul > 0:
                out.append((m.mul, m.ir))
        return Irreps(out)

    def __add__(self, other) -> "Irreps":  # type: ignore[override]
        return Irreps(tuple(self) + tuple(Irreps(other)))

    def __mul__(self, n) -> "Irreps":  # type: ignore[override]
        """The list repeated ``n`` times (``2 * "1x0e"`` is ``1x0e+1x0e``)."""
        if not isinstance(n, int):
            raise NotImplementedError("Irreps multiply only by an integer")
        return Irreps(tuple(self) * n)

    __rmul__ = __mul__

    def __repr__(self) -> str:
        return "+".join(repr(m) for m in self)

    __str__ = __repr__

    def __eq__(self, other) -> bool:
        try:
            other = Irreps(other)
        except Exception:
            return False
        return tuple.__eq__(self, other)

    def __hash__(self) -> int:
        return tuple.__hash__(self)


class SortedIrreps(NamedTuple):
    irreps: Irreps
    p: Tuple[int, ...]
    inv: Tuple[int, ...]
