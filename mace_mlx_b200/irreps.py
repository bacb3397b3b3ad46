"""O(3) irrep bookkeeping (host-side metadata only).

Same string format and ordering rules as the reference's ``mace_mlx/irreps.py``
(which follows e3nn): an irrep is ``(l, p)`` written ``"1o"``; an ``Irreps`` is an
ordered direct sum ``"128x0e + 128x1o"``.  Ordering between irreps is by
``(l, p)`` with odd parity (-1) before even (+1) for the same ``l``
(reference ``irreps.py:80-81``), and ``sort`` is a stable sort on that key
(``irreps.py:196-205``).  The layout conventions fixed here decide the slot
order of every feature table the kernels see, so they must agree with the
reference exactly.
"""

from __future__ import annotations

import re
from typing import Iterable, Iterator, NamedTuple

_IRREP_RE = re.compile(r"^\s*(\d+)\s*([eoy])\s*$")


class Irrep(NamedTuple):
    """Irreducible representation of O(3): degree ``l`` and parity ``p`` (+1/-1)."""

    l: int
    p: int

    @classmethod
    def parse(cls, s) -> "Irrep":
        if isinstance(s, Irrep):
            return s
        if isinstance(s, tuple):
            return cls(int(s[0]), int(s[1]))
        m = _IRREP_RE.match(str(s))
        if not m:
            raise ValueError(f"cannot parse irrep {s!r}")
        l = int(m.group(1))
        c = m.group(2)
        p = 1 if c == "e" else -1 if c == "o" else (-1) ** l
        return cls(l, p)

    @property
    def dim(self) -> int:
        return 2 * self.l + 1

    def __str__(self) -> str:  # noqa: D105
        return f"{self.l}{'e' if self.p == 1 else 'o'}"

    __repr__ = __str__

    def couple(self, other: "Irrep") -> list["Irrep"]:
        """Selection rule of the product ``self x other``: |l1-l2| <= l <= l1+l2."""
        p = self.p * other.p
        return [Irrep(l, p) for l in range(abs(self.l - other.l), self.l + other.l + 1)]


class MulIr(NamedTuple):
    mul: int
    ir: Irrep

    @property
    def dim(self) -> int:
        return self.mul * self.ir.dim


class Irreps(tuple):
    """Ordered direct sum of irreps with multiplicities (immutable)."""

    def __new__(cls, spec=None):
        if spec is None:
            return super().__new__(cls, ())
        if isinstance(spec, Irreps):
            return spec
        items: list[MulIr] = []
        if isinstance(spec, str):
            for part in spec.split("+"):
                part = part.strip()
                if not part:
                    continue
                if "x" in part:
                    mul_s, ir_s = part.split("x", 1)
                    items.append(MulIr(int(mul_s), Irrep.parse(ir_s)))
                else:
                    items.append(MulIr(1, Irrep.parse(part)))
        else:
            for it in spec:
                if isinstance(it, MulIr):
                    items.append(it)
                elif isinstance(it, Irrep):
                    items.append(MulIr(1, it))
                else:
                    mul, ir = it
                    items.append(MulIr(int(mul), Irrep.parse(ir)))
        return super().__new__(cls, tuple(items))

    # -- sizes -------------------------------------------------------------
    @property
    def dim(self) -> int:
        return sum(m.dim for m in self)

    @property
    def lmax(self) -> int:
        return max(m.ir.l for m in self)

    def count(self, ir) -> int:
        ir = Irrep.parse(ir)
        return sum(m.mul for m in self if m.ir == ir)

    def offsets(self) -> list[int]:
        """Start offset of every slot in the reference's irreps-major layout."""
        out, o = [], 0
        for m in self:
            out.append(o)
            o += m.dim
        return out

    def has(self, ir) -> bool:
        ir = Irrep.parse(ir)
        return any(m.ir == ir for m in self)

    # -- reorderings ---------------------------------------------------------
    def sort(self) -> tuple["Irreps", tuple[int, ...], tuple[int, ...]]:
        """Stable sort by ``(l, p)``; returns (sorted, perm, inv) like e3nn."""
        order = sorted(range(len(self)), key=lambda i: (self[i].ir.l, self[i].ir.p))
        inv = [0] * len(order)
        for new, old in enumerate(order):
            inv[old] = new
        return Irreps([self[i] for i in order]), tuple(order), tuple(inv)

    def scalars(self) -> "Irreps":
        return Irreps([m for m in self if m.ir.l == 0])

    @staticmethod
    def spherical_harmonics(lmax: int) -> "Irreps":
        return Irreps([MulIr(1, Irrep(l, (-1) ** l)) for l in range(lmax + 1)])

    def __iter__(self) -> Iterator[MulIr]:  # type: ignore[override]
        return super().__iter__()

    def __str__(self) -> str:
        return " + ".join(f"{m.mul}x{m.ir}" for m in self)

    __repr__ = __str__


def irreps(spec: str | Iterable) -> Irreps:
    return Irreps(spec)
