"""Torch-free integer expressions over named symbols.

The same constructors as the reference frontend's ``reloc_torch.symbolic``
(Const, Symbol, Add, Mul, FloorDiv, Mod, dense_strides; reference
libreloc/python/reloc_torch/symbolic.py:26-181) so recipes read alike. Adds
the postfix lowering to the wire expression opcodes used by the plan encoder.
"""
from __future__ import annotations

from dataclasses import dataclass


class UnsupportedSymbolicExpr(ValueError):
    reason = "unsupported_symbolic_expr"

    def __init__(self, detail):
        super().__init__(f"{self.reason}: {detail}")


@dataclass(frozen=True)
class Expr:
    def evaluate(self, bindings):
        if isinstance(self, Const):
            return self.value
        if isinstance(self, Symbol):
            return int(bindings[self.name])
        if isinstance(self, Add):
            return self.lhs.evaluate(bindings) + self.rhs.evaluate(bindings)
        if isinstance(self, Mul):
            return self.lhs.evaluate(bindings) * self.rhs.evaluate(bindings)
        if isinstance(self, FloorDiv):
            return self.lhs.evaluate(bindings) // self.divisor
        if isinstance(self, Mod):
            return self.lhs.evaluate(bindings) % self.divisor
        raise UnsupportedSymbolicExpr("unknown expression")

    def symbols(self):
        if isinstance(self, Symbol):
            return [self.name]
        out = []
        for child in (getattr(self, "lhs", None), getattr(self, "rhs", None)):
            if child is not None:
                for s in child.symbols():
                    if s not in out:
                        out.append(s)
        return out


@dataclass(frozen=True)
class Const(Expr):
    value: int

    def __post_init__(self):
        if type(self.value) is not int:
            raise UnsupportedSymbolicExpr("constant must be an integer")


@dataclass(frozen=True)
class Symbol(Expr):
    name: str

    def __post_init__(self):
        if not self.name.isidentifier() or not self.name.isascii():
            raise UnsupportedSymbolicExpr("invalid symbol name")


@dataclass(frozen=True)
class Add(Expr):
    lhs: Expr
    rhs: Expr


@dataclass(frozen=True)
class Mul(Expr):
    lhs: Expr
    rhs: Expr


@dataclass(frozen=True)
class FloorDiv(Expr):
    lhs: Expr
    divisor: int


@dataclass(frozen=True)
class Mod(Expr):
    lhs: Expr
    divisor: int


def expression(value) -> Expr:
    if isinstance(value, Expr):
        return value
    if type(value) is int:
        return Const(value)
    raise UnsupportedSymbolicExpr(f"not an expression: {value!r}")


def add(lhs, rhs) -> Expr:
    """``lhs + rhs`` in the plan format's simplified form (the rules of the
    reference's sym simplifier): constants fold, ``+ 0`` drops, and
    ``(x + c1) + c2`` becomes ``x + (c1 + c2)``."""
    lhs, rhs = expression(lhs), expression(rhs)
    if isinstance(lhs, Const) and isinstance(rhs, Const):
        return Const(lhs.value + rhs.value)
    if isinstance(rhs, Const) and rhs.value == 0:
        return lhs
    if isinstance(lhs, Const) and lhs.value == 0:
        return rhs
    if isinstance(rhs, Const) and isinstance(lhs, Add) and isinstance(lhs.rhs, Const):
        return add(lhs.lhs, Const(lhs.rhs.value + rhs.value))
    return Add(lhs, rhs)


def mul(lhs, rhs) -> Expr:
    """``lhs * rhs`` simplified likewise: constants fold, ``* 1`` drops and
    ``(x * c1) * c2`` becomes ``x * (c1 * c2)``."""
    lhs, rhs = expression(lhs), expression(rhs)
    if isinstance(lhs, Const) and isinstance(rhs, Const):
        return Const(lhs.value * rhs.value)
    if isinstance(rhs, Const) and rhs.value == 1:
        return lhs
    if isinstance(lhs, Const) and lhs.value == 1:
        return rhs
    if isinstance(rhs, Const) and isinstance(lhs, Mul) and isinstance(lhs.rhs, Const):
        return mul(lhs.lhs, Const(lhs.rhs.value * rhs.value))
    # (X floordiv k) * k with k constant stays as written; the encoder records
    # the divisibility that makes it equal X.
    return Mul(lhs, rhs)


def product(shape) -> Expr:
    out = Const(1)
    for d in shape:
        out = mul(out, d)
    return out


def dense_strides(shape):
    """Row-major element strides of ``shape`` (innermost 1)."""
    strides = []
    running = Const(1)
    for d in reversed(list(shape)):
        strides.append(running)
        running = mul(running, d)
    return tuple(reversed(strides))


def from_json(node) -> Expr:
    """Decode the reference manifest's expression form (["const", 3],
    ["symbol", "s0"], ["add", a, b], ["mul", a, b], ["floordiv", a, k],
    ["mod", a, k])."""
    kind = node[0]
    if kind == "const":
        return Const(int(node[1]))
    if kind == "symbol":
        return Symbol(node[1])
    if kind == "add":
        return Add(from_json(node[1]), from_json(node[2]))
    if kind == "mul":
        return Mul(from_json(node[1]), from_json(node[2]))
    if kind == "floordiv":
        return FloorDiv(from_json(node[1]), int(node[2][1] if isinstance(node[2], list) else node[2]))
    if kind == "mod":
        return Mod(from_json(node[1]), int(node[2][1] if isinstance(node[2], list) else node[2]))
    raise UnsupportedSymbolicExpr(f"unknown node {kind!r}")


# ---- canonical products (for reshape grouping) ---------------------------------

def _factors(e: Expr):
    """(constant, sorted atoms) of a product, or None when not a product."""
    if isinstance(e, Const):
        return e.value, ()
    if isinstance(e, (Symbol, FloorDiv, Add, Mod)):
        return 1, (e,)
    if isinstance(e, Mul):
        a, b = _factors(e.lhs), _factors(e.rhs)
        if a is None or b is None:
            return None
        return a[0] * b[0], tuple(sorted(a[1] + b[1], key=repr))
    return None


def product_key(factors):
    """Canonical key of a list of extents' product; FloorDiv(X, k) * k folds to X."""
    const = 1
    atoms = []
    for f in factors:
        fc = _factors(expression(f))
        if fc is None:
            return None
        const *= fc[0]
        atoms.extend(fc[1])
    changed = True
    while changed:
        changed = False
        for i, a in enumerate(atoms):
            if isinstance(a, FloorDiv) and const % a.divisor == 0:
                const //= a.divisor
                atoms[i] = a.lhs
                changed = True
                break
    return const, tuple(sorted(atoms, key=repr))
