"""Expected stdout and exit code of a Mapal program from the bench subset.

TEST INFRASTRUCTURE ONLY: the CPU restatement of the reference interpreter
(crates/mapal-interp) that the program driver's output is compared with. The
product never imports it.

Subset: `fn main() { ... }` statements `expr -> stage -> ... ;` with stages
`iota`, `map { p -> ... }`, `fold { acc, v -> ... }`, `zip`, `widen_f32`,
`widen_f64`, `println`, `print`, `time` and name bindings; expressions with
i32/f32/f64 arithmetic `+ - * / %`, unary minus, indexing `a[j]`, pair
projection `p.0`, tuples and array literals.

Semantics restated (file:line of crates/mapal-interp/src):
  * Map visits elements in order, captures read from the enclosing scope,
    a trap in any element ends the program (eval.rs:297-324);
  * Fold is a strict left fold from the seed (eval.rs:326-359);
  * Zip pairs equal-length arrays (eval.rs:371-385);
  * integer ops wrap; `/` and `%` truncate toward zero, divide-by-zero traps
    (kind 0), MIN / -1 wraps to MIN and MIN % -1 is 0; float ops are single
    IEEE operations, `%` is fmod (eval.rs:544-596);
  * Widen converts with round-to-nearest (eval.rs:238-248);
  * Index traps (kind 1) when the index is negative or not below the length
    (eval.rs:655-669);
  * `time` yields f64 milliseconds of a monotonic clock (eval.rs:433-446);
  * float literals take the float type they meet and default to f64; integer
    literals are i32 (crates/mapal-lower/src/typing.rs:160-320,
    emit.rs:1832-1866: an f32 literal is parsed directly as f32);
  * printing uses Rust's Display text (mapal-interp/src/value.rs:90-100).

Maps are evaluated vectorised over the elements with numpy (every f32 / i32
operation is still one correctly rounded or wrapping operation per element);
each element remembers the first trap it hit, and the lowest trapping element
is the one the interpreter stops at. The f32 sum fold goes through the C
restatement `or_fold_sum`; other folds loop in Python.
"""
from __future__ import annotations

import ctypes
import ctypes.util
import re
import time as _time

import numpy as np

from . import fold_sum, render_f32, render_f64

TIME_MARK = "\x00time\x00"

_libc = ctypes.CDLL(ctypes.util.find_library("c"))
_libc.strtof.restype = ctypes.c_float
_libc.strtof.argtypes = [ctypes.c_char_p, ctypes.c_void_p]


class Unsupported(Exception):
    """The program is outside the subset this evaluator restates."""


class Trap(Exception):
    def __init__(self, kind: int):
        super().__init__(kind)
        self.kind = kind


# ---- lexer / parser ---------------------------------------------------------------

_TOKEN = re.compile(r"""
    (?P<ws>\s+|//[^\n]*)
  | (?P<float>\d+\.\d+)
  | (?P<int>\d+)
  | (?P<ident>[A-Za-z_][A-Za-z_0-9]*)
  | (?P<str>"(?:[^"\\]|\\.)*")
  | (?P<arrow>->)
  | (?P<punct>[{}()\[\],;:.+\-*/%])
""", re.VERBOSE)


def _lex(src: str):
    out, pos = [], 0
    while pos < len(src):
        m = _TOKEN.match(src, pos)
        if not m:
            raise Unsupported(f"bad character {src[pos]!r}")
        pos = m.end()
        kind = m.lastgroup
        if kind == "ws":
            continue
        text = m.group(kind)
        if kind == "str":
            text = bytes(text[1:-1], "utf-8").decode("unicode_escape")
        out.append((kind, text))
    out.append(("eof", ""))
    return out


class _Parser:
    def __init__(self, src: str):
        self.t = _lex(src)
        self.p = 0

    def peek(self, k=0):
        return self.t[self.p + k]

    def at(self, text):
        return self.t[self.p][1] == text and self.t[self.p][0] in ("punct", "arrow", "ident")

    def take(self, text=None, kind=None):
        tok = self.t[self.p]
        if text is not None and tok[1] != text:
            raise Unsupported(f"expected {text!r}, found {tok[1]!r}")
        if kind is not None and tok[0] != kind:
            raise Unsupported(f"expected {kind}, found {tok[1]!r}")
        self.p += 1
        return tok

    def program(self):
        body = None
        while self.peek()[0] != "eof":
            self.take("fn")
            name = self.take(kind="ident")[1]
            if name != "main":
                raise Unsupported(f"fn {name}")
            self.take("(")
            self.take(")")
            self.take("{")
            stmts = []
            while not self.at("}"):
                stmts.append(self.chain())
                self.take(";")
            self.take("}")
            body = stmts
        if body is None:
            raise Unsupported("no fn main")
        return body

    def chain(self):
        head = self.expr()
        stages = []
        while self.at("->"):
            self.take("->")
            name = self.take(kind="ident")[1]
            if name in ("map", "fold"):
                stages.append((name, self.lam()))
            else:
                if self.at(":"):
                    self.take(":")
                    self.skip_type()
                stages.append(("name", name))
        return ("chain", head, stages)

    def skip_type(self):
        if self.at("[") or self.at("("):
            close = "]" if self.at("[") else ")"
            open_ = self.peek()[1]
            depth = 0
            while True:
                tok = self.take()
                depth += tok[1] == open_
                depth -= tok[1] == close
                if depth == 0:
                    break
        else:
            self.take(kind="ident")

    def lam(self):
        self.take("{")
        params = [self.take(kind="ident")[1]]
        while self.at(","):
            self.take(",")
            params.append(self.take(kind="ident")[1])
        self.take("->")
        stmts = [self.chain()]
        while self.at(";"):
            self.take(";")
            if self.at("}"):
                break
            stmts.append(self.chain())
        self.take("}")
        return (params, stmts)

    def expr(self):
        e = self.term()
        while self.at("+") or self.at("-"):
            op = self.take()[1]
            e = ("bin", op, e, self.term())
        return e

    def term(self):
        e = self.unary()
        while self.at("*") or self.at("/") or self.at("%"):
            op = self.take()[1]
            e = ("bin", op, e, self.unary())
        return e

    def unary(self):
        if self.at("-"):
            self.take()
            inner = self.unary()
            if inner[0] == "int":
                return ("int", -inner[1])
            if inner[0] == "float":
                return ("float", "-" + inner[1])
            return ("neg", inner)
        return self.postfix()

    def postfix(self):
        e = self.primary()
        while True:
            if self.at("["):
                self.take("[")
                e = ("index", e, self.expr())
                self.take("]")
            elif self.at(".") and self.peek(1)[0] == "int":
                self.take(".")
                e = ("proj", e, int(self.take()[1]))
            else:
                return e

    def primary(self):
        kind, text = self.peek()
        if kind == "int":
            self.p += 1
            return ("int", int(text))
        if kind == "float":
            self.p += 1
            return ("float", text)
        if kind == "str":
            self.p += 1
            return ("str", text)
        if kind == "ident":
            self.p += 1
            return ("name", text)
        if self.at("("):
            self.take("(")
            if self.at(")"):
                self.take(")")
                return ("unit",)
            items = [self.expr()]
            while self.at(","):
                self.take(",")
                items.append(self.expr())
            self.take(")")
            return items[0] if len(items) == 1 else ("tuple", items)
        if self.at("["):
            self.take("[")
            items = []
            while not self.at("]"):
                items.append(self.expr())
                if self.at(","):
                    self.take(",")
            self.take("]")
            return ("array", items)
        raise Unsupported(f"unexpected {text!r}")


# ---- values ----------------------------------------------------------------------------

class V:
    """A value. kind: i32, f32, f64, flit (an untyped float literal), str,
    unit, tuple, arr (elem i32/f32/f64, data ndarray), iota (n), zip.
    Scalars may hold an ndarray payload inside a vectorised map body."""
    __slots__ = ("kind", "val", "elem", "items", "taint")

    def __init__(self, kind, val=None, elem=None, items=None, taint=False):
        self.kind, self.val, self.elem, self.items, self.taint = kind, val, elem, items, taint


_NP = {"i32": np.int32, "f32": np.float32, "f64": np.float64}


def _f32_lit(text: str) -> np.float32:
    return np.float32(_libc.strtof(text.encode(), None))


def _resolve(v: V, want: str) -> V:
    """Give an untyped float literal its type."""
    if v.kind != "flit":
        return v
    if want == "f32":
        return V("f32", _f32_lit(v.val), taint=v.taint)
    return V("f64", float(v.val), taint=v.taint)


def _wrap(x):
    return (np.asarray(x, dtype=np.int64) & 0xFFFFFFFF).astype(np.uint32).view(np.int32)


class _Traps:
    """Per-element first trap of a vectorised site (or immediate for scalars)."""

    def __init__(self, n=None):
        self.kind = None if n is None else np.full(n, -1, dtype=np.int8)

    def hit(self, bad, kind):
        if self.kind is None:
            if np.any(bad):
                raise Trap(kind)
            return
        bad = np.broadcast_to(bad, self.kind.shape)
        self.kind[bad & (self.kind < 0)] = kind

    def raise_first(self):
        if self.kind is not None:
            hits = np.nonzero(self.kind >= 0)[0]
            if hits.size:
                raise Trap(int(self.kind[hits[0]]))


class Evaluator:
    def __init__(self):
        self.out: list[str] = []
        self.env: dict[str, V] = {}

    # -- arithmetic (eval.rs:544-596) --
    def binop(self, op, a: V, b: V, traps: _Traps) -> V:
        if a.kind == "flit" and b.kind == "flit":
            a, b = _resolve(a, "f64"), _resolve(b, "f64")
        a = _resolve(a, b.kind)
        b = _resolve(b, a.kind)
        if a.kind != b.kind or a.kind not in ("i32", "f32", "f64"):
            raise Unsupported(f"{a.kind} {op} {b.kind}")
        taint = a.taint or b.taint
        if a.kind == "i32":
            x = np.asarray(a.val, dtype=np.int64)
            y = np.asarray(b.val, dtype=np.int64)
            if op == "+":
                r = x + y
            elif op == "-":
                r = x - y
            elif op == "*":
                r = x * y
            else:
                zero = y == 0
                traps.hit(zero, 0)
                ys = np.where(zero, 1, y)
                q = np.abs(x) // np.abs(ys) * np.sign(x) * np.sign(ys)
                r = q if op == "/" else x - q * ys
            return V("i32", _wrap(r) if np.ndim(r) else np.int32(_wrap(r)[()]), taint=taint)
        t = _NP[a.kind]
        x = np.asarray(a.val, dtype=t)
        y = np.asarray(b.val, dtype=t)
        with np.errstate(all="ignore"):
            if op == "+":
                r = x + y
            elif op == "-":
                r = x - y
            elif op == "*":
                r = x * y
            elif op == "/":
                r = x / y
            else:
                r = np.fmod(x, y)
        return V(a.kind, r if np.ndim(r) else t(r), taint=taint)

    def index(self, a: V, j: V, traps: _Traps) -> V:
        if j.kind != "i32":
            raise Unsupported("index must be i32")
        jj = np.asarray(j.val, dtype=np.int64)
        if a.kind == "iota":
            bad = (jj < 0) | (jj >= a.val)
            traps.hit(bad, 1)
            return V("i32", j.val)
        if a.kind != "arr":
            raise Unsupported("indexing a non-array")
        n = a.val.shape[0]
        bad = (jj < 0) | (jj >= n)
        traps.hit(bad, 1)
        safe = np.where(bad, 0, jj) if n else np.zeros_like(jj)
        if n == 0:
            return V(a.elem, np.zeros(np.shape(jj), dtype=_NP[a.elem]))
        r = a.val[safe]
        return V(a.elem, r if np.ndim(r) else _NP[a.elem](r))

    # -- expressions --
    def eval(self, e, scope: dict, traps: _Traps) -> V:
        k = e[0]
        if k == "int":
            if not -2**31 <= e[1] < 2**31:
                raise Unsupported("integer literal beyond i32")
            return V("i32", np.int32(e[1]))
        if k == "float":
            return V("flit", e[1])
        if k == "str":
            return V("str", e[1])
        if k == "unit":
            return V("unit")
        if k == "name":
            if scope and e[1] in scope:
                return scope[e[1]]
            if e[1] in self.env:
                return self.env[e[1]]
            raise Unsupported(f"unknown name {e[1]}")
        if k == "tuple":
            items = [self.eval(x, scope, traps) for x in e[1]]
            return V("tuple", items=items)
        if k == "array":
            items = [self.eval(x, scope, traps) for x in e[1]]
            kinds = {i.kind for i in items}
            if kinds <= {"i32"}:
                return V("arr", np.array([i.val for i in items], dtype=np.int32), elem="i32")
            if kinds <= {"f32", "flit"}:
                vals = [_resolve(i, "f32").val for i in items]
                return V("arr", np.array(vals, dtype=np.float32), elem="f32")
            raise Unsupported("array literal element types")
        if k == "neg":
            a = self.eval(e[1], scope, traps)
            if a.kind == "flit":
                return V("flit", "-" + a.val)
            if a.kind == "i32":
                return V("i32", _wrap(-np.asarray(a.val, dtype=np.int64)) if np.ndim(a.val)
                         else np.int32(_wrap(-np.int64(a.val))[()]), taint=a.taint)
            if a.kind in ("f32", "f64"):
                return V(a.kind, -a.val, taint=a.taint)
            raise Unsupported("negation")
        if k == "bin":
            a = self.eval(e[2], scope, traps)
            b = self.eval(e[3], scope, traps)
            return self.binop(e[1], a, b, traps)
        if k == "index":
            a = self.eval(e[1], scope, traps)
            j = self.eval(e[2], scope, traps)
            return self.index(a, j, traps)
        if k == "proj":
            a = self.eval(e[1], scope, traps)
            if a.kind != "tuple" or e[2] >= len(a.items):
                raise Unsupported("projection")
            return a.items[e[2]]
        raise Unsupported(k)

    # -- chains --
    def chain(self, c, scope: dict, traps: _Traps) -> V:
        _, head, stages = c
        v = self.eval(head, scope, traps)
        for st in stages:
            v = self.stage(st, v, scope, traps)
        return v

    def stage(self, st, v: V, scope: dict, traps: _Traps) -> V:
        kind, arg = st
        if kind == "map":
            return self.map(arg, v, scope)
        if kind == "fold":
            return self.fold(arg, v, scope, traps)
        name = arg
        if name == "iota":
            if v.kind != "i32" or np.ndim(v.val) or int(v.val) < 0:
                raise Unsupported("iota of a non-count")
            return V("iota", int(v.val))
        if name == "zip":
            if v.kind != "tuple" or len(v.items) != 2:
                raise Unsupported("zip of a non-pair")
            lens = [self._len(x) for x in v.items]
            if lens[0] != lens[1]:
                raise Unsupported("zip of different lengths")
            return V("zip", items=v.items)
        if name == "enumerate":
            if v.kind not in ("arr", "iota"):
                raise Unsupported("enumerate of a non-array")
            return V("zip", items=[V("iota", self._len(v)), v])
        if name == "widen_f32":
            if v.kind != "i32":
                raise Unsupported("widen_f32 of non-i32")
            r = np.asarray(v.val).astype(np.float32)
            return V("f32", r if np.ndim(r) else np.float32(r), taint=v.taint)
        if name == "widen_f64":
            v = _resolve(v, "f64")
            if v.kind not in ("i32", "f32"):
                raise Unsupported("widen_f64")
            r = np.asarray(v.val).astype(np.float64)
            return V("f64", r if np.ndim(r) else float(r), taint=v.taint)
        if name in ("println", "print"):
            self.print(_resolve(v, "f64"), name == "println")
            return V("unit")
        if name == "time":
            return V("f64", _time.monotonic() * 1000.0, taint=True)
        if scope is not None and scope.get("__local__"):
            scope[name] = v
        else:
            self.env[name] = v
        return v

    def _len(self, v: V) -> int:
        if v.kind == "iota":
            return v.val
        if v.kind == "arr":
            return v.val.shape[0]
        raise Unsupported("not an array")

    def _elements(self, v: V) -> tuple[V, int]:
        if v.kind == "iota":
            return V("i32", np.arange(v.val, dtype=np.int32)), v.val
        if v.kind == "arr":
            return V(v.elem, v.val), v.val.shape[0]
        if v.kind == "zip":
            parts = [self._elements(x)[0] for x in v.items]
            return V("tuple", items=parts), self._len(v.items[0])
        raise Unsupported("map over a non-array")

    def map(self, lam, dom: V, scope) -> V:
        params, stmts = lam
        if len(params) != 1:
            raise Unsupported("map takes one parameter")
        elem, n = self._elements(dom)
        traps = _Traps(n)
        local = dict(scope or {})
        local["__local__"] = True
        local[params[0]] = elem
        r = None
        for c in stmts:
            r = self.chain(c, local, traps)
        traps.raise_first()
        r = _resolve(r, "f64")
        if r.kind not in _NP:
            raise Unsupported("map body result")
        data = np.broadcast_to(np.asarray(r.val, dtype=_NP[r.kind]), (n,)).copy()
        return V("arr", data, elem=r.kind)

    def fold(self, lam, v: V, scope, traps: _Traps) -> V:
        params, stmts = lam
        if v.kind != "tuple" or len(v.items) != 2 or len(params) != 2:
            raise Unsupported("fold takes (seed, array) and two parameters")
        seed, xs = v.items
        if xs.kind == "arr":
            seed = _resolve(seed, xs.elem)
        elif seed.kind == "flit":
            seed = _resolve(seed, "f32" if self._body_is_f32(stmts, scope) else "f64")
        n = self._len(xs)
        acc_name, x_name = params
        # the f32 sum fold at top level: the C restatement
        if (traps.kind is None and xs.kind == "arr" and xs.elem == "f32" and seed.kind == "f32"
                and len(stmts) == 1 and not stmts[0][2] and stmts[0][1] == ("bin", "+", ("name", acc_name),
                                                                              ("name", x_name))):
            return V("f32", np.float32(fold_sum(float(seed.val), xs.val)))
        if traps.kind is None and n > 200_000:
            raise Unsupported("general top-level fold beyond the evaluator's size bound")
        acc = seed
        for k in range(n):
            x = V("i32", np.int32(k)) if xs.kind == "iota" else V(xs.elem, xs.val[k])
            local = dict(scope or {})
            local["__local__"] = True
            local[acc_name] = acc
            local[x_name] = x
            r = None
            for c in stmts:
                r = self.chain(c, local, traps)
            acc = _resolve(r, acc.kind)
        return acc

    def _body_is_f32(self, stmts, scope) -> bool:
        # a fold over an index range inside a map: its seed's type is the
        # body's, which for the subset is the type of the arrays it reads
        def arrays(e):
            if isinstance(e, tuple):
                if e and e[0] == "index" and e[1][0] == "name":
                    v = (scope or {}).get(e[1][1]) or self.env.get(e[1][1])
                    if v is not None and v.kind == "arr":
                        yield v.elem
                for x in e[1:]:
                    yield from arrays(x)
            elif isinstance(e, list):
                for x in e:
                    yield from arrays(x)
        kinds = set(arrays(stmts))
        return kinds == {"f32"}

    def print(self, v: V, newline: bool):
        if v.kind == "str":
            text = v.val
        elif v.taint:
            text = TIME_MARK
        elif v.kind == "i32":
            text = str(int(v.val))
        elif v.kind == "f32":
            text = render_f32(float(v.val))
        elif v.kind == "f64":
            text = render_f64(float(v.val))
        else:
            raise Unsupported(f"printing {v.kind}")
        self.out.append(text + ("\n" if newline else ""))

    def run(self, body):
        for c in body:
            self.chain(c, None, _Traps())


def expected(src: str) -> tuple[str, int]:
    """(stdout, exit code) the interpreter gives for `src`: 0, or 101 after a trap.
    Printed values computed from `time` appear as TIME_MARK."""
    body = _Parser(src).program()
    ev = Evaluator()
    try:
        ev.run(body)
    except Trap:
        return "".join(ev.out), 101
    return "".join(ev.out), 0


def matches(actual: str, want: str) -> bool:
    """Compare stdout with an expected text whose TIME_MARKs stand for any number."""
    pattern = "".join(re.escape(p) if p != TIME_MARK else r"-?[0-9.e+-]+(?:inf|NaN)?"
                      for p in re.split(f"({re.escape(TIME_MARK)})", want))
    return re.fullmatch(pattern, actual, flags=re.S) is not None
