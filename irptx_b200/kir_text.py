"""KIR text as data: read a KIR file into its header and body tree, and write it back.

The wire format is the reference's (fe/kirdump.py:90-103, src/kir.c:553-628): the header lines
``kir 1``, ``kernel``, ``launch``, ``arg``, ``zero``, then ``body`` and one S-expression, then
``end``. In the S-expression a node is ``(Kind field=value ...)``, a list is ``[v ...]``, a
string is ``"..."``, and anything else (numbers, hex floats, ``dt:f32``, ``op:relu``, ``none``,
``false``) is an atom kept as written, so that ``write(read(text))`` returns the text as the
reference's writer emits it.

This is host-side plumbing for rewriting graphs (kernel fusion in ``irptx_b200.fuse``); the
selector in the C core remains the one reader that decides what a graph means.
"""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class Node:
    kind: str
    fields: list = field(default_factory=list)     # [(name, value)], in written order

    def get(self, name, default=None):
        for n, v in self.fields:
            if n == name:
                return v
        return default

    def set(self, name, value):
        for i, (n, _) in enumerate(self.fields):
            if n == name:
                self.fields[i] = (n, value)
                return
        self.fields.append((name, value))


@dataclass(frozen=True)
class Str:
    text: str


@dataclass(frozen=True)
class Atom:
    text: str


@dataclass
class Arg:
    name: str
    kind: str          # in / const / out
    dtype: str
    dims: list


@dataclass
class Kir:
    kernel: str
    launch: list       # gx gy gz bx by bz smem
    args: list         # [Arg], in arg order
    zero: list         # output names
    body: object       # the S-expression value (normally a list holding one Tile node)


class KirSyntaxError(ValueError):
    pass


def _parse_value(s: str, i: int):
    n = len(s)
    while i < n and s[i].isspace():
        i += 1
    if i >= n:
        raise KirSyntaxError("unexpected end of the body")
    c = s[i]
    if c == "(":
        j = i + 1
        k = j
        while k < n and not s[k].isspace() and s[k] not in ")":
            k += 1
        node = Node(s[j:k])
        i = k
        while True:
            while i < n and s[i].isspace():
                i += 1
            if i < n and s[i] == ")":
                return node, i + 1
            eq = s.find("=", i)
            if eq < 0:
                raise KirSyntaxError(f"a field without '=' at offset {i}")
            name = s[i:eq].strip()
            val, i = _parse_value(s, eq + 1)
            node.fields.append((name, val))
    if c == "[":
        items = []
        i += 1
        while True:
            while i < n and s[i].isspace():
                i += 1
            if i < n and s[i] == "]":
                return items, i + 1
            v, i = _parse_value(s, i)
            items.append(v)
    if c == '"':
        j = s.index('"', i + 1)
        return Str(s[i + 1:j]), j + 1
    j = i
    while j < n and not s[j].isspace() and s[j] not in ")]":
        j += 1
    return Atom(s[i:j]), j


def write_value(v) -> str:
    if isinstance(v, Node):
        return "(" + " ".join([v.kind] + [f"{k}={write_value(x)}" for k, x in v.fields]) + ")"
    if isinstance(v, list):
        return "[" + " ".join(write_value(x) for x in v) + "]"
    if isinstance(v, Str):
        return f'"{v.text}"'
    if isinstance(v, Atom):
        return v.text
    raise TypeError(f"not a KIR value: {v!r}")


def read(text: str) -> Kir:
    lines = text.splitlines()
    kernel, launch, args, zero, body = None, None, [], [], None
    i = 0
    while i < len(lines):
        ln = lines[i].strip()
        i += 1
        if not ln or ln == "kir 1":
            continue
        w = ln.split()
        if w[0] == "kernel":
            kernel = w[1]
        elif w[0] == "launch":
            launch = [int(x) for x in w[1:]]
        elif w[0] == "arg":
            rank = int(w[5])
            args.append(Arg(w[2], w[3], w[4], [int(x) for x in w[6:6 + rank]]))
        elif w[0] == "zero":
            zero.append(w[1])
        elif w[0] == "body":
            end = next(j for j in range(i, len(lines)) if lines[j].strip() == "end")
            src = "\n".join(lines[i:end])
            body, k = _parse_value(src, 0)
            if src[k:].strip():
                raise KirSyntaxError("text after the body's S-expression")
            i = end + 1
        elif w[0] == "end":
            break
        else:
            raise KirSyntaxError(f"unknown header line {ln!r}")
    if kernel is None or launch is None or body is None:
        raise KirSyntaxError("a KIR file without kernel, launch or body")
    return Kir(kernel, launch, args, zero, body)


def write(k: Kir) -> str:
    out = ["kir 1", f"kernel {k.kernel}", "launch " + " ".join(map(str, k.launch))]
    for i, a in enumerate(k.args):
        out.append(f"arg {i} {a.name} {a.kind} {a.dtype} {len(a.dims)} " + " ".join(map(str, a.dims)))
    out += [f"zero {z}" for z in k.zero]
    out += ["body", write_value(k.body), "end", ""]
    return "\n".join(line.rstrip() for line in out)
