"""A small PTX text builder shared by every sm_100a template.

Virtual registers are handed out per class and declared once at the top of the
entry (``ptxas`` does the real allocation), the same division of labour the
reference's ``Emitter`` uses (``compiler/emitter.py:42-84``).  Templates here are
hand-written PTX with Python doing the bookkeeping: unrolling, register naming,
predicated tails and the launch descriptor comment.
"""

from __future__ import annotations

import json
import struct
from collections import Counter

PTX_VERSION = "8.8"      # tcgen05 needs >= 8.6, three-input max 8.8; ptxas 12.9 accepts 8.6-8.8
TARGET = "sm_100a"

HEADER = f".version {PTX_VERSION}\n.target {TARGET}\n.address_size 64\n"

# register class -> (declared type, name prefix)
_CLASSES = {
    "pred": (".pred", "%p"),
    "b16": (".b16", "%h"),
    "b32": (".b32", "%r"),
    "b64": (".b64", "%rd"),
    "f32": (".f32", "%f"),
    "f64": (".f64", "%fd"),
}
_ALIAS = {"u32": "b32", "s32": "b32", "u64": "b64", "s64": "b64", "f16": "b16", "bf16": "b16",
          "u16": "b16", "s16": "b16"}


def f32_hex(v: float) -> str:
    """Exact single-precision immediate (``0fXXXXXXXX``)."""
    return "0f%08X" % struct.unpack("<I", struct.pack("<f", float(v)))[0]


def f64_hex(v: float) -> str:
    return "0d%016X" % struct.unpack("<Q", struct.pack("<d", float(v)))[0]


class Ptx:
    """Accumulates the body of one ``.entry`` and its register declarations."""

    def __init__(self):
        self.lines: list[str] = []
        self.count: Counter = Counter()
        self.named: dict[str, str] = {}   # explicitly named registers -> class
        self._labels: Counter = Counter()

    # -- registers ---------------------------------------------------------
    def reg(self, kind: str) -> str:
        cls = _ALIAS.get(kind, kind)
        _, prefix = _CLASSES[cls]
        n = self.count[cls]
        self.count[cls] += 1
        return f"{prefix}{n}"

    def regs(self, kind: str, n: int) -> list[str]:
        return [self.reg(kind) for _ in range(n)]

    def named_reg(self, name: str, kind: str) -> str:
        """A readable register name (``%tid``); declared once."""
        cls = _ALIAS.get(kind, kind)
        prev = self.named.get(name)
        if prev is not None and prev != cls:
            raise ValueError(f"register {name} redeclared as {cls} (was {prev})")
        self.named[name] = cls
        return name

    # -- text --------------------------------------------------------------
    def emit(self, text: str) -> None:
        for line in text.strip("\n").split("\n"):
            line = line.rstrip()
            if not line:
                continue
            if line.lstrip().startswith(("//", "{", "}")) or line.endswith(":"):
                self.lines.append("\t" + line.strip() if not line.endswith(":") else line.strip())
            else:
                s = line.strip()
                self.lines.append("\t" + s + ("" if s.endswith(";") else ";"))

    def comment(self, text: str) -> None:
        self.lines.append("\t// " + text)

    def label(self, stem: str) -> str:
        self._labels[stem] += 1
        return f"$L_{stem}_{self._labels[stem]}"

    def place(self, label: str) -> None:
        self.lines.append(f"{label}:")

    # -- assembly ----------------------------------------------------------
    def declarations(self) -> list[str]:
        out = []
        for cls, n in self.count.items():
            if n:
                typ, prefix = _CLASSES[cls]
                out.append(f"\t.reg {typ} \t{prefix}<{n}>;")
        for name, cls in sorted(self.named.items()):
            out.append(f"\t.reg {_CLASSES[cls][0]} \t{name};")
        return out


def module(entries: list[str], launch: dict | None = None, globals_: list[str] | None = None) -> str:
    """Assemble a module: header, launch descriptor comment, module globals, entries."""
    parts = [HEADER]
    if launch is not None:
        parts.append("// @launch " + json.dumps(launch, sort_keys=True))
    parts.extend(globals_ or [])
    parts.extend(entries)
    text = "\n".join(parts) + "\n"
    text.encode("ascii")   # PTX rejects non-ASCII anywhere
    return text


def entry(name: str, params: list[str], body: Ptx, maxntid: int | None = None,
          extra_directives: str = "") -> str:
    sig = ",\n".join("\t" + p for p in params)
    bounds = f"\n.maxntid {maxntid}, 1, 1" if maxntid else ""
    return (f".visible .entry {name}(\n{sig}\n){bounds}{extra_directives}\n{{\n"
            + "\n".join(body.declarations()) + "\n\n" + "\n".join(body.lines) + "\n}\n")


def parse_launch(ptx: str) -> dict:
    """Read the ``// @launch {...}`` descriptor back out of a module."""
    for line in ptx.splitlines():
        if line.startswith("// @launch "):
            return json.loads(line[len("// @launch "):])
    raise ValueError("module has no // @launch descriptor")
