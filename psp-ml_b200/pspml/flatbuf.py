"""Minimal FlatBuffers reader and writer (the binary format of .tflite files).

The reference parses TFLite models with the generated Rust accessors of the
`flatbuffers` crate (cargo-psp-ml/src/parse/tflite/schema_generated.rs); this
module restates the wire format those accessors read, for the handful of
tables the int8 inference path needs:

* a buffer starts with a u32 offset to the root table (an optional 4-byte
  file identifier follows it);
* a table starts with an i32 that, subtracted from the table's position,
  gives its vtable: u16 vtable bytes, u16 table bytes, then one u16 field
  offset per slot (0: field absent, use the default);
* scalars sit inline in the table; strings, vectors and sub-tables are u32
  offsets relative to the field's own position; a vector is a u32 length
  followed by its elements (tables and strings as u32 offsets again);
* a union field takes two slots, the type (u8) and the value (offset).

The writer lays the tree out front to back: a table is written, then the
objects it refers to, and each offset is patched once its target exists (all
offsets point forward, as unsigned offsets must).  Scalars and vector
elements are aligned to their size, vector bytes to `align` where asked.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field


# ------------------------------------------------------------------ reader
class Table:
    """Read access to one table of a FlatBuffers buffer."""

    __slots__ = ("buf", "pos", "vt", "vt_len")

    def __init__(self, buf: bytes, pos: int):
        self.buf = buf
        self.pos = pos
        self.vt = pos - struct.unpack_from("<i", buf, pos)[0]
        self.vt_len = struct.unpack_from("<H", buf, self.vt)[0]

    def _field(self, slot: int) -> int:
        o = 4 + 2 * slot
        if o >= self.vt_len:
            return 0
        return struct.unpack_from("<H", self.buf, self.vt + o)[0]

    def has(self, slot: int) -> bool:
        return self._field(slot) != 0

    def scalar(self, slot: int, fmt: str, default=0):
        off = self._field(slot)
        if off == 0:
            return default
        return struct.unpack_from("<" + fmt, self.buf, self.pos + off)[0]

    def _target(self, slot: int) -> int | None:
        off = self._field(slot)
        if off == 0:
            return None
        p = self.pos + off
        return p + struct.unpack_from("<I", self.buf, p)[0]

    def table(self, slot: int) -> Table | None:
        t = self._target(slot)
        return None if t is None else Table(self.buf, t)

    def string(self, slot: int) -> str | None:
        t = self._target(slot)
        if t is None:
            return None
        n = struct.unpack_from("<I", self.buf, t)[0]
        return bytes(self.buf[t + 4:t + 4 + n]).decode("utf-8", "replace")

    def vector(self, slot: int, fmt: str) -> list:
        """Vector of scalars (struct format character)."""
        t = self._target(slot)
        if t is None:
            return []
        n = struct.unpack_from("<I", self.buf, t)[0]
        return list(struct.unpack_from(f"<{n}{fmt}", self.buf, t + 4))

    def vector_bytes(self, slot: int) -> tuple[int, int] | None:
        """(absolute offset, length) of a [ubyte] vector's bytes."""
        t = self._target(slot)
        if t is None:
            return None
        n = struct.unpack_from("<I", self.buf, t)[0]
        return t + 4, n

    def tables(self, slot: int) -> list[Table]:
        t = self._target(slot)
        if t is None:
            return []
        n = struct.unpack_from("<I", self.buf, t)[0]
        out = []
        for i in range(n):
            p = t + 4 + 4 * i
            out.append(Table(self.buf, p + struct.unpack_from("<I", self.buf, p)[0]))
        return out


def root(buf: bytes) -> Table:
    return Table(buf, struct.unpack_from("<I", buf, 0)[0])


def file_identifier(buf: bytes) -> bytes:
    return bytes(buf[4:8])


# ------------------------------------------------------------------ writer
@dataclass
class Vec:
    """Vector: scalars with a struct format character, or tables/strings."""
    fmt: str                     # struct character, or "table" / "string"
    items: list
    align: int = 0               # extra alignment of the element bytes


@dataclass
class Str:
    text: str


@dataclass
class Obj:
    """Table: slot -> (struct format character, value) for scalars, or
    slot -> Obj / Vec / Str for offsets."""
    fields: dict = field(default_factory=dict)

    def scalar(self, slot: int, fmt: str, value) -> "Obj":
        self.fields[slot] = (fmt, value)
        return self

    def ref(self, slot: int, value) -> "Obj":
        self.fields[slot] = value
        return self


class _Writer:
    def __init__(self):
        self.buf = bytearray()
        self.todo: list[tuple[int, object]] = []  # (u32 field position, target)

    def align(self, n: int, extra_after: int = 0):
        # Pad so that position + extra_after is a multiple of n.
        while (len(self.buf) + extra_after) % n:
            self.buf.append(0)

    def put(self, fmt: str, value):
        self.buf += struct.pack("<" + fmt, value)

    def ref_slot(self, target) -> None:
        self.todo.append((len(self.buf), target))
        self.put("I", 0)

    def table(self, obj: Obj) -> int:
        slots = max(obj.fields) + 1 if obj.fields else 0
        # Table layout: soffset, then fields sorted by size (largest first)
        # so that each is aligned to its size relative to the table start.
        entries = []
        for slot, v in obj.fields.items():
            size = struct.calcsize("<" + v[0]) if isinstance(v, tuple) else 4
            entries.append((size, slot, v))
        entries.sort(key=lambda e: (-e[0], e[1]))
        layout = []
        off = 4
        for size, slot, v in entries:
            while off % size:
                off += 1
            layout.append((off, slot, v, size))
            off += size
        table_size = off
        # vtable right before the table
        vt = [0] * slots
        for o, slot, _, _ in layout:
            vt[slot] = o
        self.align(2)
        vt_bytes = struct.pack(f"<HH{slots}H", 4 + 2 * slots, table_size, *vt)
        # the table must start 8-aligned (for 8-byte scalars)
        pad = (-(len(self.buf) + len(vt_bytes))) % 8
        self.buf += b"\0" * pad
        vt_pos = len(self.buf)
        self.buf += vt_bytes
        t_pos = len(self.buf)
        body = bytearray(table_size)
        struct.pack_into("<i", body, 0, t_pos - vt_pos)
        self.buf += body
        for o, slot, v, size in layout:
            if isinstance(v, tuple):
                struct.pack_into("<" + v[0], self.buf, t_pos + o, v[1])
            else:
                self.todo.append((t_pos + o, v))
        return t_pos

    def vector(self, v: Vec) -> int:
        if v.fmt in ("table", "string"):
            self.align(4)
            pos = len(self.buf)
            self.put("I", len(v.items))
            for it in v.items:
                self.ref_slot(it if v.fmt == "table" else Str(it) if isinstance(it, str) else it)
            return pos
        esize = struct.calcsize("<" + v.fmt)
        self.align(max(4, esize, v.align), extra_after=4)
        pos = len(self.buf)
        self.put("I", len(v.items))
        if v.fmt == "B" and isinstance(v.items, (bytes, bytearray, memoryview)):
            self.buf += bytes(v.items)
        else:
            self.buf += struct.pack(f"<{len(v.items)}{v.fmt}", *v.items)
        return pos

    def string(self, s: Str) -> int:
        self.align(4)
        pos = len(self.buf)
        b = s.text.encode("utf-8")
        self.put("I", len(b))
        self.buf += b + b"\0"
        return pos

    def emit(self, target) -> int:
        if isinstance(target, Obj):
            return self.table(target)
        if isinstance(target, Vec):
            return self.vector(target)
        if isinstance(target, Str):
            return self.string(target)
        raise TypeError(f"cannot serialise {type(target)}")


def build(root_obj: Obj, identifier: bytes = b"") -> bytes:
    """Serialises a table tree; the result starts with the root offset (and
    the 4-byte identifier, if given)."""
    w = _Writer()
    w.put("I", 0)
    if identifier:
        assert len(identifier) == 4
        w.buf += identifier
    rpos = w.table(root_obj)
    struct.pack_into("<I", w.buf, 0, rpos)
    i = 0
    while i < len(w.todo):
        fpos, target = w.todo[i]
        tpos = w.emit(target)
        struct.pack_into("<I", w.buf, fpos, tpos - fpos)
        i += 1
    w.align(16)
    return bytes(w.buf)
