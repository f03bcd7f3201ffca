"""Build small .vmb program images for the device constant-pool tests.

The layout is the one core/src/format.rs defines and Vm::load reads
(core/src/interp.rs:123-220): a 28-byte header (magic, version, text offset and
length, const offset and length, meta offset), TEXT (16-byte instructions:
op u8, fl u8, dt u16, dst, a, b), CONST (each constant 64-byte aligned), and
META (7-word header, 24-byte constant entries: off, len, rows, cols, dtype byte,
name hash; 16-byte slot entries: kind, index or byte offset, rows, cols; a slot
name-hash table).
"""
import struct

import numpy as np

from oracle.vmb import MAGIC, hash32

OP_GEMM = 10


def ins(op, fl=0, dt=0, dst=0, a=0, b=0) -> bytes:
    return struct.pack("<BBHIII", op, fl, dt, dst, a, b)


def build(consts, slots, text=b"", act_bytes=0, state_bytes=0, grad_bytes=0, version=1):
    """consts: list of (name, array, dtype code) with the array's raw bytes stored as is;
    slots: list of (name, kind, const index or region byte offset, rows, cols)."""
    pool = b""
    table = []
    for name, arr, dt in consts:
        raw = np.ascontiguousarray(arr).tobytes()
        pool += b"\0" * (-len(pool) % 64)
        rows, cols = (arr.shape + (1,))[:2] if arr.ndim else (1, 1)
        table.append((len(pool), len(raw), rows, cols, dt, hash32(name)))
        pool += raw
    text_off = 32
    const_off = text_off + len(text)
    const_off += -const_off % 64
    meta_off = const_off + len(pool)
    meta_off += -meta_off % 4
    slots_off = 28 + 24 * len(table)
    names_off = slots_off + 16 * len(slots)
    meta = struct.pack("<7I", len(table), len(slots), slots_off, act_bytes, state_bytes, grad_bytes, names_off)
    for off, ln, rows, cols, dt, h in table:
        meta += struct.pack("<4I", off, ln, rows, cols) + struct.pack("<B3xI", dt, h)
    for _, kind, idx, rows, cols in slots:
        meta += struct.pack("<4I", kind, idx, rows, cols)
    for name, *_ in slots:
        meta += struct.pack("<I", hash32(name))
    head = struct.pack("<IHHIIIII", MAGIC, version, 0, text_off, len(text), const_off, len(pool), meta_off)
    img = bytearray(head + b"\0" * (text_off - len(head)) + text)
    img += b"\0" * (const_off - len(img))
    img += pool
    img += b"\0" * (meta_off - len(img))
    img += meta
    return bytes(img)
