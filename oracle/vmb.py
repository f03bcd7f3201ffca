"""vmb.py -- TEST INFRASTRUCTURE ONLY.

A pure-Python restatement of how the reference VM reads a .vmb program's
constant pool and slot table, used by tests/ to check the library's device
constant pool (vmlm_pool_*). Nothing in the product library imports it.

  parse          Vm::load_impl (core/src/interp.rs:123-220): header fields,
                 META header, constant table; bind_slots (:351-397): each slot's
                 region, byte offset, shape and dtype; dtype_size and hash32 of
                 core/src/format.rs (:73-95, :203-213)
  layerb         the OP_LAYERB base update (core/src/interp.rs:1019-1045)
  const_offset   const_ptr / const_ptr_based (:438-479): the layer base on a
                 CONSTANT slot and its bound
  audit          audit_const_dtypes (:241-345): the load-time check that a
                 non-f32 constant is read only as a GEMM B operand (or as a
                 bf16 EMB table with an f32 destination)
"""
import struct

MAGIC = 0x4D4C4D56
SLOT_CONST, SLOT_ACT, SLOT_STATE, SLOT_GRAD, SLOT_PARAM = range(5)
DTYPE_SIZE = {0: 4, 1: 2, 2: 1, 3: 4, 4: 2}  # f32, f16, i8, i32, bf16


class VmExit(Exception):
    """The VM printed `msg` and exited with `code`."""

    def __init__(self, code, msg):
        super().__init__(f"exit {code}: {msg}")
        self.code, self.msg = code, msg


def hash32(name: str) -> int:
    h = 0x811C9DC5
    for c in name.encode():
        h = ((h ^ c) * 0x01000193) & 0xFFFFFFFF
    return h


def parse(image: bytes):
    """-> dict(header, consts, slots) as the VM binds them. consts: (off, len, rows,
    cols, dtype, hash); slots: (kind, region, byte offset, rows, cols, dtype, name hash),
    region 0 = constant pool, 1 = activations, 2 = state, 3 = gradients."""
    u32 = lambda off: struct.unpack_from("<I", image, off)[0]  # noqa: E731
    if u32(0) != MAGIC:
        raise VmExit(3, "bad magic")
    hdr = dict(text_off=u32(8), text_len=u32(12), const_off=u32(16), const_len=u32(20), meta_off=u32(24))
    mo = hdr["meta_off"]
    n_const, n_slot, slots_off, act, state, grad, names_off = struct.unpack_from("<7I", image, mo)
    hdr.update(act_bytes=act, state_bytes=state, grad_bytes=grad)
    consts = []
    for i in range(n_const):
        e = mo + 28 + 24 * i
        off, ln, rows, cols = struct.unpack_from("<4I", image, e)
        consts.append((off, ln, rows, cols, image[e + 16], u32(e + 20)))
    slots = []
    for i in range(n_slot):
        kind, idx, rows, cols = struct.unpack_from("<4I", image, mo + slots_off + 16 * i)
        name = u32(mo + names_off + 4 * i)
        if kind in (SLOT_CONST, SLOT_PARAM):
            c = consts[idx]
            if DTYPE_SIZE.get(c[4], 0) == 0:
                raise VmExit(9, "const has unknown dtype")
            slots.append((kind, 0, c[0], rows, cols, c[4], name))
        else:
            region = {SLOT_STATE: 2, SLOT_GRAD: 3}.get(kind, 1)
            slots.append((kind, region, idx, rows, cols, 0, name))
    return dict(header=hdr, consts=consts, slots=slots)


def _to_usize(x: float) -> int:
    if x != x or x <= 0:
        return 0
    if x >= 2.0**64:
        return 2**64 - 1
    return int(x)


def layerb(base: int, delta: float) -> int:
    if delta >= 0:
        return min(base + _to_usize(delta), 2**64 - 1)
    return max(base - _to_usize(-delta), 0)


def const_offset(parsed, slot: int, base: int) -> int:
    """Byte offset of a slot's data inside its region with the layer base applied."""
    kind, region, off, rows, cols, dt, _ = parsed["slots"][slot]
    if kind != SLOT_CONST or base == 0:
        return off
    if off + base + rows * cols * DTYPE_SIZE[dt] > parsed["header"]["const_len"]:
        raise VmExit(9, "layer base walks past the constant pool")
    return off + base


# opcodes (trans/src/opcode.rs:6-94) and dtypes (core/src/format.rs:73-79) the audit names
OP_SLICE, OP_GEMM, OP_EMB, OP_SHAPE, OP_WRITECOL, OP_PUSH, OP_POP, OP_LOOP_CNT = 6, 10, 14, 52, 71, 86, 87, 89
DT_F32, DT_I8, DT_BF16 = 0, 2, 4


def audit(image: bytes, parsed) -> None:
    """audit_const_dtypes (core/src/interp.rs:241-345) over the TEXT section:
    raises VmExit(9, message) where the VM prints and exits 9. Slot numbers
    past the table count as f32 (the VM's probe skips them)."""
    hdr, slots = parsed["header"], parsed["slots"]

    def dtype(s):
        return slots[s][5] if s < len(slots) else DT_F32

    for i in range(hdr["text_len"] // 16):
        op, _fl, _dt, dst, a, b = struct.unpack_from("<BBHIII", image, hdr["text_off"] + 16 * i)
        if op == OP_GEMM:
            if dtype(b) in (DT_BF16, DT_I8, DT_F32):
                continue
            raise VmExit(9, "gemm B has no kernel for this dtype")
        if op == OP_EMB:
            if dtype(a) != DT_BF16:
                continue
            if dtype(dst) == DT_F32:
                continue
        if op == OP_SHAPE:
            checks = (False, False, False)
        elif op == OP_LOOP_CNT:
            checks = (False, True, False)
        else:
            checks = (True, True, op not in (OP_SLICE, OP_WRITECOL, OP_PUSH, OP_POP))
        for field, check in zip((dst, a, b), checks):
            if not check or field >= len(slots):
                continue
            dt = slots[field][5]
            if dt == DT_F32:
                continue
            what = {DT_BF16: "bf16", DT_I8: "i8"}.get(dt, "non-f32")
            raise VmExit(9, f"op {op} uses {what} const at slot {field} (only a GEMM may read a non-f32 operand)")
