"""The device constant pool of a .vmb program (vmlm_pool_*): Vm::load and
bind_slots (core/src/interp.rs:123-220, :351-397), the OP_LAYERB base
(:438-479, :1019-1045) and the OP_GEMM arm run on the pool's slots.

CPU tests pin the loader restatement (oracle/vmb.py) on the reference's own
program image (tests/golden/e2e_tiny: its constants against their .bin files,
their names against the .args manifest) and check the load errors the library
reports before any device work. GPU tests load images into device memory and
compare every slot's address and contents with the restatement, run the
fixture's OP_GEMM and synthetic OP_GEMMs of each B dtype against the oracle,
and walk the layer base.
"""
import os
import struct

import numpy as np
import pytest

import sparrow_b200.kernels as K
from conftest import GOLDEN
from oracle import vmb
from sparrow_b200._lib import VmlmError
from vmb_image import OP_GEMM, build, ins

ARG, SHAPE, OPERATOR = 1, 2, 8
TINY = os.path.join(GOLDEN, "e2e_tiny")


def _tiny():
    with open(os.path.join(TINY, "e2e_tiny.vmb"), "rb") as f:
        return f.read()


def _args():
    out = []
    with open(os.path.join(TINY, "e2e_tiny.args")) as f:
        for line in f:
            name, fn, rows, cols = line.strip().split(":")
            out.append((name, fn, int(rows), int(cols)))
    return out


def test_oracle_loader_on_the_reference_program():
    img = _tiny()
    p = vmb.parse(img)
    h = p["header"]
    assert len(p["consts"]) == 7 and len(p["slots"]) == 11
    pool = img[h["const_off"]:h["const_off"] + h["const_len"]]
    for (off, ln, rows, cols, dt, name_hash), (name, fn, r, c) in zip(p["consts"], _args()):
        assert name_hash == vmb.hash32(name) and (rows, cols) == (r, c) and dt == 0 and ln == 4 * r * c
        with open(os.path.join(TINY, fn), "rb") as f:
            assert pool[off:off + ln] == f.read()
    # one OP_GEMM: LINEAR_out = SPARSE_out . LINEAR_W^T
    text = img[h["text_off"]:h["text_off"] + h["text_len"]]
    gemms = [struct.unpack_from("<BBHIII", text, i) for i in range(0, len(text), 16) if text[i] == OP_GEMM]
    assert len(gemms) == 1
    _, fl, _, d, a, b = gemms[0]
    names = {s[6]: i for i, s in enumerate(p["slots"])}
    assert fl == 0 and (d, a, b) == tuple(names[vmb.hash32(n)] for n in ("LINEAR_out", "SPARSE_out", "LINEAR_W"))


def test_oracle_layerb_arithmetic():
    assert vmb.layerb(0, 100.0) == 100 and vmb.layerb(100, -40.0) == 60 and vmb.layerb(10, -40.0) == 0
    assert vmb.layerb(5, float("nan")) == 5 and vmb.layerb(0, 2.9) == 2 and vmb.layerb(3, float("inf")) == 2**64 - 1


@pytest.mark.parametrize("mutate,status,msg", [
    (lambda b: b"XXXX" + b[4:], ARG, "bad magic"),
    (lambda b: b[:20], SHAPE, "header"),
    (lambda b: b[:-8], SHAPE, "outside the image"),
])
def test_pool_load_errors_before_device_work(mutate, status, msg):
    with pytest.raises(VmlmError) as e:
        K.Pool(mutate(_tiny()))
    assert e.value.status == status and msg in str(e.value)


def test_pool_load_unknown_const_dtype():
    img = build([("W", np.zeros((2, 2), np.float32), 7)], [("W", vmb.SLOT_CONST, 0, 2, 2)])
    with pytest.raises(vmb.VmExit):
        vmb.parse(img)
    with pytest.raises(VmlmError) as e:
        K.Pool(img)
    assert e.value.status == OPERATOR and "const has unknown dtype" in str(e.value)


def test_pool_load_slot_past_the_pool():
    img = build([("W", np.zeros((2, 2), np.float32), 0)], [("W", vmb.SLOT_CONST, 0, 4, 4)])
    with pytest.raises(VmlmError) as e:
        K.Pool(img)
    assert e.value.status == SHAPE


def test_audit_passes_the_reference_program():
    img = _tiny()
    vmb.audit(img, vmb.parse(img))  # the reference's own program loads in the VM


OP_COPY, OP_EWADD = 3, 4  # any instruction other than the special cases reads its slots as f32


def _audit_image(text, dt_w=4):
    """Slots: 0 activation [2,4], 1 constant W [4,4] of dtype dt_w, 2 activation [2,4], 3 f32 constant."""
    w = np.zeros((4, 4), np.uint16 if dt_w in (1, 4) else np.int8 if dt_w == 2 else np.float32)
    return build([("W", w, dt_w), ("F", np.zeros((4, 4), np.float32), 0)],
                 [("x", vmb.SLOT_ACT, 0, 2, 4), ("W", vmb.SLOT_CONST, 0, 4, 4), ("y", vmb.SLOT_ACT, 64, 2, 4),
                  ("F", vmb.SLOT_CONST, 1, 4, 4)], text=text, act_bytes=128)


@pytest.mark.parametrize("text,dt_w,msg", [
    (ins(OP_COPY, dst=2, a=1), 4, "op 3 uses bf16 const at slot 1 (only a GEMM may read a non-f32 operand)"),
    (ins(OP_EWADD, dst=2, a=0, b=1), 2, "op 4 uses i8 const at slot 1 (only a GEMM may read a non-f32 operand)"),
    (ins(OP_COPY, dst=1, a=0), 1, "op 3 uses non-f32 const at slot 1 (only a GEMM may read a non-f32 operand)"),
    (ins(OP_GEMM, dst=2, a=0, b=1), 1, "gemm B has no kernel for this dtype"),
    (ins(vmb.OP_EMB, dst=1, a=1, b=0), 4, "op 14 uses bf16 const at slot 1"),
])
def test_audit_rejects_non_f32_constants_outside_gemm(text, dt_w, msg):
    img = _audit_image(text, dt_w)
    with pytest.raises(vmb.VmExit) as ve:
        vmb.audit(img, vmb.parse(img))
    assert ve.value.code == 9 and msg in ve.value.msg
    with pytest.raises(VmlmError) as e:
        K.Pool(img)  # rejected before any device work
    assert e.value.status == OPERATOR and msg in str(e.value)


@pytest.mark.parametrize("text,dt_w", [
    (ins(OP_GEMM, dst=2, a=0, b=1), 4),                     # bf16 B operand
    (ins(OP_GEMM, dst=2, a=0, b=1, dt=3), 2),               # i8 B operand, scale slot in dt
    (ins(vmb.OP_EMB, dst=2, a=1, b=0), 4),                  # bf16 table, f32 destination
    (ins(vmb.OP_SHAPE, dst=1, a=1, b=1), 4),                # SHAPE fields are numbers
    (ins(vmb.OP_SLICE, dst=2, a=0, b=1), 4),                # SLICE b is a column offset
    (ins(vmb.OP_LOOP_CNT, dst=1, a=0, b=1), 2),             # LOOP_CNT: only a is a slot
    (ins(OP_COPY, dst=2, a=3), 4),                          # f32 constants are fine anywhere
    (ins(OP_COPY, dst=2, a=99), 4),                         # slot numbers past the table are skipped
])
def test_audit_accepts_what_the_vm_accepts(text, dt_w):
    img = _audit_image(text, dt_w)
    vmb.audit(img, vmb.parse(img))


# --------------------------------------------------------------------- GPU

def _d2h(addr, nbytes):
    from cuda.bindings import runtime as rt
    out = np.empty(nbytes, np.uint8)
    err, = rt.cudaMemcpy(out.ctypes.data, addr, nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert int(err) == 0
    return out


def _h2d(addr, arr):
    from cuda.bindings import runtime as rt
    arr = np.ascontiguousarray(arr)
    err, = rt.cudaMemcpy(addr, arr.ctypes.data, arr.nbytes, rt.cudaMemcpyKind.cudaMemcpyHostToDevice)
    assert int(err) == 0


@pytest.mark.gpu
def test_pool_binds_the_reference_program(kernels, oracle):
    img = _tiny()
    p = vmb.parse(img)
    h = p["header"]
    with K.Pool(img) as pool:
        n_const, n_slots, sizes = pool.info()
        assert (n_const, n_slots) == (7, 11)
        assert sizes == [h["const_len"], h["act_bytes"], h["state_bytes"], h["grad_bytes"]]
        bases = [pool.region(r) for r in range(4)]
        const = _d2h(bases[0], h["const_len"]).tobytes()
        assert const == img[h["const_off"]:h["const_off"] + h["const_len"]]
        assert not _d2h(bases[1], h["act_bytes"] + 64).any()
        for i, (kind, region, off, rows, cols, dt, name) in enumerate(p["slots"]):
            assert pool.slot(i) == (bases[region] + off, rows, cols, dt, kind)
            assert pool.find_slot({vmb.hash32(n): n for n in _slot_names()}[name]) == i
        assert pool.find_const("LINEAR_W") == 5
        with pytest.raises(VmlmError):
            pool.find_const("nope")
        # the program's OP_GEMM on the device: LINEAR_out = SPARSE_out . LINEAR_W^T
        text = img[h["text_off"]:h["text_off"] + h["text_len"]]
        g = next(text[i:i + 16] for i in range(0, len(text), 16) if text[i] == OP_GEMM)
        _, _, _, d, a, b = struct.unpack("<BBHIII", g)
        x = np.array([[0.5, -1.25, 2.0, 3.5]], np.float32)
        _h2d(pool.slot(a)[0], x)
        pool.gemm(g)
        kernels.sync()
        got = _d2h(pool.slot(d)[0], 16).view(np.float32).reshape(1, 4)
        w = np.fromfile(os.path.join(TINY, "LINEAR_W.bin"), np.float32).reshape(4, 4)
        assert np.abs(got - oracle.gemm_nt_f32(x, w)).max() <= 1e-6


def _slot_names():
    return ["EMBED_out", "EMBED_E", "tiny_in", "SPARSE_col", "SPARSE_off", "SPARSE_src", "SPARSE_W", "SPARSE_out",
            "LINEAR_out", "LINEAR_W", "LINEAR_b"]


def _gemm_program(oracle, m, n, k):
    x = oracle.fill_normal(m * k, 1, 1.0).reshape(m, k)
    wf = oracle.fill_normal(n * k, 2, 0.05).reshape(n, k)
    wb = oracle.f32_to_bf16(wf).reshape(n, k)
    q, s = oracle.quant_int8(wf)
    wnn = np.ascontiguousarray(wf.T)
    consts = [("X", x, 0), ("WB", wb, 4), ("WQ", q, 2), ("S", s.reshape(1, n), 0), ("WF", wf, 0), ("WNN", wnn, 0)]
    act = 4 * m * n
    slots = [("X", 0, 0, m, k), ("WB", 0, 1, n, k), ("WQ", 0, 2, n, k), ("S", 0, 3, 1, n), ("WF", 0, 4, n, k),
             ("WNN", 0, 5, k, n), ("D1", 1, 0, m, n), ("D2", 1, act, m, n), ("D3", 1, 2 * act, m, n),
             ("D4", 1, 3 * act, m, n)]
    text = (ins(OP_GEMM, 0, 0xFFFF, 6, 0, 1) + ins(OP_GEMM, 0, 3, 7, 0, 2) + ins(OP_GEMM, 0, 0xFFFF, 8, 0, 4)
            + ins(OP_GEMM, 2, 0xFFFF, 9, 0, 5))
    img = build(consts, slots, text, act_bytes=4 * act)
    return img, text, (x, wb, q, s, wf)


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(4, 300, 256), (64, 2304, 2304)])
def test_pool_gemm_every_b_dtype(kernels, oracle, m, n, k):
    img, text, (x, wb, q, s, wf) = _gemm_program(oracle, m, n, k)
    refs = [oracle.gemm_nt_bf16(x, wb), oracle.gemm_nt_int8(x, q, s), oracle.gemm_nt_f32(x, wf),
            oracle.gemm_nt_f32(x, wf)]
    tols = [1e-4, 2e-5, 5e-5, 5e-5]  # the bounds of the bf16 / Q8 / f32 parity tests
    with K.Pool(img) as pool:
        for i, (r, tol) in enumerate(zip(refs, tols)):
            pool.gemm(text[16 * i:16 * i + 16])
            kernels.sync()
            got = _d2h(pool.slot(6 + i)[0], 4 * m * n).view(np.float32).reshape(m, n)
            assert oracle.max_rel_err(got, r) <= tol, i


@pytest.mark.gpu
def test_pool_gemm_guards(kernels, oracle):
    m, n, k = 2, 8, 16
    img, text, _ = _gemm_program(oracle, m, n, k)
    with K.Pool(img) as pool:
        with pytest.raises(VmlmError) as e:  # int8 B with the scale slot out of the table
            pool.gemm(ins(OP_GEMM, 0, 0xFFFF, 7, 0, 2))
        assert e.value.status == OPERATOR and "scale slot must be f32" in str(e.value)
        with pytest.raises(VmlmError) as e:  # bf16 NN
            pool.gemm(ins(OP_GEMM, 2, 0, 6, 0, 1))
        assert e.value.status == OPERATOR and "bf16 NN gemm unimplemented" in str(e.value)
        with pytest.raises(VmlmError) as e:
            pool.gemm(ins(OP_GEMM + 1, 0, 0, 6, 0, 1))
        assert e.value.status == ARG
        with pytest.raises(VmlmError) as e:
            pool.gemm(ins(OP_GEMM, 0, 0, 6, 0, 99))
        assert e.value.status == ARG


@pytest.mark.gpu
def test_pool_layer_base(kernels, oracle):
    """Two layers of [n, k] f32 weights one stride apart; OP_LAYERB moves every
    CONSTANT slot to the next layer and back; a base past the pool is refused."""
    m, n, k = 3, 40, 64
    x = oracle.fill_normal(m * k, 5, 1.0).reshape(m, k)
    w0 = oracle.fill_normal(n * k, 6, 0.1).reshape(n, k)
    w1 = oracle.fill_normal(n * k, 7, 0.1).reshape(n, k)
    img = build([("W0", w0, 0), ("W1", w1, 0), ("X", x, 0)],
                [("W", 0, 0, n, k), ("X", 4, 2, m, k), ("D", 1, 0, m, n)],
                ins(OP_GEMM, 0, 0xFFFF, 2, 1, 0), act_bytes=4 * m * n)
    p = vmb.parse(img)
    stride = p["consts"][1][0] - p["consts"][0][0]
    g = ins(OP_GEMM, 0, 0xFFFF, 2, 1, 0)
    with K.Pool(img) as pool:
        def run():
            pool.gemm(g)
            kernels.sync()
            return _d2h(pool.slot(2)[0], 4 * m * n).view(np.float32).reshape(m, n)
        assert oracle.max_rel_err(run(), oracle.gemm_nt_f32(x, w0)) <= 1e-6
        pool.layerb(float(stride))
        assert pool.layer_base() == stride == vmb.layerb(0, float(stride))
        assert pool.slot(0)[0] == pool.region(0) + vmb.const_offset(p, 0, stride)
        assert pool.slot(1)[0] == pool.region(0) + p["slots"][1][2]  # a PARAM slot does not move
        assert oracle.max_rel_err(run(), oracle.gemm_nt_f32(x, w1)) <= 1e-6
        pool.layerb(float(stride))
        with pytest.raises(VmlmError) as e:
            pool.gemm(g)
        assert e.value.status == OPERATOR and "layer base walks past the constant pool" in str(e.value)
        pool.layerb(-2.0 * stride)
        assert pool.layer_base() == 0
        assert oracle.max_rel_err(run(), oracle.gemm_nt_f32(x, w0)) <= 1e-6
