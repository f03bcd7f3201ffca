"""The OP_GEMM operator (core/src/interp.rs:734-812) through the C ABI.

CPU tests: every case where the VM prints a message and exits 9 returns
VMLM_ERR_OPERATOR with that message, before any device work. GPU tests: the
dtype dispatch reaches the same kernels as the direct entry points (bit-equal
results) and matches the oracle.
"""
import numpy as np
import pytest

import sparrow_b200.kernels as K
from sparrow_b200._lib import VmlmError

OPERATOR = 8  # VMLM_ERR_OPERATOR


def _refused(fl, d, a, b, scale=None):
    with pytest.raises(VmlmError) as e:
        K.op_gemm(fl, d, a, b, scale)
    assert e.value.status == OPERATOR
    return str(e.value)


A = np.zeros((2, 4), np.float32)
D = np.zeros((2, 3), np.float32)


@pytest.mark.parametrize("fl,b,scale,msg", [
    (K.FL_TRANS_B, np.zeros((4, 3), np.uint16), None, "bf16 NN gemm unimplemented"),       # interp.rs:755-759
    (K.FL_ACC, np.zeros((3, 4), np.uint16), None, "bf16 acc gemm unimplemented"),           # :760-763
    (K.FL_TRANS_B, np.zeros((4, 3), np.int8), None, "int8 NN gemm unimplemented"),          # :779-782
    (K.FL_ACC, np.zeros((3, 4), np.int8), None, "int8 acc gemm unimplemented"),             # :783-786
    (0, np.zeros((3, 4), np.int8), None, "int8 gemm: scale slot must be f32"),              # :787-791
    (0, np.zeros((3, 4), np.int8), np.zeros((3, 1), np.int32), "int8 gemm: scale slot must be f32"),
    (0, np.zeros((3, 4), np.int8), np.zeros((1, 2), np.float32), "int8 gemm: scale shorter than N rows"),  # :792-798
    (0, np.zeros((3, 4), np.int32), None, "gemm operand dtype unsupported"),                # :802-804
    (0, np.zeros((3, 4), np.float16), None, "gemm operand dtype unsupported"),
])
def test_vm_exit9_cases(fl, b, scale, msg):
    assert msg in _refused(fl, D, A, b, scale)


@pytest.mark.parametrize("fl,b,d,msg", [
    (0, np.zeros((3, 5), np.float32), D, "K of B differs"),
    (K.FL_TRANS_B, np.zeros((5, 3), np.float32), D, "K of B differs"),
    (0, np.zeros((3, 4), np.float32), np.zeros((2, 2), np.float32), "output slot smaller"),
    (0, np.zeros((3, 4), np.uint16), np.zeros((2, 3), np.int32), "must be f32"),
])
def test_bounds_the_reference_leaves_unchecked(fl, b, d, msg):
    assert msg in _refused(fl, d, A, b)


@pytest.mark.gpu
def test_op_gemm_dispatch_matches_entry_points(kernels, oracle):
    m, n, k = 96, 700, 512
    a = oracle.fill_normal(m * k, 1, 1.0).reshape(m, k)
    wf = oracle.fill_normal(n * k, 2, 0.05).reshape(n, k)
    wb = oracle.f32_to_bf16(wf)
    q, s = oracle.quant_int8(wf)

    def both(fl, b, scale, direct):
        d = np.empty((m, n), np.float32)
        K.op_gemm(fl, d, a, b, scale.reshape(-1, 1) if scale is not None else None)
        ref = np.empty((m, n), np.float32)
        direct(ref)
        assert np.array_equal(d.view(np.uint32), ref.view(np.uint32))
        return d

    got = both(0, wb, None, lambda c: K.gemm_nt_bf16(a, wb, c, m, n, k))
    assert oracle.max_rel_err(got, oracle.gemm_nt_bf16(a, wb)) < 1e-4
    got = both(0, q, s, lambda c: K.gemm_nt_int8(a, q, s, c, m, n, k))
    assert oracle.max_rel_err(got, oracle.gemm_nt_int8(a, q, s)) < 2e-5
    got = both(0, wf, None, lambda c: K.gemm_nt_f32(a, wf, c, m, n, k))
    assert oracle.max_rel_err(got, oracle.gemm_nt_f32(a, wf)) < 1e-3
    wt = np.ascontiguousarray(wf.T)
    got = both(K.FL_TRANS_B, wt, None, lambda c: K.gemm_f32(a, wt, c, m, n, k))
    assert oracle.max_rel_err(got, oracle.gemm_f32(a, wt)) < 1e-3
    c0 = oracle.fill_normal(m * n, 3, 1.0).reshape(m, n)
    d = c0.copy()
    K.op_gemm(K.FL_ACC, d, a, wf)
    assert oracle.max_rel_err(d, oracle.gemm_nt_f32(a, wf, c0)) < 1e-3


@pytest.mark.gpu
def test_op_gemm_device_slots(kernels, oracle):
    import torch
    m, n, k = 64, 300, 256
    a = oracle.fill_normal(m * k, 4, 1.0).reshape(m, k)
    q, s = oracle.quant_int8(oracle.fill_normal(n * k, 5, 0.02).reshape(n, k))
    da, dq, ds = torch.from_numpy(a).cuda(), torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda().reshape(n, 1)
    dd = torch.empty((m, n), device="cuda")
    K.op_gemm_dev(0, dd, da, dq, ds, stream=torch.cuda.current_stream())
    torch.cuda.synchronize()
    assert oracle.max_rel_err(dd.cpu().numpy(), oracle.gemm_nt_int8(a, q, s)) < 2e-5
