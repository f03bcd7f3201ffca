"""The decode-step neighbours of the quantised linear layer:
RMSNorm fused into the Q8 GEMM, OP_GEMV and OP_EMB, through the C ABI.

CPU tests pin the oracle restatements (ops/src/kernels.rs:1346-1370,
core/src/interp.rs:815-827, :1351-1420) and check OP_EMB's index guards, which
the host call applies before any device work. GPU tests compare the kernels
with the oracle: the fused RMSNorm + Q8 GEMM within the Q8 bound (the norm's
sum of squares runs in another order: ~1 ulp of inv), OP_GEMV within f32
rounding of a reordered sum, OP_EMB bit-exact.
"""
import numpy as np
import pytest

import sparrow_b200.kernels as K
from sparrow_b200._lib import VmlmError

TIGHT_Q8 = 2e-5
OPERATOR = 8


def test_oracle_rmsnorm_matches_its_definition(oracle):
    x = oracle.fill_normal(6 * 300, 1, 2.0).reshape(6, 300)
    g = oracle.fill_normal(300, 2, 1.0)
    got = oracle.rmsnorm(x, g, 1e-5)
    x64 = x.astype(np.float64)
    ref = x64 / np.sqrt((x64 * x64).mean(axis=1, keepdims=True) + 1e-5) * g
    assert np.abs(got - ref).max() / np.abs(ref).max() < 1e-6


def test_oracle_gemv_and_emb(oracle):
    a = oracle.fill_normal(40 * 33, 3, 1.0).reshape(40, 33)
    b = oracle.fill_normal(33, 4, 1.0)
    assert np.abs(oracle.gemv_f32(a, b) - a.astype(np.float64) @ b).max() < 1e-4
    tab = oracle.f32_to_bf16(oracle.fill_normal(5 * 7, 5, 1.0)).reshape(5, 7)
    st, out = oracle.emb(tab, np.array([4, 0, 2], np.float32))
    assert st == 0 and np.array_equal(out, oracle.bf16_to_f32(tab[[4, 0, 2]]))
    for bad, code in ((-1.0, 1), (5.0, 1), (np.nan, 1), (2.5, 2)):
        assert oracle.emb(tab, np.array([0, bad], np.float32))[0] == code


@pytest.mark.parametrize("bad,msg", [(-1.0, "out of range"), (7.0, "out of range"), (np.nan, "out of range"),
                                     (np.inf, "out of range"), (1.5, "not an integer")])
def test_emb_host_guards(bad, msg):
    # core/src/interp.rs:1375-1397: checked before any device work
    tab = np.zeros((7, 4), np.float32)
    with pytest.raises(VmlmError) as e:
        K.emb(tab, np.array([0.0, bad], np.float32), np.empty((2, 4), np.float32))
    assert e.value.status == OPERATOR and msg in str(e.value)


# --------------------------------------------------------------------- GPU

@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(1, 5760, 2304), (8, 2304, 2304), (32, 2304, 5760), (64, 16384, 2304),
                                   (300, 1000, 520), (3, 100, 7)])
def test_rmsnorm_gemm_nt_int8(kernels, oracle, m, n, k):
    x = oracle.fill_normal(m * k, m + 1, 3.0).reshape(m, k)
    g = oracle.fill_normal(k, 2, 1.0)
    q, s = oracle.quant_int8(oracle.fill_normal(n * k, 3, 0.02).reshape(n, k))
    c = np.empty((m, n), np.float32)
    kernels.rmsnorm_gemm_nt_int8(x, g, 1e-6, q, s, c, m, n, k)
    ref = oracle.gemm_nt_int8(oracle.rmsnorm(x, g, 1e-6), q, s, nt=16)
    assert oracle.max_rel_err(c, ref) <= TIGHT_Q8


@pytest.mark.gpu
def test_rmsnorm_gemm_nonfinite_rows(kernels, oracle):
    m, n, k = 4, 600, 512
    x = oracle.fill_normal(m * k, 7, 1.0).reshape(m, k)
    x[1, 3] = np.nan
    x[2, 9] = np.inf
    g = oracle.fill_normal(k, 8, 1.0)
    q, s = oracle.quant_int8(oracle.fill_normal(n * k, 9, 0.02).reshape(n, k))
    c = np.empty((m, n), np.float32)
    kernels.rmsnorm_gemm_nt_int8(x, g, 1e-6, q, s, c, m, n, k)
    ref = oracle.gemm_nt_int8(oracle.rmsnorm(x, g, 1e-6), q, s)
    assert np.array_equal(np.isnan(c), np.isnan(ref))
    fin = np.isfinite(ref).all(axis=1)
    assert oracle.max_rel_err(np.ascontiguousarray(c[fin]), np.ascontiguousarray(ref[fin])) <= TIGHT_Q8


@pytest.mark.gpu
def test_rmsnorm_gemm_device(kernels, oracle):
    import torch
    m, n, k = 16, 5760, 2304
    x = oracle.fill_normal(m * k, 10, 1.0).reshape(m, k)
    g = oracle.fill_normal(k, 11, 1.0)
    q, s = oracle.quant_int8(oracle.fill_normal(n * k, 12, 0.02).reshape(n, k))
    dx, dg, dq, ds = (torch.from_numpy(v).cuda() for v in (x, g, q, s))
    dc = torch.empty((m, n), device="cuda")
    kernels.rmsnorm_gemm_nt_int8_dev(dx, dg, 1e-5, dq, ds, dc, m, n, k, stream=torch.cuda.current_stream())
    torch.cuda.synchronize()
    ref = oracle.gemm_nt_int8(oracle.rmsnorm(x, g, 1e-5), q, s, nt=16)
    assert oracle.max_rel_err(dc.cpu().numpy(), ref) <= TIGHT_Q8


@pytest.mark.gpu
@pytest.mark.parametrize("m,k", [(5760, 2304), (1000, 7), (1, 1), (333, 129)])
def test_gemv_f32(kernels, oracle, m, k):
    a = oracle.fill_normal(m * k, m, 1.0).reshape(m, k)
    b = oracle.fill_normal(k, k, 1.0)
    c = np.empty(m, np.float32)
    kernels.gemv_f32(a, b, c, m, k)
    ref = oracle.gemv_f32(a, b)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    assert np.abs(c - ref).max() <= 1e-3 * max(1.0, np.abs(ref).max())
    assert np.abs(c - exact).max() <= 1e-5 * max(1.0, np.abs(exact).max())


@pytest.mark.gpu
@pytest.mark.parametrize("bf16", [True, False])
def test_emb_rows(kernels, oracle, bf16):
    rows, cols = 1000, 2304
    vals = oracle.fill_normal(rows * cols, 13, 1.0).reshape(rows, cols)
    tab = oracle.f32_to_bf16(vals).reshape(rows, cols) if bf16 else vals
    idx = np.array([999, 0, 17, 17, 512], np.float32)
    out = np.empty((idx.size, cols), np.float32)
    kernels.emb(tab, idx, out)
    st, ref = oracle.emb(tab, idx)
    assert st == 0 and np.array_equal(out.view(np.uint32), ref.view(np.uint32))
    kernels.register_weight(tab)  # a registered table is read on the device in place
    try:
        out2 = np.empty_like(out)
        kernels.emb(tab, idx, out2)
        assert np.array_equal(out2.view(np.uint32), ref.view(np.uint32))
    finally:
        kernels.unregister_weight(tab)


@pytest.mark.gpu
def test_emb_device_rows_and_guards(kernels, oracle):
    import torch
    rows, cols = 300, 520
    vals = oracle.fill_normal(rows * cols, 14, 1.0).reshape(rows, cols)
    tab = oracle.f32_to_bf16(vals).reshape(rows, cols)
    dtab = torch.from_numpy(tab.view(np.int16)).cuda()
    idx = np.array([3, 299, 0], np.float32)
    dout = torch.empty((3, cols), device="cuda")
    st = torch.cuda.current_stream()
    kernels.emb_dev(dtab, torch.from_numpy(idx).cuda(), dout, stream=st)
    kernels.sync(st)
    assert np.array_equal(dout.cpu().numpy().view(np.uint32), oracle.emb(tab, idx)[1].view(np.uint32))
    for bad, msg in ((300.0, "out of range"), (np.nan, "out of range"), (2.25, "not an integer")):
        kernels.emb_dev(dtab, torch.tensor([1.0, bad], device="cuda"), torch.empty((2, cols), device="cuda"),
                        stream=st)
        with pytest.raises(VmlmError) as e:
            kernels.sync(st)
        assert e.value.status == OPERATOR and msg in str(e.value)
