"""GPU parity: the CUDA path through the C ABI against the CPU oracle.

Tolerances: int8 x int8 -> int32 accumulators and their
scaled outputs bit-exact; f32 outputs within 1e-3 max relative error
(max|gpu-ref| / max|ref|). The kernels are tighter than that: Q8 results carry
~2^-22 relative rounding of the activations and bf16 results ~f32 accumulation
error, so the tests also assert the tighter bounds TIGHT_Q8 / TIGHT_BF16.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN
from test_oracle import EDGE_SHAPES, edge_inputs

pytestmark = pytest.mark.gpu

TOL = 1e-3        # BASELINE: fp32 outputs within 1e-3 max relative error
TIGHT_Q8 = 2e-5
TIGHT_BF16 = 1e-4
NT = os.cpu_count() or 1


def q8_case(O, m, n, k, seed=0):
    x = O.fill_normal(m * k, seed, 1.0).reshape(m, k)
    q, s = O.quant_int8(O.fill_normal(n * k, seed + 1, 0.02).reshape(n, k))
    return x, q, s


def check_q8(K, O, x, q, s, tight=TIGHT_Q8):
    got = K.q8_linear(x, q, s)
    ref = O.gemm_nt_int8(x, q, s, nt=NT)
    err = O.max_rel_err(got, ref)
    assert err <= TOL and err <= tight, err
    return got, ref


# ----------------------------------------------------------- golden fixtures

def _f32(p, shape=None):
    a = np.fromfile(os.path.join(GOLDEN, p), "<f4")
    return a.reshape(shape) if shape else a


def _i8(p, shape):
    return np.fromfile(os.path.join(GOLDEN, p), "i1").reshape(shape)


def test_golden_p13_q8_exact(kernels):
    a = _f32("p13/q8_a.f32", (1, 4))
    w = _i8("p13/q8_w.i8", (2, 4))
    s = _f32("p13/q8_scale.f32")
    assert kernels.q8_linear(a, w, s).ravel().tolist() == [-1.0, -1.0]


def test_golden_int8_bins_through_gpu(kernels, oracle):
    def lin(d, tag, x, kin):
        q = _i8(f"{d}/{tag}_Wq.bin", (4, kin))
        return kernels.q8_linear(x, q, _f32(f"{d}/{tag}_scale.bin")) + _f32(f"{d}/{tag}_b.bin")

    def lin_f32(d, tag, x, kin):
        return oracle.gemm_naive_f32(x, _f32(f"{d}/{tag}_W.bin", (4, kin))) + _f32(f"{d}/{tag}_b.bin")

    x1 = _f32("int8_bins/i8o_in.bin", (1, 1))
    assert oracle.print_f32(lin("int8_bins", "o", x1, 1)) == "0.881869 -0.907158 -0.010653 2.102990"
    x4 = _f32("int8_bins/i8t_in.bin", (1, 4))
    two = lambda d, f: f(d, "b", f(d, "a", x4, 4), 4)  # noqa: E731
    exact = two("int8_bins", lin_f32)
    assert np.abs(two("int8_bins", lin) - exact).max() <= 1e-4
    assert abs(np.abs(two("int8_bad_bins", lin) - exact).max() - 0.607249) < 1e-5
    xn = _f32("int8_naive_bins/i8t_in.bin", (1, 4))
    d4 = np.abs(lin("int8_naive_bins", "b", lin("int8_naive_bins", "a", xn, 4), 4)
                - lin_f32("int8_naive_bins", "b", lin_f32("int8_naive_bins", "a", xn, 4), 4)).max()
    assert abs(d4 - 0.009791) < 1e-5


# ------------------------------------------------------------- Q8 configs

def test_c1_q8_gemv_full(kernels, oracle):
    x, q, s = q8_case(oracle, 1, 5760, 2304)
    check_q8(kernels, oracle, x, q, s)


@pytest.mark.parametrize("m", [1, 8, 32])
def test_c3_q8_layer_set(kernels, oracle, m):
    shapes = [(2304, 2304)] * 4 + [(5760, 2304)] * 2 + [(2304, 5760)]
    for i, (n, k) in enumerate(shapes):
        x, q, s = q8_case(oracle, m, n, k, seed=10 * i)
        check_q8(kernels, oracle, x, q, s)


@pytest.mark.parametrize("m", [1, 64])
def test_c4_q8_lm_head(kernels, oracle, m):
    n, k = 122753, 2304
    x, q, s = q8_case(oracle, m, n, k, seed=40)
    got = kernels.q8_linear(x, q, s)
    rows = np.unique(np.concatenate([np.arange(256), np.arange(n - 256, n),
                                     np.random.default_rng(0).integers(0, n, 4096)]))
    ref = oracle.gemm_nt_int8(x, np.ascontiguousarray(q[rows]), np.ascontiguousarray(s[rows]), nt=NT)
    err = oracle.max_rel_err(np.ascontiguousarray(got[:, rows]), ref)
    assert err <= TOL and err <= TIGHT_Q8, err


@pytest.mark.parametrize("m,n,k", [(1, 2304, 2304), (3, 1000, 4096), (17, 130, 2304), (80, 384, 1024),
                                   (81, 640, 768), (100, 257, 512), (200, 96, 256), (64, 128, 8192)])
def test_q8_shapes_streamk_and_token_chunks(kernels, oracle, m, n, k):
    x, q, s = q8_case(oracle, m, n, k, seed=m + n)
    check_q8(kernels, oracle, x, q, s)


@pytest.mark.parametrize("m,n,k", EDGE_SHAPES)
def test_q8_edge_shapes(kernels, oracle, m, n, k):
    a, b = edge_inputs(m, n, k)
    q, s = oracle.quant_int8(b)
    check_q8(kernels, oracle, a, q, s)


@pytest.mark.parametrize("m,n,k", [(80, 76000, 256), (17, 80001, 512), (200, 30000, 256)])
def test_q8_cta_pair_tiles(kernels, oracle, m, n, k):
    # enough whole weight tiles for the CTA-pair kernel: 256 weight rows per
    # pair, each SM loading half of the digit planes (ragged N, up to 80
    # tokens per tile, several token tiles with a ragged last one)
    x, q, s = q8_case(oracle, m, n, k, seed=n % 97)
    check_q8(kernels, oracle, x, q, s)


def test_q8_cta_pair_nonfinite(kernels, oracle):
    m, n, k = 40, 76000, 256
    x, q, s = q8_case(oracle, m, n, k, seed=12)
    x[3, 17] = np.nan
    x[39, 0] = -np.inf
    got = kernels.q8_linear(x, q, s)
    ref = oracle.gemm_nt_int8(x, q, s, nt=NT)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref))
    fin = np.isfinite(ref)
    assert oracle.max_rel_err(np.ascontiguousarray(got[fin]), np.ascontiguousarray(ref[fin])) <= TIGHT_Q8


def test_q8_nonfinite_rows_match_reference(kernels, oracle):
    m, n, k = 4, 300, 512
    x, q, s = q8_case(oracle, m, n, k, seed=3)
    x[1, 7] = np.inf
    x[2, 100] = np.nan
    x[3, 5] = -np.inf
    x[3, 6] = np.inf
    got = kernels.q8_linear(x, q, s)
    ref = oracle.gemm_nt_int8(x, q, s)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref))
    fin = np.isfinite(ref)
    assert np.array_equal(np.sign(got[np.isinf(ref)]), np.sign(ref[np.isinf(ref)]))
    assert oracle.max_rel_err(np.ascontiguousarray(got[fin]), np.ascontiguousarray(ref[fin])) <= TIGHT_Q8


def test_q8_zero_rows_and_extreme_scales(kernels, oracle):
    m, n, k = 3, 200, 256
    x, q, s = q8_case(oracle, m, n, k, seed=9)
    x[0] = 0.0
    x[1] *= np.float32(1e-30)
    x[2] *= np.float32(1e30)
    got = kernels.q8_linear(x, q, s)
    ref = oracle.gemm_nt_int8(x, q, s)
    assert np.all(got[0] == 0.0)
    for r in (1, 2):
        assert oracle.max_rel_err(got[r:r + 1], ref[r:r + 1]) <= TIGHT_Q8


@pytest.mark.parametrize("m,n,k", [(32, 2304, 2304), (17, 5760, 2304), (16, 2304, 5760), (5, 640, 2304),
                                   (2, 130, 1040), (1, 18944, 512), (9, 1, 128), (8, 2304, 5760),
                                   (21, 2304, 2304), (16, 2304, 2304)])
def test_q8_decode_cluster_shapes(kernels, oracle, m, n, k):
    # decode kernel: K split over a cluster of CTAs, partial k-blocks, both
    # token halves of the accumulator, a single row; x slices of exactly one
    # register batch (8 x 2304 x 5760: 8 tokens x 8 k-blocks per CTA) and just
    # under it (21 x 3); the first three shapes exceed it and take the
    # persistent swap-mode GEMM
    x, q, s = q8_case(oracle, m, n, k, seed=m * 7 + k)
    check_q8(kernels, oracle, x, q, s)


def test_q8_decode_nonfinite_in_one_cta_range(kernels, oracle):
    # the K range of each CTA sees only part of a row: a NaN/Inf anywhere must
    # still turn the whole output row into the sequential f32 result
    m, n, k = 3, 2304, 2304
    x, q, s = q8_case(oracle, m, n, k, seed=31)
    x[0, 2200] = np.inf
    x[1, 3] = np.nan
    got = kernels.q8_linear(x, q, s)
    ref = oracle.gemm_nt_int8(x, q, s)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref))
    assert np.array_equal(np.sign(got[np.isinf(ref)]), np.sign(ref[np.isinf(ref)]))
    assert oracle.max_rel_err(got[2:3], ref[2:3]) <= TIGHT_Q8


def test_q8_decode_unaligned_activations(kernels, oracle):
    import torch
    m, n, k = 4, 1000, 2304
    x, q, s = q8_case(oracle, m, n, k, seed=77)
    buf = torch.zeros(m * k + 1, dtype=torch.float32, device="cuda")
    buf[1:].copy_(torch.from_numpy(x.ravel()))
    dx = buf[1:].view(m, k)  # 4-byte aligned only
    dq, ds = torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()
    out = torch.empty((m, n), dtype=torch.float32, device="cuda")
    kernels.gemm_nt_int8_dev(dx, dq, ds, out, m, n, k)
    torch.cuda.synchronize()
    err = oracle.max_rel_err(out.cpu().numpy(), oracle.gemm_nt_int8(x, q, s))
    assert err <= TIGHT_Q8, err


def test_q8_deterministic(kernels, oracle):
    x, q, s = q8_case(oracle, 8, 2304, 2304, seed=5)
    a = kernels.q8_linear(x, q, s)
    b = kernels.q8_linear(x, q, s)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_registered_weights_and_layer_offsets(kernels, oracle):
    # OP_LAYERB hands the kernel pointers into the middle of one constant
    # (core/src/interp.rs:438-475): register the whole stack, call on a slice.
    layers, n, k = 3, 384, 1024
    x, q, s = q8_case(oracle, 2, layers * n, k, seed=21)
    kernels.register_weight(q)
    kernels.register_weight(s)
    try:
        for l in range(layers):
            ql, sl = q[l * n:(l + 1) * n], s[l * n:(l + 1) * n]
            got = kernels.q8_linear(x, ql, sl)
            assert oracle.max_rel_err(got, oracle.gemm_nt_int8(x, ql, sl)) <= TIGHT_Q8
    finally:
        kernels.unregister_all()


# ------------------------------------------------------------- bf16 configs

def bf16_case(O, m, n, k, seed=0, exact_x=True):
    x = O.fill_normal(m * k, seed, 1.0)
    if exact_x:
        x = O.bf16_to_f32(O.f32_to_bf16(x))
    w = O.f32_to_bf16(O.fill_normal(n * k, seed + 1, 0.02)).reshape(n, k)
    return x.reshape(m, k), w


def check_bf16(K, O, x, w, tight=TIGHT_BF16):
    got = K.bf16_linear(x, w)
    ref = O.gemm_nt_bf16(x, w, nt=NT)
    err = O.max_rel_err(got, ref)
    assert err <= TOL and err <= tight, err
    return got, ref


def test_c2_bf16_prefill_full(kernels, oracle):
    x, w = bf16_case(oracle, 512, 2304, 2304)
    check_bf16(kernels, oracle, x, w)


def test_c2_shape_general_f32_activations(kernels, oracle):
    # activations that are not bf16 values: three split terms are active
    x, w = bf16_case(oracle, 512, 2304, 2304, seed=7, exact_x=False)
    check_bf16(kernels, oracle, x, w)


def test_bf16_term_planes_stay_exact_across_calls(kernels, oracle):
    # the GEMM writes a row's mid / lo term planes only where they are needed
    # now or were non-zero after the previous call: alternate activations with
    # and without sub-bf16 bits, including single rows that need them
    m, n, k = 512, 768, 1024
    w = oracle.f32_to_bf16(oracle.fill_normal(n * k, 2, 0.02)).reshape(n, k)
    general = oracle.fill_normal(m * k, 3, 1.0).reshape(m, k)
    exact = oracle.bf16_to_f32(oracle.f32_to_bf16(general))
    one = exact.copy()
    one[5, 17] += np.float32(3e-3)
    one[300, 1000] = np.float32(0.1)
    for x in (general, exact, one, general, one, exact):
        check_bf16(kernels, oracle, x, w)


@pytest.mark.parametrize("m,n,k", [(129, 4096, 512), (2000, 256, 256), (640, 2304, 2304)])
def test_bf16_row_block_waits(kernels, oracle, m, n, k):
    # many CTAs converting a few rows each; blocks with a partial last block
    x, w = bf16_case(oracle, m, n, k, seed=m + 1, exact_x=(m % 2 == 0))
    check_bf16(kernels, oracle, x, w)


@pytest.mark.parametrize("m", [1, 8, 32, 80])
def test_bf16_decode_shapes(kernels, oracle, m):
    x, w = bf16_case(oracle, m, 5760, 2304, seed=m, exact_x=False)
    check_bf16(kernels, oracle, x, w)


@pytest.mark.parametrize("m,n,k", [(81, 300, 512), (129, 257, 1000), (300, 2304, 64), (1000, 520, 2048)])
def test_bf16_ragged_tiles(kernels, oracle, m, n, k):
    x, w = bf16_case(oracle, m, n, k, seed=m, exact_x=False)
    check_bf16(kernels, oracle, x, w)


@pytest.mark.parametrize("m,n,k", EDGE_SHAPES)
def test_bf16_edge_shapes(kernels, oracle, m, n, k):
    a, b = edge_inputs(m, n, k)
    check_bf16(kernels, oracle, a, oracle.f32_to_bf16(b))


def test_bf16_nonfinite(kernels, oracle):
    x, w = bf16_case(oracle, 3, 200, 256, seed=2, exact_x=False)
    x[0, 3] = np.inf
    x[1, 9] = np.nan
    got = kernels.bf16_linear(x, w)
    ref = oracle.gemm_nt_bf16(x, w)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref))


# ------------------------------------------------------------- int8 x int8

def i8_case(O, m, n, k, seed=0):
    x = O.fill_int8(m * k, seed).reshape(m, k)
    w = O.fill_int8(n * k, seed + 1).reshape(n, k)
    s = np.abs(O.fill_normal(n, seed + 2, 0.02)) + np.float32(1e-3)
    return x, w, s


def run_i8(K, x, w, s):
    m, k = x.shape
    n = w.shape[0]
    c = np.empty((m, n), np.float32)
    acc = np.empty((m, n), np.int32)
    K.gemm_i8i8(x, w, s, c, acc, m, n, k)
    return c, acc


@pytest.mark.parametrize("m,n,k", [(512, 2048, 8192), (128, 256, 128), (300, 1000, 4096), (4096, 512, 1024)])
def test_i8i8_bit_exact(kernels, oracle, m, n, k):
    x, w, s = i8_case(oracle, m, n, k, seed=m)
    c, acc = run_i8(kernels, x, w, s)
    rc, racc = oracle.gemm_i8i8(x, w, s, nt=NT)
    assert np.array_equal(acc, racc)
    assert np.array_equal(c.view(np.uint32), rc.view(np.uint32))


@pytest.mark.parametrize("m,n,k", EDGE_SHAPES)
def test_i8i8_edge_shapes(kernels, oracle, m, n, k):
    x, w, s = i8_case(oracle, m, n, k, seed=1)
    c, acc = run_i8(kernels, x, w, s)
    rc, racc = oracle.gemm_i8i8(x, w, s)
    assert np.array_equal(acc, racc) and np.array_equal(c.view(np.uint32), rc.view(np.uint32))


def test_c5_full_size_checksums_and_blocks(kernels, oracle):
    """C5 at full size: exact row/column checksums (int64) plus exact random blocks."""
    import torch
    m, n, k = 4096, 28672, 8192
    x, w, s = i8_case(oracle, m, n, k, seed=55)
    dx, dw, ds = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda()
    dacc = torch.empty((m, n), dtype=torch.int32, device="cuda")
    dc = torch.empty((m, n), dtype=torch.float32, device="cuda")
    kernels.gemm_i8i8_dev(dx, dw, ds, dc, dacc, m, n, k)
    kernels.sync()
    # column sums: sum_m acc[m][n] = (sum_m x[m,:]) . w[n,:]
    colsum = dacc.to(torch.int64).sum(0).cpu().numpy()
    xs = x.astype(np.int64).sum(0)
    ref_col = (w.astype(np.int64) @ xs)
    assert np.array_equal(colsum, ref_col)
    rowsum = dacc.to(torch.int64).sum(1).cpu().numpy()
    ref_row = x.astype(np.int64) @ w.astype(np.int64).sum(0)
    assert np.array_equal(rowsum, ref_row)
    rng = np.random.default_rng(1)
    for _ in range(3):
        r0, c0 = int(rng.integers(0, m - 64)), int(rng.integers(0, n - 256))
        blk_c, blk_a = oracle.gemm_i8i8(np.ascontiguousarray(x[r0:r0 + 64]), np.ascontiguousarray(w[c0:c0 + 256]),
                                        np.ascontiguousarray(s[c0:c0 + 256]), nt=NT)
        assert np.array_equal(dacc[r0:r0 + 64, c0:c0 + 256].cpu().numpy(), blk_a)
        assert np.array_equal(dc[r0:r0 + 64, c0:c0 + 256].cpu().numpy().view(np.uint32), blk_c.view(np.uint32))


# ------------------------------------------------------- device entry points

def test_device_entry_points_match_host_ones(kernels, oracle):
    import torch
    x, q, s = q8_case(oracle, 8, 5760, 2304, seed=77)
    host = kernels.q8_linear(x, q, s)
    dx, dq, ds = torch.from_numpy(x).cuda(), torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()
    dc = torch.empty((8, 5760), dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream()
    kernels.gemm_nt_int8_dev(dx, dq, ds, dc, 8, 5760, 2304, stream=st)
    kernels.sync(st)
    assert np.array_equal(dc.cpu().numpy().view(np.uint32), host.view(np.uint32))
    xb, wb = bf16_case(oracle, 64, 1024, 2304, seed=3, exact_x=False)
    hb = kernels.bf16_linear(xb, wb)
    dxb = torch.from_numpy(xb).cuda()
    dwb = torch.from_numpy(wb.view(np.int16)).cuda()
    dcb = torch.empty((64, 1024), dtype=torch.float32, device="cuda")
    kernels.gemm_nt_bf16_dev(dxb, dwb, dcb, 64, 1024, 2304, stream=st)
    kernels.sync(st)
    # bf16 tiles split between CTAs are summed with f32 atomics: equal up to the last bits
    assert oracle.max_rel_err(dcb.cpu().numpy(), hb) <= 1e-6


@pytest.mark.parametrize("m", [512, 1000, 2048])
def test_pipelined_host_calls_match_device_calls(kernels, oracle, m):
    """Large host-pointer calls run in row chunks on copy streams; every chunk
    must give the bits the one device call gives (ragged last chunks too)."""
    import torch
    n, k = 2304, 2304
    st = torch.cuda.current_stream()
    x, q, s = q8_case(oracle, m, n, k, seed=m)
    host = kernels.q8_linear(x, q, s)
    dc = torch.empty((m, n), dtype=torch.float32, device="cuda")
    kernels.gemm_nt_int8_dev(torch.from_numpy(x).cuda(), torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda(),
                             dc, m, n, k, stream=st)
    kernels.sync(st)
    assert np.array_equal(dc.cpu().numpy().view(np.uint32), host.view(np.uint32))
    xb, wb = bf16_case(oracle, m, n, k, seed=m + 1, exact_x=False)
    hb = kernels.bf16_linear(xb, wb)
    kernels.gemm_nt_bf16_dev(torch.from_numpy(xb).cuda(), torch.from_numpy(wb.view(np.int16)).cuda(), dc,
                             m, n, k, stream=st)
    kernels.sync(st)
    assert np.array_equal(dc.cpu().numpy().view(np.uint32), hb.view(np.uint32))
    xi, wi, si = i8_case(oracle, m, n, k, seed=m + 2)
    c_only = np.empty((m, n), np.float32)
    acc_only = np.empty((m, n), np.int32)
    kernels.gemm_i8i8(xi, wi, si, c_only, None, m, n, k)
    kernels.gemm_i8i8(xi, wi, si, None, acc_only, m, n, k)
    rc, racc = oracle.gemm_i8i8(xi, wi, si, nt=NT)
    assert np.array_equal(acc_only, racc)
    assert np.array_equal(c_only.view(np.uint32), rc.view(np.uint32))


@pytest.mark.parametrize("m,n,k", [(2048, 4096, 1024), (1000, 3000, 520), (4096, 2048, 4096)])
def test_i8i8_cta_pairs_bit_exact(kernels, oracle, m, n, k):
    # shapes large enough for the CTA-pair kernel (256-row tiles over two SMs)
    x = oracle.fill_int8(m * k, 80).reshape(m, k)
    w = oracle.fill_int8(n * k, 81).reshape(n, k)
    s = np.abs(oracle.fill_normal(n, 82, 0.02)) + np.float32(1e-3)
    c = np.empty((m, n), np.float32)
    acc = np.empty((m, n), np.int32)
    kernels.gemm_i8i8(x, w, s, c, acc, m, n, k)
    rc, ra = oracle.gemm_i8i8(x, w, s, nt=NT)
    assert np.array_equal(acc, ra)
    assert np.array_equal(c.view(np.uint32), rc.view(np.uint32))


@pytest.mark.parametrize("m,n,k,exact", [(2048, 3072, 1024, True), (1536, 2304, 768, False)])
def test_bf16_cta_pairs(kernels, oracle, m, n, k, exact):
    x, w = bf16_case(oracle, m, n, k, seed=83, exact_x=exact)
    check_bf16(kernels, oracle, x, w)


@pytest.mark.parametrize("m,n,k,exact", [(512, 2304, 2304, True), (512, 2304, 2304, False), (256, 4096, 1024, True),
                                         (600, 3000, 520, True), (384, 2304, 2304, False)])
def test_bf16_prefill_k_split_shapes(kernels, oracle, m, n, k, exact):
    # prefill shapes whose tiles are split over K across a cluster (partials
    # exchanged through distributed shared memory), general and bf16-valued X
    x, w = bf16_case(oracle, m, n, k, seed=m + k, exact_x=exact)
    check_bf16(kernels, oracle, x, w)


# ------------------------------------------------- batches of independent calls

C3_SHAPES = [(2304, 2304)] * 4 + [(5760, 2304)] * 2 + [(2304, 5760)]


def _batch(oracle, m, shapes, seed):
    import torch
    calls, host = [], []
    for i, (n, k) in enumerate(shapes):
        x, q, s = q8_case(oracle, m, n, k, seed=seed + i)
        dx, dq, ds = (torch.from_numpy(v).cuda() for v in (x, q, s))
        calls.append((dx, dq, ds, torch.empty((m, n), device="cuda"), m, n, k))
        host.append((x, q, s))
    return calls, host


@pytest.mark.parametrize("m", [1, 3, 8, 32])
def test_q8_batch_matches_single_calls(kernels, oracle, m):
    """A decoder layer's seven Q8 linears as one batch, against the oracle and the
    seven calls one by one. Not bit-identical to them: in a grouped launch a CTA
    forms a token's digit planes over the whole K (one exponent), a single call
    split over a cluster over each CTA's K range (an exponent per range), so the
    activations are rounded on different 22-bit grids."""
    import torch
    calls, host = _batch(oracle, m, C3_SHAPES, seed=40 + m)
    st = torch.cuda.current_stream()
    kernels.gemm_nt_int8_batch_dev(calls, stream=st)
    kernels.sync(st)
    for (dx, dq, ds, dc, m_, n, k), (x, q, s) in zip(calls, host):
        single = torch.empty_like(dc)
        kernels.gemm_nt_int8_dev(dx, dq, ds, single, m_, n, k, stream=st)
        kernels.sync(st)
        ref = oracle.gemm_nt_int8(x, q, s, nt=NT)
        assert oracle.max_rel_err(dc.cpu().numpy(), ref) <= TIGHT_Q8, (n, k)
        assert oracle.max_rel_err(dc.cpu().numpy(), single.cpu().numpy()) <= TIGHT_Q8, (n, k)


def test_q8_batch_mixed_and_edge_calls(kernels, oracle):
    """Calls that do not share m, a K that is not a multiple of 16, a ragged N, a
    non-finite token, and more calls than one grouped launch takes."""
    import torch
    st = torch.cuda.current_stream()
    shapes = [(300, 1024), (129, 64), (1000, 2304)] * 7  # 21 calls: two grouped launches
    calls, host = _batch(oracle, 2, shapes, seed=90)
    host[4][0][1, 7] = np.inf
    calls[4][0].copy_(torch.from_numpy(host[4][0]))
    kernels.gemm_nt_int8_batch_dev(calls, stream=st)
    kernels.sync(st)
    for (dx, dq, ds, dc, m_, n, k), (x, q, s) in zip(calls, host):
        ref = oracle.gemm_nt_int8(x, q, s)
        got = dc.cpu().numpy()
        assert np.array_equal(np.isnan(got), np.isnan(ref)) and np.array_equal(np.isinf(got), np.isinf(ref))
        fin = np.isfinite(ref).all(axis=1)
        assert oracle.max_rel_err(np.ascontiguousarray(got[fin]), np.ascontiguousarray(ref[fin])) <= TIGHT_Q8
    mixed, mhost = _batch(oracle, 1, [(640, 2304)], seed=7)
    more, more_host = _batch(oracle, 4, [(640, 100)], seed=8)  # K % 16 != 0 and another m: one by one
    kernels.gemm_nt_int8_batch_dev(mixed + more, stream=st)
    kernels.sync(st)
    for (dx, dq, ds, dc, m_, n, k), (x, q, s) in zip(mixed + more, mhost + more_host):
        assert oracle.max_rel_err(dc.cpu().numpy(), oracle.gemm_nt_int8(x, q, s)) <= TIGHT_Q8


@pytest.mark.parametrize("m,shapes", [(2, [(2000, 1040)] * 12), (16, [(2560, 256)] * 8), (1, C3_SHAPES),
                                     (8, [(2000, 1040)] * 12), (16, [(1200, 2304)] * 16),
                                     (32, [(2000, 1040)] * 12), (32, C3_SHAPES)])
def test_q8_batch_equal_share(kernels, oracle, m, shapes):
    """Batches with more 128-row tiles than the GPU has SMs run with an equal
    share of k-blocks per CTA: tiles split between CTAs are summed through f64
    slots by the CTA that completes them. The kernel makes the digit planes
    itself (m = 1) or loads those of the planes kernel with each weight box
    (m = 2 to 32)."""
    _equal_share_case(kernels, oracle, m, shapes)


def _equal_share_case(kernels, oracle, m, shapes):
    """Ragged N, a K that ends inside a k-block, tokens holding NaN and Inf,
    and the same batch twice in a row (the slots and counters must be left at
    zero): against the oracle, and the two calls bit-identical."""
    import torch
    calls, host = _batch(oracle, m, shapes, seed=300 + m)
    a, b = 1, len(shapes) - 2
    host[a][0][m - 1, 5] = np.nan
    host[b][0][0, shapes[b][1] - 1] = -np.inf
    for i in (a, b):
        calls[i][0].copy_(torch.from_numpy(host[i][0]))
    st = torch.cuda.current_stream()
    outs = []
    for _ in range(2):
        for c in calls:
            c[3].fill_(7.0)
        kernels.gemm_nt_int8_batch_dev(calls, stream=st)
        kernels.sync(st)
        outs.append([c[3].cpu().numpy().copy() for c in calls])
    for got, again, (x, q, s) in zip(outs[0], outs[1], host):
        assert np.array_equal(got.view(np.uint32), again.view(np.uint32))
        ref = oracle.gemm_nt_int8(x, q, s, nt=NT)
        assert np.array_equal(np.isnan(got), np.isnan(ref)) and np.array_equal(np.isinf(got), np.isinf(ref))
        fin = np.isfinite(ref).all(axis=1)
        assert oracle.max_rel_err(np.ascontiguousarray(got[fin]), np.ascontiguousarray(ref[fin])) <= TIGHT_Q8


def test_q8_batch_equal_share_uneven_magnitudes_across_k(kernels, oracle):
    """One token, a decoder layer's seven linears as one batch (equal shares per
    CTA, each segment of a row with its own exponent): rows whose magnitudes
    differ by 2^40 along K. A segment over the small part gets an exponent 40
    larger; the f64 partials are then no longer on one grid and their sum may
    round in the last bits depending on the order of the atomic adds, but the
    result stays within the Q8 bound of the reference."""
    import torch
    m = 1
    calls, host = _batch(oracle, m, C3_SHAPES, seed=77)
    for (dx, _, _, _, _, _, k), (x, _, _) in zip(calls, host):
        x[:, : k // 2] *= np.float32(2.0 ** -40)
        dx.copy_(torch.from_numpy(x))
    st = torch.cuda.current_stream()
    kernels.gemm_nt_int8_batch_dev(calls, stream=st)
    kernels.sync(st)
    for (dx, dq, ds, dc, m_, n, k), (x, q, s) in zip(calls, host):
        ref = oracle.gemm_nt_int8(x, q, s, nt=NT)
        assert oracle.max_rel_err(dc.cpu().numpy(), ref) <= TIGHT_Q8, (n, k)
