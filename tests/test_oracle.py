"""CPU tests: pin the oracle to the reference's golden vectors and known answers.

The oracle (oracle/vmlm_oracle.c) restates the reference kernels; these tests
check it against every fixture and recorded output the reference holds for the
Q8/bf16 GEMM path (fixtures copied by tests/golden/make_golden.py).
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN


def _f32(path, shape=None):
    a = np.fromfile(os.path.join(GOLDEN, path), "<f4")
    return a.reshape(shape) if shape else a


def _i8(path, shape):
    return np.fromfile(os.path.join(GOLDEN, path), "i1").reshape(shape)


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLDEN, "golden.json")) as f:
        return json.load(f)


# ---------------------------------------------------------- tools/p13_q8_check.py

def test_p13_q8_known_answer(oracle, golden):
    a = _f32("p13/q8_a.f32", (1, 4))
    w = _i8("p13/q8_w.i8", (2, 4))
    s = _f32("p13/q8_scale.f32")
    c = oracle.gemm_nt_int8(a, w, s)
    assert c.ravel().tolist() == golden["p13_q8"]["expected"]
    # the non-x86 fallback gives the same answer
    assert oracle.gemm_nt_int8_scalar(a, w, s).ravel().tolist() == golden["p13_q8"]["expected"]


# ------------------------------------------------- sparrow/tools/int8_ab.ps1 criteria 1-4

def _linear_i8(d, tag, x, kin):
    q = _i8(f"{d}/{tag}_Wq.bin", (4, kin))
    s = _f32(f"{d}/{tag}_scale.bin")
    b = _f32(f"{d}/{tag}_b.bin")
    return _oracle().gemm_nt_int8(x, q, s) + b


def _linear_f32(d, tag, x, kin):
    w = _f32(f"{d}/{tag}_W.bin", (4, kin))
    b = _f32(f"{d}/{tag}_b.bin")
    return _oracle().gemm_naive_f32(x, w) + b


def _oracle():
    from oracle import oracle as O
    return O


def _printed_diff(u, v):
    O = _oracle()
    return max(abs(float(p) - float(q)) for p, q in zip(O.print_f32(u).split(), O.print_f32(v).split()))


def test_int8_k1_prints_identical(oracle, golden):
    x = _f32("int8_bins/i8o_in.bin", (1, 1))
    got_i8 = _linear_i8("int8_bins", "o", x, 1)
    got_f32 = _linear_f32("int8_bins", "o", x, 1)
    assert oracle.print_f32(got_i8) == golden["int8_one_k1"]["printed"]
    assert oracle.print_f32(got_f32) == golden["int8_one_k1"]["printed"]


def _two(d, x, lin):
    return lin(d, "b", lin(d, "a", x, 4), 4)


def test_int8_k4_exact_set(golden):
    x = _f32("int8_bins/i8t_in.bin", (1, 4))
    d = _printed_diff(_two("int8_bins", x, _linear_i8), _two("int8_bins", x, _linear_f32))
    assert d <= golden["int8_two_k4_exact"]["max_diff_bound"]
    assert d == golden["int8_two_k4_exact"]["measured"]


def test_int8_bad_scale_can_fail(golden):
    x = _f32("int8_bins/i8t_in.bin", (1, 4))
    d = _printed_diff(_two("int8_bad_bins", x, _linear_i8), _two("int8_bins", x, _linear_f32))
    assert abs(d - golden["int8_two_bad_scale"]["max_diff"]) < 2e-6


def test_int8_naive_quantisation_control(golden):
    x = _f32("int8_naive_bins/i8t_in.bin", (1, 4))
    d = _printed_diff(_two("int8_naive_bins", x, _linear_i8), _two("int8_naive_bins", x, _linear_f32))
    assert abs(d - golden["int8_two_naive"]["max_diff"]) < 2e-6


def test_quantiser_reproduces_naive_bins(oracle):
    for tag in ("a", "b"):
        w = _f32(f"int8_naive_bins/{tag}_W.bin", (4, 4))
        q, s = oracle.quant_int8(w)
        assert np.array_equal(q, _i8(f"int8_naive_bins/{tag}_Wq.bin", (4, 4)))
        assert np.array_equal(s, _f32(f"int8_naive_bins/{tag}_scale.bin"))


# ------------------------------------------------------------- bf16 fixtures

def test_bf16_widen_matches_truncated_f32(oracle, golden):
    for fn in golden["bf16_widen"]["files"]:
        bits = np.fromfile(os.path.join(GOLDEN, "bf16_bins_bf16", fn), "<u2")
        f32 = _f32(f"bf16_bins_f32/{fn}")
        assert np.array_equal(oracle.bf16_to_f32(bits).view(np.uint32), f32.view(np.uint32))


def test_bf16_kernel_vs_widened_f32(oracle):
    # tests/src/bf16.rs:211-271: M=4, N=K=512, a = rnd(.,0xAA,0.5), w = rnd(.,0xBB,1/sqrt(k)),
    # bf16 kernel vs f32 GEMM on the widened weights within 1e-5 * max|ref|.
    m, n, k = 4, 512, 512
    a = oracle.fill_uniform(m * k, 0xAA, 0.5).reshape(m, k)
    w = oracle.fill_uniform(n * k, 0xBB, 1.0 / np.sqrt(k)).reshape(n, k)
    wb = oracle.f32_to_bf16(w)
    ref = oracle.gemm_naive_f32(a, oracle.bf16_to_f32(wb))
    got = oracle.gemm_nt_bf16(a, wb)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()


# --------------------------------------------------------------- regressions

EDGE_SHAPES = [  # tests/src/main.rs:338-342
    (4, 8, 8), (1, 1, 64), (1, 32, 64), (1, 10, 32), (8, 8, 512), (512, 512, 512), (3, 5, 7),
    (5, 3, 9), (17, 23, 31), (64, 64, 64), (16, 1, 16), (1, 16, 16), (16, 16, 1),
]


def edge_inputs(m, n, k):
    """Deterministic inputs of tests/src/main.rs:298-299."""
    a = (((np.arange(m * k) * 37) % 100).astype(np.float32) / 50.0 - 1.0).reshape(m, k)
    b = (((np.arange(n * k) * 53) % 100).astype(np.float32) / 50.0 - 1.0).reshape(n, k)
    return a.astype(np.float32), b.astype(np.float32)


@pytest.mark.parametrize("m,n,k", EDGE_SHAPES)
def test_edge_shapes_int8_and_bf16_vs_naive(oracle, m, n, k):
    a, b = edge_inputs(m, n, k)
    q, s = oracle.quant_int8(b)
    deq = (q.astype(np.float32) * s[:, None]).astype(np.float32)
    ref = oracle.gemm_naive_f32(a, deq)
    got = oracle.gemm_nt_int8(a, q, s)
    # int8 scale is applied after the dot product: a different rounding order only
    assert np.abs(got - ref).max() < 1e-3 * max(1.0, np.abs(ref).max())
    wb = oracle.f32_to_bf16(b)
    refb = oracle.gemm_naive_f32(a, oracle.bf16_to_f32(wb))
    assert np.abs(oracle.gemm_nt_bf16(a, wb) - refb).max() < 1e-3


def test_scalar_fallback_close_to_avx2(oracle):
    m, n, k = 3, 17, 301
    a = oracle.fill_normal(m * k, 5, 1.0).reshape(m, k)
    q, s = oracle.quant_int8(oracle.fill_normal(n * k, 6, 0.02).reshape(n, k))
    assert oracle.max_rel_err(oracle.gemm_nt_int8_scalar(a, q, s), oracle.gemm_nt_int8(a, q, s)) < 1e-5


def test_parallel_split_is_bitwise_identical(oracle):
    m, n, k = 5, 257, 300
    a = oracle.fill_normal(m * k, 7, 1.0).reshape(m, k)
    q, s = oracle.quant_int8(oracle.fill_normal(n * k, 8, 0.02).reshape(n, k))
    one = oracle.gemm_nt_int8(a, q, s, nt=1)
    many = oracle.gemm_nt_int8(a, q, s, nt=7)
    assert np.array_equal(one.view(np.uint32), many.view(np.uint32))


def test_generator_threads_share_one_stream(oracle):
    g1 = oracle.fill_normal(10007, 42, 0.02, nt=1)
    g8 = oracle.fill_normal(10007, 42, 0.02, nt=8)
    assert np.array_equal(g1.view(np.uint32), g8.view(np.uint32))
    u1 = oracle.fill_int8(9999, 3, nt=1)
    u8 = oracle.fill_int8(9999, 3, nt=5)
    assert np.array_equal(u1, u8)
    assert u1.min() >= -127 and u1.max() <= 127


def test_generator_first_values_follow_reference_lcg(oracle):
    # lcg of tests/src/quant.rs:48-51, computed here in Python integers
    s, out = 0xAA, []
    for _ in range(4):
        s = (s * 6364136223846793005 + 1442695040888963407) % (1 << 64)
        out.append(np.float32(np.float32(s >> 33) / np.float32(2 ** 31)) - np.float32(1.0))
    got = oracle.fill_uniform(4, 0xAA, 1.0, nt=1)
    assert np.array_equal(got, np.array(out, np.float32))


def test_normal_statistics(oracle):
    g = oracle.fill_normal(400000, 0, 1.0)
    assert abs(float(g.mean())) < 0.01 and abs(float(g.std()) - 1.0) < 0.01
    assert abs(float(np.mean(g ** 4)) - 3.0) < 0.1  # Gaussian kurtosis


def test_reference_generator_quirk_is_restated(oracle):
    # lcg() of tests/src/quant.rs:48-51 lies in [-1, 0): rnd() is all negative and the
    # reference Box-Muller radius is at least sqrt(2 ln 2).
    u = oracle.fill_uniform(100000, 0xBB, 1.0)
    assert u.max() < 0.0 and u.min() >= -1.0
    g = oracle.fill_gauss_ref(100000, 0xDEADBEEF, 1.0)
    assert abs(float(g.std()) - 1.30) < 0.02


def test_i8i8_oracle_exact(oracle):
    m, n, k = 7, 33, 1000
    x = oracle.fill_int8(m * k, 1).reshape(m, k)
    w = oracle.fill_int8(n * k, 2).reshape(n, k)
    s = np.abs(oracle.fill_normal(n, 3, 0.02)) + np.float32(1e-3)
    c, acc = oracle.gemm_i8i8(x, w, s)
    ref = x.astype(np.int64) @ w.astype(np.int64).T
    assert np.array_equal(acc, ref.astype(np.int32))
    assert np.array_equal(c, (ref.astype(np.float32) * s[None, :]).astype(np.float32))


@pytest.mark.parametrize("m,n,k", EDGE_SHAPES)
def test_f32_gemm_restatements_match_the_reference_naive_loop(oracle, m, n, k):
    # gemm_nt_scalar (ops/src/kernels.rs:947-967) sums in the order of the
    # reference test's naive loop (tests/src/main.rs:283-295): bit-identical;
    # gemm_scalar (NN, :383-403) on B^T too; acc adds the old C once
    a, b = edge_inputs(m, n, k)
    ref = oracle.gemm_naive_f32(a, b)
    got = oracle.gemm_nt_f32(a, b)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    got_nn = oracle.gemm_f32(a, np.ascontiguousarray(b.T))
    assert np.array_equal(got_nn.view(np.uint32), ref.view(np.uint32))
    c0 = (np.arange(m * n, dtype=np.float32).reshape(m, n) % 7) - 3.0
    got_acc = oracle.gemm_nt_f32(a, b, c0)
    assert np.array_equal(got_acc.view(np.uint32), (ref + c0).astype(np.float32).view(np.uint32))
