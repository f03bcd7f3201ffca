"""Python handle on the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Loads oracle/_build/libvmlm_oracle.so (built by oracle/Makefile) and wraps its
functions for numpy arrays. Only tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py use this module; the product library never does.

Each wrapper names the reference function it restates (paths inside the
shouzugzs-AI/Sparrow tree); the C file holds the arithmetic.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libvmlm_oracle.so")

_lib = None


def build() -> None:
    """Compile the oracle with its Makefile (gcc, -mavx2 -mfma -ffp-contract=off)."""
    subprocess.check_call(["make", "-s", "-C", HERE])


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, S, I, U64, F = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_uint64, ctypes.c_float
        sig = {
            "oracle_gemm_nt_int8": [P, P, P, P, S, S, S],
            "oracle_gemm_nt_int8_scalar": [P, P, P, P, S, S, S],
            "oracle_gemm_nt_bf16": [P, P, P, S, S, S],
            "oracle_gemm_naive_f32": [P, P, P, S, S, S],
            "oracle_gemm_i8i8": [P, P, P, P, P, S, S, S],
            "oracle_gemm_nt_int8_par": [P, P, P, P, S, S, S, I],
            "oracle_gemm_nt_bf16_par": [P, P, P, S, S, S, I],
            "oracle_gemm_i8i8_par": [P, P, P, P, P, S, S, S, I],
            "oracle_gemm_nt_f32_par": [P, P, P, S, S, S, I, I],
            "oracle_gemm_f32_par": [P, P, P, S, S, S, I, I],
            "oracle_rmsnorm": [P, P, P, S, S, F],
            "oracle_gemv_f32": [P, P, P, S, S],
            "oracle_fill_uniform": [P, S, U64, F, I],
            "oracle_fill_normal": [P, S, U64, F, I],
            "oracle_fill_gauss_ref": [P, S, U64, F, I],
            "oracle_fill_int8": [P, S, U64, I],
            "oracle_fill_gauss_k": [P, S, U64, F, I],
            "oracle_quant_int4_grouped": [P, S, S, S, P, P],
            "oracle_gemm_nt_int4_gs": [P, P, P, P, S, S, S, S, I],
            "oracle_gemm_nt_int8_outlier": [P, P, P, P, P, S, P, S, S, S],
            "oracle_quant_int8": [P, S, S, P, P, I],
            "oracle_f32_to_bf16_n": [P, P, S],
            "oracle_bf16_to_f32_n": [P, P, S],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = None
        L.oracle_emb.argtypes = [P, I, S, S, P, S, P]
        L.oracle_emb.restype = I
        L.oracle_quant_int8_outliers.argtypes = [P, S, S, F, P, P, P]
        L.oracle_quant_int8_outliers.restype = S
        L.oracle_max_rel_err.argtypes = [P, P, S]
        L.oracle_max_rel_err.restype = ctypes.c_double
        _lib = L
    return _lib


def _p(x: np.ndarray):
    assert x.flags["C_CONTIGUOUS"]
    return ctypes.c_void_p(x.ctypes.data)


def _threads(nt):
    return (os.cpu_count() or 1) if nt is None else nt


# ---------------------------------------------------------------- kernels

def gemm_nt_int8(a, q, scale, nt=1):
    """ops/src/kernels.rs:1256-1287: C[M,N] = (A[M,K] . f32(q[N,K])^T) * scale[N]."""
    a = np.ascontiguousarray(a, np.float32)
    q = np.ascontiguousarray(q, np.int8)
    scale = np.ascontiguousarray(scale, np.float32)
    m, k = a.shape
    n = q.shape[0]
    assert q.shape == (n, k) and scale.shape[0] >= n
    c = np.empty((m, n), np.float32)
    lib().oracle_gemm_nt_int8_par(_p(a), _p(q), _p(scale), _p(c), m, n, k, nt)
    return c


def gemm_nt_int8_scalar(a, q, scale):
    """ops/src/kernels.rs:1289-1305 (non-x86 sequential fallback)."""
    a = np.ascontiguousarray(a, np.float32)
    q = np.ascontiguousarray(q, np.int8)
    scale = np.ascontiguousarray(scale, np.float32)
    m, k = a.shape
    n = q.shape[0]
    c = np.empty((m, n), np.float32)
    lib().oracle_gemm_nt_int8_scalar(_p(a), _p(q), _p(scale), _p(c), m, n, k)
    return c


def gemm_nt_bf16(a, b_bits, nt=1):
    """ops/src/kernels.rs:1199-1227: C[M,N] = A[M,K] . widen(B_bf16[N,K])^T."""
    a = np.ascontiguousarray(a, np.float32)
    b_bits = np.ascontiguousarray(b_bits, np.uint16)
    m, k = a.shape
    n = b_bits.shape[0]
    assert b_bits.shape == (n, k)
    c = np.empty((m, n), np.float32)
    lib().oracle_gemm_nt_bf16_par(_p(a), _p(b_bits), _p(c), m, n, k, nt)
    return c


def gemm_naive_f32(a, b):
    """tests/src/main.rs:283-295: naive sequential f32 NT GEMM."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m, k = a.shape
    n = b.shape[0]
    c = np.empty((m, n), np.float32)
    lib().oracle_gemm_naive_f32(_p(a), _p(b), _p(c), m, n, k)
    return c


def gemm_nt_f32(a, b, c=None, nt=1):
    """ops/src/kernels.rs:947-967 (gemm_nt_scalar): C[M,N] = A[M,K] . B[N,K]^T, plus the
    old C (one add per element) when c is given (acc)."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m, k = a.shape
    n = b.shape[0]
    assert b.shape == (n, k)
    out = np.array(c, np.float32, order="C", copy=True) if c is not None else np.empty((m, n), np.float32)
    lib().oracle_gemm_nt_f32_par(_p(a), _p(b), _p(out), m, n, k, int(c is not None), _threads(nt))
    return out


def gemm_f32(a, b, c=None, nt=1):
    """ops/src/kernels.rs:383-403 (gemm_scalar, which gemm at :407-419 calls): C[M,N] =
    A[M,K] . B[K,N], plus the old C when c is given (acc)."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m, k = a.shape
    n = b.shape[1]
    assert b.shape == (k, n)
    out = np.array(c, np.float32, order="C", copy=True) if c is not None else np.empty((m, n), np.float32)
    lib().oracle_gemm_f32_par(_p(a), _p(b), _p(out), m, n, k, int(c is not None), _threads(nt))
    return out


def rmsnorm(x, g, eps):
    """ops/src/kernels.rs:1346-1370: per row x * (1 / sqrt(mean(x^2) + eps)) * g."""
    x = np.ascontiguousarray(x, np.float32)
    g = np.ascontiguousarray(g, np.float32)
    rows, cols = x.shape
    out = np.empty_like(x)
    lib().oracle_rmsnorm(_p(out), _p(x), _p(g), rows, cols, float(eps))
    return out


def gemv_f32(a, b):
    """core/src/interp.rs:815-827 (OP_GEMV): c[i] = sum_p a[i, p] * b[p], sequential."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m, k = a.shape
    c = np.empty(m, np.float32)
    lib().oracle_gemv_f32(_p(a), _p(b), _p(c), m, k)
    return c


def emb(table, idx):
    """core/src/interp.rs:1351-1420 (OP_EMB) for every index: (status, out); status 1 = row index out
    of range, 2 = not an integer (where the VM exits 9)."""
    rows, cols = table.shape
    table = np.ascontiguousarray(table)
    idx = np.ascontiguousarray(idx, np.float32)
    out = np.zeros((idx.size, cols), np.float32)
    st = lib().oracle_emb(_p(table), 4 if table.dtype == np.uint16 else 0, rows, cols, _p(idx), idx.size, _p(out))
    return st, out


def gemm_i8i8(x, w, scale, nt=1, want_acc=True):
    """Exact int8 x int8 -> int32 GEMM, then float(acc) * scale[n] (no reference kernel)."""
    x = np.ascontiguousarray(x, np.int8)
    w = np.ascontiguousarray(w, np.int8)
    scale = np.ascontiguousarray(scale, np.float32)
    m, k = x.shape
    n = w.shape[0]
    c = np.empty((m, n), np.float32)
    acc = np.empty((m, n), np.int32) if want_acc else None
    lib().oracle_gemm_i8i8_par(_p(x), _p(w), _p(scale), _p(acc) if want_acc else None,
                               _p(c), m, n, k, nt)
    return (c, acc) if want_acc else c


# ------------------------------------------------------------- generators

def fill_normal(n, seed, sigma, nt=None):
    """N(0, sigma): Box-Muller with full-range uniforms on the reference lcg (configuration inputs)."""
    out = np.empty(n, np.float32)
    lib().oracle_fill_normal(_p(out), n, seed, sigma, _threads(nt))
    return out


def fill_gauss_ref(n, seed, sigma, nt=None):
    """The reference's Box-Muller as written (tests/src/quant.rs:605-613): lcg() lies in
    [-1, 0), so the values are not N(0,1) (std ~1.30 * sigma)."""
    out = np.empty(n, np.float32)
    lib().oracle_fill_gauss_ref(_p(out), n, seed, sigma, _threads(nt))
    return out


def fill_uniform(n, seed, scale, nt=None):
    """rnd(n, seed, scale) of tests/src/quant.rs:52-55 (values lie in [-scale, 0))."""
    out = np.empty(n, np.float32)
    lib().oracle_fill_uniform(_p(out), n, seed, scale, _threads(nt))
    return out


def fill_gauss_k(n, seed, k, nt=None):
    """The quantisation benchmark's weights (tests/src/quant.rs:595-602): the reference
    Box-Muller divided by sqrt(k)."""
    out = np.empty(n, np.float32)
    lib().oracle_fill_gauss_k(_p(out), n, seed, float(np.sqrt(np.float32(k), dtype=np.float32)), _threads(nt))
    return out


def quant_weights_with_outlier_channels(n, k):
    """tests/src/quant.rs:595-609: fill_gauss_k (seed 0xDEADBEEF), then every 64th
    column (0, 64, ...) times 12."""
    w = fill_gauss_k(n * k, 0xDEADBEEF, k).reshape(n, k)
    w[:, ::64] *= np.float32(12.0)
    return w


def quant_int4_grouped(w, group):
    """tests/src/quant.rs:114-152 -> (packed uint8 [n, (k+1)//2], scale f32 [n, ceil(k/group)])."""
    w = np.ascontiguousarray(w, np.float32)
    n, k = w.shape
    packed = np.empty((n, (k + 1) // 2), np.uint8)
    scale = np.empty((n, (k + group - 1) // group), np.float32)
    lib().oracle_quant_int4_grouped(_p(w), n, k, group, _p(packed), _p(scale))
    return packed, scale


def gemm_nt_int4_gs(a, packed, scale, k, group, order=0):
    """tests/src/quant.rs:298-362: order 1 = the AVX2 step as shipped, order 0 = the
    same arithmetic on the packer's nibble order."""
    a = np.ascontiguousarray(a, np.float32)
    m = a.shape[0]
    n = packed.shape[0]
    c = np.empty((m, n), np.float32)
    lib().oracle_gemm_nt_int4_gs(_p(a), _p(np.ascontiguousarray(packed, np.uint8)),
                                 _p(np.ascontiguousarray(scale, np.float32)), _p(c), m, n, k, group, int(order))
    return c


def quant_int8_outliers(w, thresh):
    """tests/src/quant.rs:458-515 -> (q int8 [n,k], scale f32 [n], outlier column indices uint32)."""
    w = np.ascontiguousarray(w, np.float32)
    n, k = w.shape
    q = np.empty((n, k), np.int8)
    s = np.empty(n, np.float32)
    idx = np.empty(max(k, 1), np.uint32)
    cnt = lib().oracle_quant_int8_outliers(_p(w), n, k, thresh, _p(q), _p(s), _p(idx))
    assert cnt <= k
    return q, s, idx[:cnt].copy()


def gemm_nt_int8_outlier(a, q, scale, w, idx):
    """tests/src/quant.rs:524-565: the int8 body times scale, plus a[jj] * w[j][jj] per outlier."""
    a = np.ascontiguousarray(a, np.float32)
    m, k = a.shape
    n = q.shape[0]
    c = np.empty((m, n), np.float32)
    idx = np.ascontiguousarray(idx, np.uint32)
    lib().oracle_gemm_nt_int8_outlier(_p(a), _p(np.ascontiguousarray(q, np.int8)),
                                      _p(np.ascontiguousarray(scale, np.float32)),
                                      _p(np.ascontiguousarray(w, np.float32)), _p(idx), idx.size, _p(c), m, n, k)
    return c


def fill_int8(n, seed, nt=None):
    """Uniform int8 in [-127,127] from the same lcg: ((s>>33) % 255) - 127."""
    out = np.empty(n, np.int8)
    lib().oracle_fill_int8(_p(out), n, seed, _threads(nt))
    return out


def quant_int8(w, nt=None):
    """tests/src/quant.rs:78-104: per-row absmax/127 scale, round half away, clamp +-127."""
    w = np.ascontiguousarray(w, np.float32)
    n, k = w.shape
    q = np.empty((n, k), np.int8)
    s = np.empty(n, np.float32)
    lib().oracle_quant_int8(_p(w), n, k, _p(q), _p(s), _threads(nt))
    return q, s


def f32_to_bf16(x):
    """tensor/src/dtype.rs:38-45 (round to nearest even, high 16 bits)."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().oracle_f32_to_bf16_n(_p(x), _p(out), x.size)
    return out


def bf16_to_f32(h):
    """tensor/src/dtype.rs:47-51 (exact widening)."""
    h = np.ascontiguousarray(h, np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().oracle_bf16_to_f32_n(_p(h), _p(out), h.size)
    return out


def max_rel_err(got, ref):
    """max|got-ref| / max|ref| (tests/src/quant.rs:381-418 convention)."""
    got = np.ascontiguousarray(got, np.float32)
    ref = np.ascontiguousarray(ref, np.float32)
    assert got.size == ref.size
    return lib().oracle_max_rel_err(_p(got), _p(ref), got.size)


def print_f32(values):
    """The engine's truncating printer (core/src/interp.rs:2416-2473), in f32 arithmetic."""
    out = []
    for v in np.asarray(values, np.float32).ravel():
        neg = v < np.float32(0.0)
        av = np.float32(-v if neg else v)
        ip = int(av)
        s = ("-" if neg else "") + str(ip) + "."
        frac = np.float32(av - np.float32(ip))
        for _ in range(6):
            frac = np.float32(frac * np.float32(10.0))
            dig = int(frac)
            s += str(dig % 10)
            frac = np.float32(frac - np.float32(dig))
        out.append(s)
    return " ".join(out)
