"""Python mirror of `vmlm_ops::kernels` for the quantised-linear path.

Same operator names, argument order and meaning as the reference
(ops/src/kernels.rs in the shouzugzs-AI/Sparrow tree):

    gemm_nt_int8(a, q, scale, c, m, n, k)   ops/src/kernels.rs:1256-1287
    gemm_nt_bf16(a, b, c, m, n, k)          ops/src/kernels.rs:1199-1227

`a`, `q`/`b`, `scale` and `c` are host buffers (numpy arrays, contiguous, of
the stated element type and at least the stated length); `c` is overwritten.
The reference kernels check nothing and the VM calls exit(9) on misuse
(core/src/interp.rs:752-806); here a bad argument raises VmlmError (or
ValueError for a Python-side type or size mismatch) before any GPU work.

The `_dev` variants take device buffers: torch CUDA tensors (or raw device
addresses as ints) and an optional CUDA stream, and return without waiting.
"""
import ctypes

import numpy as np

from ._lib import Slot, check, lib


def _host_ptr(x, dtype, count, name):
    if not isinstance(x, np.ndarray):
        raise ValueError(f"{name}: expected a numpy array, got {type(x).__name__}")
    if x.dtype != dtype:
        raise ValueError(f"{name}: expected {np.dtype(dtype).name}, got {x.dtype.name}")
    if not x.flags["C_CONTIGUOUS"]:
        raise ValueError(f"{name}: must be C-contiguous")
    if x.size < count:
        raise ValueError(f"{name}: needs {count} elements, has {x.size}")
    return ctypes.c_void_p(x.ctypes.data) if x.size else None


def _dev_ptr(x, dtype_name, count, name):
    if x is None:
        return None
    if isinstance(x, int):
        return ctypes.c_void_p(x)
    if not getattr(x, "is_cuda", False):
        raise ValueError(f"{name}: expected a CUDA tensor or a device address")
    if str(x.dtype) != f"torch.{dtype_name}":
        raise ValueError(f"{name}: expected torch.{dtype_name}, got {x.dtype}")
    if not x.is_contiguous():
        raise ValueError(f"{name}: must be contiguous")
    if x.numel() < count:
        raise ValueError(f"{name}: needs {count} elements, has {x.numel()}")
    return ctypes.c_void_p(x.data_ptr())


CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy: the legacy default stream


def _stream_ptr(stream):
    """None -> the library's own stream. A torch stream whose handle is 0 is the
    legacy default stream, which the C ABI must receive as cudaStreamLegacy
    (a NULL handle there selects the library stream)."""
    if stream is None:
        return None
    h = stream if isinstance(stream, int) else stream.cuda_stream
    return ctypes.c_void_p(h if h else CUDA_STREAM_LEGACY)


# ------------------------------------------------------------------ setup

def init(device: int = 0) -> None:
    """Select the device for the host-pointer entry points (creates its context)."""
    check(lib().vmlm_init(device))


def shutdown() -> None:
    check(lib().vmlm_shutdown())


def register_weight(w: np.ndarray) -> None:
    """Keep a device copy of an immutable host weight (or scale) array."""
    if not isinstance(w, np.ndarray) or not w.flags["C_CONTIGUOUS"]:
        raise ValueError("register_weight: expected a C-contiguous numpy array")
    check(lib().vmlm_register_weight(ctypes.c_void_p(w.ctypes.data), w.nbytes))


def unregister_weight(w: np.ndarray) -> None:
    check(lib().vmlm_unregister_weight(ctypes.c_void_p(w.ctypes.data)))


def unregister_all() -> None:
    check(lib().vmlm_unregister_all())


def sync(stream=None) -> None:
    check(lib().vmlm_sync(_stream_ptr(stream)))


def launch_count() -> int:
    return int(lib().vmlm_launch_count())


def probe_mma_peak(kind: str, iters: int):
    """Dense tensor-core rate of the current device from back-to-back tcgen05.mma
    on shared-memory operands: kind "bf16" (kind::f16) or "int8" (kind::i8).
    Returns (TFLOP/s or TOP/s, kernel ms)."""
    code = {"bf16": 0, "int8": 1}[kind]
    tops, ms = ctypes.c_double(), ctypes.c_double()
    check(lib().vmlm_probe_mma_peak(code, int(iters), ctypes.byref(tops), ctypes.byref(ms)))
    return tops.value, ms.value


def profile_enable(on: bool) -> None:
    """Bracket each tensor-core GEMM launch with CUDA events (diagnostics)."""
    check(lib().vmlm_profile_enable(1 if on else 0))


def trace_enable(max_ctas: int) -> None:
    """Record per-CTA phase timestamps of each GEMM launch (0 disables)."""
    check(lib().vmlm_trace_enable(max_ctas))


def trace_take(n_ctas: int) -> np.ndarray:
    """The last traced launch: [n_ctas, 16] values (8 globaltimer stamps, 4 summed waits and
    3 summed split-tile phases in ns, then items * 65536 + tiles finished)."""
    out = np.zeros((n_ctas, 16), np.uint64)
    check(lib().vmlm_trace_take(ctypes.c_void_p(out.ctypes.data), out.size))
    return out


def profile_take():
    """(summed device ms, launches) of the GEMM launches recorded since the last take."""
    ms = ctypes.c_double(0.0)
    n = ctypes.c_uint64(0)
    check(lib().vmlm_profile_take(ctypes.byref(ms), ctypes.byref(n)))
    return ms.value, n.value


def profile_kernel() -> str:
    """Kernel and tile plan of the last profiled GEMM launch."""
    buf = ctypes.create_string_buffer(256)
    check(lib().vmlm_profile_kernel(buf, len(buf)))
    return buf.value.decode()


# ------------------------------------------------------- reference operators

def gemm_nt_int8(a, q, scale, c, m, n, k) -> None:
    """C[M,N] = (A[M,K] . f32(q[N,K])^T) * scale[N]  (ops/src/kernels.rs:1256-1287)."""
    check(lib().vmlm_gemm_nt_int8(
        _host_ptr(a, np.float32, m * k, "a"), _host_ptr(q, np.int8, n * k, "q"),
        _host_ptr(scale, np.float32, n, "scale"), _host_ptr(c, np.float32, m * n, "c"), m, n, k))


def gemm_nt_bf16(a, b, c, m, n, k) -> None:
    """C[M,N] = A[M,K] . widen(B_bf16[N,K])^T  (ops/src/kernels.rs:1199-1227); b holds bf16 bits as uint16."""
    check(lib().vmlm_gemm_nt_bf16(
        _host_ptr(a, np.float32, m * k, "a"), _host_ptr(b, np.uint16, n * k, "b"),
        _host_ptr(c, np.float32, m * n, "c"), m, n, k))


def gemm_i8i8(x, w, scale, c, acc, m, n, k) -> None:
    """int8 x int8 -> exact int32 acc[M,N]; C = f32(acc) * scale[N]. c or acc may be None."""
    check(lib().vmlm_gemm_i8i8(
        _host_ptr(x, np.int8, m * k, "x"), _host_ptr(w, np.int8, n * k, "w"),
        _host_ptr(scale, np.float32, n, "scale") if c is not None else None,
        _host_ptr(c, np.float32, m * n, "c") if c is not None else None,
        _host_ptr(acc, np.int32, m * n, "acc") if acc is not None else None, m, n, k))


def gemm_nt_f32(a, b, c, m, n, k, acc=False) -> None:
    """C[M,N] = A[M,K] . B[N,K]^T, plus the old C when acc  (ops/src/kernels.rs:987-1015)."""
    check(lib().vmlm_gemm_nt_f32(
        _host_ptr(a, np.float32, m * k, "a"), _host_ptr(b, np.float32, n * k, "b"),
        _host_ptr(c, np.float32, m * n, "c"), m, n, k, int(bool(acc))))


def gemm_f32(a, b, c, m, n, k, acc=False) -> None:
    """C[M,N] = A[M,K] . B[K,N], plus the old C when acc  (ops/src/kernels.rs:383-419)."""
    check(lib().vmlm_gemm_f32(
        _host_ptr(a, np.float32, m * k, "a"), _host_ptr(b, np.float32, k * n, "b"),
        _host_ptr(c, np.float32, m * n, "c"), m, n, k, int(bool(acc))))


# ----------------------------------------------------------- device variants

def gemm_nt_int8_dev(a, q, scale, c, m, n, k, stream=None) -> None:
    check(lib().vmlm_gemm_nt_int8_dev(
        _dev_ptr(a, "float32", m * k, "a"), _dev_ptr(q, "int8", n * k, "q"),
        _dev_ptr(scale, "float32", n, "scale"), _dev_ptr(c, "float32", m * n, "c"), m, n, k,
        _stream_ptr(stream)))


def gemm_nt_int8_dev_noalloc(a, q, scale, c, m, n, k, stream=None) -> None:
    """gemm_nt_int8_dev without any device allocation: its scratch is a fixed
    array inside the library (m <= 16, n <= 131072, k <= 16384). For callers
    that reserve all device memory up front and must not allocate per call.
    Calls that overlap on the GPU share that scratch and race.

    stream=None runs on the CUDA legacy default stream (the C entry point's
    NULL), not on the library stream that None selects for the other *_dev
    calls; pass a stream to order it with other work."""
    st = ctypes.c_void_p(CUDA_STREAM_LEGACY) if stream is None else _stream_ptr(stream)
    check(lib().vmlm_gemm_nt_int8_dev_noalloc(
        _dev_ptr(a, "float32", m * k, "a"), _dev_ptr(q, "int8", n * k, "q"),
        _dev_ptr(scale, "float32", n, "scale"), _dev_ptr(c, "float32", m * n, "c"), m, n, k, st))


def gemm_nt_bf16_dev(a, b, c, m, n, k, stream=None) -> None:
    """b: a bfloat16 (or int16/uint16 bit-pattern) CUDA tensor [n, k]."""
    if b is not None and not isinstance(b, int) and str(b.dtype) in ("torch.int16", "torch.uint16"):
        bptr = _dev_ptr(b, str(b.dtype)[6:], n * k, "b")
    else:
        bptr = _dev_ptr(b, "bfloat16", n * k, "b")
    check(lib().vmlm_gemm_nt_bf16_dev(
        _dev_ptr(a, "float32", m * k, "a"), bptr, _dev_ptr(c, "float32", m * n, "c"), m, n, k,
        _stream_ptr(stream)))


def gemm_i8i8_dev(x, w, scale, c, acc, m, n, k, stream=None) -> None:
    check(lib().vmlm_gemm_i8i8_dev(
        _dev_ptr(x, "int8", m * k, "x"), _dev_ptr(w, "int8", n * k, "w"),
        _dev_ptr(scale, "float32", n, "scale"), _dev_ptr(c, "float32", m * n, "c"),
        _dev_ptr(acc, "int32", m * n, "acc"), m, n, k, _stream_ptr(stream)))


def gemm_nt_f32_dev(a, b, c, m, n, k, acc=False, stream=None) -> None:
    check(lib().vmlm_gemm_nt_f32_dev(
        _dev_ptr(a, "float32", m * k, "a"), _dev_ptr(b, "float32", n * k, "b"),
        _dev_ptr(c, "float32", m * n, "c"), m, n, k, int(bool(acc)), _stream_ptr(stream)))


def gemm_f32_dev(a, b, c, m, n, k, acc=False, stream=None) -> None:
    check(lib().vmlm_gemm_f32_dev(
        _dev_ptr(a, "float32", m * k, "a"), _dev_ptr(b, "float32", k * n, "b"),
        _dev_ptr(c, "float32", m * n, "c"), m, n, k, int(bool(acc)), _stream_ptr(stream)))


# ------------------------------------------------ decode-step neighbours

def rmsnorm_gemm_nt_int8(a, g, eps, q, scale, c, m, n, k) -> None:
    """C = gemm_nt_int8(rmsnorm(a, g, eps), q, scale) (ops/src/kernels.rs:1346-1370, then :1256-1287)."""
    check(lib().vmlm_rmsnorm_gemm_nt_int8(
        _host_ptr(a, np.float32, m * k, "a"), _host_ptr(g, np.float32, k, "g"), float(eps),
        _host_ptr(q, np.int8, n * k, "q"), _host_ptr(scale, np.float32, n, "scale"),
        _host_ptr(c, np.float32, m * n, "c"), m, n, k))


def rmsnorm_gemm_nt_int8_dev(a, g, eps, q, scale, c, m, n, k, stream=None) -> None:
    check(lib().vmlm_rmsnorm_gemm_nt_int8_dev(
        _dev_ptr(a, "float32", m * k, "a"), _dev_ptr(g, "float32", k, "g"), float(eps),
        _dev_ptr(q, "int8", n * k, "q"), _dev_ptr(scale, "float32", n, "scale"),
        _dev_ptr(c, "float32", m * n, "c"), m, n, k, _stream_ptr(stream)))


def gemv_f32(a, b, c, m, k) -> None:
    """OP_GEMV (core/src/interp.rs:815-827): c[i] = sum_p a[i, p] * b[p]."""
    check(lib().vmlm_gemv_f32(_host_ptr(a, np.float32, m * k, "a"), _host_ptr(b, np.float32, k, "b"),
                              _host_ptr(c, np.float32, m, "c"), m, k))


def gemv_f32_dev(a, b, c, m, k, stream=None) -> None:
    check(lib().vmlm_gemv_f32_dev(_dev_ptr(a, "float32", m * k, "a"), _dev_ptr(b, "float32", k, "b"),
                                  _dev_ptr(c, "float32", m, "c"), m, k, _stream_ptr(stream)))


class Pool:
    """A .vmb program's constant pool, scratch regions and slot table in device
    memory (vmlm_pool_*; Vm::load, core/src/interp.rs:123-220)."""

    def __init__(self, image: bytes, weights: bytes = None):
        self._h = ctypes.c_void_p()
        img = bytes(image)
        w = bytes(weights) if weights is not None else None
        check(lib().vmlm_pool_load(img, len(img), w, len(w) if w is not None else 0, ctypes.byref(self._h)))

    def close(self) -> None:
        if self._h:
            check(lib().vmlm_pool_free(self._h))
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def info(self):
        """-> (n_const, n_slots, [const, act, state, grad] bytes)."""
        nc, ns = ctypes.c_size_t(), ctypes.c_size_t()
        rb = (ctypes.c_size_t * 4)()
        check(lib().vmlm_pool_info(self._h, ctypes.byref(nc), ctypes.byref(ns), rb))
        return nc.value, ns.value, list(rb)

    def region(self, r: int) -> int:
        p = ctypes.c_void_p()
        check(lib().vmlm_pool_region(self._h, r, ctypes.byref(p)))
        return p.value or 0

    def slot(self, i: int):
        """-> (device address, rows, cols, dtype, kind)."""
        s, kind = Slot(), ctypes.c_int()
        check(lib().vmlm_pool_slot(self._h, i, ctypes.byref(s), ctypes.byref(kind)))
        return s.ptr or 0, s.rows, s.cols, s.dtype, kind.value

    def layerb(self, delta: float) -> None:
        check(lib().vmlm_pool_layerb(self._h, ctypes.c_float(delta)))

    def layer_base(self) -> int:
        b = ctypes.c_size_t()
        check(lib().vmlm_pool_layer_base(self._h, ctypes.byref(b)))
        return b.value

    def find_const(self, name: str) -> int:
        i = ctypes.c_size_t()
        check(lib().vmlm_pool_find_const(self._h, name.encode(), ctypes.byref(i)))
        return i.value

    def find_slot(self, name: str) -> int:
        i = ctypes.c_size_t()
        check(lib().vmlm_pool_find_slot(self._h, name.encode(), ctypes.byref(i)))
        return i.value

    def gemm(self, ins: bytes, stream=None) -> None:
        """Run one 16-byte OP_GEMM instruction on the pool's slots."""
        assert len(ins) == 16
        check(lib().vmlm_pool_gemm(self._h, ins, _stream_ptr(stream)))


class Q8Call(ctypes.Structure):
    """vmlm_q8_call: one Q8 call of a batch (device pointers)."""
    _fields_ = [("a", ctypes.c_void_p), ("q", ctypes.c_void_p), ("scale", ctypes.c_void_p), ("c", ctypes.c_void_p),
                ("m", ctypes.c_size_t), ("n", ctypes.c_size_t), ("k", ctypes.c_size_t)]


def gemm_nt_int8_batch_dev(calls, stream=None) -> None:
    """Independent Q8 calls [(a, q, scale, c, m, n, k), ...] on CUDA tensors, as one grouped launch where they fit."""
    arr = (Q8Call * len(calls))()
    for i, (a, q, s, c, m, n, k) in enumerate(calls):
        arr[i] = Q8Call(_dev_ptr(a, "float32", m * k, "a"), _dev_ptr(q, "int8", n * k, "q"),
                        _dev_ptr(s, "float32", n, "scale"), _dev_ptr(c, "float32", m * n, "c"), m, n, k)
    check(lib().vmlm_gemm_nt_int8_batch_dev(arr, len(calls), _stream_ptr(stream)))


def set_host_pipeline(max_chunks: int) -> None:
    """Most row chunks a large host-pointer call is pipelined in (1 = off, 0 = default)."""
    check(lib().vmlm_set_host_pipeline(int(max_chunks)))


def gemm_nt_int4_gs(a, packed, scale, c, m, n, k, group, order=0) -> None:
    """int4 weights, a scale per group of columns (tests/src/quant.rs:298-362); packed
    [n, (k+1)//2] uint8, scale [n, ceil(k/group)]; order 1 = the AVX2 step as shipped."""
    gpr = (k + group - 1) // group if group else 0
    check(lib().vmlm_gemm_nt_int4_gs(
        _host_ptr(a, np.float32, m * k, "a"), _host_ptr(packed, np.uint8, n * ((k + 1) // 2), "packed"),
        _host_ptr(scale, np.float32, n * gpr, "scale"), _host_ptr(c, np.float32, m * n, "c"),
        m, n, k, group, int(order)))


def gemm_nt_int4_gs_dev(a, packed, scale, c, m, n, k, group, order=0, stream=None) -> None:
    gpr = (k + group - 1) // group if group else 0
    check(lib().vmlm_gemm_nt_int4_gs_dev(
        _dev_ptr(a, "float32", m * k, "a"), _dev_ptr(packed, "uint8", n * ((k + 1) // 2), "packed"),
        _dev_ptr(scale, "float32", n * gpr, "scale"), _dev_ptr(c, "float32", m * n, "c"),
        m, n, k, group, int(order), _stream_ptr(stream)))


def _idx_dev_ptr(idx, count):
    if idx is None or isinstance(idx, int):
        return _dev_ptr(idx, "int32", count, "idx")
    return _dev_ptr(idx, "uint32" if str(idx.dtype) == "torch.uint32" else "int32", count, "idx")


def gemm_nt_int8_outlier(a, q, scale, w, idx, c, m, n, k) -> None:
    """int8 plus f32 outlier columns (tests/src/quant.rs:524-565); idx uint32 column indices."""
    idx = np.ascontiguousarray(idx, np.uint32)
    check(lib().vmlm_gemm_nt_int8_outlier(
        _host_ptr(a, np.float32, m * k, "a"), _host_ptr(q, np.int8, n * k, "q"),
        _host_ptr(scale, np.float32, n, "scale"), _host_ptr(w, np.float32, n * k, "w") if idx.size else None,
        _host_ptr(idx, np.uint32, idx.size, "idx") if idx.size else None, idx.size,
        _host_ptr(c, np.float32, m * n, "c"), m, n, k))


def gemm_nt_int8_outlier_dev(a, q, scale, w, idx, n_idx, c, m, n, k, compact=False, stream=None) -> None:
    """w: the f32 weight [n, k] (compact False) or the gathered outlier columns [n, n_idx]."""
    check(lib().vmlm_gemm_nt_int8_outlier_dev(
        _dev_ptr(a, "float32", m * k, "a"), _dev_ptr(q, "int8", n * k, "q"), _dev_ptr(scale, "float32", n, "scale"),
        _dev_ptr(w, "float32", n * (n_idx if compact else k), "w") if n_idx else None, int(bool(compact)),
        _idx_dev_ptr(idx, n_idx) if n_idx else None, n_idx, _dev_ptr(c, "float32", m * n, "c"), m, n, k,
        _stream_ptr(stream)))


def gather_columns_dev(w, idx, n_idx, n, k, wo, stream=None) -> None:
    """wo[j, t] = w[j, idx[t]] (device tensors)."""
    check(lib().vmlm_gather_columns_dev(_dev_ptr(w, "float32", n * k, "w"), _idx_dev_ptr(idx, n_idx), n_idx, n, k,
                                        _dev_ptr(wo, "float32", n * n_idx, "wo"), _stream_ptr(stream)))


def emb(table, idx, out) -> None:
    """OP_EMB (core/src/interp.rs:1351-1420) for every index: out[t] = f32(table[idx[t]]);
    table: a [rows, cols] bf16-bit (uint16) or float32 array, idx: float32 row numbers."""
    rows, cols = table.shape
    dt = DT_BF16 if table.dtype == np.uint16 else DT_F32
    m = idx.size
    check(lib().vmlm_emb(_host_ptr(table, table.dtype, rows * cols, "table"), dt, rows, cols,
                         _host_ptr(idx, np.float32, m, "idx"), m, _host_ptr(out, np.float32, m * cols, "out")))


def emb_dev(table, idx, out, stream=None) -> None:
    """OP_EMB on CUDA tensors (bfloat16 / int16 bits or float32 table); a bad index is reported by sync()."""
    rows, cols = table.shape
    name = str(table.dtype)[6:]
    dt = DT_BF16 if name in ("bfloat16", "int16", "uint16") else DT_F32
    m = idx.numel()
    check(lib().vmlm_emb_dev(_dev_ptr(table, name, rows * cols, "table"), dt, rows, cols,
                             _dev_ptr(idx, "float32", m, "idx"), m, _dev_ptr(out, "float32", m * cols, "out"),
                             _stream_ptr(stream)))


# ------------------------------------------------------ the OP_GEMM operator

DT_F32, DT_F16, DT_I8, DT_I32, DT_BF16 = 0, 1, 2, 3, 4  # core/src/format.rs:73-79
FL_ACC, FL_TRANS_B = 1, 2                                # trans/src/opcode.rs:303-304
_NP_DT = {"float32": DT_F32, "float16": DT_F16, "int8": DT_I8, "int32": DT_I32, "uint16": DT_BF16}


def slot(x, dtype=None):
    """A VM slot over a 2-D numpy array or CUDA tensor (uint16 / bfloat16 / int16 data is bf16)."""
    from ._lib import Slot
    if x is None:
        return None
    rows, cols = x.shape
    if isinstance(x, np.ndarray):
        if not x.flags["C_CONTIGUOUS"]:
            raise ValueError("slot: must be C-contiguous")
        ptr, dt = x.ctypes.data, _NP_DT.get(x.dtype.name, -1)
    else:
        if not x.is_contiguous():
            raise ValueError("slot: must be contiguous")
        name = str(x.dtype)[6:]
        ptr, dt = x.data_ptr(), DT_BF16 if name in ("bfloat16", "int16") else _NP_DT.get(name, -1)
    return Slot(ptr, rows, cols, dt if dtype is None else dtype)


def _slot_ref(s):
    return ctypes.byref(s) if s is not None else None


def op_gemm(fl, d, a, b, scale=None) -> None:
    """The VM's OP_GEMM (core/src/interp.rs:734-812) on host arrays: d = a . op(b) (+ d with FL_ACC)."""
    sd, sa, sb, ss = slot(d), slot(a), slot(b), slot(scale)
    check(lib().vmlm_op_gemm(fl, _slot_ref(sd), _slot_ref(sa), _slot_ref(sb), _slot_ref(ss)))


def op_gemm_dev(fl, d, a, b, scale=None, stream=None) -> None:
    """OP_GEMM on CUDA tensors, on `stream`."""
    sd, sa, sb, ss = slot(d), slot(a), slot(b), slot(scale)
    check(lib().vmlm_op_gemm_dev(fl, _slot_ref(sd), _slot_ref(sa), _slot_ref(sb), _slot_ref(ss),
                                 _stream_ptr(stream)))


# ---------------------------------------------------------- conveniences

def q8_linear(x: np.ndarray, q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """x[M,K] f32, q[N,K] int8, scale[N] f32 -> C[M,N] f32 through gemm_nt_int8."""
    m, k = x.shape
    n = q.shape[0]
    c = np.empty((m, n), np.float32)
    gemm_nt_int8(np.ascontiguousarray(x, np.float32), np.ascontiguousarray(q, np.int8),
                 np.ascontiguousarray(scale, np.float32), c, m, n, k)
    return c


def bf16_linear(x: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """x[M,K] f32, b_bits[N,K] uint16 (bf16 bits) -> C[M,N] f32 through gemm_nt_bf16."""
    m, k = x.shape
    n = b_bits.shape[0]
    c = np.empty((m, n), np.float32)
    gemm_nt_bf16(np.ascontiguousarray(x, np.float32), np.ascontiguousarray(b_bits, np.uint16), c, m, n, k)
    return c
