"""ctypes binding of include/vmlm_cuda.h (the library's C ABI)."""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(HERE, "lib", "libvmlm_cuda.so")

STATUS = {
    0: "VMLM_OK",
    1: "VMLM_ERR_ARG",
    2: "VMLM_ERR_SHAPE",
    3: "VMLM_ERR_CUDA",
    4: "VMLM_ERR_NO_DEVICE",
    5: "VMLM_ERR_STATE",
    6: "VMLM_ERR_OOM",
    7: "VMLM_ERR_DEVICE_TIMEOUT",
    8: "VMLM_ERR_OPERATOR",
}

P, S, I = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int


class Slot(ctypes.Structure):
    """vmlm_slot: a VM slot as the OP_GEMM operator reads it."""
    _fields_ = [("ptr", ctypes.c_void_p), ("rows", ctypes.c_size_t), ("cols", ctypes.c_size_t),
                ("dtype", ctypes.c_int)]


SP = ctypes.POINTER(Slot)

# name -> (restype, argtypes); must list every symbol the header declares.
SIGNATURES = {
    "vmlm_version": (I, []),
    "vmlm_init": (I, [I]),
    "vmlm_shutdown": (I, []),
    "vmlm_last_error": (ctypes.c_char_p, []),
    "vmlm_register_weight": (I, [P, S]),
    "vmlm_unregister_weight": (I, [P]),
    "vmlm_unregister_all": (I, []),
    "vmlm_gemm_nt_int8": (I, [P, P, P, P, S, S, S]),
    "vmlm_gemm_nt_bf16": (I, [P, P, P, S, S, S]),
    "vmlm_gemm_i8i8": (I, [P, P, P, P, P, S, S, S]),
    "vmlm_gemm_nt_f32": (I, [P, P, P, S, S, S, I]),
    "vmlm_gemm_f32": (I, [P, P, P, S, S, S, I]),
    "vmlm_gemm_nt_f32_dev": (I, [P, P, P, S, S, S, I, P]),
    "vmlm_gemm_f32_dev": (I, [P, P, P, S, S, S, I, P]),
    "vmlm_gemm_nt_int8_dev": (I, [P, P, P, P, S, S, S, P]),
    "vmlm_gemm_nt_bf16_dev": (I, [P, P, P, S, S, S, P]),
    "vmlm_gemm_i8i8_dev": (I, [P, P, P, P, P, S, S, S, P]),
    "vmlm_gemm_nt_int8_dev_noalloc": (I, [P, P, P, P, S, S, S, P]),
    "vmlm_sync": (I, [P]),
    "vmlm_sharded_gemm_nt_int8_dev": (I, [P, P, P, P, P, I, I, S, S, S, P]),
    "vmlm_sharded_gemm_i8i8_dev": (I, [P, P, P, P, P, I, I, S, S, S, P]),
    "vmlm_sharded_reset": (I, [P]),
    "vmlm_ipc_handle": (I, [P, P]),
    "vmlm_ipc_open": (I, [P, ctypes.POINTER(ctypes.c_void_p)]),
    "vmlm_ipc_close": (I, [P]),
    "vmlm_launch_count": (ctypes.c_uint64, []),
    "vmlm_profile_enable": (I, [I]),
    "vmlm_profile_take": (I, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_uint64)]),
    "vmlm_profile_kernel": (I, [ctypes.c_char_p, ctypes.c_size_t]),
    "vmlm_probe_mma_peak": (I, [I, I, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]),
    "vmlm_trace_enable": (I, [I]),
    "vmlm_trace_take": (I, [P, S]),
    "vmlm_op_gemm": (I, [ctypes.c_uint, SP, SP, SP, SP]),
    "vmlm_rmsnorm_gemm_nt_int8": (I, [P, P, ctypes.c_float, P, P, P, S, S, S]),
    "vmlm_rmsnorm_gemm_nt_int8_dev": (I, [P, P, ctypes.c_float, P, P, P, S, S, S, P]),
    "vmlm_gemv_f32": (I, [P, P, P, S, S]),
    "vmlm_gemv_f32_dev": (I, [P, P, P, S, S, P]),
    "vmlm_emb": (I, [P, I, S, S, P, S, P]),
    "vmlm_emb_dev": (I, [P, I, S, S, P, S, P, P]),
    "vmlm_set_host_pipeline": (I, [I]),
    "vmlm_gemm_nt_int8_batch_dev": (I, [P, S, P]),
    "vmlm_pool_load": (I, [P, S, P, S, P]),
    "vmlm_pool_free": (I, [P]),
    "vmlm_pool_info": (I, [P, P, P, P]),
    "vmlm_pool_region": (I, [P, I, P]),
    "vmlm_pool_slot": (I, [P, S, P, P]),
    "vmlm_pool_layerb": (I, [P, ctypes.c_float]),
    "vmlm_pool_layer_base": (I, [P, P]),
    "vmlm_pool_find_const": (I, [P, ctypes.c_char_p, P]),
    "vmlm_pool_find_slot": (I, [P, ctypes.c_char_p, P]),
    "vmlm_pool_gemm": (I, [P, P, P]),
    "vmlm_gemm_nt_int4_gs": (I, [P, P, P, P, S, S, S, S, I]),
    "vmlm_gemm_nt_int4_gs_dev": (I, [P, P, P, P, S, S, S, S, I, P]),
    "vmlm_gemm_nt_int8_outlier": (I, [P, P, P, P, P, S, P, S, S, S]),
    "vmlm_gemm_nt_int8_outlier_dev": (I, [P, P, P, P, I, P, S, P, S, S, S, P]),
    "vmlm_gather_columns_dev": (I, [P, P, S, S, S, P, P]),
    "vmlm_op_gemm_dev": (I, [ctypes.c_uint, SP, SP, SP, SP, P]),
}


class VmlmError(RuntimeError):
    """A non-zero status from the C ABI (the reference VM prints and exits 9)."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS.get(status, status)}: {message}")


_lib = None


def lib_path() -> str:
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    """Load the CUDA library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise ImportError(
                f"{_LIB_PATH} is missing: build it with `python -m sparrow_b200.build` "
                "(there is no CPU fallback)")
        L = ctypes.CDLL(_LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != 0:
        msg = lib().vmlm_last_error()
        raise VmlmError(status, msg.decode() if msg else "")
