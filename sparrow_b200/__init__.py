"""sparrow_b200 -- B200 (sm_100a) implementation of the VMLM quantised-linear path.

The product is the C-ABI library sparrow_b200/lib/libvmlm_cuda.so
(declared in include/vmlm_cuda.h). This package is its Python host mirror:
`sparrow_b200.kernels` keeps the names, argument meaning and error behaviour of
the reference operators `vmlm_ops::kernels::{gemm_nt_int8, gemm_nt_bf16}`
(ops/src/kernels.rs:1200-1287 in the shouzugzs-AI/Sparrow tree).

There is no CPU fallback: importing the kernels without the built library, or
calling them without an sm_100 GPU, raises.
"""
from ._lib import VmlmError, lib, lib_path  # noqa: F401
from . import kernels  # noqa: F401

__all__ = ["kernels", "VmlmError", "lib", "lib_path"]
