"""CPU tests of the C ABI boundary: the library loads, exports every symbol the
header declares, and rejects bad arguments on the host before any GPU work.
No kernel is launched here."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import ROOT, gpu_available

HEADER = os.path.join(ROOT, "include", "vmlm_cuda.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"VMLM_API\s+[\w\s\*]+?\b(vmlm_\w+)\s*\(", text)))


def test_library_builds_and_loads():
    from sparrow_b200 import build, lib
    build.build()
    assert os.path.exists(build.OUT)
    lib()


def test_every_declared_symbol_is_exported_and_bound():
    from sparrow_b200 import _lib
    names = declared_symbols()
    assert len(names) >= 15
    out = subprocess.check_output(["nm", "-D", "--defined-only", _lib.lib_path()], text=True)
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    assert sorted(_lib.SIGNATURES) == names
    L = _lib.lib()
    for n in names:
        assert getattr(L, n) is not None


def test_library_has_no_cpu_compute_path():
    # The product library links no oracle and no host BLAS: only libc/libstdc++/libm.
    from sparrow_b200 import _lib
    out = subprocess.check_output(["ldd", _lib.lib_path()], text=True)
    assert "oracle" not in out and "blas" not in out.lower()
    syms = subprocess.check_output(["nm", "-D", _lib.lib_path()], text=True)
    assert "oracle_" not in syms


def test_version_and_errors():
    from sparrow_b200 import _lib
    L = _lib.lib()
    assert L.vmlm_version() == 100
    assert isinstance(L.vmlm_last_error(), bytes)


def test_null_pointers_rejected_before_device():
    from sparrow_b200 import _lib
    L = _lib.lib()
    rc = L.vmlm_gemm_nt_int8(None, None, None, None, 2, 3, 4)
    assert rc == 1  # VMLM_ERR_ARG
    assert b"null" in L.vmlm_last_error()
    assert L.vmlm_gemm_nt_bf16(None, None, None, 2, 3, 4) == 1
    assert L.vmlm_gemm_nt_int8_dev(None, None, None, None, 2, 3, 4, None) == 1


def test_empty_shapes_are_noops():
    # m == 0 or n == 0: the reference loops do nothing; no device is touched.
    from sparrow_b200 import _lib
    L = _lib.lib()
    assert L.vmlm_gemm_nt_int8(None, None, None, None, 0, 5, 7) == 0
    assert L.vmlm_gemm_nt_bf16(None, None, None, 3, 0, 7) == 0
    assert L.vmlm_gemm_i8i8(None, None, None, None, None, 0, 0, 0) == 0


def test_oversized_dims_rejected():
    from sparrow_b200 import _lib
    L = _lib.lib()
    assert L.vmlm_gemm_nt_int8(None, None, None, None, 1, 1 << 31, 16) == 2  # VMLM_ERR_SHAPE
    assert L.vmlm_gemm_i8i8(None, None, None, None, None, 4, 4, 200000) == 2


def test_python_mirror_validates_buffers():
    import sparrow_b200.kernels as K
    a = np.zeros(8, np.float32)
    q = np.zeros(8, np.int8)
    s = np.zeros(2, np.float32)
    c = np.zeros(4, np.float32)
    with pytest.raises(ValueError):
        K.gemm_nt_int8(a.astype(np.float64), q, s, c, 2, 2, 4)
    with pytest.raises(ValueError):
        K.gemm_nt_int8(a, q, s[:1], c, 2, 2, 4)
    with pytest.raises(ValueError):
        K.gemm_nt_bf16(a, q, c, 2, 2, 4)


@pytest.mark.skipif(gpu_available(), reason="checks the no-device error path")
def test_no_device_is_a_loud_error():
    import sparrow_b200.kernels as K
    from sparrow_b200 import VmlmError
    a = np.ones(8, np.float32)
    q = np.ones(8, np.int8)
    s = np.ones(2, np.float32)
    c = np.zeros(4, np.float32)
    with pytest.raises(VmlmError):
        K.gemm_nt_int8(a, q, s, c, 2, 2, 4)


def test_oracle_not_importable_from_product():
    # the product package never imports the oracle
    for fn in os.listdir(os.path.join(ROOT, "sparrow_b200")):
        if fn.endswith(".py"):
            assert "oracle" not in open(os.path.join(ROOT, "sparrow_b200", fn)).read()
