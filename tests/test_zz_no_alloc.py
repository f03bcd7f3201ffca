"""GPU test of the allocation-free Q8 entry point, vmlm_gemm_nt_int8_dev_noalloc.

Some callers cannot allocate device memory once they are running (an engine
that reserves all of its memory at start-up and must not fail or stall on
cudaMalloc in its decode loop). This entry point serves them from a fixed
scratch array inside the library. The test calls it through the C ABI twice
in a row (the second call sees whatever the first left in the shared scratch)
and checks both results against the allocating entry point,
vmlm_gemm_nt_int8_dev, within the parity tolerance the other tests use. The
file name makes pytest collect it last.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-3        # BASELINE: f32 outputs within 1e-3 max relative error
TIGHT_Q8 = 2e-5   # the Q8 path's own bound, as in test_parity_gpu.py


@pytest.mark.parametrize("m,n,k", [
    (1, 5760, 2304),     # config 1; tiles split between CTAs (stream-K)
    (16, 2304, 2304),    # largest token count; split tiles with 16 tokens
    (1, 122753, 2304),   # config-4 shape; whole tiles round-robin
    (5, 300, 7),         # K not a multiple of 16: CUDA-core path
])
def test_noalloc_matches_allocating_entry_point_twice(kernels, oracle, m, n, k):
    import torch
    x = oracle.fill_normal(m * k, 100 + m, 1.0).reshape(m, k)
    q, s = oracle.quant_int8(oracle.fill_normal(n * k, 101 + m, 0.02).reshape(n, k))
    dx, dq, ds = torch.from_numpy(x).cuda(), torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()
    st = torch.cuda.current_stream()
    ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
    kernels.gemm_nt_int8_dev(dx, dq, ds, ref, m, n, k, stream=st)
    torch.cuda.synchronize()
    ref_h = ref.cpu().numpy()
    for _ in range(2):
        out = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        kernels.gemm_nt_int8_dev_noalloc(dx, dq, ds, out, m, n, k, stream=st)
        torch.cuda.synchronize()
        err = oracle.max_rel_err(out.cpu().numpy(), ref_h)
        assert err <= TOL and err <= TIGHT_Q8, err


def test_noalloc_rejects_sizes_beyond_its_scratch(kernels):
    import torch
    from sparrow_b200 import VmlmError
    m, n, k = 17, 64, 64
    a = torch.zeros((m, k), dtype=torch.float32, device="cuda")
    q = torch.zeros((n, k), dtype=torch.int8, device="cuda")
    s = torch.ones((n,), dtype=torch.float32, device="cuda")
    c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    with pytest.raises(VmlmError) as info:
        kernels.gemm_nt_int8_dev_noalloc(a, q, s, c, m, n, k)
    assert info.value.status == 2 and "m <= 16" in str(info.value)


def test_noalloc_calls_leave_device_memory_unchanged(kernels, oracle):
    """The point of the entry point: after one warm-up call per kernel it uses
    (the first launch of a kernel may load its code), further calls of any size
    within the limits leave the device's free memory exactly as it was, and
    vmlm_sync (which reads the array's own error word) reports no error."""
    import torch
    shapes = [(1, 5760, 2304), (16, 2304, 2304), (3, 300, 7), (8, 40000, 4096)]
    bufs = []
    for i, (m, n, k) in enumerate(shapes):
        x = torch.from_numpy(oracle.fill_normal(m * k, 200 + i, 1.0).reshape(m, k)).cuda()
        q, s = oracle.quant_int8(oracle.fill_normal(n * k, 210 + i, 0.02).reshape(n, k))
        bufs.append((x, torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda(),
                     torch.empty((m, n), dtype=torch.float32, device="cuda"), m, n, k))
    st = torch.cuda.current_stream()
    for x, q, s, c, m, n, k in bufs[:1] + bufs[2:3]:
        kernels.gemm_nt_int8_dev_noalloc(x, q, s, c, m, n, k, stream=st)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        for x, q, s, c, m, n, k in bufs:
            kernels.gemm_nt_int8_dev_noalloc(x, q, s, c, m, n, k, stream=st)
    torch.cuda.synchronize()
    kernels.sync(st)
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    for x, q, s, c, m, n, k in bufs:
        ref = oracle.gemm_nt_int8(x.cpu().numpy(), q.cpu().numpy(), s.cpu().numpy())
        assert oracle.max_rel_err(c.cpu().numpy(), ref) <= TIGHT_Q8
