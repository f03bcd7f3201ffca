"""Device entry points captured in a CUDA graph.

An engine that runs a decode or prefill loop captures its steps in a CUDA
graph, so that the host does not launch kernel by kernel. After one eager call
of a shape (which sizes the library's workspace), the same call captured in a
graph and replayed must give the same bits as the eager call, on every replay.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

C3_SHAPES = [(2304, 2304)] * 4 + [(5760, 2304)] * 2 + [(2304, 5760)]


def _gen(torch, shape, seed, sd):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(shape, generator=g, device="cuda") * sd


def _q8(torch, n, k, seed):
    w = _gen(torch, (n, k), seed, 0.02)
    s = w.abs().amax(dim=1) / 127.0
    q = torch.clamp(torch.round(w / s[:, None]), -127, 127).to(torch.int8)
    return q, s.contiguous()


def _capture_and_compare(torch, calls, outs, replays=3):
    """Run `calls` eagerly, keep the outputs, capture them in one graph on a
    side stream, replay and compare bit for bit after every replay."""
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        for f in calls:
            f(st)
    torch.cuda.synchronize()
    ref = [o.clone() for o in outs]
    for o in outs:
        o.fill_(float("nan"))
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for f in calls:
            f(st)
    for _ in range(replays):
        for o in outs:
            o.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        for o, r in zip(outs, ref):
            assert torch.equal(o.view(torch.int32), r.view(torch.int32))
    del g


def test_graph_bf16_prefill_and_q8_decode_calls(kernels):
    import torch
    K = kernels
    torch.cuda.set_device(0)
    K.init(0)
    m2, n2, k2 = 512, 2304, 2304
    x2 = _gen(torch, (m2, k2), 1, 1.0).to(torch.bfloat16).float().contiguous()
    w2 = _gen(torch, (n2, k2), 2, 0.02).to(torch.bfloat16)
    c2 = torch.empty((m2, n2), device="cuda")
    x1 = _gen(torch, (1, 2304), 3, 1.0)
    q1, s1 = _q8(torch, 5760, 2304, 4)
    c1 = torch.empty((1, 5760), device="cuda")
    calls = [lambda st: K.gemm_nt_bf16_dev(x2, w2, c2, m2, n2, k2, stream=st),
             lambda st: K.gemm_nt_int8_dev(x1, q1, s1, c1, 1, 5760, 2304, stream=st)] * 2  # even: flag parity
    _capture_and_compare(torch, calls, [c2, c1])


@pytest.mark.parametrize("m", [1, 8])
def test_graph_q8_layer_batch(kernels, m):
    import torch
    K = kernels
    torch.cuda.set_device(0)
    K.init(0)
    batch, outs = [], []
    for i, (n, k) in enumerate(C3_SHAPES):
        x = _gen(torch, (m, k), 10 + i, 1.0)
        q, s = _q8(torch, n, k, 20 + i)
        c = torch.empty((m, n), device="cuda")
        batch.append((x, q, s, c, m, n, k))
        outs.append(c)
    _capture_and_compare(torch, [lambda st: K.gemm_nt_int8_batch_dev(batch, stream=st)] * 3, outs)


def test_graph_int8_prefill(kernels):
    import torch
    K = kernels
    torch.cuda.set_device(0)
    K.init(0)
    m, n, k = 1024, 4096, 2048
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    x = torch.randint(-127, 128, (m, k), generator=g, device="cuda", dtype=torch.int8)
    w = torch.randint(-127, 128, (n, k), generator=g, device="cuda", dtype=torch.int8)
    s = (_gen(torch, (n,), 8, 0.02).abs() + 1e-3).contiguous()
    c = torch.empty((m, n), device="cuda")
    _capture_and_compare(torch, [lambda st: K.gemm_i8i8_dev(x, w, s, c, None, m, n, k, stream=st)] * 2, [c])
    assert np.isfinite(c.cpu().numpy()).all()


def test_graph_profiled_gemm_launches_report_times(kernels):
    """Launch profiling inside a capture: the event pairs around each GEMM
    launch become graph nodes, and after a replay every pair holds a time."""
    import torch
    K = kernels
    torch.cuda.set_device(0)
    K.init(0)
    m, n, k = 512, 2304, 2304
    x = _gen(torch, (m, k), 1, 1.0).to(torch.bfloat16).float().contiguous()
    w = _gen(torch, (n, k), 2, 0.02).to(torch.bfloat16)
    c = torch.empty((m, n), device="cuda")
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        K.gemm_nt_bf16_dev(x, w, c, m, n, k, stream=st)
    torch.cuda.synchronize()
    ref = c.clone()
    K.profile_enable(True)
    K.profile_take()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for _ in range(4):
            K.gemm_nt_bf16_dev(x, w, c, m, n, k, stream=st)
    K.profile_enable(False)
    c.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    ms, launches = K.profile_take()
    del g
    assert launches == 4
    assert 0.0 < ms / launches < 1.0
    assert torch.equal(c.view(torch.int32), ref.view(torch.int32))
