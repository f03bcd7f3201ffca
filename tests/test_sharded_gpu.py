"""GPU tests of the row-sharded entry points, whose GEMM epilogue stores every
output into every rank's C (the all-gather fused into the kernel).

One GPU: a single-rank group (the rank is its own only peer) against the
oracle, twice in a row so the inbox count advances. Two or more GPUs: two
processes, one per GPU, exchange IPC handles over gloo and must both end with
the full result, equal to the single-GPU call on the whole weight."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TIGHT_Q8 = 2e-5


@pytest.mark.parametrize("m,n,k", [(1, 20000, 2304), (64, 16384, 2304), (5, 300, 256), (64, 80000, 1024)])
def test_single_rank_sharded_q8_matches_oracle(kernels, oracle, m, n, k):
    import torch
    from sparrow_b200.sharded import PeerOutputs, sharded_gemm_nt_int8
    x = oracle.fill_normal(m * k, 60 + m, 1.0).reshape(m, k)
    q, s = oracle.quant_int8(oracle.fill_normal(n * k, 61 + m, 0.02).reshape(n, k))
    ref = oracle.gemm_nt_int8(x, q, s, nt=os.cpu_count() or 1)
    dx, dq, ds = torch.from_numpy(x).cuda(), torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()
    peers = PeerOutputs(m, n)
    try:
        for _ in range(2):
            peers.c.fill_(float("nan"))
            sharded_gemm_nt_int8(dx, dq, ds, peers, m, n, k, stream=torch.cuda.current_stream())
            torch.cuda.synchronize()
            kernels.sync()
            err = oracle.max_rel_err(peers.c.cpu().numpy(), ref)
            assert err <= TIGHT_Q8, err
    finally:
        peers.close()


@pytest.mark.parametrize("m,n,k", [(300, 1000, 512), (1024, 4096, 1024)])
def test_single_rank_sharded_i8i8_bit_exact(kernels, oracle, m, n, k):
    import torch
    from sparrow_b200.sharded import PeerOutputs, sharded_gemm_i8i8
    x = oracle.fill_int8(m * k, 70).reshape(m, k)
    w = oracle.fill_int8(n * k, 71).reshape(n, k)
    s = np.abs(oracle.fill_normal(n, 72, 0.02)) + np.float32(1e-3)
    rc, _ = oracle.gemm_i8i8(x, w, s, nt=os.cpu_count() or 1)
    peers = PeerOutputs(m, n)
    try:
        for _ in range(2):
            peers.c.zero_()
            sharded_gemm_i8i8(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda(),
                              peers, m, n, k, stream=torch.cuda.current_stream())
            torch.cuda.synchronize()
            kernels.sync()
            assert np.array_equal(peers.c.cpu().numpy().view(np.uint32), rc.view(np.uint32))
    finally:
        peers.close()


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _two_gpu_rank(rank, world, port, errors):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    import sparrow_b200.kernels as K
    from sparrow_b200.sharded import PeerOutputs, shard_rows, sharded_gemm_i8i8, sharded_gemm_nt_int8
    K.init(rank)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        g = torch.Generator(device="cuda")
        # Q8 LM-head shape, M = 1 and 64 (the all-gather in the GEMM epilogue), and one whose
        # output per rank is large enough for the copy-engine gather: full weight on every rank
        for m, n, k in ((1, 30011, 2304), (64, 16384, 2304), (128, 65536, 2304)):
            g.manual_seed(7 + m)
            x = torch.randn((m, k), generator=g, device="cuda")
            q = torch.randint(-127, 128, (n, k), generator=g, device="cuda", dtype=torch.int8)
            s = torch.rand((n,), generator=g, device="cuda") * 0.01 + 1e-3
            full = torch.empty((m, n), device="cuda")
            st = torch.cuda.current_stream()
            K.gemm_nt_int8_dev(x, q, s, full, m, n, k, stream=st)
            r0, r1 = shard_rows(n, world, rank)
            qs, ss = q[r0:r1].contiguous(), s[r0:r1].contiguous()
            peers = PeerOutputs(m, n)
            for _ in range(2):
                peers.c.fill_(float("nan"))
                torch.cuda.synchronize()  # no peer may write into C before it is reset
                dist.barrier()
                sharded_gemm_nt_int8(x, qs, ss, peers, m, n, k, stream=st)
                torch.cuda.synchronize()
                K.sync()
                got = peers.c.cpu().numpy()
                ref = full.cpu().numpy()
                err = float(np.abs(got - ref).max() / np.abs(ref).max())
                if not err <= TIGHT_Q8:
                    errors.put(f"rank {rank} q8 {m}x{n}: max rel err {err}")
            dist.barrier()
            peers.close()
            dist.barrier()
        # int8 x int8 FFN shapes (smaller), bit-exact: a K-split plan with the peer
        # stores, and one large enough for the copy-engine gather of a chunked GEMM
        for m, n, k in ((512, 8192, 1024), (2048, 8192, 1024)):
            g.manual_seed(99 + m)
            x = torch.randint(-127, 128, (m, k), generator=g, device="cuda", dtype=torch.int8)
            w = torch.randint(-127, 128, (n, k), generator=g, device="cuda", dtype=torch.int8)
            s = torch.rand((n,), generator=g, device="cuda") * 0.01 + 1e-3
            full = torch.empty((m, n), device="cuda")
            st = torch.cuda.current_stream()
            K.gemm_i8i8_dev(x, w, s, full, None, m, n, k, stream=st)
            r0, r1 = shard_rows(n, world, rank)
            ws, ss = w[r0:r1].contiguous(), s[r0:r1].contiguous()
            peers = PeerOutputs(m, n)
            torch.cuda.synchronize()
            dist.barrier()
            sharded_gemm_i8i8(x, ws, ss, peers, m, n, k, stream=st)
            torch.cuda.synchronize()
            K.sync()
            if not torch.equal(peers.c.view(torch.int32), full.view(torch.int32)):
                errors.put(f"rank {rank} i8i8 {m}x{n}: results differ")
            dist.barrier()
            peers.close()
            dist.barrier()
    except Exception as e:  # reported to the parent, which fails the test
        errors.put(f"rank {rank}: {type(e).__name__}: {e}")
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_gpu_sharded_calls_give_every_rank_the_whole_result():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_gpu_rank, args=(r, 2, port, errors)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join(timeout=10)
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert all(p.exitcode == 0 for p in procs), msgs
    assert not msgs, msgs


@pytest.mark.timeout(120)
def test_missing_rank_makes_the_bounded_wait_run_out_and_the_next_call_is_correct(kernels, oracle):
    """Failure detection without a GPU fault. A two-rank call is made on one GPU
    for rank 0 only: rank 1's C and inbox are local buffers that no process
    serves, so rank 1's count never arrives (a flag that nothing sets). The
    kernel's bounded wait for it (5 s) runs out, it records the timeout and
    returns; vmlm_sync reports VMLM_ERR_DEVICE_TIMEOUT. After
    vmlm_sharded_reset the context is usable and the next call (a single-rank
    call on the same buffers) matches the oracle."""
    import ctypes
    import torch
    from sparrow_b200 import VmlmError
    from sparrow_b200._lib import lib
    from sparrow_b200.sharded import shard_rows
    m, n, k = 1, 4096, 2304
    x = oracle.fill_normal(m * k, 80, 1.0).reshape(m, k)
    q, s = oracle.quant_int8(oracle.fill_normal(n * k, 81, 0.02).reshape(n, k))
    ref = oracle.gemm_nt_int8(x, q, s, nt=os.cpu_count() or 1)
    dx, dq, ds = torch.from_numpy(x).cuda(), torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()
    c = [torch.zeros((m, n), dtype=torch.float32, device="cuda") for _ in range(2)]
    inbox = [torch.zeros(4, dtype=torch.int32, device="cuda") for _ in range(2)]
    for b in inbox:
        assert lib().vmlm_sharded_reset(ctypes.c_void_p(b.data_ptr())) == 0
    c_ptrs = (ctypes.c_void_p * 2)(*[t.data_ptr() for t in c])
    in_ptrs = (ctypes.c_void_p * 2)(*[t.data_ptr() for t in inbox])
    st = torch.cuda.current_stream()
    sp = ctypes.c_void_p(st.cuda_stream or 1)
    r0, r1 = shard_rows(n, 2, 0)
    qs, ss = dq[r0:r1].contiguous(), ds[r0:r1].contiguous()
    rc = lib().vmlm_sharded_gemm_nt_int8_dev(
        ctypes.c_void_p(dx.data_ptr()), ctypes.c_void_p(qs.data_ptr()), ctypes.c_void_p(ss.data_ptr()),
        c_ptrs, in_ptrs, 0, 2, m, n, k, sp)
    assert rc == 0
    with pytest.raises(VmlmError) as info:
        kernels.sync(st)
    assert info.value.status == 7, str(info.value)  # VMLM_ERR_DEVICE_TIMEOUT
    # rank 0's own columns reached both Cs before the wait; rank 1's never came
    got = c[0].cpu().numpy()
    assert oracle.max_rel_err(got[:, r0:r1], ref[:, r0:r1]) <= TIGHT_Q8
    assert np.all(got[:, r1:] == 0)
    for b in inbox:
        assert lib().vmlm_sharded_reset(ctypes.c_void_p(b.data_ptr())) == 0
    for _ in range(2):
        c[0].fill_(float("nan"))
        rc = lib().vmlm_sharded_gemm_nt_int8_dev(
            ctypes.c_void_p(dx.data_ptr()), ctypes.c_void_p(dq.data_ptr()), ctypes.c_void_p(ds.data_ptr()),
            c_ptrs, in_ptrs, 0, 1, m, n, k, sp)
        assert rc == 0
        kernels.sync(st)
        assert oracle.max_rel_err(c[0].cpu().numpy(), ref) <= TIGHT_Q8


@pytest.mark.parametrize("kind,m,n,k", [("i8i8", 512, 12288, 1024), ("q8", 64, 98304, 1024)])
def test_four_rank_forms_push_one_rank_slice_to_every_peer(kernels, oracle, kind, m, n, k):
    """The forms used on more than two GPUs (int8 x int8 with a large output:
    row chunks pushed to every peer by peer_push_kernel; Q8: the fused
    epilogue), run on one GPU for rank 1 of a four-rank group whose C buffers
    and inboxes are local. The other ranks' counts are added to rank 1's inbox
    before each call, on the call's stream, so the call's bounded wait ends
    without waiting on any other launch. Every rank's C must then hold rank 1's
    column slice: bit for bit for int8 x int8, within the Q8 bound for Q8; the
    rest of each C is untouched. Two calls in a row (the inbox count advances)."""
    import ctypes
    import torch
    from sparrow_b200._lib import lib
    from sparrow_b200.sharded import shard_rows
    world, rank = 4, 1
    r0, r1 = shard_rows(n, world, rank)
    if kind == "i8i8":
        x = oracle.fill_int8(m * k, 90).reshape(m, k)
        w = oracle.fill_int8((r1 - r0) * k, 91).reshape(r1 - r0, k)
        s = np.abs(oracle.fill_normal(r1 - r0, 92, 0.02)) + np.float32(1e-3)
        ref, _ = oracle.gemm_i8i8(x, w, s, nt=os.cpu_count() or 1)
    else:
        x = oracle.fill_normal(m * k, 93, 1.0).reshape(m, k)
        w, s = oracle.quant_int8(oracle.fill_normal((r1 - r0) * k, 94, 0.02).reshape(r1 - r0, k))
        ref = oracle.gemm_nt_int8(x, w, s, nt=os.cpu_count() or 1)
    dx, dw, ds = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda()
    c = [torch.zeros((m, n), dtype=torch.float32, device="cuda") for _ in range(world)]
    inbox = [torch.zeros(4, dtype=torch.int32, device="cuda") for _ in range(world)]
    for b in inbox:
        assert lib().vmlm_sharded_reset(ctypes.c_void_p(b.data_ptr())) == 0
    c_ptrs = (ctypes.c_void_p * world)(*[t.data_ptr() for t in c])
    in_ptrs = (ctypes.c_void_p * world)(*[t.data_ptr() for t in inbox])
    st = torch.cuda.current_stream()
    sp = ctypes.c_void_p(st.cuda_stream or 1)
    fn = lib().vmlm_sharded_gemm_i8i8_dev if kind == "i8i8" else lib().vmlm_sharded_gemm_nt_int8_dev
    try:
        for _ in range(2):
            for t in c:
                t.zero_()
            inbox[rank][0] += world - 1  # the other ranks' counts for this call
            rc = fn(ctypes.c_void_p(dx.data_ptr()), ctypes.c_void_p(dw.data_ptr()), ctypes.c_void_p(ds.data_ptr()),
                    c_ptrs, in_ptrs, rank, world, m, n, k, sp)
            assert rc == 0
            kernels.sync(st)
            for q in range(world):
                got = c[q].cpu().numpy()
                if kind == "i8i8":
                    assert np.array_equal(got[:, r0:r1].view(np.uint32), ref.view(np.uint32)), q
                else:
                    assert oracle.max_rel_err(got[:, r0:r1], ref) <= TIGHT_Q8, q
                assert np.all(got[:, :r0] == 0) and np.all(got[:, r1:] == 0), q
    finally:
        for b in inbox:
            lib().vmlm_sharded_reset(ctypes.c_void_p(b.data_ptr()))
