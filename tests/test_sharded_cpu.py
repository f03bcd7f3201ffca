"""CPU tests of the row-sharded (multi-GPU) boundary: argument checks of the C
ABI entry points (rejected before any device work) and, over a world-size-2
gloo process group, the split of output rows between ranks that the sharded
entry points and `sparrow_b200.sharded` agree on."""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from sparrow_b200.sharded import shard_rows


def test_shard_rows_cover_every_row_once():
    for n in (8, 9, 122753, 28672, 15, 1000):
        for world in range(1, 9):
            try:
                spans = [shard_rows(n, world, r) for r in range(world)]
            except ValueError:
                rows = -(-n // world)
                assert rows * (world - 1) >= n  # only when some rank would get no rows
                continue
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert all(r1 > r0 for r0, r1 in spans)


def test_shard_rows_rejects_bad_ranks():
    with pytest.raises(ValueError):
        shard_rows(100, 9, 0)
    with pytest.raises(ValueError):
        shard_rows(100, 2, 2)
    with pytest.raises(ValueError):
        shard_rows(10, 8, 0)  # ceil(10/8) = 2 rows per rank leaves ranks 5..7 empty


def _ptrs(vals):
    return (ctypes.c_void_p * len(vals))(*vals)


def test_sharded_entry_points_check_arguments_first():
    from sparrow_b200 import _lib
    L = _lib.lib()
    one = _ptrs([16])
    args = (ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16))
    # world out of range, rank out of range, null peer lists
    assert L.vmlm_sharded_gemm_nt_int8_dev(*args, one, one, 0, 9, 1, 64, 64, None) == 1
    assert L.vmlm_sharded_gemm_nt_int8_dev(*args, one, one, 1, 1, 1, 64, 64, None) == 1
    assert L.vmlm_sharded_gemm_i8i8_dev(*args, None, one, 0, 1, 1, 64, 64, None) == 1
    assert b"rank" in L.vmlm_last_error() or b"null" in L.vmlm_last_error()
    # a rank without rows, and k not a multiple of 16
    eight = _ptrs([16] * 8)
    assert L.vmlm_sharded_gemm_i8i8_dev(*args, eight, eight, 0, 8, 1, 10, 64, None) == 2
    assert L.vmlm_sharded_gemm_nt_int8_dev(*args, one, one, 0, 1, 1, 64, 60, None) == 2
    assert L.vmlm_ipc_close(ctypes.c_void_p(12345)) == 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r0, r1 = shard_rows(n, world, rank)
        spans = [None] * world
        dist.all_gather_object(spans, (r0, r1))
        if rank == 0:
            out.put(spans)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_world2_ranks_agree_on_the_row_split():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    n = 122753
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, n, q)) for r in range(2)]
    for p in procs:
        p.start()
    spans = q.get(timeout=100)
    for p in procs:
        p.join(timeout=100)
        assert p.exitcode == 0
    assert spans[0] == (0, 61377) and spans[1] == (61377, n)
    covered = np.zeros(n, np.int32)
    for r0, r1 in spans:
        covered[r0:r1] += 1
    assert np.all(covered == 1)


def _gate_rank(rank, world, port, mode, out):
    """Two gloo ranks step through row-sharded Q8 products computed by the
    oracle on the CPU (each rank its rows, then an all-gather). Rank 1 leaves
    after two steps: by announcing it (mode "leave") or by exiting without a
    word (mode "vanish"). Rank 0 must learn of it at the gate of step 3, before
    launching anything, and a collective after that must fail, not hang."""
    import datetime
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from oracle import oracle as O
    from sparrow_b200.sharded import RankLost, StepGate
    store = dist.distributed_c10d._get_default_store()
    gate = StepGate(store, rank, world, timeout_s=3.0)
    m, n, k = 2, 96, 64
    x = O.fill_normal(m * k, 1, 1.0).reshape(m, k)
    q, s = O.quant_int8(O.fill_normal(n * k, 2, 0.02).reshape(n, k))
    full = O.gemm_nt_int8(x, q, s)
    r0, r1 = shard_rows(n, world, rank)
    import torch
    for step in range(1, 4):
        if rank == 1 and step == 3:
            if mode == "leave":
                gate.leave()
            out.close()
            out.join_thread()
            os._exit(0)  # between steps: nothing of this rank in flight
        t0 = time.monotonic()
        try:
            gate.enter(step)
        except RankLost as e:
            out.put(("lost", step, e.rank, time.monotonic() - t0))
            break
        part = torch.from_numpy(O.gemm_nt_int8(x, q[r0:r1], s[r0:r1]))
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        ok = np.array_equal(torch.cat(parts, 1).numpy(), full)
        if rank == 0:
            out.put(("step", step, ok))
    if rank == 0:
        t0 = time.monotonic()
        try:
            dist.barrier()
            out.put(("barrier", "returned", 0.0))
        except Exception as e:  # noqa: BLE001 - any error ends the wait
            out.put(("barrier", type(e).__name__, time.monotonic() - t0))
    out.close()
    out.join_thread()  # flush the queue before leaving without clean-up
    os._exit(0)


@pytest.mark.timeout(120)
@pytest.mark.parametrize("mode", ["leave", "vanish"])
def test_world2_rank_loss_between_steps_is_detected_on_the_host(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gate_rank, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    events = [q.get(timeout=60) for _ in range(4)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert events[0] == ("step", 1, True) and events[1] == ("step", 2, True)
    kind, step, who, waited = events[2]
    assert (kind, step, who) == ("lost", 3, 1)
    assert waited < (1.0 if mode == "leave" else 4.5)
    assert events[3][0] == "barrier" and events[3][1] != "returned" and events[3][2] < 30
