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
