"""Row-sharded Q8 / int8 linear layers across the GPUs of one node.

One process per GPU. Each rank holds rows [r0, r1) of W (see `shard_rows`)
and calls `sharded_gemm_nt_int8` / `sharded_gemm_i8i8`; the kernel stores
every output value straight into every rank's full output C over NVLink, so
after the call each rank's C holds the whole [m, n] result (the all-gather is
part of the GEMM). `PeerOutputs` sets up what those calls need: this rank's
C and inbox word, and the other ranks' C and inbox mapped into this process
through CUDA IPC handles exchanged over torch.distributed.
"""
import ctypes

from ._lib import check, lib

IPC_HANDLE_BYTES = 72  # VMLM_IPC_HANDLE_BYTES
MAX_RANKS = 8


def shard_rows(n: int, world: int, rank: int):
    """Output rows (= rows of W) owned by `rank`: [r0, r1), blocks of ceil(n / world)."""
    if not 1 <= world <= MAX_RANKS or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    rows = -(-n // world)
    if rows * (world - 1) >= n:
        raise ValueError(f"n={n} leaves a rank without rows at world={world}")
    r0 = rank * rows
    return r0, min(n, r0 + rows)


def ipc_handle(dev_ptr: int) -> bytes:
    """Handle naming the device allocation that holds dev_ptr (and the offset)."""
    buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    check(lib().vmlm_ipc_handle(ctypes.c_void_p(dev_ptr), buf))
    return buf.raw


def ipc_open(handle: bytes) -> int:
    """Map another process's allocation; returns the address of the named pointer here."""
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError("bad IPC handle")
    out = ctypes.c_void_p()
    check(lib().vmlm_ipc_open(handle, ctypes.byref(out)))
    return out.value


def ipc_close(dev_ptr: int) -> None:
    check(lib().vmlm_ipc_close(ctypes.c_void_p(dev_ptr)))


class PeerOutputs:
    """This rank's output C [m, n] (f32) and inbox, plus every rank's, mapped here.

    Collective: every rank of `group` constructs it with the same m, n. With no
    initialised process group it is a single-rank setup. Keep the object alive
    (on every rank) while calls use it; `close()` unmaps the peers' buffers and
    must run on every rank before any rank frees its own.
    """

    def __init__(self, m: int, n: int, group=None, device=None):
        import torch
        import torch.distributed as dist
        self.m, self.n = m, n
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.c = torch.zeros((m, n), dtype=torch.float32, device=device)
        self.inbox = torch.zeros(4, dtype=torch.int32, device=device)  # one word used, 16-byte aligned
        if dist.is_available() and dist.is_initialized():
            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        if self.world > MAX_RANKS:
            raise ValueError(f"at most {MAX_RANKS} ranks")
        # a new inbox starts at zero calls (its address may be one the library has seen before)
        check(lib().vmlm_sharded_reset(ctypes.c_void_p(self.inbox.data_ptr())))
        mine = (ipc_handle(self.c.data_ptr()), ipc_handle(self.inbox.data_ptr()))
        if self.world > 1:
            torch.cuda.synchronize()
            handles = [None] * self.world
            dist.all_gather_object(handles, mine, group=group)
        else:
            handles = [mine]
        self._opened = []
        c_ptrs, in_ptrs = [], []
        for q, (hc, hi) in enumerate(handles):
            if q == self.rank:
                c_ptrs.append(self.c.data_ptr())
                in_ptrs.append(self.inbox.data_ptr())
            else:
                pc, pi = ipc_open(hc), ipc_open(hi)
                self._opened += [pc, pi]
                c_ptrs.append(pc)
                in_ptrs.append(pi)
        self.c_ptrs = (ctypes.c_void_p * self.world)(*c_ptrs)
        self.inbox_ptrs = (ctypes.c_void_p * self.world)(*in_ptrs)

    def reset(self) -> None:
        """Zero this rank's inbox after a failed call (every rank, after a host barrier)."""
        check(lib().vmlm_sharded_reset(ctypes.c_void_p(self.inbox.data_ptr())))

    def close(self) -> None:
        for p in self._opened:
            ipc_close(p)
        self._opened = []
        self.reset()


class RankLost(RuntimeError):
    """A rank of a sharded group left, or stopped answering, between steps."""

    def __init__(self, rank: int, how: str):
        self.rank = rank
        super().__init__(f"rank {rank} {how}")


class StepGate:
    """Host-side liveness check before each step of row-sharded calls.

    A sharded call ends only when every rank's outputs have landed, so a rank
    that is gone makes the others' kernels wait until their bounded wait runs
    out. The gate finds that out on the host first: `enter(step)` posts this
    rank's step number to the process group's key-value store and waits, for at
    most `timeout_s`, until every rank has posted that step; a rank that has
    called `leave()` (between steps, with nothing of its own in flight) raises
    RankLost at once, and one that posts nothing in time raises RankLost when
    the limit runs out. Only then is the step's kernel launched. The store is
    torch.distributed's (any object with set / get / check works)."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 10.0, prefix: str = "vmlm_gate"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix = timeout_s, prefix

    def _key(self, what: str, q: int) -> str:
        return f"{self.prefix}/{what}/{q}"

    def enter(self, step: int) -> None:
        import time
        self.store.set(self._key("step", self.rank), str(step))
        waiting = [q for q in range(self.world) if q != self.rank]
        deadline = time.monotonic() + self.timeout_s
        while waiting:
            for q in list(waiting):
                if self.store.check([self._key("left", q)]):
                    raise RankLost(q, f"left the group before step {step}")
                key = self._key("step", q)
                if self.store.check([key]) and int(self.store.get(key)) >= step:
                    waiting.remove(q)
            if waiting and time.monotonic() > deadline:
                raise RankLost(waiting[0], f"did not reach step {step} within {self.timeout_s} s")
            if waiting:
                time.sleep(0.001)

    def leave(self) -> None:
        """Announce that this rank takes no further steps (call between steps)."""
        self.store.set(self._key("left", self.rank), "1")


def _dev(x, dtype, count, name):
    from .kernels import _dev_ptr
    return _dev_ptr(x, dtype, count, name)


def sharded_gemm_nt_int8(a, q_shard, scale_shard, peers: PeerOutputs, m, n, k, stream=None) -> None:
    """C = x . dequant(W)^T over all ranks; this rank passes its rows of W (int8) and scales."""
    from .kernels import _stream_ptr
    r0, r1 = shard_rows(n, peers.world, peers.rank)
    check(lib().vmlm_sharded_gemm_nt_int8_dev(
        _dev(a, "float32", m * k, "a"), _dev(q_shard, "int8", (r1 - r0) * k, "q_shard"),
        _dev(scale_shard, "float32", r1 - r0, "scale_shard"), peers.c_ptrs, peers.inbox_ptrs,
        peers.rank, peers.world, m, n, k, _stream_ptr(stream)))


def sharded_gemm_i8i8(x, w_shard, scale_shard, peers: PeerOutputs, m, n, k, stream=None) -> None:
    """C = f32(X . W^T) * scale over all ranks; this rank passes its rows of W and scales."""
    from .kernels import _stream_ptr
    r0, r1 = shard_rows(n, peers.world, peers.rank)
    check(lib().vmlm_sharded_gemm_i8i8_dev(
        _dev(x, "int8", m * k, "x"), _dev(w_shard, "int8", (r1 - r0) * k, "w_shard"),
        _dev(scale_shard, "float32", r1 - r0, "scale_shard"), peers.c_ptrs, peers.inbox_ptrs,
        peers.rank, peers.world, m, n, k, _stream_ptr(stream)))
