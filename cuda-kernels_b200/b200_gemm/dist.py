"""Single-node multi-GPU driver for the row-sharded BF16 GEMM.

The job (BASELINE config "row-sharded large GEMM"): C = A @ B with A split
into contiguous row panels, one per rank (one process per GPU); B is
broadcast once from a source rank with NCCL over NVLink; each rank multiplies
its panel with the local copy of B on its own GPU; C stays sharded, and an
optional all-gather assembles it.

The reference has no multi-GPU code at all (typr7/CUDA-Kernels is a
single-GPU kernel collection); this driver is new.  Design points:

  * B is broadcast in column chunks when it is stored [N,K] (each chunk is a
    contiguous block of B's rows), on a side stream; the GEMM of chunk j runs
    on the compute stream as soon as chunk j has arrived (CUDA event), so
    the broadcast overlaps the GEMM of the chunks before it.  [K,N] B is
    broadcast whole (its column chunks are not contiguous).
  * The persistent GEMM occupies every SM, so an NCCL kernel queued behind
    it starts only between two GEMM launches.  On B200 (NVLink 5, NVSwitch)
    one whole-B broadcast before the GEMM measured fastest at 4 and 8 GPUs
    (128 MiB at ~560 GB/s, 0.24 ms): chunking adds a serialised broadcast
    per chunk, and leaving SMs free for the broadcast (GEMM grid limited,
    NCCL limited to as many CTAs) cost the GEMM more than it hid.  `chunks`
    stays available; 1 is the default.
  * No kernel reads another GPU's memory: B lands in each GPU's own HBM
    first.
  * The GEMM is pluggable (`gemm_fn`) so the host logic can be tested with
    CPU ranks (gloo) and a CPU GEMM; the default is b200_gemm.gemm.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist

from . import _lib as _abi


def shard_rows(M: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's contiguous row panel; the first M % world ranks get one extra row."""
    if world <= 0 or not (0 <= rank < world) or M < 0:
        raise ValueError(f"bad shard request M={M} world={world} rank={rank}")
    base, extra = divmod(M, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


def chunk_bounds(N: int, chunks: int, align: int = 64) -> list[tuple[int, int]]:
    """Split [0, N) into at most `chunks` pieces whose starts are multiples of `align`
    (keeps every output column offset 16-byte aligned for TMA)."""
    if N <= 0:
        return []
    chunks = max(1, min(chunks, (N + align - 1) // align))
    step = ((N + chunks - 1) // chunks + align - 1) // align * align
    out = []
    s = 0
    while s < N:
        out.append((s, min(s + step, N)))
        s += step
    return out


GemmFn = Callable[..., torch.Tensor]


def _default_gemm(a, b, *, b_layout, out):
    import b200_gemm
    return b200_gemm.gemm(a, b, b_layout=b_layout, out=out)


@dataclass
class ShardedResult:
    c_local: torch.Tensor  # this rank's row panel of C
    row_start: int
    row_stop: int


def broadcast_b(b: torch.Tensor, src: int = 0, group=None) -> None:
    """Broadcast B from `src` to every rank of `group` in place."""
    dist.broadcast(b, src=src, group=group)


def row_sharded_gemm(a_local: torch.Tensor, b: torch.Tensor, *, M: int, b_layout: str = "kn", src: int = 0,
                     group=None, chunks: int = 1, out: torch.Tensor | None = None,
                     gemm_fn: GemmFn | None = None, broadcast: bool = True) -> ShardedResult:
    """One row-sharded GEMM step on this rank.

    a_local : this rank's panel A[start:stop, :] (shape [stop-start, K])
    b       : on `src`, the full B; on the other ranks, a buffer of the same
              shape and dtype that receives it (unless broadcast=False, in
              which case every rank already holds B)
    M       : global number of rows of A (used to check the panel size)
    chunks  : number of column chunks of an [N,K] B to broadcast and
              multiply one after another (1 = whole B, then the GEMM)
    """
    gemm_fn = gemm_fn or _default_gemm
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    start, stop = shard_rows(M, world, rank)
    if a_local.shape[0] != stop - start:
        raise ValueError(f"rank {rank}: A panel has {a_local.shape[0]} rows, expected {stop - start}")
    K = a_local.shape[1]
    N = b.shape[0] if b_layout == "nk" else b.shape[1]
    if (b.shape[1] if b_layout == "nk" else b.shape[0]) != K:
        raise ValueError("inner dimensions of the A panel and B differ")
    if out is None:
        out = torch.empty((stop - start, N), dtype=a_local.dtype, device=a_local.device)

    use_streams = a_local.is_cuda
    if not broadcast or world == 1:
        gemm_fn(a_local, b, b_layout=b_layout, out=out)
        return ShardedResult(out, start, stop)

    if b_layout != "nk" or chunks <= 1:
        broadcast_b(b, src, group)
        gemm_fn(a_local, b, b_layout=b_layout, out=out)
        return ShardedResult(out, start, stop)

    # [N,K] B: broadcast row blocks of B on a side stream, multiply each block
    # as soon as it has arrived.
    bounds = chunk_bounds(N, chunks)
    if use_streams:
        compute = torch.cuda.current_stream(a_local.device)
        comm = _comm_stream(a_local.device)
        comm.wait_stream(compute)
        events = []
        with torch.cuda.stream(comm):
            for (s, e) in bounds:
                dist.broadcast(b[s:e], src=src, group=group)
                ev = torch.cuda.Event()
                ev.record(comm)
                events.append(ev)
        for (s, e), ev in zip(bounds, events):
            compute.wait_event(ev)
            gemm_fn(a_local, b[s:e], b_layout="nk", out=out[:, s:e])
        b.record_stream(comm)
    else:
        for (s, e) in bounds:
            dist.broadcast(b[s:e], src=src, group=group)
            gemm_fn(a_local, b[s:e], b_layout="nk", out=out[:, s:e])
    return ShardedResult(out, start, stop)


_COMM_STREAMS: dict = {}


def _comm_stream(device) -> "torch.cuda.Stream":
    """One side stream per device for the broadcasts (reused across calls)."""
    key = torch.device(device).index
    if key not in _COMM_STREAMS:
        _COMM_STREAMS[key] = torch.cuda.Stream(device=device)
    return _COMM_STREAMS[key]


class _DevBuf:
    """__cuda_array_interface__ view of raw device memory (int16 words; viewed as bf16 by the caller)."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<i2", "data": (ptr, False),
                                         "version": 3, "strides": None}


class GatheredC:
    """Gathered-C buffers for the fused GEMM + all-gather: every rank owns a
    [M, ldc] bf16 buffer (allocated with b200_ipc_alloc) and maps every other
    rank's into its process (b200_ipc_open), so the gathering kernel can store
    its C tiles straight into all of them over NVLink.  Collective: every rank
    of `group` constructs it (and closes it) in the same order."""

    def __init__(self, M: int, N: int, group=None, device=None):
        import ctypes
        from . import _lib
        self._lib = _lib.load()
        self.M, self.N = M, N
        self.ldc = (N + 7) // 8 * 8
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the gathering GEMM stores to at most 8 ranks")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        nbytes = max(M * self.ldc * 2, 16)
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * _lib.B200_IPC_HANDLE_BYTES)()
        with torch.cuda.device(self.device):
            rc = self._lib.b200_ipc_alloc(nbytes, ctypes.byref(ptr), ctypes.cast(handle, ctypes.c_void_p))
        if rc != _lib.B200_OK:
            raise _lib.B200GemmError(rc, "b200_ipc_alloc")
        self._own = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.ptrs = []
        self._opened = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.ptrs.append(self._own)
                    continue
                hb = (ctypes.c_ubyte * _lib.B200_IPC_HANDLE_BYTES).from_buffer_copy(h)
                peer = ctypes.c_void_p()
                rc = self._lib.b200_ipc_open(ctypes.cast(hb, ctypes.c_void_p), ctypes.byref(peer))
                if rc != _lib.B200_OK:
                    raise _lib.B200GemmError(rc, f"b200_ipc_open(rank {r})")
                self.ptrs.append(peer.value)
                self._opened.append(peer.value)
        full = torch.as_tensor(_DevBuf(self._own, (M, self.ldc)), device=self.device).view(torch.bfloat16)
        self.local = full[:, :N]  # this rank's gathered C

    def close(self) -> None:
        """Unmap the peers' buffers, then (after every rank has) free this rank's."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                self._lib.b200_ipc_close(p)
        self._opened = []
        dist.barrier(group=self.group)
        self.local = None
        with torch.cuda.device(self.device):
            self._lib.b200_ipc_free(self._own)
        self._own = None


def broadcast_chunks(nbytes: int, world: int, align: int = 256) -> list[tuple[int, int]]:
    """Byte ranges [(offset, length)] of the pieces PeerBroadcast scatters: one
    per receiving rank (ranks 1 .. world-1 in order), starts aligned to
    `align` bytes, together covering [0, nbytes) exactly once."""
    if world < 2 or nbytes <= 0:
        return []
    parts = world - 1
    bounds = [min(nbytes, (nbytes * i // parts + align - 1) // align * align) for i in range(parts)] + [nbytes]
    return [(bounds[i], bounds[i + 1] - bounds[i]) for i in range(parts)]


class PeerBroadcast:
    """Broadcast of one device buffer from rank 0 to every rank, once per step,
    on the copy engines over NVLink, overlapped with the GEMMs.

    A collective kernel needs SMs, and the persistent GEMM occupies every SM,
    so an NCCL broadcast queued beside a GEMM only runs between GEMMs (B200,
    2 GPUs, 32 MiB of B per 4096^3 step: broadcast then GEMM 156 us a step,
    NCCL on a side stream 119 us, copy engines 100 us against 95 us for the
    GEMM alone).  Here every rank owns three IPC-mapped receive slots (step s
    uses slot s % 3) and a small flag array; rank 0 scatters piece q-1 of the
    buffer to rank q (broadcast_chunks), and each receiving rank forwards its
    piece to the other receivers as soon as it has landed, so every byte
    crosses rank 0's links once.  Copies go into the peers' slots on the copy
    engines, each followed by a flag write into the reader's memory; a
    reader's compute stream waits for its flags before the GEMM of that step,
    and after the GEMM tells every writer that the slot is free again.  No SM
    is used by any of it.  The per-step protocol is native (b200_bcast_* in
    include/b200_gemm.h): a step costs three calls whatever the world size.
    This class allocates and maps the buffers and exchanges their handles.

    Per step s, on every rank, in the same order:
        pb.issue(s + 2, src)      # rank 0: the buffer two steps on (others: None)
        pb.wait(s, stream)        # the slot of step s has arrived (no-op on rank 0)
        ... GEMM reading pb.data(s, src) on `stream` ...
        pb.release(s, stream)     # this rank is done reading slot s % 3
    with pb.issue(0, src) and pb.issue(1, src) once before the first step (an
    issue may run at most two steps ahead of the oldest unreleased step: the
    writers of step s wait for the release of step s - 3).  Steps count up from 0
    and are never reused (flags compare step numbers).  Rank 0 reads `src`
    in place; it must not change until the copies of that step are done
    (pb.copied(s) is an event for that).  Every rank of `group` constructs,
    steps and closes it together; a rank that stops stepping leaves the
    others' streams waiting on its flags (stream waits have no time limit)."""

    SLOTS = _abi.B200_BCAST_SLOTS

    def __init__(self, nbytes: int, group=None, device=None):
        import ctypes
        from . import _lib
        self._lib = _lib.load()
        self.nbytes = int(nbytes)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("PeerBroadcast supports up to 8 ranks")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        W = self.world
        flag_bytes = max(int(self._lib.b200_bcast_flag_bytes(W)), 16)
        own, handles = [], []
        with torch.cuda.device(self.device):
            for nb in [self.nbytes] * self.SLOTS + [flag_bytes]:
                p = ctypes.c_void_p()
                h = (ctypes.c_ubyte * _lib.B200_IPC_HANDLE_BYTES)()
                rc = self._lib.b200_ipc_alloc(max(nb, 16), ctypes.byref(p), ctypes.cast(h, ctypes.c_void_p))
                if rc != _lib.B200_OK:
                    raise _lib.B200GemmError(rc, "b200_ipc_alloc")
                own.append(p.value)
                handles.append(bytes(h))
        self._own = own
        flags = torch.as_tensor(_DevBuf(own[self.SLOTS], ((flag_bytes + 1) // 2,)), device=self.device)
        flags.zero_()
        torch.cuda.synchronize(self.device)
        all_h = [None] * W
        dist.all_gather_object(all_h, handles, group=group)
        self._opened = []
        ptrs = {self.rank: own}
        with torch.cuda.device(self.device):
            for r in range(W):
                if r == self.rank:
                    continue
                mapped = []
                for h in all_h[r]:
                    hb = (ctypes.c_ubyte * _lib.B200_IPC_HANDLE_BYTES).from_buffer_copy(h)
                    pp = ctypes.c_void_p()
                    rc = self._lib.b200_ipc_open(ctypes.cast(hb, ctypes.c_void_p), ctypes.byref(pp))
                    if rc != _lib.B200_OK:
                        raise _lib.B200GemmError(rc, f"b200_ipc_open(rank {r})")
                    mapped.append(pp.value)
                    self._opened.append(pp.value)
                ptrs[r] = mapped
        slots = (ctypes.c_void_p * (W * self.SLOTS))(*[ptrs[r][k] for r in range(W) for k in range(self.SLOTS)])
        flagp = (ctypes.c_void_p * W)(*[ptrs[r][self.SLOTS] for r in range(W)])
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):  # its copy streams belong to this device
            rc = self._lib.b200_bcast_create(self.rank, W, self.nbytes, slots, flagp, ctypes.byref(handle))
        if rc != _lib.B200_OK:
            raise _lib.B200GemmError(rc, "b200_bcast_create")
        self._h = handle
        self.slot_ptr = own[:self.SLOTS]
        # Steps alternate between two copy streams: the copies of step s+1
        # need not wait for the last copies of step s (rank 0's pieces of s+1
        # go out while the others still forward the pieces of s).  Each
        # step's copies are joined back into its stream.
        self.comms = [torch.cuda.Stream(self.device) for _ in range(2)]
        self._copied = [torch.cuda.Event() for _ in range(self.SLOTS)]
        dist.barrier(group=group)  # every rank's flags are zero before anyone signals

    def _check(self, rc: int, what: str) -> None:
        from . import _lib
        if rc != _lib.B200_OK:
            raise _lib.B200GemmError(rc, what)

    def issue(self, step: int, src: torch.Tensor | None = None, offset: int = 0, length: int | None = None) -> None:
        """Queue the copies of step `step` on the copy stream (rank 0: from `src`,
        a contiguous tensor of nbytes on this device; others: forwarding).  With
        offset / length only those bytes move (offset a multiple of 256), to the
        same offsets of the step's slot."""
        import ctypes
        if self.world == 1:
            return
        length = self.nbytes - offset if length is None else length
        ptr = None
        if self.rank == 0:
            if src is None or not src.is_contiguous() or src.numel() * src.element_size() != self.nbytes:
                raise ValueError("rank 0 needs a contiguous source tensor of nbytes")
            ptr = src.data_ptr()
        self._check(self._lib.b200_bcast_issue_range(self._h, step, ctypes.c_void_p(ptr), offset, length,
                                                     ctypes.c_void_p(self.comms[step % 2].cuda_stream)),
                    "b200_bcast_issue")
        if self.rank == 0:
            self._copied[step % self.SLOTS].record(self.comms[step % 2])

    def wait(self, step: int, stream) -> None:
        """Make `stream` wait until this rank's slot of `step` is complete."""
        import ctypes
        self._check(self._lib.b200_bcast_wait(self._h, step, ctypes.c_void_p(stream.cuda_stream)), "b200_bcast_wait")

    def data(self, step: int, src: torch.Tensor | None = None) -> torch.Tensor:
        """The buffer of `step` on this rank as flat bytes (rank 0: src itself)."""
        if self.rank == 0 or self.world == 1:
            return src
        p = self.slot_ptr[step % self.SLOTS]
        return torch.as_tensor(_DevBuf(p, ((self.nbytes + 1) // 2,)), device=self.device).view(torch.uint8)[:self.nbytes]

    def release(self, step: int, stream) -> None:
        """After the work on `stream` that reads the slot of `step`: tell every
        rank that writes into this rank's slots that it may overwrite it."""
        import ctypes
        self._check(self._lib.b200_bcast_release(self._h, step, ctypes.c_void_p(stream.cuda_stream)),
                    "b200_bcast_release")

    def gemm(self, step: int, a: torch.Tensor, b_shape, *, out: torch.Tensor, b_layout: str = "kn",
             src: torch.Tensor | None = None, stream=None, b_offset: int = 0, ldb: int | None = None) -> torch.Tensor:
        """out = a @ op(B of step `step`) through b200_bcast_gemm, in place of
        wait / gemm / release: the CTA-pair kernel waits for the step's data and
        releases the slot itself, so consecutive GEMMs on `stream` keep their
        programmatic overlap.  b_shape is the shape of the B this GEMM reads,
        starting at byte b_offset of the step's buffer with row pitch ldb
        (default: b_shape's columns); rank 0 passes that B as `src`."""
        import ctypes
        from . import _lib
        stream = stream if stream is not None else torch.cuda.current_stream(self.device)
        M, K = a.shape
        rows, cols = b_shape
        N = rows if b_layout == "nk" else cols
        if (cols if b_layout == "nk" else rows) != K or tuple(out.shape) != (M, N):
            raise ValueError("shapes of A, B and out do not match")
        if a.dtype != torch.bfloat16 or out.dtype != torch.bfloat16 or a.stride(1) != 1 or out.stride(1) != 1:
            raise ValueError("A and out must be row-major bf16")
        b0 = src.data_ptr() if (self.rank == 0 and src is not None) else None
        ldb = cols if ldb is None else ldb
        rc = self._lib.b200_bcast_gemm(self._h, step, b_offset, ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b0),
                                       ctypes.c_void_p(out.data_ptr()), M, N, K, max(a.stride(0), 1), ldb,
                                       max(out.stride(0), 1), _lib.B200_B_NK if b_layout == "nk" else _lib.B200_B_KN,
                                       ctypes.c_void_p(stream.cuda_stream))
        self._check(rc, f"b200_bcast_gemm step {step}")
        return out

    def copied(self, step: int) -> "torch.cuda.Event":
        """Rank 0: event after its copies of `step` (src may change once it has completed)."""
        return self._copied[step % self.SLOTS]

    def close(self) -> None:
        """Wait for everything queued, then unmap the peers' buffers and free
        this rank's (every rank together)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._lib.b200_bcast_destroy(self._h)
        with torch.cuda.device(self.device):
            for p in self._opened:
                self._lib.b200_ipc_close(p)
        self._opened = []
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._own:
                self._lib.b200_ipc_free(p)
        self._own = None


def row_sharded_gemm_peer(a_local: torch.Tensor, b: torch.Tensor, *, M: int, exchange: "PeerBroadcast", step: int,
                          out: torch.Tensor | None = None, first_rows: int | None = None,
                          stream=None) -> ShardedResult:
    """One row-sharded GEMM job with B (stored [N, K], the reference's layout:
    its rows are columns of C and contiguous) moved from rank 0 on the copy
    engines (`exchange`, a PeerBroadcast of B's bytes) in two parts: the first
    `first_rows` rows as exchange step `step`, the rest as step `step + 1`.
    The GEMM of the first column block of C starts as soon as its rows have
    arrived, and the rest of B moves while it runs; each GEMM waits for its
    rows and releases them inside the kernel (b200_bcast_gemm).  Uses exchange
    steps `step` and `step + 1`.  On rank 0, `b` is the source."""
    world = dist.get_world_size()
    rank = dist.get_rank()
    start, stop = shard_rows(M, world, rank)
    if a_local.shape[0] != stop - start:
        raise ValueError(f"rank {rank}: A panel has {a_local.shape[0]} rows, expected {stop - start}")
    N, K = b.shape
    if a_local.shape[1] != K:
        raise ValueError("inner dimensions of the A panel and B differ")
    if exchange.nbytes != N * K * b.element_size():
        raise ValueError("the exchange must be sized for B")
    if first_rows is None:  # about an eighth of B, whole 256-row blocks
        first_rows = max(256, (N // 8) // 256 * 256)
    first_rows = min(first_rows, N)
    if first_rows % 256 != 0 and first_rows != N:
        raise ValueError("first_rows must be a multiple of 256")
    bytes0 = first_rows * K * b.element_size()
    if out is None:
        out = torch.empty((stop - start, N), dtype=a_local.dtype, device=a_local.device)
    src = b if rank == 0 else None
    exchange.issue(step, src, offset=0, length=bytes0)
    if first_rows < N:
        exchange.issue(step + 1, src, offset=bytes0, length=exchange.nbytes - bytes0)
    exchange.gemm(step, a_local, (first_rows, K), out=out[:, :first_rows], b_layout="nk",
                  src=b[:first_rows] if rank == 0 else None, stream=stream, b_offset=0, ldb=K)
    if first_rows < N:
        exchange.gemm(step + 1, a_local, (N - first_rows, K), out=out[:, first_rows:], b_layout="nk",
                      src=b[first_rows:] if rank == 0 else None, stream=stream, b_offset=bytes0, ldb=K)
    else:  # keep the step count of every job at two
        exchange.issue(step + 1, src, offset=0, length=0)
        exchange.wait(step + 1, stream if stream is not None else torch.cuda.current_stream(a_local.device))
        exchange.release(step + 1, stream if stream is not None else torch.cuda.current_stream(a_local.device))
    return ShardedResult(out, start, stop)


def row_sharded_gemm_gather(a_local: torch.Tensor, b: torch.Tensor, *, gathered: GatheredC, M: int,
                            b_layout: str = "nk", src: int = 0, group=None, broadcast: bool = True) -> torch.Tensor:
    """One row-sharded GEMM step with the C all-gather fused into the GEMM
    (b200_gemm_bf16_allgather): every rank's epilogue stores its C tiles into
    every rank's gathered C.  Returns this rank's full [M, N] C.

    Ordering: before the kernel, the ranks meet in the B broadcast (or a
    barrier collective when broadcast=False), so no rank is still reading the
    previous step's gathered C when the others start writing it; after the
    kernel, a barrier collective on the same stream makes the result complete
    on every rank."""
    import ctypes
    from . import _lib
    lib = _lib.load()
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    start, stop = shard_rows(M, world, rank)
    if a_local.shape[0] != stop - start:
        raise ValueError(f"rank {rank}: A panel has {a_local.shape[0]} rows, expected {stop - start}")
    K = a_local.shape[1]
    N = b.shape[0] if b_layout == "nk" else b.shape[1]
    if gathered.M != M or gathered.N != N:
        raise ValueError("gathered-C buffers have another shape")
    dev = a_local.device
    token = torch.zeros(1, device=dev)
    if broadcast:
        broadcast_b(b, src, group)
    else:
        dist.all_reduce(token, group=group)
    outs = (ctypes.c_void_p * world)(*gathered.ptrs)
    s = torch.cuda.current_stream(dev)
    rc = lib.b200_gemm_bf16_allgather(ctypes.c_void_p(a_local.data_ptr()), ctypes.c_void_p(b.data_ptr()), outs, world,
                                      stop - start, N, K, max(a_local.stride(0), 1), max(b.stride(0), 1),
                                      gathered.ldc, start, M, _lib.B200_B_NK if b_layout == "nk" else _lib.B200_B_KN,
                                      ctypes.c_void_p(s.cuda_stream))
    if rc != _lib.B200_OK:
        raise _lib.B200GemmError(rc, "b200_gemm_bf16_allgather")
    dist.all_reduce(token, group=group)  # every rank's stores are complete after this
    return gathered.local


def gather_rows(c_local: torch.Tensor, M: int, group=None) -> torch.Tensor:
    """All-gather the row panels of C into the full [M, N] matrix on every rank."""
    world = dist.get_world_size(group)
    sizes = [shard_rows(M, world, r) for r in range(world)]
    N = c_local.shape[1]
    if all((e - s) == (sizes[0][1] - sizes[0][0]) for s, e in sizes):
        full = torch.empty((M, N), dtype=c_local.dtype, device=c_local.device)
        dist.all_gather_into_tensor(full, c_local.contiguous(), group=group)
        return full
    # Ragged panels: gather padded panels, then drop the padding rows.
    rows = sizes[0][1] - sizes[0][0]
    padded = torch.zeros((rows, N), dtype=c_local.dtype, device=c_local.device)
    padded[: c_local.shape[0]] = c_local
    stacked = torch.empty((world * rows, N), dtype=c_local.dtype, device=c_local.device)
    dist.all_gather_into_tensor(stacked, padded, group=group)
    return torch.cat([stacked[r * rows: r * rows + (e - s)] for r, (s, e) in enumerate(sizes)], dim=0)
