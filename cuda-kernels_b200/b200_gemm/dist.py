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
