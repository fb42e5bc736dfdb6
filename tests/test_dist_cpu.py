"""CPU (gloo) tests of the row-sharded multi-GPU driver's host logic
(b200_gemm/dist.py): panel partitioning, chunked broadcast of B, gather of C,
and a rank that fails before the broadcast.  The GEMM is the CPU oracle here;
the same driver runs b200_gemm.gemm over NCCL on GPUs."""
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests._util import spawn_ranks

from b200_gemm.dist import chunk_bounds, gather_rows, row_sharded_gemm, shard_rows


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_rows_cover_and_balance():
    for M in (0, 1, 7, 8, 37, 131072):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_rows(M, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == M
            for (s0, e0), (s1, _) in zip(spans, spans[1:]):
                assert e0 == s1
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_rows(8, 2, 2)


def test_chunk_bounds_aligned():
    for N in (1, 63, 64, 65, 1000, 4096, 8192):
        for chunks in (1, 2, 3, 4, 7):
            b = chunk_bounds(N, chunks)
            assert b[0][0] == 0 and b[-1][1] == N
            assert all(s % 64 == 0 for s, _ in b)
            assert len(b) <= chunks


def _cpu_gemm(a, b, *, b_layout, out):
    from oracle import oracle as o
    from tests._util import bits, from_bits
    c = o.gemm_bf16(bits(a), bits(b.contiguous()), 0 if b_layout == "nk" else 1, threads=1)
    out.copy_(from_bits(c))
    return out


def _worker(rank, world, port, M, N, K, layout, chunks, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    try:
        from tests._util import uniform_bf16
        a_full = uniform_bf16((M, K), 1)
        b_full = uniform_bf16((N, K) if layout == "nk" else (K, N), 2)
        s, e = shard_rows(M, world, rank)
        b = b_full.clone() if rank == 0 else torch.zeros_like(b_full)
        res = row_sharded_gemm(a_full[s:e].contiguous(), b, M=M, b_layout=layout, chunks=chunks, gemm_fn=_cpu_gemm)
        assert torch.equal(b, b_full), "broadcast did not deliver B"
        full = gather_rows(res.c_local, M)
        if rank == 0:
            torch.save(full, os.path.join(result_dir, "c.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("layout,chunks", [("nk", 3), ("kn", 1), ("nk", 1)])
def test_row_sharded_gemm_two_ranks(tmp_path, layout, chunks):
    M, N, K = 37, 200, 72  # ragged panels (19 + 18 rows), N not a multiple of the chunk
    world = 2
    spawn_ranks(_worker, lambda port: (world, port, M, N, K, layout, chunks, str(tmp_path)), world)
    c = torch.load(os.path.join(tmp_path, "c.pt"))
    from oracle import oracle as o
    from tests._util import bits, uniform_bf16
    a = uniform_bf16((M, K), 1)
    b = uniform_bf16((N, K) if layout == "nk" else (K, N), 2)
    ref = o.gemm_bf16(bits(a), bits(b), 0 if layout == "nk" else 1)
    assert np.array_equal(bits(c), ref)


def _failing_worker(rank, world, port, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        # Injected failure on the host: this rank leaves before the broadcast.
        os._exit(0)
    t0 = time.time()
    err = None
    try:
        b = torch.ones((64, 64), dtype=torch.bfloat16)
        row_sharded_gemm(torch.ones((32, 64), dtype=torch.bfloat16), b, M=64, b_layout="nk", chunks=1,
                         gemm_fn=_cpu_gemm)
    except Exception as e:  # the surviving rank must get an error, not hang
        err = type(e).__name__
    with open(os.path.join(result_dir, "rank0.txt"), "w") as f:
        f.write(f"{err} {time.time() - t0:.1f}")
    os._exit(0)


def test_rank_failure_surfaces_as_error(tmp_path):
    ctx = mp.spawn(_failing_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False)
    deadline = time.time() + 90
    while not ctx.join(timeout=1):
        assert time.time() < deadline, "surviving rank hung"
    err, secs = open(os.path.join(tmp_path, "rank0.txt")).read().split()
    assert err != "None", "broadcast with a missing rank did not raise"
    assert float(secs) < 60


@pytest.mark.parametrize("world", [2, 3, 4, 8])
@pytest.mark.parametrize("nbytes", [16, 1000, 32 << 20, (128 << 20) + 258])
def test_broadcast_chunks_cover_once_aligned(world, nbytes):
    """PeerBroadcast's pieces: one per receiving rank, 256-byte aligned starts,
    together covering the buffer exactly once."""
    from b200_gemm.dist import broadcast_chunks
    ch = broadcast_chunks(nbytes, world)
    assert len(ch) == world - 1
    pos = 0
    for off, n in ch:
        assert off == pos and n >= 0 and (off % 256 == 0 or off == nbytes)
        pos += n
    assert pos == nbytes
    assert broadcast_chunks(nbytes, 1) == []
