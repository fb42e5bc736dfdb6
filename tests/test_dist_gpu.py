"""Multi-GPU test of the row-sharded driver over NCCL with the B200 kernel
(b200_gemm/dist.py).  Needs >= 2 GPUs; each rank is its own process on its
own GPU.  B is broadcast from rank 0 in chunks overlapped with the GEMM."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tests._util import spawn_ranks

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, N, K, layout, chunks, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta
    import torch.distributed as dist
    import b200_gemm
    from b200_gemm.dist import gather_rows, row_sharded_gemm, shard_rows
    from tests._util import uniform_bf16
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        a_full = uniform_bf16((M, K), 11)
        b_full = uniform_bf16((N, K) if layout == "nk" else (K, N), 12)
        s, e = shard_rows(M, world, rank)
        a = a_full[s:e].cuda()
        b = b_full.cuda() if rank == 0 else torch.zeros(b_full.shape, dtype=torch.bfloat16, device="cuda")
        res = row_sharded_gemm(a, b, M=M, b_layout=layout, chunks=chunks)
        full = gather_rows(res.c_local, M)
        torch.cuda.synchronize()
        assert b200_gemm.check_status() == 0
        assert torch.equal(b.cpu(), b_full)
        if rank == 0:
            torch.save(full.cpu(), os.path.join(result_dir, "c.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("layout,chunks", [("nk", 4), ("kn", 1)])
def test_row_sharded_gemm_nccl(tmp_path, layout, chunks):
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs at least 2 GPUs")
    world = min(world, 8)
    M, N, K = 4099, 1000, 520  # ragged panels and a ragged last chunk
    spawn_ranks(_worker, lambda port: (world, port, M, N, K, layout, chunks, str(tmp_path)), world)
    c = torch.load(os.path.join(tmp_path, "c.pt"))
    from oracle import oracle as o
    from tests._util import bits, check_parity, uniform_bf16
    a = uniform_bf16((M, K), 11)
    b = uniform_bf16((N, K) if layout == "nk" else (K, N), 12)
    ref = o.gemm_bf16(bits(a), bits(b), 0 if layout == "nk" else 1)
    c32 = o.gemm_f32acc(bits(a), bits(b), 0 if layout == "nk" else 1).astype(np.float64)
    check_parity(bits(c), c32, ref, ctx=f"row-sharded x{world} {layout}")


def _gather_worker(rank, world, port, M, N, K, layout, steps, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta
    import torch.distributed as dist
    import b200_gemm
    from b200_gemm.dist import GatheredC, row_sharded_gemm_gather, shard_rows
    from tests._util import uniform_bf16
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    g = None
    try:
        g = GatheredC(M, N)
        s, e = shard_rows(M, world, rank)
        outs = []
        for step in range(steps):  # consecutive steps reuse the gathered buffers
            a_full = uniform_bf16((M, K), 21 + step)
            b_full = uniform_bf16((N, K) if layout == "nk" else (K, N), 31 + step)
            a = a_full[s:e].cuda()
            b = b_full.cuda() if rank == 0 else torch.zeros(b_full.shape, dtype=torch.bfloat16, device="cuda")
            full = row_sharded_gemm_gather(a, b, gathered=g, M=M, b_layout=layout)
            outs.append(full.cpu().clone())
        torch.cuda.synchronize()
        assert b200_gemm.check_status() == 0
        torch.save(outs, os.path.join(result_dir, f"c{rank}.pt"))
    finally:
        if g is not None:
            g.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("layout", ["nk", "kn"])
def test_gemm_with_fused_allgather(tmp_path, layout):
    """b200_gemm_bf16_allgather: every rank ends with the whole C, equal on all
    ranks and within the parity bounds of the oracle; two steps in a row."""
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs at least 2 GPUs")
    world = min(world, 8)
    M, N, K, steps = 2051, 1000, 520, 2  # ragged panels, N not a multiple of the tile
    spawn_ranks(_gather_worker, lambda port: (world, port, M, N, K, layout, steps, str(tmp_path)), world)
    from oracle import oracle as o
    from tests._util import bits, check_parity, uniform_bf16
    per_rank = [torch.load(os.path.join(tmp_path, f"c{r}.pt")) for r in range(world)]
    for step in range(steps):
        a = uniform_bf16((M, K), 21 + step)
        b = uniform_bf16((N, K) if layout == "nk" else (K, N), 31 + step)
        ref = o.gemm_bf16(bits(a), bits(b), 0 if layout == "nk" else 1)
        c32 = o.gemm_f32acc(bits(a), bits(b), 0 if layout == "nk" else 1).astype(np.float64)
        c0 = per_rank[0][step]
        check_parity(bits(c0), c32, ref, ctx=f"gather x{world} {layout} step {step}")
        for r in range(1, world):
            assert torch.equal(per_rank[r][step], c0), f"rank {r} gathered a different C at step {step}"


def _peer_bcast_worker(rank, world, port, nbytes, steps, ahead, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta
    import torch.distributed as dist
    import b200_gemm
    from b200_gemm.dist import PeerBroadcast
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        dev = torch.device("cuda", rank)

        def payload(s):  # the bytes rank 0 sends at step s, reproducible on every rank
            g = torch.Generator(device=dev).manual_seed(1000 + s)
            return torch.randint(0, 256, (nbytes,), generator=g, device=dev, dtype=torch.uint8)

        pb = PeerBroadcast(nbytes)
        stream = torch.cuda.current_stream(dev)
        srcs = [payload(s) for s in range(steps + ahead)] if rank == 0 else None
        for s in range(ahead):
            pb.issue(s, srcs[s] if rank == 0 else None)
        ok = True
        K, N = 256, 1024  # B [K, N] read from the front of each step's buffer
        for s in range(steps):
            pb.issue(s + ahead, srcs[s + ahead] if rank == 0 else None)
            ref_b = payload(s)[:K * N * 2].view(torch.bfloat16).view(K, N)
            src_b = srcs[s][:K * N * 2].view(torch.bfloat16).view(K, N) if rank == 0 else None
            if s % 3 == 0:
                # explicit wait / read / release
                pb.wait(s, stream)
                got = pb.data(s, srcs[s] if rank == 0 else None)
                ok &= bool(torch.equal(got, payload(s)))  # on `stream`, after the wait
                a = torch.ones((64, K), dtype=torch.bfloat16, device=dev)
                c = b200_gemm.gemm(a, got[:K * N * 2].view(torch.bfloat16).view(K, N), b_layout="kn")
                pb.release(s, stream)
            else:
                # the GEMM waits and releases itself: M = 2048 takes the CTA-pair
                # kernel (in-kernel flags), M = 64 the skinny kernel (stream operations)
                m = 2048 if s % 3 == 1 else 64
                a = torch.ones((m, K), dtype=torch.bfloat16, device=dev)
                c = torch.empty((m, N), dtype=torch.bfloat16, device=dev)
                pb.gemm(s, a, (K, N), out=c, b_layout="kn", src=src_b, stream=stream)
            ref = b200_gemm.gemm(a, ref_b, b_layout="kn")
            ok &= bool(torch.equal(torch.nan_to_num(c, nan=0.0), torch.nan_to_num(ref, nan=0.0)))
        torch.cuda.synchronize()
        pb.close()
        assert b200_gemm.check_status() == 0
        flag = torch.tensor([int(ok)], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if rank == 0:
            torch.save(bool(flag.item()), os.path.join(result_dir, "ok.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("ahead", [1, 2])
@pytest.mark.parametrize("nbytes", [(2 << 20) + 258, 32 << 20])
def test_peer_broadcast_delivers_every_step(tmp_path, nbytes, ahead):
    """PeerBroadcast (copy engines + stream-ordered flags): over several steps,
    with the three receive slots reused in turn and the copies issued one or
    two steps ahead of the step being read, every rank receives exactly the
    bytes rank 0 sent for that step, and a GEMM reading them sees them — after
    an explicit wait, and through b200_bcast_gemm, which waits and releases
    inside the CTA-pair kernel or with stream operations around the others."""
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs at least 2 GPUs")
    world = min(world, 8)
    spawn_ranks(_peer_bcast_worker, lambda port: (world, port, nbytes, 7, ahead, str(tmp_path)), world)
    assert torch.load(os.path.join(tmp_path, "ok.pt"))


def _peer_job_worker(rank, world, port, M, N, K, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta
    import torch.distributed as dist
    import b200_gemm
    from b200_gemm.dist import PeerBroadcast, row_sharded_gemm, row_sharded_gemm_peer, shard_rows
    from tests._util import uniform_bf16
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        s, e = shard_rows(M, world, rank)
        ok = True
        pb = PeerBroadcast(N * K * 2)
        for job in range(2):  # two jobs: both slots are reused
            a = uniform_bf16((M, K), 30 + job)[s:e].cuda()
            b_full = uniform_bf16((N, K), 40 + job).cuda()
            b_src = b_full.clone() if rank == 0 else torch.zeros_like(b_full)
            got = row_sharded_gemm_peer(a, b_src, M=M, exchange=pb, step=2 * job, first_rows=256).c_local
            ref = row_sharded_gemm(a, b_full, M=M, b_layout="nk", broadcast=False).c_local
            torch.cuda.synchronize()
            ok &= bool(torch.equal(got, ref))
        pb.close()
        assert b200_gemm.check_status() == 0
        flag = torch.tensor([int(ok)], device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if rank == 0:
            torch.save(bool(flag.item()), os.path.join(result_dir, "ok.pt"))
    finally:
        dist.destroy_process_group()


def test_row_sharded_job_on_copy_engines(tmp_path):
    """The row-sharded job with B moved in two parts on the copy engines
    (dist.row_sharded_gemm_peer: the first block's GEMM waits for its rows and
    starts while the rest of B moves) gives every rank the same panel of C as
    the plain GEMM on a local copy of B, bit for bit, over two jobs."""
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs at least 2 GPUs")
    world = min(world, 8)
    spawn_ranks(_peer_job_worker, lambda port: (world, port, 1031 * world, 1280, 520, str(tmp_path)), world)
    assert torch.load(os.path.join(tmp_path, "ok.pt"))
