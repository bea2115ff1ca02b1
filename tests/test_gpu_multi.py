"""The multi-GPU long row on real GPUs: one process per GPU over NCCL, each
holding a contiguous shard of a long row's keys. Both of multi.long_decode's
GPU branches must equal one GPU's call over the whole row and the CPU
oracle, on every rank, three calls in a row (the plan's buffers are reused;
the third call takes the first half of the peer buffers again): the peer
exchange (one kernel that stores each rank's merged partial into every
rank's buffer over NVLink and waits for the others', the production branch)
and, with WPT_B200_PEER=0, the all-gather branch (each rank's partials
merged into its chunk of a shared buffer, one in-place all-gather, the
grouped merge). The peer branch is also replayed from a CUDA graph (three
captured calls, two replays), which its on-device call count must survive.
Skipped with fewer than two GPUs (each rank needs its own GPU: the ranks'
exchange kernels wait for one another); the all-gather logic runs on gloo
ranks on CPU in tests/test_multi_cpu.py."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

C, H = 128, 32


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(N, seed):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(1, 1, H, C, generator=g) * 0.5).bfloat16()
    e = (torch.randn(1, N, 2 * C, generator=g) * 0.5).bfloat16()
    sink = torch.randn(H, generator=g) * 0.5
    return q, e, sink


def _rank(rank, world, port, N, peer, result):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WPT_B200_PEER="1" if peer else "0")
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=device)
    try:
        import wpt_b200
        from wpt_b200 import multi
        start, stop = multi.key_shard(N, world, rank)
        for seed in (1, 2, 3):
            q, e, sink = _inputs(N, seed)
            shard = e[:, start:stop].to(device)
            pos = torch.tensor([[N - 1 - 7 * seed]], device=device)
            out, lse = multi.long_decode(q.to(device), shard[..., :C], shard[..., C:], start, pos, C ** -0.5,
                                         sink=sink.to(device))
            torch.cuda.synchronize()
            result[(rank, seed)] = (out.float().cpu().numpy(), lse.cpu().numpy(), wpt_b200.device_status())
        result[(rank, "peer")] = isinstance(next(iter(multi._PLANS.values()))[3], multi.PeerExchange)
        if peer:  # seed 1's call captured three times in a graph, replayed twice
            q, e, sink = _inputs(N, 1)
            qd, shard, sd = q.to(device), e[:, start:stop].to(device), sink.to(device)
            pos = torch.tensor([[N - 1 - 7]], device=device)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(3):
                    out, lse = multi.long_decode(qd, shard[..., :C], shard[..., C:], start, pos, C ** -0.5, sink=sd)
            for _ in range(2):
                graph.replay()
            torch.cuda.synchronize()
            result[(rank, "graph")] = (out.float().cpu().numpy(), lse.cpu().numpy(), wpt_b200.device_status())
            del graph
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("peer", [True, False])
def test_long_row_over_nccl_ranks_equals_one_gpu_and_oracle(peer):
    import wpt_b200
    from oracle import attention as oat
    from wpt_b200 import build
    build.build()
    world, N = min(4, torch.cuda.device_count()), 50000
    manager = mp.get_context("spawn").Manager()
    result = manager.dict()
    mp.start_processes(_rank, args=(world, _free_port(), N, peer, result), nprocs=world, start_method="spawn",
                       join=True)
    assert all(result[(rank, "peer")] == peer for rank in range(world))
    for seed in (1, 2, 3):
        q, e, sink = _inputs(N, seed)
        pos = torch.tensor([[N - 1 - 7 * seed]])
        whole, whole_lse = wpt_b200.forward_with_lse(q.cuda(), e.cuda()[..., :C], e.cuda()[..., C:], pos.cuda(),
                                                     C ** -0.5, sink=sink.cuda())
        ref, ref_lse = oat.range_attention(q.float().numpy(), e[..., :C].float().numpy(),
                                           e[..., C:].float().numpy(), pos.numpy(), C ** -0.5,
                                           sink=sink.double().numpy())
        for rank in range(world):
            out, lse, status = result[(rank, seed)]
            assert status == 0
            assert np.abs(out - whole.float().cpu().numpy()).max() < 1e-2
            assert np.abs(lse - whole_lse.cpu().numpy()).max() < 1e-4
            assert np.abs(out - ref).max() < 2e-2
            assert np.abs(lse - ref_lse).max() < 1e-3
            if peer and seed == 1:
                g_out, g_lse, g_status = result[(rank, "graph")]
                assert g_status == 0
                assert np.array_equal(g_out, out) and np.array_equal(g_lse, lse)


def _skip_rank(rank, world, port, N, result):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WPT_B200_PEER="1", NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=device)
    try:
        import wpt_b200
        from wpt_b200 import multi
        start, stop = multi.key_shard(N, world, rank)
        q, e, sink = _inputs(N, 1)
        qd, shard, sd = q.to(device), e[:, start:stop].to(device), sink.to(device)
        pos = torch.tensor([[N - 8]], device=device)
        multi.long_decode(qd, shard[..., :C], shard[..., C:], start, pos, C ** -0.5, sink=sd)
        torch.cuda.synchronize()
        first = wpt_b200.device_status()
        dist.barrier()  # between steps: nothing of either rank in flight
        if rank == 0:  # rank 1 skips this call: rank 0's wait for its partial runs out
            t = __import__("time").perf_counter()
            multi.long_decode(qd, shard[..., :C], shard[..., C:], start, pos, C ** -0.5, sink=sd)
            torch.cuda.synchronize()
            result[rank] = (first, wpt_b200.device_status(), __import__("time").perf_counter() - t)
        else:
            result[rank] = (first, wpt_b200.device_status(), 0.0)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_a_rank_that_skips_a_call_makes_the_others_wait_run_out():
    """Rank 1 skips a call between steps: rank 0's exchange kernel waits for
    its partial for the bounded 2 s, then returns with status bit 0 set (no
    fault, no hang); the first call, made by both ranks, reported nothing.
    Child processes on two GPUs, NVLS off, plain peer stores only."""
    from wpt_b200 import build
    build.build()
    world, N = 2, 20000
    manager = mp.get_context("spawn").Manager()
    result = manager.dict()
    mp.start_processes(_skip_rank, args=(world, _free_port(), N, result), nprocs=world, start_method="spawn",
                       join=True)
    first0, after0, seconds = result[0]
    first1, after1, _ = result[1]
    assert first0 == 0 and first1 == 0 and after1 == 0
    assert after0 & 1 and 1.5 < seconds < 30
