"""One-shot NVLink peer all-reduce (cb_peer_allreduce) on two GPUs: every rank's
result equals the fp32 sum of the partials in rank order, rounded once (exact
comparison), across repeated calls (both buffer parities), in-place calls and
CUDA-graph replays. Skipped with fewer than two GPUs."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _expected(parts, dtype):
    acc = torch.zeros_like(parts[0], dtype=torch.float32)
    for p in parts:
        acc += p.float()
    return acc.to(dtype)


def _rank(rank, world, port):
    import sys

    sys.path.insert(0, os.path.join(ROOT, "cache-barrier_b200"))
    import torch.distributed as dist

    from cb200.peer import PeerAllReduce

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        ar = PeerAllReduce(64 * 5120, device=dev)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        for dtype in (torch.bfloat16, torch.float16):
            for n in (5120, 8 * 5120, 64 * 5120, 1000, 3):
                for _rep in range(3):
                    x = torch.randn(n, generator=g, device=dev).to(dtype)
                    parts = [torch.empty_like(x) for _ in range(world)]
                    dist.all_gather(parts, x)
                    out = ar(x)
                    torch.cuda.synchronize()
                    assert torch.equal(out, _expected(parts, dtype)), (dtype, n)
        # in place
        x = torch.randn(8 * 5120, generator=g, device=dev).to(torch.bfloat16)
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x)
        ar(x, out=x)
        torch.cuda.synchronize()
        assert torch.equal(x, _expected(parts, torch.bfloat16))
        # inside a CUDA graph (three calls per replay)
        xs = [torch.empty(5120, device=dev, dtype=torch.bfloat16) for _ in range(3)]
        outs = [torch.empty_like(t) for t in xs]
        for t, o in zip(xs, outs):
            ar(t, out=o)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for t, o in zip(xs, outs):
                ar(t, out=o)
        for _replay in range(2):
            for t in xs:
                t.copy_(torch.randn(5120, generator=g, device=dev).to(torch.bfloat16))
            torch.cuda.synchronize()
            gathered = []
            for t in xs:
                parts = [torch.empty_like(t) for _ in range(world)]
                dist.all_gather(parts, t)
                gathered.append(parts)
            graph.replay()
            torch.cuda.synchronize()
            for o, parts in zip(outs, gathered):
                assert torch.equal(o, _expected(parts, torch.bfloat16))
        del graph
        assert int(ar.status.item()) == 0
        ar.close()
    finally:
        dist.destroy_process_group()


def test_peer_allreduce_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_rank, args=(2, port), nprocs=2, join=True, start_method="spawn")
