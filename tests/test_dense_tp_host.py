"""Tensor-parallel sharding and all-reduce placement of the dense projection harness,
run as two gloo ranks on CPU with an fp32 matmul standing in for the GPU kernels."""

import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HARNESS = os.path.join(ROOT, "cache-barrier_b200", "harness")
sys.path.insert(0, HARNESS)

import dense_tp as D  # noqa: E402

DIMS = D.Dims(hidden=256, qkv=384, inter=512, layers=2)
T = 3


class CpuMatmul(D.Backend):
    name = "cpu_fp32"

    def prepare(self, w):
        return w.float().contiguous()

    def weight_bytes(self, N, K):
        return 4 * N * K

    def run(self, x, h, out, scratch):
        out.copy_(x.float() @ h.t())


def full_problem():
    g = torch.Generator().manual_seed(0)
    weights = []
    for _ in range(DIMS.layers):
        weights.append({p: torch.randn(*D.full_shape(DIMS, p), generator=g) * 0.02 for p in D.PROJS})
    x = torch.randn(T, DIMS.hidden, generator=g)
    o_in = torch.randn(T, DIMS.hidden, generator=g)
    act_in = torch.randn(T, DIMS.inter, generator=g)
    return weights, x, o_in, act_in


def _rank_main(rank, world, port, errs):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        weights, x, o_in, act_in = full_problem()
        stack = D.TPStack(DIMS, world, rank, CpuMatmul(), torch.device("cpu"), full_weights=weights).bind(T)
        hk, ik = DIMS.hidden // world, DIMS.inter // world
        stack.x.copy_(x)
        stack.o_in.copy_(o_in[:, rank * hk:(rank + 1) * hk])
        stack.act_in.copy_(act_in[:, rank * ik:(rank + 1) * ik])
        for layer in range(DIMS.layers):
            stack.layer(layer, reduce=True)
            w = weights[layer]
            # row-parallel outputs are complete after the all-reduce
            torch.testing.assert_close(stack.o_out, o_in @ w["o"].t(), rtol=1e-5, atol=1e-5)
            torch.testing.assert_close(stack.d_out, act_in @ w["down"].t(), rtol=1e-5, atol=1e-5)
            # column-parallel outputs are this rank's slice
            q = DIMS.qkv // world
            torch.testing.assert_close(stack.qkv_out, (x @ w["qkv"].t())[:, rank * q:(rank + 1) * q])
            gu = x @ w["gate_up"].t()
            gate, up = gu[:, :DIMS.inter], gu[:, DIMS.inter:]
            mine = torch.cat([gate[:, rank * ik:(rank + 1) * ik], up[:, rank * ik:(rank + 1) * ik]], dim=1)
            torch.testing.assert_close(stack.gu_out, mine)
        # the local silu(gate) * up of each rank concatenates to the full activation
        g_loc, u_loc = stack.gu_out[:, :ik], stack.gu_out[:, ik:]
        act_loc = torch.nn.functional.silu(g_loc) * u_loc
        parts = [torch.empty_like(act_loc) for _ in range(world)]
        dist.all_gather(parts, act_loc)
        gu = x @ weights[-1]["gate_up"].t()
        full_act = torch.nn.functional.silu(gu[:, :DIMS.inter]) * gu[:, DIMS.inter:]
        torch.testing.assert_close(torch.cat(parts, dim=1), full_act)
    except Exception as e:  # noqa: BLE001
        errs.put(f"rank {rank}: {e!r}")
        raise
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_shapes_27b():
    d = D.Dims()
    for tp in (1, 2, 4, 8):
        shapes = {p: D.shard_shape(d, p, tp) for p in D.PROJS}
        assert shapes["qkv"] == (7168 // tp, 5120)
        assert shapes["o"] == (5120, 5120 // tp)
        assert shapes["gate_up"] == (2 * 17408 // tp, 5120)
        assert shapes["down"] == (5120, 17408 // tp)
        # every K shard stays a whole number of 128-wide groups (g128 int4, 128-byte k-blocks)
        assert all(K % 128 == 0 for _, K in shapes.values())
    with pytest.raises(ValueError):
        D.shard_shape(d, "qkv", 3)


def test_tp2_gloo_matches_unsharded():
    ctx = mp.get_context("spawn")
    errs = ctx.SimpleQueue()
    mp.start_processes(_rank_main, args=(2, _free_port(), errs), nprocs=2, join=True, start_method="spawn")
    assert errs.empty()
