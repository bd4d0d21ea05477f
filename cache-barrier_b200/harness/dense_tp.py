"""Tensor-parallel dense decoder projections on 1..8 B200s (27B-class decoder).

The reference times the dense projections of one GPU with vLLM kernels
(profiling/dense_qwen/bench_dense_proj.py:55-65, 80-150) and has no multi-GPU
code. This harness runs the same projections of a 64-layer decoder (hidden
5120, 40 query and 8 KV heads of 128, FFN 17408) sharded Megatron-style over
``WORLD_SIZE`` ranks, one process per GPU:

  QKV      [5120 -> 7168]      column-parallel (each rank 7168/tp output rows)
  O        [5120 -> 5120]      row-parallel (each rank K = 5120/tp), then all-reduce
  gate-up  [5120 -> 2 x 17408] column-parallel; rank r holds gate rows and up rows
                               [r*I/tp, (r+1)*I/tp) so its silu(gate)*up is local
  down     [17408 -> 5120]     row-parallel (K = 17408/tp), then all-reduce

The all-reduce (sum of the [T, 5120] bf16 partial outputs) is NCCL over
NVLink/NVSwitch through torch.distributed. Attention and the gate activation
are outside the measured path: the row-parallel projections read synthetic
shard inputs of the right shape. Each precision's weights (W8A8 per-channel
int8, W4A16 g128 int4, bf16 for the cuBLAS baseline) are random N(0, 0.02),
generated per shard from a seed of (layer, projection, rank); 64 distinct
layers keep the per-GPU working set far above L2.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 cache-barrier_b200/harness/dense_tp.py \\
        --tokens 1,8,32,64 --precisions w8a8,w4a16,bf16 --allreduce nccl,peer --out dense_tp_tp8.json

The projection backend is injectable (``Backend``) so the sharding and
reduction logic runs on CPU with gloo ranks and an fp32 matmul in the tests.
"""

from __future__ import annotations

import argparse
import datetime
import os
import sys
from dataclasses import dataclass

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


@dataclass(frozen=True)
class Dims:
    hidden: int = 5120
    qkv: int = 7168  # (40 + 2 * 8) heads x 128
    inter: int = 17408
    layers: int = 64


PROJS = ("qkv", "o", "gate_up", "down")


def full_shape(d: Dims, proj: str) -> tuple[int, int]:
    """(N, K) of the unsharded weight, stored [N, K] like torch.nn.Linear."""
    return {"qkv": (d.qkv, d.hidden), "o": (d.hidden, d.hidden), "gate_up": (2 * d.inter, d.hidden),
            "down": (d.hidden, d.inter)}[proj]


def shard_shape(d: Dims, proj: str, tp: int) -> tuple[int, int]:
    N, K = full_shape(d, proj)
    if proj in ("qkv", "gate_up"):
        if N % tp:
            raise ValueError(f"{proj}: N={N} not divisible by tp={tp}")
        return N // tp, K
    if K % tp:
        raise ValueError(f"{proj}: K={K} not divisible by tp={tp}")
    return N, K // tp


def shard_weight(w: torch.Tensor, d: Dims, proj: str, tp: int, rank: int) -> torch.Tensor:
    """Rank ``rank``'s shard of the full [N, K] weight ``w``."""
    N, K = w.shape
    if proj == "qkv":
        n = N // tp
        return w[rank * n:(rank + 1) * n]
    if proj == "gate_up":
        i = d.inter // tp
        gate, up = w[:d.inter], w[d.inter:]
        return torch.cat([gate[rank * i:(rank + 1) * i], up[rank * i:(rank + 1) * i]], dim=0)
    k = K // tp
    return w[:, rank * k:(rank + 1) * k]


class Backend:
    """One precision's projection: ``prepare`` turns a bf16 [N, K] shard into the
    operand the kernel reads, ``run`` computes out[T, N] = x[T, K] @ W^T."""

    name = "base"

    def prepare(self, w: torch.Tensor):
        raise NotImplementedError

    def weight_bytes(self, N: int, K: int) -> int:
        raise NotImplementedError

    def run(self, x, handle, out, scratch):
        raise NotImplementedError


class Bf16Cublas(Backend):
    name = "bf16"

    def prepare(self, w):
        return w.to(torch.bfloat16).contiguous()

    def weight_bytes(self, N, K):
        return 2 * N * K

    def run(self, x, h, out, scratch):
        torch.mm(x, h.t(), out=out)


class W8A8(Backend):
    """Per-channel int8 weights (s = amax_K/127, round half to even), dynamic
    per-token activation quantization and the tcgen05 kind::i8 GEMM."""

    name = "w8a8"

    def prepare(self, w):
        wf = w.float()
        s = torch.clamp(wf.abs().amax(dim=1) / 127.0, min=1e-8)
        q = torch.clamp(torch.round(wf / s[:, None]), -127, 127).to(torch.int8).contiguous()  # [N, K] K-major
        return q, s.contiguous()

    def weight_bytes(self, N, K):
        return N * K + 4 * N

    def run(self, x, h, out, scratch):
        from cb200 import ops

        q, s = h
        T, K = x.shape
        ops.w8a8_gemm_dynamic(x, q, s, q=scratch["q"][:T * K], s=scratch["s"], out=out)


class W4A16(Backend):
    """int4 g128 weights (dense_ops.quantize_w4a16) and the tcgen05 kind::f16 dequant GEMM."""

    name = "w4a16"

    def prepare(self, w):
        import dense_ops

        native, scales = dense_ops.quantize_w4a16(w.to(torch.bfloat16), 128)
        return native, scales, w.shape[0]

    def weight_bytes(self, N, K):
        return N * K // 2 + (K // 128) * N * 2

    def run(self, x, h, out, scratch):
        from cb200 import ops

        native, scales, N = h
        ops.w4a16_gemm(x, native, scales, N, 128, out=out)


BACKENDS = {"bf16": Bf16Cublas, "w8a8": W8A8, "w4a16": W4A16}


class TPStack:
    """The layers' weight shards of one rank, and one decode step over them."""

    def __init__(self, d: Dims, tp: int, rank: int, backend: Backend, device, seed: int = 0,
                 full_weights=None, group=None, allreduce=None):
        self.d, self.tp, self.rank, self.backend = d, tp, rank, backend
        self.device, self.group = device, group
        self.allreduce = allreduce  # None: NCCL through torch.distributed; else a callable(x, out=x)
        self.handles = []
        for layer in range(d.layers):
            hs = {}
            for pi, proj in enumerate(PROJS):
                if full_weights is not None:
                    w = shard_weight(full_weights[layer][proj], d, proj, tp, rank).to(device)
                else:
                    N, K = shard_shape(d, proj, tp)
                    g = torch.Generator(device=device).manual_seed(seed + 1000003 * layer + 7919 * pi + 104729 * rank)
                    w = (torch.randn(N, K, generator=g, device=device, dtype=torch.float32) * 0.02).to(torch.bfloat16)
                hs[proj] = backend.prepare(w)
                del w
            self.handles.append(hs)

    def bind(self, T: int, seed: int = 7):
        """Allocates the step's activations and outputs for T tokens."""
        d, tp, device = self.d, self.tp, self.device
        self.T = T
        g = torch.Generator(device=device).manual_seed(seed + self.rank)
        dt = torch.bfloat16 if device.type == "cuda" else torch.float32
        H, Q, I = d.hidden, d.qkv, d.inter
        self.x = torch.randn(T, H, generator=g, device=device, dtype=torch.float32).to(dt)
        self.o_in = torch.randn(T, H // tp, generator=g, device=device, dtype=torch.float32).to(dt)
        self.act_in = torch.randn(T, I // tp, generator=g, device=device, dtype=torch.float32).to(dt)
        self.qkv_out = torch.empty(T, Q // tp, device=device, dtype=dt)
        self.o_out = torch.empty(T, H, device=device, dtype=dt)
        self.gu_out = torch.empty(T, 2 * I // tp, device=device, dtype=dt)
        self.d_out = torch.empty(T, H, device=device, dtype=dt)
        kmax = max(H, I // tp)
        self.scratch = {"q": torch.empty(T * kmax, device=device, dtype=torch.int8),
                        "s": torch.empty(T, device=device, dtype=torch.float32)}
        return self

    def layer(self, i: int, reduce: bool = True):
        h, b, sc = self.handles[i], self.backend, self.scratch
        b.run(self.x, h["qkv"], self.qkv_out, sc)
        b.run(self.o_in, h["o"], self.o_out, sc)
        if reduce and self.tp > 1:
            self._reduce(self.o_out)
        b.run(self.x, h["gate_up"], self.gu_out, sc)
        b.run(self.act_in, h["down"], self.d_out, sc)
        if reduce and self.tp > 1:
            self._reduce(self.d_out)

    def _reduce(self, t):
        if self.allreduce is None:
            dist.all_reduce(t, group=self.group)
        else:
            self.allreduce(t, out=t)

    def step(self, reduce: bool = True):
        for i in range(self.d.layers):
            self.layer(i, reduce)

    def proj_step(self, proj: str):
        """One projection's GEMM in every layer (no all-reduce): per-GEMM timing of one shard shape."""
        b, sc = self.backend, self.scratch
        x, out = {"qkv": (self.x, self.qkv_out), "o": (self.o_in, self.o_out), "gate_up": (self.x, self.gu_out),
                  "down": (self.act_in, self.d_out)}[proj]
        for i in range(self.d.layers):
            b.run(x, self.handles[i][proj], out, sc)

    def weight_bytes(self) -> int:
        return self.d.layers * sum(self.backend.weight_bytes(*shard_shape(self.d, p, self.tp)) for p in PROJS)


def _time_graph(fn, steps: int, warmup: int) -> float:
    """Milliseconds per replay of a CUDA graph holding one call of ``fn``."""
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        g.replay()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    del g
    return ms


def _max_over_ranks(v: float, device) -> float:
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def measure(world: int, rank: int, dev, tokens, precisions, modes, steps: int = 10, warmup: int = 3,
            layers: int = 64, per_projection: bool = True, log=print):
    """Times the decode step of the tensor-parallel stack at tp = world on this rank (every rank calls it
    with the same arguments). Returns the rows (max over ranks of CUDA-event time) and a summary."""
    from common import ClockSampler

    d = Dims(layers=layers)
    peer = None
    if world > 1 and "peer" in modes:
        sys.path.insert(0, os.path.dirname(HERE))
        from cb200.peer import PeerAllReduce

        peer = PeerAllReduce(max(tokens) * d.hidden, device=dev)
    if world == 1:
        modes = ["none"]
    rows, proj_rows = [], []
    for prec in precisions:
        backend = BACKENDS[prec]()
        stack = TPStack(d, world, rank, backend, dev, seed=1234)
        for T in tokens:
            stack.bind(T)
            ms_noar = None
            for mode in modes:
                stack.allreduce = peer if mode == "peer" else None
                if world > 1:
                    dist.barrier()
                with ClockSampler(dev.index) as clk:
                    ms = _max_over_ranks(_time_graph(lambda: stack.step(world > 1), steps, warmup), dev)
                    if ms_noar is None:
                        ms_noar = _max_over_ranks(_time_graph(lambda: stack.step(False), steps, warmup), dev)
                wb = stack.weight_bytes()
                row = {"precision": prec, "tokens": T, "tp": world, "layers": d.layers, "allreduce": mode,
                       "step_ms": round(ms, 4), "us_per_layer": round(ms * 1e3 / d.layers, 3),
                       "step_ms_without_allreduce": round(ms_noar, 4),
                       "allreduce_us_per_layer": round((ms - ms_noar) * 1e3 / d.layers, 3),
                       "tokens_per_s": round(T / (ms * 1e-3), 1),
                       "weight_bytes_per_gpu": wb,
                       "weight_gbs_per_gpu": round(wb / (ms_noar * 1e-3) / 1e9, 1),
                       "clocks": clk.info}
                rows.append(row)
                log(f"tp={world} {prec:6s} T={T:3d} [{mode}]: {row['us_per_layer']:9.2f} us/layer "
                    f"(all-reduce {row['allreduce_us_per_layer']:.2f}), {row['weight_gbs_per_gpu']} GB/s/GPU")
            if per_projection:
                for proj in PROJS:
                    N, K = shard_shape(d, proj, world)
                    ms = _max_over_ranks(_time_graph(lambda: stack.proj_step(proj), steps, warmup), dev)
                    proj_rows.append({"precision": prec, "tokens": T, "tp": world, "proj": proj, "N": N, "K": K,
                                      "bf16_shard_mb": round(2 * N * K / 1e6, 2),
                                      "us_per_gemm": round(ms * 1e3 / d.layers, 3)})
        del stack
        torch.cuda.empty_cache()
    if peer is not None:
        assert int(peer.status.item()) == 0, "peer all-reduce reported a timeout"
        peer.close()
    return rows, proj_rows, summarize(rows, proj_rows, world)


def summarize(rows, proj_rows, world: int) -> dict:
    """Per token count: the best exchange per precision, the all-reduce share, quantized vs bf16, and the
    gate at this tp: the per-GPU projection shards (bf16-equivalent MB) where each quantized kernel wins."""
    out = {"tp": world, "per_tokens": {}}
    tokens = sorted({r["tokens"] for r in rows})
    for T in tokens:
        best = {}
        for r in rows:
            if r["tokens"] != T:
                continue
            cur = best.get(r["precision"])
            if cur is None or r["us_per_layer"] < cur["us_per_layer"]:
                best[r["precision"]] = r
        ent = {}
        for prec, r in best.items():
            e = {"us_per_layer": r["us_per_layer"], "allreduce": r["allreduce"],
                 "allreduce_us_per_layer": r["allreduce_us_per_layer"],
                 "allreduce_share": round(r["allreduce_us_per_layer"] / r["us_per_layer"], 3) if world > 1 else 0.0,
                 "weight_gbs_per_gpu": r["weight_gbs_per_gpu"]}
            modes = {x["allreduce"]: x["allreduce_us_per_layer"] for x in rows
                     if x["tokens"] == T and x["precision"] == prec}
            if len(modes) > 1:
                e["allreduce_us_per_layer_by_exchange"] = modes
            if "bf16" in best and prec != "bf16":
                e["speedup_vs_bf16"] = round(best["bf16"]["us_per_layer"] / r["us_per_layer"], 3)
            ent[prec] = e
        gate = {}
        bf = {p["proj"]: p for p in proj_rows if p["tokens"] == T and p["precision"] == "bf16"}
        for prec in {p["precision"] for p in proj_rows} - {"bf16"}:
            shards = []
            for p in proj_rows:
                if p["tokens"] == T and p["precision"] == prec and p["proj"] in bf:
                    shards.append({"proj": p["proj"], "bf16_shard_mb": p["bf16_shard_mb"], "us": p["us_per_gemm"],
                                   "bf16_us": bf[p["proj"]]["us_per_gemm"],
                                   "speedup": round(bf[p["proj"]]["us_per_gemm"] / p["us_per_gemm"], 3)})
            shards.sort(key=lambda x: x["bf16_shard_mb"])
            wins = [x["bf16_shard_mb"] for x in shards if x["speedup"] > 1.0]
            loses = [x["bf16_shard_mb"] for x in shards if x["speedup"] <= 1.0]
            gate[prec] = {"shards": shards,
                          "smallest_winning_shard_mb": min(wins) if wins else None,
                          "largest_losing_shard_mb": max(loses) if loses else None}
        out["per_tokens"][str(T)] = {"layer": ent, "gate": gate}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", default="1,8,32,64")
    ap.add_argument("--precisions", default="w8a8,w4a16,bf16")
    ap.add_argument("--layers", type=int, default=64)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--allreduce", default="nccl,peer", help="comma-separated: nccl, peer (NVLink one-shot kernel)")
    ap.add_argument("--no-per-projection", action="store_true")
    ap.add_argument("--out", default=None)
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from common import gpu_info, save_json

    rows, proj_rows, summary = measure(world, rank, dev, [int(t) for t in args.tokens.split(",")],
                                       args.precisions.split(","), args.allreduce.split(","), args.steps,
                                       args.warmup, args.layers, not args.no_per_projection,
                                       log=(lambda m: print(m, flush=True)) if rank == 0 else (lambda m: None))
    if rank == 0:
        out = {"experiment": "dense_tp_projections", "dims": Dims(layers=args.layers).__dict__, "tp": world,
               "gpu": gpu_info(),
               "method": "one CUDA graph per decode step (64 layers x 4 projections + 2 all-reduces per layer); "
                         "max over ranks of CUDA-event time; weights rotate naturally across layers; "
                         "per-projection rows: a graph of one projection's GEMM in all 64 layers",
               "rows": rows, "projections": proj_rows, "summary": summary}
        if args.out:
            save_json(args.out, out)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
