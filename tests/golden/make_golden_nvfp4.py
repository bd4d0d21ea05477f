"""Generate the NVFP4 golden vectors in this directory from vLLM's reference code.

The reference runs its native-FP4 path through vLLM
(profiling/cuda_validation/bench_moe_nvfp4_native.py:97-108, vLLM's
``scaled_fp4_quant`` and ``run_cutlass_moe_fp4``). vLLM ships a CPU restatement of
that quantizer, ``ref_nvfp4_quant`` (vllm 0.22.0,
vllm/model_executor/layers/quantization/utils/nvfp4_emulation_utils.py:439-453),
and the inverse of its scale swizzle, ``convert_swizzled_to_linear`` (:348-355).
This script runs both on the CPU on seeded inputs and writes
``nvfp4_quant_*.npz`` (inputs, vLLM's fp4 values and scales) and
``nvfp4_swizzle.npz`` (a swizzled buffer with vLLM's linear reading of it).
It is only needed to regenerate the fixtures; nothing imports it.

    python tests/golden/make_golden_nvfp4.py
"""

from __future__ import annotations

import os

import numpy as np
import torch

from vllm.model_executor.layers.quantization.utils.nvfp4_emulation_utils import (
    convert_swizzled_to_linear,
    ref_nvfp4_quant,
)

HERE = os.path.dirname(os.path.abspath(__file__))


def quant_case(name, rows, K, gs_mode, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, K, generator=g).to(dtype)
    x[0, :16] = torch.tensor([0.0, -0.0, 1e-3, -1e-3, 6.0, -6.0, 3.0, 2.5, 0.25, 0.75, 1.25, 1.75, 3.5, 5.0, -5.5, 0.1])
    if rows > 2:
        x[2] = 0  # an all-zero row (scale 0)
    if gs_mode == "amax":
        gs = torch.tensor(448.0 * 6.0 / float(x.float().abs().max()), dtype=torch.float32)
    else:
        gs = torch.tensor(float(gs_mode), dtype=torch.float32)
    q, s = ref_nvfp4_quant(x.float(), gs, 16)
    bits = x.view(torch.int16).numpy().view(np.uint16)
    np.savez_compressed(os.path.join(HERE, f"nvfp4_quant_{name}.npz"), x_bits=bits,
                        x_is_bf16=np.bool_(dtype == torch.bfloat16), gs=np.float32(gs.item()),
                        q_values=q.numpy().astype(np.float32), scales=s.numpy().astype(np.float32))


def swizzle_case():
    rng = np.random.default_rng(7)
    rows, K = 200, 640  # 2 row blocks of 128 (the second ragged), 40 scale columns (10 atoms)
    rp, cp = 256, 40
    buf = rng.integers(0, 127, rp * cp, dtype=np.uint8)
    lin = convert_swizzled_to_linear(torch.from_numpy(buf.copy()), rows, K, 16).numpy()
    np.savez_compressed(os.path.join(HERE, "nvfp4_swizzle.npz"), swizzled=buf, rows=np.int64(rows), K=np.int64(K),
                        linear=np.ascontiguousarray(lin))


def main():
    quant_case("bf16_r5_k256_amax", 5, 256, "amax", torch.bfloat16, 1)
    quant_case("f16_r3_k128_g1", 3, 128, 1.0, torch.float16, 2)
    quant_case("bf16_r130_k64_g37", 130, 64, 37.5, torch.bfloat16, 3)
    swizzle_case()
    print("wrote nvfp4 fixtures to", HERE)


if __name__ == "__main__":
    main()
