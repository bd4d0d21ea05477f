"""Fused RMSNorm -> int8 quantization (cb_rmsnorm_quant_i8) against the oracle.

Tolerance (floating point): the kernel and the oracle sum x^2 in different orders,
so r can differ in its last bit and a normalized value y can land on the other
side of a 16-bit rounding boundary. Per row: either the scale is identical and at
most 0.5 % of q differ, each by 1; or the scale differs by at most 1 % (one
16-bit ulp of amax) and every q differs by at most 1. y differs from the oracle
in at most 0.1 % of the elements, each by one 16-bit ulp.
"""

import numpy as np
import pytest
import torch

from oracle import quant_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("w_dtype", ["same", torch.float32])
@pytest.mark.parametrize("rows,H", [(1, 5120), (16, 5120), (7, 4096), (64, 17408), (3, 100)])
def test_rmsnorm_quant_matches_oracle(cuda_device, rows, H, dtype, w_dtype):
    from cb200 import ops

    g = torch.Generator().manual_seed(rows * 7 + H)
    x = (torch.randn(rows, H, generator=g) * 2.0).to(dtype)
    wd = dtype if w_dtype == "same" else w_dtype
    w = (1.0 + 0.1 * torch.randn(H, generator=g)).to(wd)
    y = torch.empty(rows, H, dtype=dtype, device=cuda_device)
    q, s = ops.rmsnorm_quant_i8(x.to(cuda_device), w.to(cuda_device), 1e-6, y=y)
    torch.cuda.synchronize()
    qr, sr, yr = O.rmsnorm_quant_i8(x.float().numpy(), w.float().numpy(), 1e-6, "bf16" if dtype == torch.bfloat16 else "f16")
    qg, sg, yg = q.cpu().numpy().astype(np.int32), s.cpu().numpy(), y.float().cpu().numpy()
    for i in range(rows):
        d = np.abs(qg[i] - qr[i].astype(np.int32))
        assert d.max() <= 1
        if sg[i] == sr[i]:
            assert (d != 0).mean() <= 0.005
        else:
            assert abs(sg[i] - sr[i]) <= 0.01 * sr[i]
    ulp = np.abs(yr) * (2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10) + 1e-30
    diff = np.abs(yg - yr)
    assert (diff > 0).mean() <= 0.001
    assert np.all(diff <= ulp)
    # q and s are exactly the act-quant of the kernel's own y
    qy, sy = ops.quant_act_i8(y)
    torch.cuda.synchronize()
    assert torch.equal(qy.cpu(), q.cpu()) and torch.equal(sy.cpu(), s.cpu())


def test_rmsnorm_quant_rejects_bad_args(cuda_device):
    from cb200 import ops

    x = torch.randn(4, 64, device=cuda_device).to(torch.bfloat16)
    with pytest.raises(ValueError):
        ops.rmsnorm_quant_i8(x, torch.ones(63, device=cuda_device, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        ops.rmsnorm_quant_i8(x.t(), torch.ones(4, device=cuda_device, dtype=torch.bfloat16))
