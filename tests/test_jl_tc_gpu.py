"""GPU checks of the JL contraction at archive-block sizes, where it runs on the tensor cores
(tcgen05, accumulator in tensor memory): C[b] = A @ X[b] for the reconstruction R [1024 x 128] @ Y
and the projection W [128 x 1024] @ X of 1024-token blocks, and smaller tensor-core shapes.

Bar: every output within one fp16 ulp (plus 1e-4) of the fp32 product of the same fp16 operands
rounded once to fp16 (the two sums differ only in accumulation order)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [
    # batch, M, K, N
    (1, 128, 64, 16),
    (2, 128, 128, 128),
    (3, 256, 192, 64),
    (2, 128, 64, 256),
    (8, 1024, 128, 128),   # reconstruction of 1024-token blocks: R [1024 x 128] @ Y [128 x 128]
    (8, 128, 1024, 128),   # projection of 1024-token blocks:     W [128 x 1024] @ X [1024 x 128]
]


@pytest.mark.parametrize("batch,M,K,N", SHAPES)
def test_tensor_core_contraction(batch, M, K, N):
    from argus_b200 import attention as A
    from argus_b200.core import jl
    g = torch.Generator(device="cpu").manual_seed(M * 7 + K * 3 + N + batch)
    a = (torch.randn(M, K, generator=g) / K ** 0.5).half().cuda()
    x = torch.randn(batch, K, N, generator=g).half().cuda()
    for _ in range(2):  # twice: tensor-memory allocation is per launch
        got = jl.apply_left(a, x)
        torch.cuda.synchronize()
        assert A.device_status() == 0
        ref = torch.matmul(a.float(), x.float()).half().float()
        diff = (got.float() - ref).abs()
        ulp = torch.clamp(ref.abs(), min=2.0 ** -14) * 2.0 ** -10
        assert bool((diff <= ulp + 1e-4).all()), float((diff - ulp).max())
