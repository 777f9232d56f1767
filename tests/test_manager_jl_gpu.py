"""PagedDynamicKVCache with 512- and 256-token pages (128- and 64-row JL blocks) at head_dim 128 and
64: inplace_paged_attention attends the JL pages without rebuilding them (JLAttention + LSE merge) and gives the same output (attention bar
plus the JL slack of the other manager tests), per-page attention mass and tier moves as the path
that rebuilds them into the fp16 scratch arena."""
import math
import os

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def run_cache(fused, tmp_path, pushes, q, page=512):
    from argus_b200.core.memory_manager import PagedDynamicKVCache
    os.environ["ARGUS_LOG_LEVEL"] = "quiet"
    cwd = os.getcwd()
    os.chdir(tmp_path)
    try:
        c = PagedDynamicKVCache(page_size=page, max_active_pages=1, max_fp8_pages=1, max_int8_pages=1,
                                max_int4_pages=1, max_int2_pages=1, max_one_bit_pages=1, sink_tokens=16,
                                threshold_sigma=0.0)
        c.fused_jl_attention = fused
        for k, v in pushes:
            c.push_new_tokens(k.cuda(), v.cuda())
        K, V = c.get_all_keys_values()
        out = c.inplace_paged_attention(q.cuda())
        torch.cuda.synchronize()
    finally:
        os.chdir(cwd)
    return c, out, K, V


@pytest.mark.parametrize("page,D", [(512, 128), (256, 128), (512, 64), (256, 64)])
def test_fused_jl_pages_match_rebuilt_pages(tmp_path, page, D):
    from argus_b200 import attention as A
    g = torch.Generator().manual_seed(9)
    B, H = 1, 2
    pushes = [(torch.randn(B, H, page, D, generator=g).half(), torch.randn(B, H, page, D, generator=g).half())
              for _ in range(10)]
    q = (torch.randn(B, H * 4, 1, D, generator=g) * 2.0 / math.sqrt(D)).half()
    c1, out1, K1, V1 = run_cache(True, tmp_path, pushes, q, page)
    c0, out0, K0, V0 = run_cache(False, tmp_path, pushes, q, page)
    assert A.device_status() == 0
    # the fused path built its JL attention; the other rebuilt the pages instead
    assert len(c1.jl_pages) >= 2 and c1._jl_attention is not None and c0._jl_attention is None
    ref = oracle.sdpa_f64(q.numpy(), K0.cpu().numpy(), V0.cpu().numpy(), 1.0 / math.sqrt(D))
    a, b = out1.cpu().numpy().astype(np.float64), out0.cpu().numpy().astype(np.float64)
    bar = 2e-3 + np.abs(ref) * 2.0 ** -11 + 4e-3
    assert (np.abs(a - ref) <= bar).all(), np.abs(a - ref).max()
    assert (np.abs(b - ref) <= bar).all(), np.abs(b - ref).max()
    # same per-page mass and the same tier moves
    tiers = ("active_pages", "fp8_pages", "int8_pages", "int4_pages", "int2_pages", "one_bit_pages", "jl_pages")
    assert [len(getattr(c1, t)) for t in tiers] == [len(getattr(c0, t)) for t in tiers]
    for t in tiers:
        for p1, p0 in zip(getattr(c1, t), getattr(c0, t)):
            assert p1["page_id"] == p0["page_id"]
            assert abs(p1["attention_sum"] - p0["attention_sum"]) <= 1e-3 * max(1e-3, abs(p0["attention_sum"])) + 1e-6
    assert c1.num_resurrections == c0.num_resurrections
