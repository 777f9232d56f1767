"""Attention over a spilled (pinned host) record arena streamed through device staging buffers
(StreamedArenaAttention) equals attention over the same arena resident in HBM, within the
attention bar, and the float64 reference; runs of every length, including a short last run."""
import math

import numpy as np
import pytest
import torch

import attn_util as U

pytestmark = pytest.mark.gpu
ATOL = 2e-3


@pytest.mark.parametrize("tier,chunk", [("one_bit", 16), ("int4", 7), ("int8", 40), ("fp16", 5)])
def test_streamed_spilled_tier_matches_resident(tier, chunk):
    from argus_b200 import attention as A
    from argus_b200 import spill
    B, Hkv, G, D, P, n = 2, 2, 4, 128, 16, 40
    rng = np.random.default_rng(3)
    pages = U.random_pages(rng, [(tier, n * P)], B, Hkv, D, P)
    arenas, plist = U.arenas_from_pages(pages)
    q = torch.from_numpy((rng.standard_normal((B, Hkv * G, 1, D)) / math.sqrt(D)).astype(np.float16)).cuda()
    plan = A.AttentionPlan(arenas, plist, batch=B, heads_kv=Hkv, group=G, head_dim=D)
    lse_ref = torch.empty(B, Hkv * G, 1, dtype=torch.float32, device="cuda")
    ref = plan.run(q, lse=lse_ref)
    host = spill.arenas_to_host(arenas)[0]
    st = spill.StreamedArenaAttention(host, group=G, chunk_slots=chunk)
    for _ in range(2):  # the staging buffers are reused across calls
        out, lse = st.run(q)
        torch.cuda.synchronize()
        assert A.device_status() == 0
        a, b = out.cpu().numpy().astype(np.float64), ref.cpu().numpy().astype(np.float64)
        assert (np.abs(a - b) <= ATOL + np.abs(b) * 2.0 ** -11).all(), np.abs(a - b).max()
        assert torch.allclose(lse, lse_ref, rtol=0, atol=1e-4)
    K, V = U.reference_kv(pages)
    f64 = U.f64_attention(q.cpu().numpy(), K, V)
    got = out.cpu().numpy().astype(np.float64)
    assert (np.abs(got - f64) <= ATOL + np.abs(f64) * 2.0 ** -11).all(), np.abs(got - f64).max()
