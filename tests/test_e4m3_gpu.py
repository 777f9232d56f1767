"""The true-e4m3 tier (ARGUS_TIER_E4M3), a separately named non-parity storage mode beside the
reference's simulated FP8: the GPU codec bit for bit against the oracle's restatement (every finite
fp16 value through the encoder, zero / NaN / inf / -0 rows), the fused decode attention over e4m3
pages within the attention bar of float64 attention over the oracle's dequantized pages, page moves
(e4m3 -> INT8 demotion, dequantization), and a cache run with fp8_format="e4m3" end to end."""
import math
import os

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
ATOL = 2e-3


def within(out, ref):
    return np.abs(out - ref) <= ATOL + np.abs(ref) * 2.0 ** -11


def same_f16(a, b):
    """fp16 arrays equal bit for bit, NaNs at the same places (NaN payloads may differ)."""
    na, nb = np.isnan(a), np.isnan(b)
    return bool((na == nb).all() and (a[~na].view(np.uint16) == b[~nb].view(np.uint16)).all())


def test_codec_matches_oracle_on_random_and_special_rows():
    from argus_b200.core import quantization as Q
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((512, 128)) * rng.choice([1e-3, 1.0, 40.0, 3000.0], (512, 1))).astype(np.float16)
    x[0] = 0.0
    x[1, 5] = np.nan
    x[2, 7] = np.inf
    x[3, :] = -0.0
    x[4, ::2] = -0.0
    x[5] = np.float16(6.0e-8)                  # fp16 subnormals
    q, s = Q.quantize_to_e4m3(torch.from_numpy(x).cuda())
    qo, so = oracle.quantize_to_e4m3(x)
    assert same_f16(s.cpu().numpy(), so)
    assert (q.cpu().numpy() == qo).all()
    y = Q.dequantize_from_e4m3(q, s).cpu().numpy()
    yo = oracle.dequantize_from_e4m3(qo, so)
    assert same_f16(y, yo)


def test_encoder_on_every_finite_fp16_value():
    """Rows whose first value is 448 have scale 1, so their codes are e4m3(x) of the other values:
    all 63,488 finite fp16 values (saturating from 448 up)."""
    from argus_b200.core import quantization as Q
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    h = h[np.isfinite(h)]
    h = h[np.abs(h.astype(np.float32)) <= 448.0]   # the row max must stay 448
    D = 128
    n = -(-h.size // (D - 1))
    x = np.zeros((n, D), np.float16)
    x[:, 0] = 448.0
    flat = np.zeros(n * (D - 1), np.float16)
    flat[:h.size] = h
    x[:, 1:] = flat.reshape(n, D - 1)
    q, s = Q.quantize_to_e4m3(torch.from_numpy(x).cuda())
    assert (s.cpu().numpy() == 1.0).all()
    got = q.cpu().numpy()[:, 1:].reshape(-1)[:h.size]
    assert (got == oracle.e4m3_encode(h.astype(np.float32))).all()


def _arena_with_pages(tier, k, v, page):
    from argus_b200 import attention as A
    from argus_b200 import paged
    B, H, L, D = k.shape
    arena = A.KVArena.allocate(tier, B, H, L // page, page, D, "cuda")
    for j in range(L // page):
        paged.quantize_page(arena, j, k[:, :, j * page:(j + 1) * page].cuda(), v[:, :, j * page:(j + 1) * page].cuda())
    return arena


@pytest.mark.parametrize("D,G,ql", [(128, 4, 1), (64, 8, 1), (128, 2, 3)])
def test_decode_attention_over_e4m3_pages(D, G, ql):
    from argus_b200 import attention as A
    from argus_b200 import paged
    g = torch.Generator().manual_seed(D + G + ql)
    B, H, page, n = 2, 2, 16, 24
    L = page * n
    k = (torch.randn(B, H, L, D, generator=g) * 2).half()
    v = torch.randn(B, H, L, D, generator=g).half()
    arena = _arena_with_pages(A.TIER_E4M3, k, v, page)
    # the pages hold the oracle's codes and scales, and dequantize to the oracle's values
    Kd, Vd = [], []
    for j in range(n):
        kq, ks = oracle.quantize_to_e4m3(k[:, :, j * page:(j + 1) * page].numpy())
        vq, vs = oracle.quantize_to_e4m3(v[:, :, j * page:(j + 1) * page].numpy())
        assert (arena.view("k", j).cpu().numpy() == kq).all() and (arena.view("v", j).cpu().numpy() == vq).all()
        Kd.append(oracle.dequantize_from_e4m3(kq, ks))
        Vd.append(oracle.dequantize_from_e4m3(vq, vs))
        kk, vv = paged.dequantize_page(arena, j)
        assert (kk.cpu().numpy().view(np.uint16) == Kd[-1].view(np.uint16)).all()
        assert (vv.cpu().numpy().view(np.uint16) == Vd[-1].view(np.uint16)).all()
    K, V = np.concatenate(Kd, axis=2), np.concatenate(Vd, axis=2)
    q = (torch.randn(B, H * G, ql, D, generator=g) / math.sqrt(D)).half()
    plan = A.AttentionPlan([arena], [(0, j, page) for j in range(n)], batch=B, heads_kv=H, group=G, head_dim=D,
                           q_len=ql)
    out = plan.run(q.cuda()).cpu().numpy().astype(np.float64)
    assert A.device_status() == 0
    ref = oracle.sdpa_f64(q.numpy(), K, V, 1.0 / math.sqrt(D))
    assert within(out, ref).all(), np.abs(out - ref).max()


def test_e4m3_page_demotes_to_int8_like_its_values():
    """The fused demotion reads an e4m3 page through its exact values: the INT8 page equals the
    oracle's INT8 quantization of the e4m3 page's fp16 values."""
    from argus_b200 import attention as A
    from argus_b200 import paged
    g = torch.Generator().manual_seed(11)
    B, H, page, D = 1, 2, 32, 128
    k = (torch.randn(B, H, page, D, generator=g) * 3).half()
    v = torch.randn(B, H, page, D, generator=g).half()
    src = _arena_with_pages(A.TIER_E4M3, k, v, page)
    dst = A.KVArena.allocate(A.TIER_INT8, B, H, 1, page, D, "cuda")
    paged.requant_page(src, 0, dst, 0)
    kd, vd = paged.dequantize_page(src, 0)
    kq, _ = oracle.quantize_to_int8(kd.cpu().numpy())
    vq, _ = oracle.quantize_to_int8(vd.cpu().numpy())
    assert (dst.view("k", 0).cpu().numpy() == kq).all() and (dst.view("v", 0).cpu().numpy() == vq).all()


def test_cache_with_e4m3_fp8_tier(tmp_path):
    """fp8_format="e4m3": pages demoted from fp16 land in an e4m3 arena, move on down the cascade,
    and the fused attention of the cache equals float64 attention over the cache's own K/V."""
    from argus_b200 import attention as A
    from argus_b200.core.memory_manager import PagedDynamicKVCache
    os.environ["ARGUS_LOG_LEVEL"] = "quiet"
    cwd = os.getcwd()
    os.chdir(tmp_path)
    try:
        c = PagedDynamicKVCache(page_size=16, max_active_pages=2, max_fp8_pages=3, max_int8_pages=2,
                                max_int4_pages=2, max_int2_pages=2, max_one_bit_pages=8, sink_tokens=4,
                                fp8_format="e4m3")
        g = torch.Generator().manual_seed(5)
        B, H, G, D = 1, 2, 4, 64
        c.push_new_tokens((torch.randn(B, H, 200, D, generator=g) * 1.5).half().cuda(),
                          torch.randn(B, H, 200, D, generator=g).half().cuda())
        assert c.arenas["fp8"].tier == A.TIER_E4M3 and len(c.fp8_pages) > 0 and c.cascade_counts["fp8_to_int8"] > 0
        for step in range(6):
            c.push_new_tokens((torch.randn(B, H, 1, D, generator=g) * 1.5).half().cuda(),
                              torch.randn(B, H, 1, D, generator=g).half().cuda())
            q = (torch.randn(B, H * G, 1, D, generator=g) / math.sqrt(D) * 2).half()
            K, V = c.get_all_keys_values()
            ref = oracle.sdpa_f64(q.numpy(), K.cpu().numpy(), V.cpu().numpy(), 1.0 / math.sqrt(D))
            out = (c.attend(q.cuda()) if step % 2 else c.inplace_paged_attention(q.cuda())).cpu().numpy()
            assert A.device_status() == 0
            assert within(out.astype(np.float64), ref).all(), (step, np.abs(out - ref).max())
    finally:
        os.chdir(cwd)
