"""GPU parity of the fused mixed-tier decode attention (through the C ABI).

Bar: within 2e-3 max-abs, plus the fp16 output's own half-ulp (2^-11 |ref|; the output is fp16 like
the reference's), of the exact (float64) softmax attention over the K/V the reference reconstructs
from the same pages (which the oracle reproduces bit for bit); and within that bar plus the
reference's own deviation of the reference's fp16 reconstruct-then-SDPA output."""
import math

import numpy as np
import pytest
import torch

import attn_util as U

pytestmark = pytest.mark.gpu
ATOL = 2e-3


def within(out, ref, extra=0.0):
    return np.abs(out - ref) <= ATOL + np.abs(ref) * 2.0 ** -11 + extra


def run_plan(pages, B, Hkv, G, D, q, n_splits=None, scale=None, precise=False):
    from argus_b200 import attention as A
    arenas, plist = U.arenas_from_pages(pages)
    plan = A.AttentionPlan(arenas, plist, batch=B, heads_kv=Hkv, group=G, head_dim=D, q_len=q.shape[2],
                           n_splits=n_splits, precise_pv=precise)
    out = plan.run(torch.from_numpy(q).cuda(), scale=scale)
    torch.cuda.synchronize()
    assert A.device_status() == 0
    return out.cpu().numpy().astype(np.float64), plan


@pytest.mark.parametrize("case", ["mixed", "peaky"])
@pytest.mark.parametrize("n_splits", [1, 3])
def test_golden_cases(golden, case, n_splits):
    z = golden("attention")
    B, Hq, Hkv, D, P, L = (int(v) for v in z[f"{case}/meta"])
    pages = U.golden_pages(z, case)
    out, _ = run_plan(pages, B, Hkv, Hq // Hkv, D, z[f"{case}/q"], n_splits=n_splits)
    f64 = z[f"{case}/out_f64"]
    ref16 = z[f"{case}/out_ref16"].astype(np.float64)
    assert within(out, f64).all(), np.abs(out - f64).max()
    assert within(out, ref16, np.abs(f64 - ref16)).all()


SHAPES = [
    # B, Hkv, G, D, P, q_len, tiers
    (2, 2, 4, 128, 16, 1, [("one_bit", 64), ("int2", 64), ("int4", 64), ("int8", 32), ("fp8", 32), ("fp16", 48)]),
    (1, 4, 8, 64, 16, 1, [("int8", 128), ("fp16", 32)]),
    (1, 2, 1, 128, 16, 1, [("int4", 32), ("int2", 32), ("fp16", 16)]),
    (1, 1, 4, 16, 8, 1, [("one_bit", 16), ("int2", 16), ("int4", 16), ("int8", 8), ("fp8", 8), ("fp16", 8)]),
    (2, 2, 2, 64, 32, 2, [("one_bit", 64), ("int4", 64), ("fp16", 32)]),
    (1, 1, 16, 128, 16, 1, [("int8", 32), ("fp16", 16)]),
    (1, 2, 4, 32, 16, 3, [("int2", 48), ("fp8", 32), ("fp16", 16)]),
    (1, 1, 4, 256, 16, 1, [("int4", 32), ("one_bit", 32), ("fp16", 16)]),
    # pages larger than a tile (records staged tile by tile) and 8-token pages
    (1, 2, 4, 128, 64, 1, [("one_bit", 128), ("int2", 64), ("int4", 128), ("int8", 64), ("fp8", 64), ("fp16", 64)]),
    (2, 1, 4, 64, 8, 1, [("one_bit", 32), ("int2", 32), ("int4", 32), ("int8", 16), ("fp8", 16), ("fp16", 16)]),
    (1, 1, 8, 128, 48, 2, [("int4", 96), ("fp16", 48)]),
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"B{s[0]}H{s[1]}G{s[2]}D{s[3]}P{s[4]}q{s[5]}")
@pytest.mark.parametrize("n_splits,precise", [(1, False), (None, False), (None, True)])
def test_random_mixed_tiers(shape, n_splits, precise):
    B, Hkv, G, D, P, qlen, tiers = shape
    rng = np.random.default_rng(hash(shape[:6]) % 2**32)
    pages = U.random_pages(rng, tiers, B, Hkv, D, P)
    q = rng.standard_normal((B, Hkv * G, qlen, D)).astype(np.float16)
    out, plan = run_plan(pages, B, Hkv, G, D, q, n_splits=n_splits, precise=precise)
    K, V = U.reference_kv(pages)
    ref = U.f64_attention(q, K, V)
    assert within(out, ref).all(), np.abs(out - ref).max()


def test_partial_fp16_tiles_and_custom_scale():
    """An fp16 staging buffer whose length is not a multiple of 16 (garbage beyond it must not
    leak), plus a non-default softmax scale."""
    from argus_b200 import attention as A
    rng = np.random.default_rng(7)
    B, Hkv, G, D = 2, 2, 4, 64
    Lbuf, cap = 21, 32
    kb = torch.full((B, Hkv, cap, D), float("nan"), dtype=torch.float16, device="cuda")
    vb = torch.full((B, Hkv, cap, D), float("inf"), dtype=torch.float16, device="cuda")
    kr = rng.standard_normal((B, Hkv, Lbuf, D)).astype(np.float16)
    vr = rng.standard_normal((B, Hkv, Lbuf, D)).astype(np.float16)
    kb[:, :, :Lbuf] = torch.from_numpy(kr).cuda()
    vb[:, :, :Lbuf] = torch.from_numpy(vr).cuda()
    pages = U.random_pages(rng, [("int4", 32)], B, Hkv, D, 16)
    arenas, plist = U.arenas_from_pages(pages)
    arenas.append(A.KVArena.from_fp16(kb, vb))
    plist += [(len(arenas) - 1, 0, 16), (len(arenas) - 1, 1, Lbuf - 16)]
    q = rng.standard_normal((B, Hkv * G, 1, D)).astype(np.float16)
    plan = A.AttentionPlan(arenas, plist, batch=B, heads_kv=Hkv, group=G, head_dim=D)
    out = plan.run(torch.from_numpy(q).cuda(), scale=0.3).cpu().numpy().astype(np.float64)
    K, V = U.reference_kv(pages)
    K = np.concatenate([K, kr], axis=2)
    V = np.concatenate([V, vr], axis=2)
    ref = U.f64_attention(q, K, V, scale=0.3)
    assert np.isfinite(out).all()
    assert within(out, ref).all(), np.abs(out - ref).max()


def test_lse_output():
    from argus_b200 import attention as A
    rng = np.random.default_rng(3)
    B, Hkv, G, D = 1, 2, 4, 128
    pages = U.random_pages(rng, [("int8", 64), ("fp16", 32)], B, Hkv, D, 16)
    arenas, plist = U.arenas_from_pages(pages)
    q = rng.standard_normal((B, Hkv * G, 1, D)).astype(np.float16)
    for ns in (1, 4):
        plan = A.AttentionPlan(arenas, plist, batch=B, heads_kv=Hkv, group=G, head_dim=D, n_splits=ns)
        lse = torch.empty(B, Hkv * G, 1, dtype=torch.float32, device="cuda")
        plan.run(torch.from_numpy(q).cuda(), lse=lse)
        K, V = U.reference_kv(pages)
        Kr = np.repeat(K.astype(np.float64), G, axis=1)
        w = np.einsum("bhqd,bhkd->bhqk", q.astype(np.float64), Kr) / math.sqrt(D)
        ref = np.log(np.exp(w - w.max(-1, keepdims=True)).sum(-1)) + w.max(-1)
        assert np.abs(lse.cpu().numpy() - ref).max() < 1e-3


def test_run_host_graph_matches_run():
    """AttentionPlan.run_host (copy in, fused kernel, copy out, replayed as one CUDA graph) gives the
    same bits as run() on device tensors, also after the pinned query buffer is refilled."""
    from argus_b200 import attention as A
    B, Hkv, G, D, P = 2, 2, 4, 128, 16
    rng = np.random.default_rng(21)
    pages = U.random_pages(rng, [("int4", 64), ("int8", 32), ("fp16", 32)], B, Hkv, D, P)
    arenas, plist = U.arenas_from_pages(pages)
    plan = A.AttentionPlan(arenas, plist, batch=B, heads_kv=Hkv, group=G, head_dim=D, n_splits=3)
    q_host = torch.empty(B, Hkv * G, 1, D, dtype=torch.float16).pin_memory()
    out_host = torch.empty_like(q_host).pin_memory()
    for step in range(3):
        q = torch.from_numpy((rng.standard_normal((B, Hkv * G, 1, D)) / 8).astype(np.float16))
        q_host.copy_(q)
        plan.run_host(q_host, out_host)
        torch.cuda.synchronize()
        ref = plan.run(q.cuda())
        torch.cuda.synchronize()
        assert torch.equal(out_host.view(torch.int16), ref.cpu().view(torch.int16)), step
    # more buffer pairs than the plan keeps graphs for: the least recently used graphs are dropped
    for step in range(A.RUN_HOST_GRAPHS + 2):
        qh = torch.from_numpy((rng.standard_normal((B, Hkv * G, 1, D)) / 8).astype(np.float16)).pin_memory()
        oh = torch.empty_like(qh).pin_memory()
        plan.run_host(qh, oh)
        torch.cuda.synchronize()
        assert torch.equal(oh.view(torch.int16), plan.run(qh.cuda()).cpu().view(torch.int16)), step
        assert len(plan._graphs) <= A.RUN_HOST_GRAPHS
    assert A.device_status() == 0


def test_llama8b_layer_full_size_sampled_heads():
    """The Llama-3-8B mixed-tier layer at full size (batch 8, 32 q / 8 kv heads, D 128, 32K context:
    1-bit 8192, INT2 8192, INT4 8192, INT8 4096, FP8-sim 3072, FP16 1024 tokens, oldest first) in one
    launch with the default split plan; every (batch, kv head) pair against float64 attention over the
    oracle's dequantization of the same pages."""
    from argus_b200 import attention as A
    B, Hkv, G, D, P = 8, 8, 4, 128, 16
    rng = np.random.default_rng(8)
    tiers = [("one_bit", 8192), ("int2", 8192), ("int4", 8192), ("int8", 4096), ("fp8", 3072), ("fp16", 1024)]
    pages = U.random_pages(rng, tiers, B, Hkv, D, P)
    q = (rng.standard_normal((B, Hkv * G, 1, D)) / math.sqrt(D)).astype(np.float16)
    out, plan = run_plan(pages, B, Hkv, G, D, q)
    assert plan.n_tokens == 32768 and plan.n_splits > 1
    for b in range(B):  # all 8 KV heads of one sequence at a time (64 pairs in all)
        sub = {t: [{k: v[b:b + 1] for k, v in pg.items()} for pg in lst] for t, lst in pages.items()}
        K, V = U.reference_kv(sub)
        ref = U.f64_attention(q[b:b + 1], K, V)
        got = out[b:b + 1]
        for h in range(Hkv):
            sl = slice(h * G, (h + 1) * G)
            assert within(got[:, sl], ref[:, sl]).all(), ((b, h), np.abs(got[:, sl] - ref[:, sl]).max())


def test_bounded_wait_times_out_and_the_context_stays_usable():
    """A device wait that nothing completes (the bounded mbarrier wait the decode kernel's staging
    rings use) gives up after its poll limit and reports ARGUS_ERR_TIMEOUT through
    argus_device_status, without a fault; launches afterwards run normally."""
    import ctypes

    from argus_b200 import _lib
    from argus_b200 import attention as A
    gave_up = ctypes.c_int(0)
    _lib.call("argus_selftest_wait_timeout", 1000, ctypes.byref(gave_up), _lib.stream_handle())
    assert gave_up.value == 1
    assert A.device_status() == _lib.ERR_TIMEOUT
    assert A.device_status() == 0  # read once, then cleared
    B, Hkv, G, D, P = 1, 2, 4, 64, 16
    rng = np.random.default_rng(5)
    pages = U.random_pages(rng, [("int4", 32), ("fp16", 16)], B, Hkv, D, P)
    q = (rng.standard_normal((B, Hkv * G, 1, D)) / 8).astype(np.float16)
    out, _ = run_plan(pages, B, Hkv, G, D, q)
    K, V = U.reference_kv(pages)
    assert within(out, U.f64_attention(q, K, V)).all()
