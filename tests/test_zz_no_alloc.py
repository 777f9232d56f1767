"""The allocation-free decode attention entry point, argus_decode_attention_noalloc, called through the
C ABI and checked against argus_decode_attention (which takes a caller-allocated workspace).

Some callers cannot allocate device memory while they decode (a runtime that owns a fixed memory
budget, or code inside a region where allocation is not allowed); this entry point keeps its split-K
partials in a fixed 8 MiB array that the library holds.  Each check runs two calls in a row with
different shapes, so the second call reads scratch that the first one left behind.

Bar: the attention tests' tolerance, 2e-3 max-abs plus the fp16 output's half-ulp (2^-11 |ref|).
This file is collected last so that a run stopping at the first failure has run every other test."""
import ctypes

import numpy as np
import pytest
import torch

import attn_util as U

pytestmark = pytest.mark.gpu
ATOL = 2e-3
CAPACITY_ERROR = 6  # ARGUS_ERR_CAPACITY


def within(out, ref):
    return np.abs(out - ref) <= ATOL + np.abs(ref) * 2.0 ** -11


def make_plan(seed, B, Hkv, G, D, P, qlen, tiers, n_splits, with_pages=False):
    from argus_b200 import attention as A
    rng = np.random.default_rng(seed)
    pages = U.random_pages(rng, tiers, B, Hkv, D, P)
    arenas, plist = U.arenas_from_pages(pages)
    plan = A.AttentionPlan(arenas, plist, batch=B, heads_kv=Hkv, group=G, head_dim=D, q_len=qlen,
                           n_splits=n_splits)
    q = torch.from_numpy(rng.standard_normal((B, Hkv * G, qlen, D)).astype(np.float16)).cuda()
    return (plan, q, pages) if with_pages else (plan, q)


def call_noalloc(plan, q):
    from argus_b200 import attention as A
    L = A._bind()
    out = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], dtype=torch.float32, device=q.device)
    st = torch.cuda.current_stream(q.device).cuda_stream
    rc = L.argus_decode_attention_noalloc(ctypes.byref(plan._shape), plan._arena_c, plan.chunks_dev.data_ptr(),
                                          plan.splits_dev.data_ptr(), q.data_ptr(), out.data_ptr(),
                                          lse.data_ptr(), None, ctypes.c_void_p(st))
    assert rc == 0, L.argus_last_error().decode()
    return out, lse


def call_workspace(plan, q):
    lse = torch.empty(q.shape[:3], dtype=torch.float32, device=q.device)
    out = plan.run(q, lse=lse)
    return out, lse


CASES = [
    # seed, B, Hkv, G, D, P, q_len, tiers, n_splits
    (70, 2, 2, 4, 128, 16, 1, [("one_bit", 64), ("int2", 64), ("int4", 64), ("int8", 32), ("fp8", 32),
                                ("fp16", 48)], 5),
    (71, 1, 4, 8, 64, 16, 2, [("int4", 128), ("int8", 64), ("fp16", 32)], 7),
]


def test_noalloc_matches_workspace_entry_twice():
    from argus_b200 import attention as A
    runs = [make_plan(*c) for c in CASES]
    for plan, q in runs:
        assert plan.n_splits > 1  # the split-K partials go through the built-in scratch
    for plan, q in runs:  # two calls in a row, the second over the first one's scratch contents
        out_n, lse_n = call_noalloc(plan, q)
        out_w, lse_w = call_workspace(plan, q)
        torch.cuda.synchronize()
        assert A.device_status() == 0
        a, b = out_n.cpu().numpy().astype(np.float64), out_w.cpu().numpy().astype(np.float64)
        assert np.isfinite(a).all()
        assert within(a, b).all(), np.abs(a - b).max()
        assert torch.allclose(lse_n, lse_w, rtol=0, atol=1e-5)


def test_noalloc_rejects_oversized_partials():
    from argus_b200 import attention as A
    L = A._bind()
    cap = L.argus_decode_attention_noalloc_capacity()
    assert cap == 8 << 20
    plan, q = make_plan(72, 1, 1, 4, 128, 16, 1, [("int8", 32), ("fp16", 16)], 2)
    shape = A.ShapeC.from_buffer_copy(plan._shape)
    shape.batch, shape.heads_kv, shape.n_splits = 64, 8, 64  # partials far beyond the built-in scratch
    assert L.argus_decode_attention_workspace_size(ctypes.byref(shape)) > cap
    out = torch.empty_like(q)
    rc = L.argus_decode_attention_noalloc(ctypes.byref(shape), plan._arena_c, plan.chunks_dev.data_ptr(),
                                          plan.splits_dev.data_ptr(), q.data_ptr(), out.data_ptr(), None, None,
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == CAPACITY_ERROR
    assert "scratch" in L.argus_last_error().decode()


def test_noalloc_matches_the_float64_oracle_twice():
    """The same two calls against float64 softmax attention over the K/V the CPU oracle rebuilds from
    the same pages (the reference's dequantization, bit for bit)."""
    from argus_b200 import attention as A
    runs = [make_plan(*c, with_pages=True) for c in CASES]
    for plan, q, pages in runs:
        out_n, _ = call_noalloc(plan, q)
        torch.cuda.synchronize()
        assert A.device_status() == 0
        K, V = U.reference_kv(pages)
        ref = U.f64_attention(q.cpu().numpy(), K, V)
        got = out_n.cpu().numpy().astype(np.float64)
        assert within(got, ref).all(), np.abs(got - ref).max()
