"""GPU parity of the outlier sidecars inside the fused decode attention: pages stay compressed and
their COO sidecars (argus_outlier_corrections blocks) are applied by the kernel.

Reference: the reader dequantizes each page and overwrites the sidecar positions with the sidecar's
fp16 values before attending (core/memory_manager.py:1190-1199, 1402-1409); the oracle reproduces
those K/V bit for bit.  Bar: 2e-3 max-abs plus the fp16 output's half-ulp (2^-11 |ref|) of float64
attention over them, as for every other tier."""
import math

import numpy as np
import pytest
import torch

import attn_util as U

pytestmark = pytest.mark.gpu
ATOL = 2e-3


def within(out, ref, extra=0.0):
    return np.abs(out - ref) <= ATOL + np.abs(ref) * 2.0 ** -11 + extra


def run(pages, B, Hkv, G, D, q, n_splits=None, sidecars=True, tile_lse=False, precise=False):
    from argus_b200 import attention as A
    arenas, plist = U.arenas_from_pages(pages, sidecars=sidecars)
    plan = A.AttentionPlan(arenas, plist, batch=B, heads_kv=Hkv, group=G, head_dim=D, q_len=q.shape[2],
                           n_splits=n_splits, precise_pv=precise)
    tl = torch.full(plan.tile_lse_shape(), float("nan"), device="cuda") if tile_lse else None
    out = plan.run(torch.from_numpy(q).cuda(), tile_lse=tl)
    torch.cuda.synchronize()
    assert A.device_status() == 0
    return out.cpu().numpy().astype(np.float64), plan, tl


@pytest.mark.parametrize("case", ["sidecars", "tiny"])
@pytest.mark.parametrize("n_splits", [1, 3])
def test_golden_sidecar_cases(golden, case, n_splits):
    z = golden("attention")
    B, Hq, Hkv, D, P, L = (int(v) for v in z[f"{case}/meta"])
    pages = U.golden_pages(z, case)
    assert any(pg.get("key_out_indices") is not None and len(pg["key_out_indices"])
               for lst in pages.values() for pg in lst)
    out, _, _ = run(pages, B, Hkv, Hq // Hkv, D, z[f"{case}/q"], n_splits=n_splits)
    f64 = z[f"{case}/out_f64"]
    ref16 = z[f"{case}/out_ref16"].astype(np.float64)
    assert within(out, f64).all(), np.abs(out - f64).max()
    assert within(out, ref16, np.abs(f64 - ref16)).all()


ALL = [("one_bit", 64), ("int2", 64), ("int4", 64), ("int8", 32), ("fp8", 32), ("fp16", 32)]
SHAPES = [
    # B, Hkv, G, D, P, q_len, tiers
    (2, 2, 4, 128, 16, 1, ALL),
    (1, 2, 4, 64, 64, 1, [("one_bit", 128), ("int2", 64), ("int4", 128), ("int8", 64), ("fp8", 64), ("fp16", 64)]),
    (1, 1, 4, 16, 8, 1, [("one_bit", 16), ("int2", 16), ("int4", 16), ("int8", 8), ("fp8", 8), ("fp16", 8)]),
    (1, 2, 2, 256, 16, 2, [("int4", 32), ("one_bit", 32), ("fp16", 16)]),
    (2, 1, 8, 32, 48, 3, [("int8", 96), ("int2", 48), ("fp16", 48)]),
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"B{s[0]}H{s[1]}G{s[2]}D{s[3]}P{s[4]}q{s[5]}")
@pytest.mark.parametrize("sigma,shared", [(3.0, False), (3.0, True), (1.0, True)])
@pytest.mark.parametrize("n_splits", [1, None])
def test_random_pages_with_sidecars(shape, sigma, shared, n_splits):
    B, Hkv, G, D, P, ql, tiers = shape
    rng = np.random.default_rng(B * 1000 + D + P + int(sigma * 7) + shared)
    pages = U.random_pages(rng, tiers, B, Hkv, D, P, sigma=sigma, shared_sidecar=shared)
    q = (rng.standard_normal((B, Hkv * G, ql, D)) / math.sqrt(D) * 2.0).astype(np.float16)
    out, _, _ = run(pages, B, Hkv, G, D, q, n_splits=n_splits)
    K, V = U.reference_kv(pages)
    ref = U.f64_attention(q, K, V)
    assert within(out, ref).all(), np.abs(out - ref).max()
    # the corrections matter: without them the output moves off the reference
    if sigma == 1.0:
        plain, _, _ = run(pages, B, Hkv, G, D, q, n_splits=n_splits, sidecars=False)
        assert not within(plain, ref).all()


def test_tile_mass_includes_key_outliers():
    """Per-tile log2-sum-exp (the page-mass signal) is taken over the corrected scores."""
    B, Hkv, G, D, P = 1, 2, 4, 64, 16
    rng = np.random.default_rng(4)
    pages = U.random_pages(rng, [("int4", 64), ("int8", 32), ("fp16", 16)], B, Hkv, D, P, sigma=1.5)
    q = (rng.standard_normal((B, Hkv * G, 1, D)) / math.sqrt(D) * 3.0).astype(np.float16)
    out, plan, tl = run(pages, B, Hkv, G, D, q, n_splits=1, tile_lse=True)
    K, V = U.reference_kv(pages)
    Kx = np.repeat(K.astype(np.float64), G, axis=1)
    s = np.einsum("bhqd,bhkd->bhqk", q.astype(np.float64), Kx) / math.sqrt(D)  # [B, Hq, 1, L]
    tl = tl.cpu().numpy()  # [B*Hkv*nqg, n_chunks, 16, 8], log2 units
    # token offset of each page in reference_kv order (tiers in TIER_ORDER, pages in order)
    starts, off = {}, 0
    for tier in U.TIER_ORDER:
        for j, _ in enumerate(pages.get(tier, [])):
            starts[(tier, j)] = off
            off += P
    tier_of_arena = [t for t in U.TIER_ORDER if t in pages and t != "jl"]
    checked = 0
    for c, src in enumerate(plan.chunk_pages):
        for i, pi in enumerate(src):
            ai, slot, _ = plan_pages(plan)[pi]
            t0 = starts[(tier_of_arena[ai], slot)]
            for h in range(Hkv):
                for n in range(G):
                    seg = s[0, h * G + n, 0, t0:t0 + P]
                    ref = (seg.max() + np.log(np.exp(seg - seg.max()).sum())) / math.log(2.0)
                    assert abs(tl[h, c, i, n] - ref) < 2e-3, (c, i, h, n)
                    checked += 1
    assert checked == 7 * Hkv * G


def plan_pages(plan):
    return plan.pages


def _one_int8_page(sigma=1.0, seed=0):
    rng = np.random.default_rng(seed)
    return U.random_pages(rng, [("int8", 16)], 1, 2, 64, 16, sigma=sigma)


def test_correction_block_layout():
    """The block written for each (b, h), as the header describes: key offsets per token pair, value
    offsets per (tile, dim group), key entries in (token, dim) order, value entries by tile, dim,
    token; each entry carries sidecar value minus dequantized value."""
    from argus_b200 import paged
    import oracle
    pages = _one_int8_page()
    pg = pages["int8"][0]
    D, P = 64, 16
    arenas, _ = U.arenas_from_pages(pages, sidecars=False)
    a = arenas[0]
    t = lambda key: torch.from_numpy(np.ascontiguousarray(pg[key])).cuda()  # noqa: E731
    blocks, addr = paged.outlier_corrections(a, 0, t("key_out_indices"), t("key_out_values"),
                                             t("value_out_indices"), t("value_out_values"))
    torch.cuda.synchronize()
    raw = blocks.cpu().numpy()
    base = blocks.data_ptr()
    kd = oracle.dequantize_from_int8(pg["key_q"], pg["key_scales"]).astype(np.float32)
    vd = oracle.dequantize_from_int8(pg["value_q"], pg["value_scales"]).astype(np.float32)
    NH = 8 * 1 + 1
    for bh, ad in enumerate(addr.cpu().numpy().tolist()):
        h = bh % 2
        sel_k = pg["key_out_indices"][:, 1] == h
        sel_v = pg["value_out_indices"][:, 1] == h
        ki, kv = pg["key_out_indices"][sel_k], pg["key_out_values"][sel_k].astype(np.float32)
        vi, vv = pg["value_out_indices"][sel_v], pg["value_out_values"][sel_v].astype(np.float32)
        order = np.lexsort((vi[:, 2], vi[:, 3], vi[:, 2] // 16))  # tile, then dim, then token
        vi, vv = vi[order], vv[order]
        assert ad != 0
        off = ad - base
        hdr = raw[off:off + 8 * NH].view(np.uint32)
        koff, voff = hdr[:NH], hdr[NH:]
        assert koff.tolist() == [int(np.sum(ki[:, 2] < 2 * j)) for j in range(NH)]
        assert voff.tolist() == [len(ki) + int(np.sum(vi[:, 3] < g * (D // 8))) for g in range(8)] + [len(ki) + len(vi)]
        ent = raw[off + 8 * NH:off + 8 * NH + 8 * (len(ki) + len(vi))].view(np.uint16).reshape(-1, 4)
        delta = ent[:, 2:].copy().view(np.float32).reshape(-1)
        assert (ent[:len(ki), 0] == ki[:, 2]).all() and (ent[:len(ki), 1] == ki[:, 3]).all()
        assert (ent[len(ki):, 0] == vi[:, 2]).all() and (ent[len(ki):, 1] == vi[:, 3]).all()
        np.testing.assert_array_equal(delta[:len(ki)], kv - kd[0, h, ki[:, 2], ki[:, 3]])
        np.testing.assert_array_equal(delta[len(ki):], vv - vd[0, h, vi[:, 2], vi[:, 3]])


@pytest.mark.parametrize("defect", ["unsorted", "out_of_range"])
def test_bad_sidecar_is_rejected_without_corrections(defect):
    """A sidecar out of row-major order or outside the page gives no corrections (every address 0)
    and a status argus_device_status reports; the attention then reads the bare page."""
    from argus_b200 import attention as A
    from argus_b200 import paged
    pages = _one_int8_page(seed=1)
    pg = pages["int8"][0]
    idx = np.ascontiguousarray(pg["key_out_indices"]).copy()
    if defect == "unsorted":
        idx[[0, 1]] = idx[[1, 0]]
    else:
        idx[-1, 3] = 64
    arenas, plist = U.arenas_from_pages(pages, sidecars=False)
    a = arenas[0]
    paged.attach_outliers(a, 0, torch.from_numpy(idx).cuda(), torch.from_numpy(pg["key_out_values"]).cuda(),
                          None, None)
    torch.cuda.synchronize()
    assert A.device_status() == 1  # ARGUS_ERR_INVALID_ARGUMENT
    assert int(a.outlier_dir.abs().sum().item()) == 0
    q = (np.random.default_rng(2).standard_normal((1, 8, 1, 64)) / 8.0).astype(np.float16)
    plan = A.AttentionPlan(arenas, plist, batch=1, heads_kv=2, group=4, head_dim=64)
    got = plan.run(torch.from_numpy(q).cuda()).cpu().numpy().astype(np.float64)
    assert A.device_status() == 0
    bare = {"int8": [{k: v for k, v in pg.items() if "out_" not in k}]}
    K, V = U.reference_kv(bare)
    assert within(got, U.f64_attention(q, K, V)).all()


@pytest.mark.parametrize("D", [64, 128, 256])
def test_sidecars_with_precise_weights(D):
    """The fp16 hi + lo weight split (ARGUS_ATTN_PRECISE_PV) also feeds the value corrections."""
    B, Hkv, G, P = 1, 2, 4, 16
    rng = np.random.default_rng(D)
    pages = U.random_pages(rng, [("int2", 32), ("int8", 32), ("fp16", 16)], B, Hkv, D, P, sigma=2.0,
                           shared_sidecar=True)
    q = (rng.standard_normal((B, Hkv * G, 1, D)) / math.sqrt(D) * 3.0).astype(np.float16)
    out, _, _ = run(pages, B, Hkv, G, D, q, n_splits=2, precise=True)
    K, V = U.reference_kv(pages)
    ref = U.f64_attention(q, K, V)
    assert within(out, ref).all(), np.abs(out - ref).max()


def test_sidecars_through_the_allocation_free_entry():
    """argus_decode_attention_noalloc applies the same corrections (the arena struct carries them)."""
    import ctypes

    from argus_b200 import _lib
    from argus_b200 import attention as A
    B, Hkv, G, D, P = 1, 2, 4, 64, 16
    rng = np.random.default_rng(8)
    pages = U.random_pages(rng, [("int4", 48), ("fp16", 16)], B, Hkv, D, P, sigma=1.5)
    arenas, plist = U.arenas_from_pages(pages)
    plan = A.AttentionPlan(arenas, plist, batch=B, heads_kv=Hkv, group=G, head_dim=D, n_splits=2)
    q = (rng.standard_normal((B, Hkv * G, 1, D)) / 8.0).astype(np.float16)
    qd = torch.from_numpy(q).cuda()
    out = torch.empty_like(qd)
    L = _lib.lib()
    rc = L.argus_decode_attention_noalloc(ctypes.byref(plan._shape), plan._arena_c, ctypes.c_void_p(plan.chunks_dev.data_ptr()),
                                          ctypes.c_void_p(plan.splits_dev.data_ptr()), ctypes.c_void_p(qd.data_ptr()),
                                          ctypes.c_void_p(out.data_ptr()), None, None,
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert A.device_status() == 0
    K, V = U.reference_kv(pages)
    ref = U.f64_attention(q, K, V)
    got = out.cpu().numpy().astype(np.float64)
    assert within(got, ref).all(), np.abs(got - ref).max()
