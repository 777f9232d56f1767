"""GPU checks of the JL archive contraction, of attention over pages with outlier sidecars and JL
pages (rebuilt on the GPU, then the fused kernel), and of host spill / prefetch round trips.

Bars: JL contractions within fp16 rounding of the reference's fp16 matmul (one output ulp plus
accumulation-order slack); sidecar pages bit-exact; attention 2e-3 + 2^-11 |ref| (plus 4e-3 when
JL pages are present, as the JL rows themselves differ by fp16 matmul rounding); spill and
prefetch bit-exact."""
import math
import os

import numpy as np
import pytest
import torch

import attn_util as U

pytestmark = pytest.mark.gpu


def host(t):
    return t.detach().cpu().contiguous().numpy()


def assert_fp16_close(got, ref, ulps=2):
    got, ref = got.astype(np.float32), ref.astype(np.float32)
    ulp = np.maximum(np.abs(ref), 2.0 ** -14) * 2.0 ** -10
    assert (np.abs(got - ref) <= ulps * ulp + 1e-4).all(), np.abs(got - ref).max()


@pytest.mark.parametrize("P", [16, 64])
def test_jl_manager_project_and_reconstruct(golden, P):
    from argus_b200.core import jl
    z = golden("jl")
    W = torch.from_numpy(z[f"mgr{P}/W"]).cuda()
    R = torch.from_numpy(z[f"mgr{P}/R"]).cuda()
    y = jl.apply_left(W, torch.from_numpy(z[f"mgr{P}/x"]).cuda())
    assert_fp16_close(host(y), z[f"mgr{P}/y"])
    xr = jl.apply_left(R, torch.from_numpy(z[f"mgr{P}/y"]).cuda())
    assert_fp16_close(host(xr), z[f"mgr{P}/xr"])
    # the manager's W drawn on the host is the reference's W bit for bit
    W_host = jl.projection_matrix(P, device="cuda")
    assert (host(W_host).view(np.uint16) == z[f"mgr{P}/W"].view(np.uint16)).all()


@pytest.mark.parametrize("ratio", [4, 8])
def test_jl_quantization_entry_points(golden, ratio):
    from argus_b200.core import quantization as Q
    z = golden("jl")
    pre = f"q256_{ratio}/"
    x = torch.from_numpy(z[pre + "x"]).cuda()
    W = torch.from_numpy(z[pre + "W"]).cuda()
    y, w2 = Q.quantize_to_jl_projection(x, ratio=ratio)
    assert y.shape == torch.Size(z[pre + "y"].shape) and w2.shape == W.shape
    xr = Q.dequantize_from_jl_projection(torch.from_numpy(z[pre + "y"]).cuda(), W)
    ref = z[pre + "xr"].astype(np.float32)
    # R is built on the host in fp32 like the reference's; its fp16 rounding can move by one ulp
    np.testing.assert_allclose(host(xr).astype(np.float32), ref, rtol=4e-3, atol=4e-3)


def gpu_reconstruct(z, case):
    """K, V [B, H, L, D] fp16 on the GPU from the golden pages: page dequant kernels + COO sidecar
    scatter for quantized pages, R @ Y for JL pages, copies for fp16 pages."""
    from argus_b200 import paged
    from argus_b200.core import jl
    B, Hq, Hkv, D, P, L = (int(v) for v in z[f"{case}/meta"])
    pages = U.golden_pages(z, case)
    K = torch.empty(B, Hkv, L, D, dtype=torch.float16, device="cuda")
    V = torch.empty_like(K)
    R = torch.from_numpy(z[f"{case}/R"]).cuda() if f"{case}/R" in z else None
    arenas, plist = U.arenas_from_pages({t: p for t, p in pages.items() if t not in ("jl", "fp16")})
    quant = iter(plist)
    off = 0
    for tier in U.TIER_ORDER:
        for pg in pages.get(tier, []):
            if tier == "fp16":
                K[:, :, off:off + P] = torch.from_numpy(pg["key"]).cuda()
                V[:, :, off:off + P] = torch.from_numpy(pg["value"]).cuda()
            elif tier == "jl":
                K[:, :, off:off + P] = jl.apply_left(R, torch.from_numpy(pg["key_proj"]).cuda())
                V[:, :, off:off + P] = jl.apply_left(R, torch.from_numpy(pg["value_proj"]).cuda())
            else:
                ai, slot, _ = next(quant)
                paged.dequantize_page(arenas[ai], slot, K, V, tok0=off)
                for side, out in (("key", K), ("value", V)):
                    idx = pg.get(f"{side}_out_indices")
                    if idx is not None and idx.size:
                        paged.scatter_coo(out, torch.from_numpy(idx).cuda(),
                                          torch.from_numpy(pg[f"{side}_out_values"]).cuda(), tok0=off,
                                          page_tokens=P)
            off += P
    return K, V


@pytest.mark.parametrize("case", ["tiny", "sidecars", "jl"])
def test_attention_over_rebuilt_pages(golden, case):
    from argus_b200 import attention as A
    z = golden("attention")
    B, Hq, Hkv, D, P, L = (int(v) for v in z[f"{case}/meta"])
    K, V = gpu_reconstruct(z, case)
    has_jl = f"{case}/R" in z
    split = dict(s.split(":") for s in z[f"{case}/split"])
    n_jl = int(split.get("jl", 0))
    for got, ref in ((host(K), z[f"{case}/K"]), (host(V), z[f"{case}/V"])):
        assert_fp16_close(got[:, :, :n_jl], ref[:, :, :n_jl], ulps=4)
        assert (got[:, :, n_jl:].view(np.uint16) == ref[:, :, n_jl:].view(np.uint16)).all()
    arena = A.KVArena.from_fp16(K, V)
    plan = A.AttentionPlan([arena], [(0, j, 16) for j in range(L // 16)], batch=B, heads_kv=Hkv, group=Hq // Hkv,
                           head_dim=D)
    out = host(plan.run(torch.from_numpy(z[f"{case}/q"]).cuda())).astype(np.float64)
    torch.cuda.synchronize()
    assert A.device_status() == 0
    f64 = z[f"{case}/out_f64"]
    ref16 = z[f"{case}/out_ref16"].astype(np.float64)
    bar = 2e-3 + np.abs(f64) * 2.0 ** -11 + 4e-3 * has_jl
    assert (np.abs(out - f64) <= bar).all(), np.abs(out - f64).max()
    assert (np.abs(out - ref16) <= bar + np.abs(f64 - ref16)).all()


def replay_cascade(z, name, tmp_path):
    from argus_b200.core.memory_manager import PagedDynamicKVCache
    P, maxp, sinks, sigma = {"t1": (8, 1, 8, 3.0), "t2": (16, 2, 4, 3.0)}[name]
    os.environ["ARGUS_LOG_LEVEL"] = "quiet"
    cwd = os.getcwd()
    os.chdir(tmp_path)
    try:
        cache = PagedDynamicKVCache(page_size=P, max_active_pages=maxp, max_fp8_pages=maxp, max_int8_pages=maxp,
                                    max_int4_pages=maxp, max_int2_pages=maxp, max_one_bit_pages=maxp,
                                    sink_tokens=sinks, threshold_sigma=sigma)
        for i in range(int(z[f"{name}/n_pushes"])):
            cache.push_new_tokens(torch.from_numpy(z[f"{name}/push{i}/k"]).cuda(),
                                  torch.from_numpy(z[f"{name}/push{i}/v"]).cuda())
    finally:
        os.chdir(cwd)
    return cache


@pytest.mark.parametrize("name", ["t1", "t2"])
def test_swap_out_and_in_round_trip(golden, name, tmp_path):
    z = golden("cascade")
    cache = replay_cascade(z, name, tmp_path)
    K0, V0 = (host(t) for t in cache.get_all_keys_values())
    used = cache.get_vram_usage()
    cache.swap_out_to_host()
    assert cache.is_swapped_out
    assert cache.get_vram_usage() < used
    from argus_b200.core import memory_manager as mm
    for tier in mm._TIERS:
        a = cache.arenas[tier]
        assert not a.k.is_cuda and a.k.is_pinned(), tier
    cache.swap_in_to_device()
    assert not cache.is_swapped_out
    K1, V1 = (host(t) for t in cache.get_all_keys_values())
    assert (K0.view(np.uint16) == K1.view(np.uint16)).all() and (V0.view(np.uint16) == V1.view(np.uint16)).all()
    # a read while spilled brings the tiers back first (memory_manager.py:1163)
    cache.swap_out_to_host()
    K2, V2 = (host(t) for t in cache.get_all_keys_values())
    assert not cache.is_swapped_out
    assert (K0.view(np.uint16) == K2.view(np.uint16)).all() and (V0.view(np.uint16) == V2.view(np.uint16)).all()
    q = torch.from_numpy(z[f"{name}/q"]).cuda()
    out = host(cache.inplace_paged_attention(q)).astype(np.float64)
    import oracle
    ref = oracle.sdpa_f64(z[f"{name}/q"], z[f"{name}/K"], z[f"{name}/V"], 1.0 / math.sqrt(q.shape[-1]))
    bar = 2e-3 + np.abs(ref) * 2.0 ** -11 + 4e-3 * (len(cache.jl_pages) > 0)
    assert (np.abs(out - ref) <= bar).all()


@pytest.mark.parametrize("name", ["t1", "t2"])
def test_speculate_and_prefetch_serves_identical_pages(golden, name, tmp_path):
    z = golden("cascade")
    cache = replay_cascade(z, name, tmp_path)
    K0, V0 = (host(t) for t in cache.get_all_keys_values())
    hits = cache.prefetch_hits
    cache.speculate_and_prefetch()
    assert len(cache.prefetch_cache) >= 1
    K1, V1 = (host(t) for t in cache.get_all_keys_values())
    assert cache.prefetch_hits > hits
    assert (K0.view(np.uint16) == K1.view(np.uint16)).all() and (V0.view(np.uint16) == V1.view(np.uint16)).all()
