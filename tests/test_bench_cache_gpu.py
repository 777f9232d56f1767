"""The cache the benchmark times (bench.build_cache: seeded N(0,1) K/V drawn on the device and
quantized there by the tier codecs, at the full Llama-3-8B layer size) checked against the oracle:
the arena bytes of sampled (batch, kv head) pairs equal the oracle's quantization of the same fp16
K/V bit for bit, and the fused attention of the benchmark's own queries over the whole cache is
within the attention bar (2e-3 + the fp16 output's half-ulp) of float64 attention over the oracle's
reconstruction, for those pairs."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
SAMPLE = [(0, 0), (7, 7), (3, 5)]


def oracle_page(tier, k, v):
    """The oracle's page dict for fp16 [n, P, D] K/V (every page quantized along its own tokens)."""
    if tier == "fp16":
        return {"key": k, "value": v}
    if tier in ("int8", "fp8"):
        f = oracle.quantize_to_int8 if tier == "int8" else oracle.quantize_to_fp8_simulated
        (kq, ks), (vq, vs) = f(k), f(v)
        return {"key_q": kq, "key_scales": ks, "value_q": vq, "value_scales": vs}
    if tier in ("int4", "int2"):
        f = oracle.quantize_to_int4_packed if tier == "int4" else oracle.quantize_to_int2_packed
        (kp, ks, km), (vp, vs, vm) = f(k), f(v)
        return {"key_packed": kp, "key_scales": ks, "key_min": km, "value_packed": vp, "value_scales": vs,
                "value_min": vm}
    (kp, ks), (vp, vs) = oracle.quantize_to_1bit_packed(k), oracle.quantize_to_1bit_packed(v)
    return {"key_packed": kp, "key_scales": ks, "value_packed": vp, "value_scales": vs}


ARENA_PARTS = {"key": "k", "value": "v", "key_q": "k", "value_q": "v", "key_packed": "k", "value_packed": "v",
               "key_scales": "ks", "value_scales": "vs", "key_min": "km", "value_min": "vm"}


def test_bench_cache_matches_the_oracle():
    import bench
    from argus_b200 import attention as A

    dev = torch.device("cuda", 0)
    plan, q, src = bench.build_cache(dev, seed=1234, sample=SAMPLE)
    out = plan.run(q)
    torch.cuda.synchronize()
    assert A.device_status() == 0
    qn, on = q.cpu().numpy(), out.cpu().numpy().astype(np.float64)
    G = bench.HQ // bench.HKV
    for b, h in SAMPLE:
        ks, vs = [], []
        for ai, (tier, _) in enumerate(bench.SPLIT):
            k, v = src[tier][(b, h)]
            pg = oracle_page(tier, k, v)
            arena = plan.arenas[ai]
            for name, arr in pg.items():
                dev_part = arena.view(ARENA_PARTS[name], 0, arena.slots)[:, b, h].cpu().numpy()
                assert dev_part.shape == arr.shape, (tier, name)
                assert np.array_equal(dev_part.view(np.uint8), np.ascontiguousarray(arr).view(np.uint8)), \
                    (tier, name, (b, h))
            kk, vv = oracle.page_kv(tier, pg)  # [n, P, D] (the page dict without batch/head dims)
            ks.append(kk.reshape(-1, bench.D))
            vs.append(vv.reshape(-1, bench.D))
        K = np.concatenate(ks)[None, None]
        V = np.concatenate(vs)[None, None]
        ref = oracle.sdpa_f64(qn[b:b + 1, h * G:(h + 1) * G], K, V, 1.0 / np.sqrt(bench.D))
        got = on[b:b + 1, h * G:(h + 1) * G]
        assert (np.abs(got - ref) <= 2e-3 + np.abs(ref) * 2.0 ** -11).all(), ((b, h), np.abs(got - ref).max())
