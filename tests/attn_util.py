"""Helpers shared by the attention tests: build arenas/pages from golden page dicts or from
seeded random data, and the float64 reference over oracle-dequantized pages."""
import math

import numpy as np
import torch

import oracle

TIER_ORDER = ("jl", "one_bit", "int2", "int4", "int8", "fp8", "fp16")


def golden_pages(z, case):
    """{tier: [page dict of numpy arrays]} for one golden attention case."""
    B, Hq, Hkv, D, P, L = (int(v) for v in z[f"{case}/meta"])
    split = dict(s.split(":") for s in z[f"{case}/split"])
    pages = {}
    for tier in TIER_ORDER:
        if tier not in split:
            continue
        lst = []
        for j in range(int(split[tier]) // P):
            pre = f"{case}/{tier}/{j}/"
            lst.append({k[len(pre):]: z[k] for k in z.files if k.startswith(pre)})
        pages[tier] = lst
    return pages


def arenas_from_pages(pages, device="cuda", sidecars=True):
    """Writes each tier's pages into a record arena and returns (arenas, page list); pages with COO
    sidecars get their outlier corrections attached (sidecars=True)."""
    from argus_b200 import attention as A

    tier_id = {"fp16": A.TIER_FP16, "fp8": A.TIER_FP8SIM, "int8": A.TIER_INT8, "int4": A.TIER_INT4,
               "int2": A.TIER_INT2, "one_bit": A.TIER_1BIT}
    arenas, plist = [], []
    for tier in TIER_ORDER:
        if tier not in pages or tier == "jl":
            continue
        lst = pages[tier]
        stack = lambda key: torch.from_numpy(np.stack([p[key] for p in lst])).to(device)  # noqa: E731
        first = lst[0]["key"] if tier == "fp16" else lst[0]["key_scales"]
        B, H, P = first.shape[0], first.shape[1], first.shape[2]
        D = (lst[0]["key"] if tier == "fp16" else lst[0].get("key_q", lst[0].get("key_packed"))).shape[-1]
        a = A.KVArena.allocate(tier_id[tier], B, H, len(lst), P, D, device)
        if tier == "fp16":
            a.write_pages(0, stack("key"), stack("value"))
        elif tier in ("fp8", "int8"):
            a.write_pages(0, stack("key_q"), stack("value_q"), stack("key_scales"), stack("value_scales"))
        elif tier in ("int4", "int2"):
            a.write_pages(0, stack("key_packed"), stack("value_packed"), stack("key_scales"), stack("value_scales"),
                          stack("key_min"), stack("value_min"))
        else:
            a.write_pages(0, stack("key_packed"), stack("value_packed"), stack("key_scales"), stack("value_scales"))
        if sidecars and tier != "fp16":
            from argus_b200 import paged
            for j, pg in enumerate(lst):
                ki, vi = pg.get("key_out_indices"), pg.get("value_out_indices")
                if (ki is None or not len(ki)) and (vi is None or not len(vi)):
                    continue
                t = lambda key: torch.from_numpy(np.ascontiguousarray(pg[key])).to(device) \
                    if pg.get(key) is not None and len(pg[key]) else None  # noqa: E731
                paged.attach_outliers(a, j, t("key_out_indices"), t("key_out_values"), t("value_out_indices"),
                                      t("value_out_values"))
        ai = len(arenas)
        arenas.append(a)
        plist += [(ai, j, P) for j in range(len(lst))]
    return arenas, plist


def random_pages(rng, tiers_tokens, B, Hkv, D, P, outlier_frac=0.01, sigma=None, shared_sidecar=False):
    """Seeded fp16 pages quantized by the CPU oracle: {tier: [page dicts]}, tokens per tier.  With
    sigma, quantized pages first have their outliers isolated into COO sidecars, as the reference's
    first demotion does (shared_sidecar: the V sidecar is the K sidecar, as the reference's INT8 and
    lower tiers store it)."""
    pages = {}
    for tier, ntok in tiers_tokens:
        lst = []
        for _ in range(ntok // P):
            k = rng.standard_normal((B, Hkv, P, D)).astype(np.float32)
            v = rng.standard_normal((B, Hkv, P, D)).astype(np.float32)
            for t in (k, v):
                m = rng.random(t.shape) < outlier_frac
                t[m] = rng.laplace(0, 4, m.sum())
            k, v = k.astype(np.float16), v.astype(np.float16)
            pg = {}
            if sigma is not None and tier != "fp16":
                kn, ko, km = oracle.isolate_outliers(k, sigma)
                vn, vo, vm = oracle.isolate_outliers(v, sigma)
                pg["key_out_indices"], pg["key_out_values"] = oracle.sidecar(km, ko)
                if shared_sidecar:
                    pg["value_out_indices"], pg["value_out_values"] = pg["key_out_indices"], pg["key_out_values"]
                else:
                    pg["value_out_indices"], pg["value_out_values"] = oracle.sidecar(vm, vo)
                k, v = kn, vn
            if tier == "fp16":
                pg = {"key": k, "value": v}
            elif tier in ("fp8", "int8"):
                f = oracle.quantize_to_int8 if tier == "int8" else oracle.quantize_to_fp8_simulated
                pg["key_q"], pg["key_scales"] = f(k)
                pg["value_q"], pg["value_scales"] = f(v)
            elif tier in ("int4", "int2"):
                f = oracle.quantize_to_int4_packed if tier == "int4" else oracle.quantize_to_int2_packed
                pg["key_packed"], pg["key_scales"], pg["key_min"] = f(k)
                pg["value_packed"], pg["value_scales"], pg["value_min"] = f(v)
            else:
                pg["key_packed"], pg["key_scales"] = oracle.quantize_to_1bit_packed(k)
                pg["value_packed"], pg["value_scales"] = oracle.quantize_to_1bit_packed(v)
            lst.append(pg)
        pages[tier] = lst
    return pages


def reference_kv(pages, R=None):
    ks, vs = [], []
    for tier in TIER_ORDER:
        for pg in pages.get(tier, []):
            k, v = oracle.page_kv(tier, pg, R)
            ks.append(k)
            vs.append(v)
    return np.concatenate(ks, axis=2), np.concatenate(vs, axis=2)


def f64_attention(q, K, V, scale=None):
    D = q.shape[-1]
    return oracle.sdpa_f64(q, K, V, (1.0 / math.sqrt(D)) if scale is None else scale)
