"""Generate the golden input/output vectors that pin the CPU oracle and the CUDA path.

This script imports the ARGUS reference package (argus_cache 0.1.8) read-only and runs it
on CPU tensors, so the reference's own torch fallback is the code path exercised
(argus_cache/core/triton_kernels.py:177,217,264,334 take the fallback when a tensor is
not on CUDA).  It writes small ``.npz`` fixtures next to this file.  The GPU box never
runs this script; the committed fixtures are what travels.

Usage (from the repository root, with the reference checked out read-only):

    python tests/golden/make_golden.py --reference /path/to/ARGUS-reference

Fixture groups
--------------
codecs.npz     every quantize_* / dequantize_* pair on random, outlier-heavy and edge rows
outliers.npz   isolate_outliers (NaN/Inf cleanse, mean|x|*sigma threshold, COO sidecar)
jl.npz         JL projection matrix W, Laplacian reconstruction operator R, project/reconstruct
attention.npz  reconstruct-then-SDPA outputs of the reference for mixed-tier page sets
cascade.npz    a full PagedDynamicKVCache run through all seven tiers (pages, K/V, attention)
"""
import argparse
import math
import os
import sys
import tempfile

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(t):
    # a copy: numpy views of CPU tensors would alias pool memory that later calls overwrite
    return t.detach().cpu().contiguous().numpy().copy()


def load_reference(path):
    os.environ["ARGUS_LOG_LEVEL"] = "quiet"
    sys.path.insert(0, path)
    import argus_cache.core.quantization as rq  # noqa: E402
    import argus_cache.core.memory_manager as rm  # noqa: E402
    return rq, rm


# ----------------------------------------------------------------------------------
# codecs
# ----------------------------------------------------------------------------------
def edge_rows(D):
    """Rows that exercise the corners of the codecs' fp16 arithmetic."""
    g = torch.Generator().manual_seed(7)
    rows = []
    rows.append(torch.zeros(D))                                   # all-zero row: scale 0, 0/0
    rows.append(torch.full((D,), 1.5))                            # constant row: int4/int2 range 0
    rows.append(torch.randn(D, generator=g) * 1e-6)               # subnormal magnitudes
    rows.append(torch.randn(D, generator=g) * 2e4)                # near the fp16 range
    r = torch.randn(D, generator=g); r[0] = 60000.0; r[1] = -60000.0
    rows.append(r)                                                # mx - mn overflows to inf
    r = torch.randn(D, generator=g); r[::3] = -0.0
    rows.append(r)                                                # negative zeros (1-bit sign)
    r = torch.randn(D, generator=g); r[2] = float("inf")
    rows.append(r)                                                # +inf
    r = torch.randn(D, generator=g); r[5] = float("-inf")
    rows.append(r)                                                # -inf
    r = torch.randn(D, generator=g); r[4] = float("nan")
    rows.append(r)                                                # NaN
    r = torch.arange(D, dtype=torch.float32) - D / 2
    rows.append(r * 0.5)                                          # exact halves: round-half-even
    r = torch.randn(D, generator=g); r[0] = 8.0
    rows.append(r * 3.0)                                          # fp8-sim wrap region
    rows.append(-torch.rand(D, generator=g) * 3 - 0.1)            # all negative
    rows.append(torch.rand(D, generator=g) * 3 + 0.1)             # all positive
    rows.append(torch.full((D,), 6.1e-5))                         # tiny constant
    rows.append(torch.randn(D, generator=g) * 100)                # large spread
    rows.append(torch.full((D,), -2.0))                           # negative constant
    return torch.stack(rows).view(1, 1, len(rows), D).half()


def laplace_outliers(shape, seed, frac=0.01, scale=4.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g)
    mask = torch.rand(*shape, generator=g) < frac
    u = torch.rand(*shape, generator=g) - 0.5
    lap = -scale * torch.sign(u) * torch.log1p(-2 * u.abs())
    return torch.where(mask, lap, x).half()


def gen_codecs(rq):
    out = {}
    cases = {
        "lap": laplace_outliers((2, 3, 32, 64), seed=0),
        "d128": (torch.randn(1, 2, 32, 128, generator=torch.Generator().manual_seed(1)) * 3).half(),
        "d16": torch.randn(1, 1, 16, 16, generator=torch.Generator().manual_seed(2)).half(),
        "edge64": edge_rows(64),
        "edge16": edge_rows(16),
        "d40": torch.randn(2, 1, 8, 40, generator=torch.Generator().manual_seed(3)).half(),
    }
    for name, x in cases.items():
        out[f"{name}/x"] = _np(x)
        q, s = rq.quantize_to_int8(x)
        out[f"{name}/int8_q"], out[f"{name}/int8_s"] = _np(q), _np(s)
        out[f"{name}/int8_deq"] = _np(rq.dequantize_from_int8(q, s))
        q, s = rq.quantize_to_fp8_simulated(x)
        out[f"{name}/fp8_q"], out[f"{name}/fp8_s"] = _np(q), _np(s)
        out[f"{name}/fp8_deq"] = _np(rq.dequantize_from_fp8_simulated(q, s))
        p, s, mn = rq.quantize_to_int4_packed(x)
        out[f"{name}/int4_p"], out[f"{name}/int4_s"], out[f"{name}/int4_mn"] = _np(p), _np(s), _np(mn)
        out[f"{name}/int4_deq"] = _np(rq.dequantize_from_int4_packed(p, s, mn))
        p, s, mn = rq.quantize_to_int2_packed(x)
        out[f"{name}/int2_p"], out[f"{name}/int2_s"], out[f"{name}/int2_mn"] = _np(p), _np(s), _np(mn)
        out[f"{name}/int2_deq"] = _np(rq.dequantize_from_int2_packed(p, s, mn))
        p, s = rq.quantize_to_1bit_packed(x)
        out[f"{name}/1bit_p"], out[f"{name}/1bit_s"] = _np(p), _np(s)
        out[f"{name}/1bit_deq"] = _np(rq.dequantize_from_1bit_packed(p, s))
    # packing along a sequence axis that is not the second-to-last one
    x = laplace_outliers((2, 16, 3, 32), seed=4)
    out["seq1/x"] = _np(x)
    p, s, mn = rq.quantize_to_int4_packed(x, seq_dim=1)
    out["seq1/int4_p"], out["seq1/int4_s"], out["seq1/int4_mn"] = _np(p), _np(s), _np(mn)
    out["seq1/int4_deq"] = _np(rq.dequantize_from_int4_packed(p, s, mn, seq_dim=1))
    p, s, mn = rq.quantize_to_int2_packed(x, seq_dim=1)
    out["seq1/int2_p"], out["seq1/int2_s"], out["seq1/int2_mn"] = _np(p), _np(s), _np(mn)
    out["seq1/int2_deq"] = _np(rq.dequantize_from_int2_packed(p, s, mn, seq_dim=1))
    p, s = rq.quantize_to_1bit_packed(x, seq_dim=1)
    out["seq1/1bit_p"], out["seq1/1bit_s"] = _np(p), _np(s)
    out["seq1/1bit_deq"] = _np(rq.dequantize_from_1bit_packed(p, s, seq_dim=1))
    out["_cases"] = np.array(list(cases.keys()))
    return out


# ----------------------------------------------------------------------------------
# outlier isolation
# ----------------------------------------------------------------------------------
def outlier_page(shape, seed, n_channels=4, factor=8.0):
    g = torch.Generator().manual_seed(seed)
    B, H, P, D = shape
    x = torch.randn(*shape, generator=g)
    for h in range(H):
        ch = torch.randperm(D, generator=g)[:n_channels]
        x[:, h, :, ch] *= factor
    return x.half()


def gen_outliers(rm):
    out = {}
    cases = {}
    cases["s3"] = (outlier_page((2, 2, 16, 64), seed=10), 3.0)
    cases["s25"] = (outlier_page((1, 2, 16, 128), seed=11), 2.5)
    x = outlier_page((1, 2, 16, 64), seed=12)
    x[0, 0, 3, 7] = float("nan"); x[0, 1, 9, 1] = float("inf"); x[0, 1, 2, 60] = float("-inf")
    cases["naninf"] = (x, 3.0)
    cases["zero_sigma"] = (outlier_page((1, 1, 16, 16), seed=13), 0.0)
    cases["d16"] = (outlier_page((1, 1, 8, 16), seed=14, n_channels=2), 3.0)
    for name, (x, sig) in cases.items():
        normal, outv, mask = rm.isolate_outliers(x, sig)
        out[f"{name}/x"] = _np(x)
        out[f"{name}/sigma"] = np.array(sig, dtype=np.float64)
        out[f"{name}/normal"] = _np(normal)
        out[f"{name}/outv"] = _np(outv)
        out[f"{name}/mask"] = _np(mask)
        out[f"{name}/idx"] = _np(torch.nonzero(mask).to(torch.int16))
        out[f"{name}/vals"] = _np(outv[mask])
    out["_cases"] = np.array(list(cases.keys()))
    return out


# ----------------------------------------------------------------------------------
# JL archive
# ----------------------------------------------------------------------------------
def gen_jl(rq, rm):
    out = {}
    # The manager's matrices (ratio 4, seed 42 drawn on the CPU device).
    for P in (16, 64):
        mgr = rm.PagedDynamicKVCache(page_size=P, sink_tokens=0)
        W = mgr.get_jl_projection_matrix(torch.device("cpu"), torch.float16)
        R = mgr.get_jl_reconstruction_operator(torch.device("cpu"), torch.float16)
        out[f"mgr{P}/W"] = _np(W)
        out[f"mgr{P}/R"] = _np(R)
        x = torch.randn(1, 2, P, 32, generator=torch.Generator().manual_seed(20 + P)).half()
        y = torch.matmul(W, x)
        out[f"mgr{P}/x"], out[f"mgr{P}/y"] = _np(x), _np(y)
        out[f"mgr{P}/xr"] = _np(torch.matmul(R, y))
    # quantization.py's solve-form operator for a caller-supplied W (ratio 4 and 8).
    for N, ratio in ((256, 4), (256, 8)):
        torch.manual_seed(30 + ratio)
        x = torch.randn(1, 1, N, 32).half()
        y, W = rq.quantize_to_jl_projection(x, ratio=ratio)
        xr = rq.dequantize_from_jl_projection(y, W)
        out[f"q{N}_{ratio}/x"], out[f"q{N}_{ratio}/y"], out[f"q{N}_{ratio}/W"] = _np(x), _np(y), _np(W)
        out[f"q{N}_{ratio}/xr"] = _np(xr)
    return out


# ----------------------------------------------------------------------------------
# attention over page sets (reference reconstruct-then-SDPA)
# ----------------------------------------------------------------------------------
def ref_sdpa(q, k, v, scale):
    """The reference's dense attention, fp16 CPU ops as in memory_manager.py:1424-1430,
    with the GQA expansion transformers applies after PagedDynamicQuantizedCache.update."""
    g = q.shape[1] // k.shape[1]
    k = k.repeat_interleave(g, dim=1)
    v = v.repeat_interleave(g, dim=1)
    w = torch.matmul(q, k.transpose(-1, -2)) * scale
    p = torch.softmax(w, dim=-1)
    return torch.matmul(p, v)


def f64_sdpa(q, k, v, scale):
    g = q.shape[1] // k.shape[1]
    k = k.double().repeat_interleave(g, dim=1)
    v = v.double().repeat_interleave(g, dim=1)
    w = torch.matmul(q.double(), k.transpose(-1, -2)) * scale
    return torch.matmul(torch.softmax(w, dim=-1), v)


def build_tier_page(rq, rm, tier, k, v, sigma):
    """One page dict built the way the _demote_* methods lay them out
    (memory_manager.py:944-1155), from an FP16 page; each tier is quantized directly."""
    page = {}
    if tier == "fp16":
        return {"key": k, "value": v}
    if sigma > 0 and tier in ("fp8", "int8", "int4", "int2", "one_bit"):
        kn, ko, km = rm.isolate_outliers(k, sigma)
        vn, vo, vm = rm.isolate_outliers(v, sigma)
        page["key_out_indices"] = torch.nonzero(km).to(torch.int16)
        page["key_out_values"] = ko[km]
        page["value_out_indices"] = torch.nonzero(vm).to(torch.int16)
        page["value_out_values"] = vo[vm]
    else:
        kn, vn = k, v
        page["key_out_indices"] = None
        page["value_out_indices"] = None
    if tier == "fp8":
        page["key_q"], page["key_scales"] = rq.quantize_to_fp8_simulated(kn)
        page["value_q"], page["value_scales"] = rq.quantize_to_fp8_simulated(vn)
    elif tier == "int8":
        page["key_q"], page["key_scales"] = rq.quantize_to_int8(kn)
        page["value_q"], page["value_scales"] = rq.quantize_to_int8(vn)
    elif tier == "int4":
        page["key_packed"], page["key_scales"], page["key_min"] = rq.quantize_to_int4_packed(kn)
        page["value_packed"], page["value_scales"], page["value_min"] = rq.quantize_to_int4_packed(vn)
    elif tier == "int2":
        page["key_packed"], page["key_scales"], page["key_min"] = rq.quantize_to_int2_packed(kn)
        page["value_packed"], page["value_scales"], page["value_min"] = rq.quantize_to_int2_packed(vn)
    elif tier == "one_bit":
        page["key_packed"], page["key_scales"] = rq.quantize_to_1bit_packed(kn)
        page["value_packed"], page["value_scales"] = rq.quantize_to_1bit_packed(vn)
    elif tier == "jl":
        raise ValueError("jl pages are built by the caller")
    return page


PAGE_FIELDS = ("key", "value", "key_q", "value_q", "key_packed", "value_packed", "key_scales",
               "value_scales", "key_min", "value_min", "key_out_indices", "key_out_values",
               "value_out_indices", "value_out_values", "key_proj", "value_proj")


def gen_attention(rq, rm):
    out = {}
    tiers_order = ("jl", "one_bit", "int2", "int4", "int8", "fp8", "fp16")

    def run_case(name, B, Hq, Hkv, D, P, split, sigma, seed, outlier_channels=0, q_scale=1.0):
        """split: list of (tier, n_tokens) from oldest to newest."""
        g = torch.Generator().manual_seed(seed)
        L = sum(n for _, n in split)
        k = torch.randn(B, Hkv, L, D, generator=g)
        v = torch.randn(B, Hkv, L, D, generator=g)
        if outlier_channels:
            for h in range(Hkv):
                ch = torch.randperm(D, generator=g)[:outlier_channels]
                k[:, h, :, ch] *= 8.0
                v[:, h, :, ch] *= 8.0
        k, v = k.half(), v.half()
        q = (torch.randn(B, Hq, 1, D, generator=g) * q_scale).half()
        mgr = rm.PagedDynamicKVCache(page_size=P, sink_tokens=0, threshold_sigma=sigma)
        recon = None
        t0 = 0
        for tier, n in split:
            assert n % P == 0
            for j in range(n // P):
                kp = k[:, :, t0:t0 + P, :]
                vp = v[:, :, t0:t0 + P, :]
                if tier == "jl":
                    W = mgr.get_jl_projection_matrix(torch.device("cpu"), torch.float16)
                    page = {"key_proj": torch.matmul(W, kp), "value_proj": torch.matmul(W, vp)}
                else:
                    page = build_tier_page(rq, rm, tier, kp, vp, sigma)
                page.update({"page_id": t0 // P + 1, "attention_sum": 0.0,
                             "last_step_accessed": 0, "entropy": 0.0, "importance_score": 0.0})
                lst = {"jl": mgr.jl_pages, "one_bit": mgr.one_bit_pages, "int2": mgr.int2_pages,
                       "int4": mgr.int4_pages, "int8": mgr.int8_pages, "fp8": mgr.fp8_pages,
                       "fp16": mgr.active_pages}[tier]
                lst.append(page)
                for f in PAGE_FIELDS:
                    if page.get(f) is not None:
                        out[f"{name}/{tier}/{j}/{f}"] = _np(page[f])
                t0 += P
        K, V = mgr.get_all_keys_values()
        scale = 1.0 / math.sqrt(D)
        o16 = ref_sdpa(q, K, V, scale)
        o64 = f64_sdpa(q, K, V, scale)
        out[f"{name}/q"] = _np(q)
        out[f"{name}/K"], out[f"{name}/V"] = _np(K), _np(V)
        out[f"{name}/out_ref16"] = _np(o16)
        out[f"{name}/out_f64"] = o64.numpy()
        out[f"{name}/scale"] = np.array(scale)
        out[f"{name}/meta"] = np.array([B, Hq, Hkv, D, P, L])
        out[f"{name}/split"] = np.array([f"{t}:{n}" for t, n in split])
        if mgr.w_proj is not None:
            out[f"{name}/W"] = _np(mgr.w_proj)
            out[f"{name}/R"] = _np(mgr.get_jl_reconstruction_operator(torch.device("cpu"), torch.float16))

    # TinyLlama-shaped: INT8 pages with their own outlier sidecars, then FP16 pages.
    run_case("tiny", B=1, Hq=8, Hkv=2, D=64, P=16, split=[("int8", 192), ("fp16", 64)],
             sigma=3.0, seed=40, outlier_channels=4)
    # Llama-3-8B-shaped mixed tiers, no sidecars.
    run_case("mixed", B=2, Hq=8, Hkv=2, D=128, P=16,
             split=[("one_bit", 64), ("int2", 64), ("int4", 64), ("int8", 32), ("fp8", 32), ("fp16", 32)],
             sigma=0.0, seed=41, q_scale=1.0 / math.sqrt(128))
    # Every tier with sidecars (INT8 and below carry their own, as built directly).
    run_case("sidecars", B=1, Hq=4, Hkv=2, D=64, P=16,
             split=[("one_bit", 32), ("int2", 32), ("int4", 32), ("int8", 16), ("fp8", 16), ("fp16", 16)],
             sigma=3.0, seed=42, outlier_channels=4)
    # JL pages (ratio 4 of the manager) next to an FP16 page, GQA 4.
    run_case("jl", B=1, Hq=8, Hkv=2, D=64, P=16, split=[("jl", 48), ("int4", 16), ("fp16", 16)],
             sigma=0.0, seed=43)
    # GQA 8, head_dim 128, larger query magnitude (peakier softmax).
    run_case("peaky", B=1, Hq=16, Hkv=2, D=128, P=16,
             split=[("int4", 32), ("int8", 32), ("fp16", 16)], sigma=0.0, seed=44, q_scale=2.0)
    return out


# ----------------------------------------------------------------------------------
# a full manager run through the cascade
# ----------------------------------------------------------------------------------
def gen_cascade(rm):
    out = {}

    def run(name, P, maxp, D, H, pushes, seed, sigma=3.0, sinks=4, attn_queries=1):
        g = torch.Generator().manual_seed(seed)
        mgr = rm.PagedDynamicKVCache(page_size=P, max_active_pages=maxp, max_fp8_pages=maxp,
                                     max_int8_pages=maxp, max_int4_pages=maxp, max_int2_pages=maxp,
                                     max_one_bit_pages=maxp, sink_tokens=sinks, threshold_sigma=sigma)
        ks, vs = [], []
        for i, n in enumerate(pushes):
            k = torch.randn(1, H, n, D, generator=g)
            v = torch.randn(1, H, n, D, generator=g)
            k[..., 3] *= 6.0
            v[..., 5] *= 6.0
            k, v = k.half(), v.half()
            ks.append(k); vs.append(v)
            out[f"{name}/push{i}/k"], out[f"{name}/push{i}/v"] = _np(k), _np(v)
            mgr.push_new_tokens(k, v)
        out[f"{name}/n_pushes"] = np.array(len(pushes))
        counts = [len(mgr.active_pages), len(mgr.fp8_pages), len(mgr.int8_pages), len(mgr.int4_pages),
                  len(mgr.int2_pages), len(mgr.one_bit_pages), len(mgr.jl_pages)]
        out[f"{name}/tier_counts"] = np.array(counts)
        for tier, lst in (("fp16", mgr.active_pages), ("fp8", mgr.fp8_pages), ("int8", mgr.int8_pages),
                          ("int4", mgr.int4_pages), ("int2", mgr.int2_pages),
                          ("one_bit", mgr.one_bit_pages), ("jl", mgr.jl_pages)):
            out[f"{name}/{tier}/page_ids"] = np.array([p["page_id"] for p in lst], dtype=np.int64)
            for j, page in enumerate(lst):
                for f in PAGE_FIELDS:
                    if isinstance(page.get(f), torch.Tensor):
                        out[f"{name}/{tier}/{j}/{f}"] = _np(page[f])
        K, V = mgr.get_all_keys_values()
        out[f"{name}/K"], out[f"{name}/V"] = _np(K), _np(V)
        q = torch.randn(1, H, attn_queries, D, generator=g).half()
        out[f"{name}/q"] = _np(q)
        o = mgr.inplace_paged_attention(q)
        out[f"{name}/attn"] = _np(o)
        counts = [len(mgr.active_pages), len(mgr.fp8_pages), len(mgr.int8_pages), len(mgr.int4_pages),
                  len(mgr.int2_pages), len(mgr.one_bit_pages), len(mgr.jl_pages)]
        out[f"{name}/tier_counts_after_attn"] = np.array(counts)

    # test_kv_cache.py:10-190 shape: one page per tier, page 8, D 16, all seven tiers reached.
    run("t1", P=8, maxp=1, D=16, H=1, pushes=[8, 4, 4, 8, 8, 8, 8, 8, 8], seed=50, sinks=8)
    # Two pages per tier, page 16, D 64, two heads: the importance policy picks victims.
    run("t2", P=16, maxp=2, D=64, H=2, pushes=[20] + [16] * 14 + [5], seed=51)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of the ARGUS reference (read-only)")
    args = ap.parse_args()
    rq, rm = load_reference(os.path.abspath(args.reference))
    torch.set_num_threads(1)
    cwd = os.getcwd()
    # The reference's manager appends a trace to ./tests/argus_attention_trace.jsonl.
    with tempfile.TemporaryDirectory() as tmp:
        os.chdir(tmp)
        try:
            groups = {
                "codecs": gen_codecs(rq),
                "outliers": gen_outliers(rm),
                "jl": gen_jl(rq, rm),
                "attention": gen_attention(rq, rm),
                "cascade": gen_cascade(rm),
            }
        finally:
            os.chdir(cwd)
    for name, arrs in groups.items():
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **arrs)
        print(f"{path}: {len(arrs)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
