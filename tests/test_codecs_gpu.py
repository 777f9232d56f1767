"""GPU parity of the tier codecs (through the C ABI) against the reference's golden vectors and
the CPU oracle: bit-exact for every code, scale, min and dequantized value."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

TIERS = ("int8", "fp8", "int4", "int2", "1bit")


def q():
    from argus_b200.core import quantization
    return quantization


def tk():
    from argus_b200.core import triton_kernels
    return triton_kernels


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.detach().cpu().contiguous().numpy()


def same(a, b, what):
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    assert a.shape == b.shape and a.dtype == b.dtype, (what, a.shape, b.shape, a.dtype, b.dtype)
    if a.dtype == np.float16:
        na, nb = np.isnan(a), np.isnan(b)
        assert (na == nb).all(), f"{what}: NaN positions differ"
        a, b = a[~na].view(np.uint16), b[~nb].view(np.uint16)
    bad = np.flatnonzero(a != b)
    assert bad.size == 0, f"{what}: {bad.size} mismatches of {a.size}, first {bad[:6]}"


def run_tier(tier, x, seq_dim=-2):
    """GPU quantize + dequantize of x (numpy fp16) for one tier; returns numpy outputs."""
    Q = q()
    t = cuda(x)
    if tier == "int8":
        c, s = Q.quantize_to_int8(t)
        return [host(c), host(s), host(Q.dequantize_from_int8(c, s))]
    if tier == "fp8":
        c, s = Q.quantize_to_fp8_simulated(t)
        return [host(c), host(s), host(Q.dequantize_from_fp8_simulated(c, s))]
    if tier == "int4":
        p, s, m = Q.quantize_to_int4_packed(t, seq_dim=seq_dim)
        return [host(p), host(s), host(m), host(Q.dequantize_from_int4_packed(p, s, m, seq_dim=seq_dim))]
    if tier == "int2":
        p, s, m = Q.quantize_to_int2_packed(t, seq_dim=seq_dim)
        return [host(p), host(s), host(m), host(Q.dequantize_from_int2_packed(p, s, m, seq_dim=seq_dim))]
    p, s = Q.quantize_to_1bit_packed(t, seq_dim=seq_dim)
    return [host(p), host(s), host(Q.dequantize_from_1bit_packed(p, s, seq_dim=seq_dim))]


def run_oracle(tier, x, seq_dim=-2):
    if tier == "int8":
        c, s = oracle.quantize_to_int8(x)
        return [c, s, oracle.dequantize_from_int8(c, s)]
    if tier == "fp8":
        c, s = oracle.quantize_to_fp8_simulated(x)
        return [c, s, oracle.dequantize_from_fp8_simulated(c, s)]
    if tier == "int4":
        p, s, m = oracle.quantize_to_int4_packed(x, seq_dim=seq_dim)
        return [p, s, m, oracle.dequantize_from_int4_packed(p, s, m, seq_dim=seq_dim)]
    if tier == "int2":
        p, s, m = oracle.quantize_to_int2_packed(x, seq_dim=seq_dim)
        return [p, s, m, oracle.dequantize_from_int2_packed(p, s, m, seq_dim=seq_dim)]
    p, s = oracle.quantize_to_1bit_packed(x, seq_dim=seq_dim)
    return [p, s, oracle.dequantize_from_1bit_packed(p, s, seq_dim=seq_dim)]


GOLD_KEYS = {"int8": ("int8_q", "int8_s", "int8_deq"), "fp8": ("fp8_q", "fp8_s", "fp8_deq"),
             "int4": ("int4_p", "int4_s", "int4_mn", "int4_deq"),
             "int2": ("int2_p", "int2_s", "int2_mn", "int2_deq"), "1bit": ("1bit_p", "1bit_s", "1bit_deq")}


@pytest.mark.parametrize("tier", TIERS)
def test_codec_golden(golden, tier):
    z = golden("codecs")
    cases = [str(c) for c in z["_cases"]] + ["seq1"]
    for case in cases:
        if f"{case}/{GOLD_KEYS[tier][0]}" not in z:
            continue
        sd = 1 if case == "seq1" else -2
        got = run_tier(tier, z[f"{case}/x"], seq_dim=sd)
        for g, key in zip(got, GOLD_KEYS[tier]):
            same(g, z[f"{case}/{key}"], f"{case}/{key}")


@pytest.mark.parametrize("tier", TIERS)
@pytest.mark.parametrize("shape", [(2, 8, 64, 128), (1, 3, 48, 64), (1, 1, 256, 16), (2, 2, 32, 256)])
def test_codec_vs_oracle_random(tier, shape):
    g = np.random.default_rng(hash((tier, shape)) % 2**32)
    x = g.standard_normal(shape).astype(np.float32)
    mask = g.random(shape) < 0.01
    x[mask] = g.laplace(0, 4, mask.sum())
    x = x.astype(np.float16)
    for a, b, i in zip(run_tier(tier, x), run_oracle(tier, x), range(4)):
        same(a, b, f"{tier}{shape} out{i}")


def test_triton_entry_points(golden):
    z = golden("codecs")
    x = z["lap/x"]
    codes = np.random.default_rng(0).integers(0, 16, size=x.shape, dtype=np.uint8)
    packed = host(tk().triton_pack_int4(cuda(codes)))
    ref = (codes.reshape(*codes.shape[:-2], -1, 2, codes.shape[-1])[..., 0, :]
           | (codes.reshape(*codes.shape[:-2], -1, 2, codes.shape[-1])[..., 1, :] << 4))
    same(packed, ref, "pack_int4 codes")
    same(host(tk().triton_pack_1bit(cuda(x))), z["lap/1bit_p"], "pack_1bit")
    same(host(tk().triton_unpack_1bit(cuda(z["lap/1bit_p"]), cuda(z["lap/1bit_s"]))), z["lap/1bit_deq"], "unpack_1bit")
    same(host(tk().triton_unpack_int4(cuda(z["lap/int4_p"]), cuda(z["lap/int4_s"]), cuda(z["lap/int4_mn"]))),
         z["lap/int4_deq"], "unpack_int4")


def test_isolate_outliers_golden(golden):
    from argus_b200.core import memory_manager as mm
    z = golden("outliers")
    for case in z["_cases"]:
        case = str(case)
        normal, outv, mask = mm.isolate_outliers(cuda(z[f"{case}/x"]), float(z[f"{case}/sigma"]))
        same(host(normal), z[f"{case}/normal"], f"{case} normal")
        same(host(outv), z[f"{case}/outv"], f"{case} outv")
        assert (host(mask) == z[f"{case}/mask"]).all(), case


def test_divisibility_asserts():
    x = torch.randn(1, 1, 6, 64, device="cuda").half()
    with pytest.raises(AssertionError):
        q().quantize_to_1bit_packed(x)
    with pytest.raises(AssertionError):
        q().quantize_to_int2_packed(x)


def test_no_cpu_fallback():
    with pytest.raises(ValueError):
        q().quantize_to_int8(torch.randn(1, 1, 8, 64).half())


@pytest.mark.parametrize("tier", TIERS)
def test_full_size_sampled_rows(tier):
    """The cascade microbenchmark shape (1,048,576 tokens x 8 KV heads x 128, 1% Laplace(0,4)):
    the whole tensor is coded on the GPU and a random sample of packing groups is checked
    bit-exact against the oracle."""
    torch.manual_seed(0)
    B, H, T, D = 1, 8, 1048576, 128
    x = torch.randn(B, H, T, D, device="cuda", dtype=torch.float16)
    lap = torch.distributions.Laplace(0.0, 4.0).sample((B, H, T, D)).to("cuda", torch.float16)
    x = torch.where(torch.rand(B, H, T, D, device="cuda") < 0.01, lap, x)
    gpu = run_tier_torch(tier, x)
    per = {"int8": 1, "fp8": 1, "int4": 2, "int2": 4, "1bit": 8}[tier]
    rng = np.random.default_rng(1)
    heads = rng.integers(0, H, 64)
    groups = rng.integers(0, T // 8, 64) * 8  # 8-token groups cover every packing factor
    for h, t0 in zip(heads, groups):
        xs = host(x[0, h, t0:t0 + 8])[None]
        ref = run_oracle(tier, xs)
        for i, (g_full, r) in enumerate(zip(gpu, ref)):
            sl = g_full[0, h, t0 // per:(t0 + 8) // per] if i == 0 and per > 1 else g_full[0, h, t0:t0 + 8]
            same(host(sl)[None], r, f"{tier} h{h} t{t0} out{i}")
    del gpu
    torch.cuda.empty_cache()


def run_tier_torch(tier, t):
    Q = q()
    if tier == "int8":
        c, s = Q.quantize_to_int8(t)
        return [c, s, Q.dequantize_from_int8(c, s)]
    if tier == "fp8":
        c, s = Q.quantize_to_fp8_simulated(t)
        return [c, s, Q.dequantize_from_fp8_simulated(c, s)]
    if tier == "int4":
        p, s, m = Q.quantize_to_int4_packed(t)
        return [p, s, m, Q.dequantize_from_int4_packed(p, s, m)]
    if tier == "int2":
        p, s, m = Q.quantize_to_int2_packed(t)
        return [p, s, m, Q.dequantize_from_int2_packed(p, s, m)]
    p, s = Q.quantize_to_1bit_packed(t)
    return [p, s, Q.dequantize_from_1bit_packed(p, s)]


def test_fast_quotient_matches_ieee_divide_for_every_fp16_pair():
    """The quantizers divide by a per-token scale with a reciprocal + FMA correction; it must equal
    the IEEE-rounded fp32 divide for every finite fp16 dividend and positive finite fp16 divisor
    (the reference's x / s on fp16 tensors), checked exhaustively (2.0e9 pairs)."""
    import ctypes

    from argus_b200 import _lib
    n = ctypes.c_ulonglong(12345)
    _lib.call("argus_selftest_fp16_quotients", ctypes.byref(n), _lib.stream_handle())
    assert n.value == 0
