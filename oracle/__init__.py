"""CPU oracle for the ARGUS tiered-KV hot path -- TEST INFRASTRUCTURE ONLY.

Restates the reference's CPU arithmetic (argus_cache 0.1.8) so that the CUDA path can be
checked against it.  The codecs and the outlier filter run in plain C (argus_oracle.c,
built by the Makefile beside it into _build/liboracle.so); attention and the page
reconstruction run in numpy float64.  Only tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py import this package.

Function -> reference file:line
  quantize_to_int8 / dequantize_from_int8                 core/quantization.py:3-28
  quantize_to_fp8_simulated / dequantize_from_fp8_sim...  core/quantization.py:203-222
  quantize_to_int4_packed / dequantize_from_int4_packed   core/quantization.py:30-67,
                                                          core/triton_kernels.py:178-189,218-239
  quantize_to_int2_packed / dequantize_from_int2_packed   core/quantization.py:69-171
  quantize_to_1bit_packed / dequantize_from_1bit_packed   core/quantization.py:173-201,
                                                          core/triton_kernels.py:264-308,334-386
  isolate_outliers                                        core/memory_manager.py:89-113
  page_kv (dequant + COO sidecar scatter of one page)     core/memory_manager.py:1170-1290
  sdpa_f64 (reconstruct-then-SDPA, GQA expanded)          core/memory_manager.py:1424-1430
  jl_projection_matrix / jl_reconstruction_operator       core/memory_manager.py:227-282
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

_u16p = ctypes.POINTER(ctypes.c_uint16)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i8p = ctypes.POINTER(ctypes.c_int8)
_f32p = ctypes.POINTER(ctypes.c_float)
_i64 = ctypes.c_int64
_int = ctypes.c_int
_flt = ctypes.c_float


def build():
    """Compile argus_oracle.c with the Makefile beside it."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO):
            build()
        L = ctypes.CDLL(_SO)
        L.oracle_quant_sym8.argtypes = [_u16p, _i64, _int, _flt, _flt, _flt, _i8p, _u16p]
        L.oracle_dequant_sym8.argtypes = [_i8p, _u16p, _i64, _int, _u16p]
        L.oracle_quant_asym.argtypes = [_u16p, _i64, _int, _int, _int, _u8p, _u16p, _u16p]
        L.oracle_dequant_asym.argtypes = [_u8p, _u16p, _u16p, _i64, _int, _int, _int, _u16p]
        L.oracle_quant_1bit.argtypes = [_u16p, _i64, _int, _int, _u8p, _u16p]
        L.oracle_dequant_1bit.argtypes = [_u8p, _u16p, _i64, _int, _int, _u16p]
        L.oracle_isolate_outliers.argtypes = [_u16p, _i64, _int, _flt, _u16p, _u16p, _u8p]
        L.oracle_f32_to_f16.argtypes = [_f32p, _i64, _u16p]
        L.oracle_torch_mean_abs.argtypes = [_u16p, _int]
        L.oracle_quant_e4m3.argtypes = [_u16p, _i64, _int, _u8p, _u16p]
        L.oracle_dequant_e4m3.argtypes = [_u8p, _u16p, _i64, _int, _u16p]
        L.oracle_e4m3_encode.argtypes = [_f32p, _i64, _u8p]
        L.oracle_torch_mean_abs.restype = ctypes.c_float
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t)


def _h(a):
    """fp16 ndarray -> contiguous uint16 view."""
    a = np.ascontiguousarray(a, dtype=np.float16)
    return a, a.view(np.uint16)


# ------------------------------------------------------------------ symmetric 8-bit
def _quant_sym8(x, div, lo, hi):
    x, xb = _h(x)
    D = x.shape[-1]
    rows = x.size // D
    q = np.empty(x.shape, np.int8)
    s = np.empty(x.shape[:-1] + (1,), np.float16)
    lib().oracle_quant_sym8(_p(xb, _u16p), rows, D, div, lo, hi, _p(q, _i8p), _p(s.view(np.uint16), _u16p))
    return q, s


def quantize_to_int8(x, dim=-1):
    if dim not in (-1, x.ndim - 1):
        q, s = quantize_to_int8(np.moveaxis(x, dim, -1))
        return np.moveaxis(q, -1, dim), np.moveaxis(s, -1, dim)
    return _quant_sym8(x, 127.0, -128.0, 127.0)


def quantize_to_fp8_simulated(x, dim=-1):
    if dim not in (-1, x.ndim - 1):
        q, s = quantize_to_fp8_simulated(np.moveaxis(x, dim, -1))
        return np.moveaxis(q, -1, dim), np.moveaxis(s, -1, dim)
    return _quant_sym8(x, 240.0, -240.0, 240.0)


def dequantize_from_int8(q, s):
    q = np.ascontiguousarray(q, np.int8)
    s = np.ascontiguousarray(np.broadcast_to(s, q.shape[:-1] + (1,)), np.float16)
    D = q.shape[-1]
    out = np.empty(q.shape, np.float16)
    lib().oracle_dequant_sym8(_p(q, _i8p), _p(s.view(np.uint16), _u16p), q.size // D, D,
                              _p(out.view(np.uint16), _u16p))
    return out


dequantize_from_fp8_simulated = dequantize_from_int8


# ------------------------------------------------------------- true e4m3 (non-parity tier)
def quantize_to_e4m3(x):
    """Per-row e4m3 codes (uint8) and fp16 scales (last dim): s = fp16(amax / 448),
    code = e4m3(x / s) rounded to nearest even, saturating at 448, NaN -> 0."""
    x, xb = _h(x)
    D = x.shape[-1]
    q = np.empty(x.shape, np.uint8)
    s = np.empty(x.shape[:-1] + (1,), np.float16)
    lib().oracle_quant_e4m3(_p(xb, _u16p), x.size // D, D, _p(q, _u8p), _p(s.view(np.uint16), _u16p))
    return q, s


def dequantize_from_e4m3(q, s):
    q = np.ascontiguousarray(q, np.uint8)
    s = np.ascontiguousarray(np.broadcast_to(s, q.shape[:-1] + (1,)), np.float16)
    D = q.shape[-1]
    out = np.empty(q.shape, np.float16)
    lib().oracle_dequant_e4m3(_p(q, _u8p), _p(s.view(np.uint16), _u16p), q.size // D, D,
                              _p(out.view(np.uint16), _u16p))
    return out


def e4m3_encode(v):
    """The e4m3 encoder alone on fp32 values (uint8 codes)."""
    v = np.ascontiguousarray(v, np.float32)
    q = np.empty(v.shape, np.uint8)
    lib().oracle_e4m3_encode(_p(v, _f32p), v.size, _p(q, _u8p))
    return q


# ------------------------------------------------------------- sequence-packed codes
def _to_seq_last2(x, seq_dim):
    sd = seq_dim % x.ndim
    assert sd != x.ndim - 1, "packing along the quantization dim is not supported"
    return np.moveaxis(x, sd, -2), sd


def _from_seq_last2(a, sd):
    return np.moveaxis(a, -2, sd)


def _quant_asym(x, bits, seq_dim):
    x, sd = _to_seq_last2(x, seq_dim)
    x, xb = _h(x)
    T, D = x.shape[-2], x.shape[-1]
    per = 8 // bits
    assert T % per == 0, f"Sequence dimension size ({T}) must be a multiple of {per}"
    groups = x.size // (T * D)
    packed = np.empty(x.shape[:-2] + (T // per, D), np.uint8)
    s = np.empty(x.shape[:-1] + (1,), np.float16)
    mn = np.empty(x.shape[:-1] + (1,), np.float16)
    lib().oracle_quant_asym(_p(xb, _u16p), groups, T, D, bits, _p(packed, _u8p),
                            _p(s.view(np.uint16), _u16p), _p(mn.view(np.uint16), _u16p))
    return _from_seq_last2(packed, sd), _from_seq_last2(s, sd), _from_seq_last2(mn, sd)


def _dequant_asym(packed, s, mn, bits, seq_dim):
    packed, sd = _to_seq_last2(packed, seq_dim)
    s = np.moveaxis(s, sd, -2)
    mn = np.moveaxis(mn, sd, -2)
    packed = np.ascontiguousarray(packed, np.uint8)
    per = 8 // bits
    Tp, D = packed.shape[-2], packed.shape[-1]
    T = Tp * per
    s = np.ascontiguousarray(s, np.float16)
    mn = np.ascontiguousarray(mn, np.float16)
    groups = packed.size // (Tp * D)
    out = np.empty(packed.shape[:-2] + (T, D), np.float16)
    lib().oracle_dequant_asym(_p(packed, _u8p), _p(s.view(np.uint16), _u16p), _p(mn.view(np.uint16), _u16p),
                              groups, T, D, bits, _p(out.view(np.uint16), _u16p))
    return _from_seq_last2(out, sd)


def quantize_to_int4_packed(x, seq_dim=-2, quant_dim=-1):
    assert quant_dim in (-1, x.ndim - 1)
    return _quant_asym(x, 4, seq_dim)


def dequantize_from_int4_packed(packed, s, mn, seq_dim=-2):
    return _dequant_asym(packed, s, mn, 4, seq_dim)


def quantize_to_int2_packed(x, seq_dim=-2, quant_dim=-1):
    assert quant_dim in (-1, x.ndim - 1)
    return _quant_asym(x, 2, seq_dim)


def dequantize_from_int2_packed(packed, s, mn, seq_dim=-2):
    return _dequant_asym(packed, s, mn, 2, seq_dim)


def quantize_to_1bit_packed(x, seq_dim=-2, quant_dim=-1):
    assert quant_dim in (-1, x.ndim - 1)
    x, sd = _to_seq_last2(x, seq_dim)
    x, xb = _h(x)
    T, D = x.shape[-2], x.shape[-1]
    assert T % 8 == 0, f"Sequence dimension size ({T}) must be a multiple of 8"
    groups = x.size // (T * D)
    packed = np.empty(x.shape[:-2] + (T // 8, D), np.uint8)
    s = np.empty(x.shape[:-1] + (1,), np.float16)
    lib().oracle_quant_1bit(_p(xb, _u16p), groups, T, D, _p(packed, _u8p), _p(s.view(np.uint16), _u16p))
    return _from_seq_last2(packed, sd), _from_seq_last2(s, sd)


def dequantize_from_1bit_packed(packed, s, seq_dim=-2):
    packed, sd = _to_seq_last2(packed, seq_dim)
    s = np.ascontiguousarray(np.moveaxis(s, sd, -2), np.float16)
    packed = np.ascontiguousarray(packed, np.uint8)
    Tp, D = packed.shape[-2], packed.shape[-1]
    groups = packed.size // (Tp * D)
    out = np.empty(packed.shape[:-2] + (Tp * 8, D), np.float16)
    lib().oracle_dequant_1bit(_p(packed, _u8p), _p(s.view(np.uint16), _u16p), groups, Tp * 8, D,
                              _p(out.view(np.uint16), _u16p))
    return _from_seq_last2(out, sd)


# ------------------------------------------------------------------- outlier filter
def isolate_outliers(x, threshold_sigma=3.0):
    """Returns (normal, outlier_values, mask) as the reference does."""
    x, xb = _h(x)
    D = x.shape[-1]
    normal = np.empty_like(x)
    outv = np.empty_like(x)
    mask = np.empty(x.shape, np.uint8)
    lib().oracle_isolate_outliers(_p(xb, _u16p), x.size // D, D, float(threshold_sigma),
                                  _p(normal.view(np.uint16), _u16p), _p(outv.view(np.uint16), _u16p),
                                  _p(mask, _u8p))
    return normal, outv, mask.astype(bool)


def sidecar(mask, outv):
    """COO sidecar as _demote_active_to_fp8 stores it: int16 (b,h,t,d) rows, fp16 values."""
    idx = np.argwhere(mask).astype(np.int16)
    return idx, outv[mask]


def f32_to_f16(a):
    a = np.ascontiguousarray(a, np.float32)
    out = np.empty(a.shape, np.uint16)
    lib().oracle_f32_to_f16(_p(a, _f32p), a.size, _p(out, _u16p))
    return out.view(np.float16)


# ----------------------------------------------------------------- pages, attention
def page_kv(tier, page, R=None):
    """Dequantize one page dict to fp16 K, V and overwrite its sidecar entries."""
    if tier == "fp16":
        return page["key"], page["value"]
    if tier in ("fp8", "int8"):
        k = dequantize_from_int8(page["key_q"], page["key_scales"])
        v = dequantize_from_int8(page["value_q"], page["value_scales"])
    elif tier == "int4":
        k = dequantize_from_int4_packed(page["key_packed"], page["key_scales"], page["key_min"])
        v = dequantize_from_int4_packed(page["value_packed"], page["value_scales"], page["value_min"])
    elif tier == "int2":
        k = dequantize_from_int2_packed(page["key_packed"], page["key_scales"], page["key_min"])
        v = dequantize_from_int2_packed(page["value_packed"], page["value_scales"], page["value_min"])
    elif tier == "one_bit":
        k = dequantize_from_1bit_packed(page["key_packed"], page["key_scales"])
        v = dequantize_from_1bit_packed(page["value_packed"], page["value_scales"])
    elif tier == "jl":
        k = (R.astype(np.float64) @ page["key_proj"].astype(np.float64)).astype(np.float16)
        v = (R.astype(np.float64) @ page["value_proj"].astype(np.float64)).astype(np.float16)
    else:
        raise ValueError(tier)
    for name, t in (("key", k), ("value", v)):
        idx = page.get(f"{name}_out_indices")
        if idx is not None and len(idx):
            idx = idx.astype(np.int64)
            t[idx[:, 0], idx[:, 1], idx[:, 2], idx[:, 3]] = page[f"{name}_out_values"]
    return k, v


def sdpa_f64(q, k, v, scale):
    """softmax(q K^T * scale) V in float64 with K/V expanded over the GQA group."""
    g = q.shape[1] // k.shape[1]
    k = np.repeat(k.astype(np.float64), g, axis=1)
    v = np.repeat(v.astype(np.float64), g, axis=1)
    w = np.einsum("bhqd,bhkd->bhqk", q.astype(np.float64), k) * scale
    w -= w.max(axis=-1, keepdims=True)
    p = np.exp(w)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, v)


def jl_projection_matrix(page_size, ratio=4, seed=42):
    """W = Q^T of qr(randn(N, M)) drawn on the CPU with the given seed, as fp16 [M, N]
    (memory_manager.py:227-239 with the draw on the CPU device)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    raw = torch.randn(page_size, page_size // ratio, dtype=torch.float32, generator=g)
    qm, _ = torch.linalg.qr(raw)
    return qm.t().to(torch.float16).numpy()


def jl_reconstruction_operator(W, alpha=1e-3):
    """R = A^-1 W^T (W A^-1 W^T)^-1 with A the corner-fixed Laplacian + alpha I, in float64."""
    M, N = W.shape
    L = np.zeros((N, N))
    L[np.arange(N), np.arange(N)] = 2.0
    L[np.arange(N - 1), np.arange(1, N)] = -1.0
    L[np.arange(1, N), np.arange(N - 1)] = -1.0
    L[0, 0] = L[N - 1, N - 1] = 1.0
    A = L + alpha * np.eye(N)
    Wf = W.astype(np.float64)
    Ai = np.linalg.inv(A)
    return Ai @ Wf.T @ np.linalg.inv(Wf @ Ai @ Wf.T)
