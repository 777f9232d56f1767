"""Page-level operations on record arenas (libargus_b200 page codecs and sidecars).

These are the device halves of the tier cascade (core/memory_manager.py:944-1155) and of the page
readers (get_all_keys_values, _resurrect_page, speculate_and_prefetch): quantize an fp16 page into
a tier, move a page one tier down in one fused kernel, dequantize a page into fp16 rows, and build
or apply the COO outlier sidecars.
"""
import ctypes

import torch

from . import _lib
from .attention import ArenaC, KVArena

BOUND_SYMBOLS = ("argus_page_quantize", "argus_page_requant", "argus_page_dequantize", "argus_outlier_blocks_bytes",
                 "argus_outlier_corrections")


def _bind():
    L = _lib.lib()
    if not getattr(L, "_argus_pages_bound", False):
        P = ctypes.POINTER(ArenaC)
        L.argus_page_quantize.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int, P,
                                          ctypes.c_int32, ctypes.c_void_p]
        L.argus_page_requant.argtypes = [P, ctypes.c_int32, P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int,
                                         ctypes.c_void_p]
        L.argus_page_dequantize.argtypes = [P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int, ctypes.c_void_p,
                                            ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
        L.argus_outlier_blocks_bytes.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64]
        L.argus_outlier_corrections.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                                ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                                ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        for f in BOUND_SYMBOLS:
            getattr(L, f).restype = ctypes.c_int
        L.argus_outlier_blocks_bytes.restype = ctypes.c_int64
        L._argus_pages_bound = True
    return L


def _check(name, rc):
    if rc != 0:
        raise _lib.ArgusError(name, rc, _lib.lib().argus_last_error().decode())


def quantize_page(arena: KVArena, slot, k, v):
    """fp16 k, v [B, H, P, D] -> slot of a record arena of any tier."""
    k = k.contiguous()
    v = v.contiguous()
    a = arena.c_struct()
    _check("argus_page_quantize", _bind().argus_page_quantize(
        k.data_ptr(), v.data_ptr(), arena.B * arena.H, arena.D, ctypes.byref(a), slot,
        _lib.stream_handle(k.device)))


def requant_page(src: KVArena, src_slot, dst: KVArena, dst_slot):
    """Fused demotion: page src_slot of src (exact reference dequantization) -> dst tier, slot dst_slot."""
    a, b = src.c_struct(), dst.c_struct()
    _check("argus_page_requant", _bind().argus_page_requant(
        ctypes.byref(a), src_slot, ctypes.byref(b), dst_slot, src.B * src.H, src.D, _lib.stream_handle(src.k.device)))


def dequantize_page(src: KVArena, slot, k_out=None, v_out=None, tok0=0):
    """Page slot of src -> fp16 K, V.  With k_out/v_out ([B, H, L, D], contiguous rows), writes
    tokens tok0 .. tok0+P-1 in place; otherwise returns new [B, H, P, D] tensors."""
    P = src.page_tokens
    if k_out is None:
        k_out = torch.empty(src.B, src.H, P, src.D, dtype=torch.float16, device=src.k.device)
        v_out = torch.empty_like(k_out)
        tok0 = 0
    assert k_out.stride(-1) == 1 and k_out.stride(-2) == src.D and k_out.stride() == v_out.stride()
    assert k_out.stride(0) == k_out.shape[1] * k_out.stride(1)
    a = src.c_struct()
    _check("argus_page_dequantize", _bind().argus_page_dequantize(
        ctypes.byref(a), slot, src.B * src.H, src.D, k_out.data_ptr(), v_out.data_ptr(), k_out.stride(1), tok0,
        _lib.stream_handle(k_out.device)))
    return k_out, v_out


def scatter_coo(out, idx, vals, tok0=0, page_tokens=None):
    """out[b, h, tok0 + t, d] = vals[i] for idx[i] = (b, h, t, d); out is [B, H, L, D] fp16."""
    if idx is None or idx.numel() == 0:
        return out
    B, H, L, D = out.shape
    P = page_tokens if page_tokens is not None else L - tok0
    assert out.stride(-1) == 1 and out.stride(-2) == D and out.stride(0) == H * out.stride(1)
    idx = idx.contiguous()
    vals = vals.contiguous()
    _lib.call("argus_scatter_coo", _lib.ptr(out), out.stride(1), tok0, B, H, P, D, _lib.ptr(idx), _lib.ptr(vals),
              idx.shape[0], _lib.stream_handle(out.device))
    return out


def outliers_to_coo(mask, outv):
    """(torch.nonzero(mask).to(int16), outv[mask]) of a [B, H, P, D] page, computed on the GPU.
    Reads the entry count back to the host (as torch.nonzero does) to size the outputs."""
    B, H, P, D = mask.shape
    dev = mask.device
    count = torch.zeros(1, dtype=torch.int64, device=dev)
    cap = max(1, min(mask.numel(), 4096))
    idx = torch.empty(cap, 4, dtype=torch.int16, device=dev)
    vals = torch.empty(cap, dtype=torch.float16, device=dev)
    m = mask.contiguous().view(torch.uint8)
    o = outv.contiguous()
    st = _lib.stream_handle(dev)
    _lib.call("argus_outliers_to_coo", _lib.ptr(m), _lib.ptr(o), B, H, P, D, _lib.ptr(idx), _lib.ptr(vals), cap,
              _lib.ptr(count), st)
    n = int(count.item())
    if n > cap:
        idx = torch.empty(n, 4, dtype=torch.int16, device=dev)
        vals = torch.empty(n, dtype=torch.float16, device=dev)
        _lib.call("argus_outliers_to_coo", _lib.ptr(m), _lib.ptr(o), B, H, P, D, _lib.ptr(idx), _lib.ptr(vals), n,
                  _lib.ptr(count), st)
    return idx[:n], vals[:n]


def outlier_corrections(arena: KVArena, slot, k_idx, k_val, v_idx, v_val, k_deq=None, v_deq=None):
    """Correction blocks of page `slot` of a quantized record arena from its COO sidecars
    (row-major (b, h, t, d) int16 indices and fp16 values, as outliers_to_coo returns them): returns
    (blocks, block_addr) for KVArena.set_outliers.  k_deq / v_deq: the page dequantized without its
    sidecars ([B, H, P, D] fp16); computed here when not given."""
    if k_deq is None:
        k_deq, v_deq = dequantize_page(arena, slot)
    dev = arena.k.device
    empty_i = torch.zeros(0, 4, dtype=torch.int16, device=dev)
    empty_v = torch.zeros(0, dtype=torch.float16, device=dev)
    k_idx = (k_idx if k_idx is not None else empty_i).contiguous()
    v_idx = (v_idx if v_idx is not None else empty_i).contiguous()
    k_val = (k_val if k_val is not None else empty_v).contiguous().view(torch.float16).reshape(-1)
    v_val = (v_val if v_val is not None else empty_v).contiguous().view(torch.float16).reshape(-1)
    nk, nv = k_idx.shape[0], v_idx.shape[0]
    L = _bind()
    BH = arena.B * arena.H
    nbytes = L.argus_outlier_blocks_bytes(BH, arena.page_tokens, nk, nv)
    blocks = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    addr = torch.empty(BH, dtype=torch.int64, device=dev)
    k_deq, v_deq = k_deq.contiguous(), v_deq.contiguous()
    _check("argus_outlier_corrections", L.argus_outlier_corrections(
        k_idx.data_ptr() if nk else None, k_val.data_ptr() if nk else None, nk,
        v_idx.data_ptr() if nv else None, v_val.data_ptr() if nv else None, nv,
        k_deq.data_ptr(), v_deq.data_ptr(), arena.B, arena.H, arena.page_tokens, arena.D, blocks.data_ptr(),
        addr.data_ptr(), _lib.stream_handle(dev)))
    return blocks, addr


def attach_outliers(arena: KVArena, slot, k_idx, k_val, v_idx, v_val):
    """Builds page `slot`'s correction blocks and points the arena's directory at them."""
    blocks, addr = outlier_corrections(arena, slot, k_idx, k_val, v_idx, v_val)
    arena.set_outliers(slot, blocks, addr)
