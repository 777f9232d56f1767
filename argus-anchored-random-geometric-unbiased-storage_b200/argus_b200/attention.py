"""Host side of the fused mixed-tier decode attention (libargus_b200 argus_decode_attention).

A KV cache is described by up to eight *arenas* (a tier pool laid out [slot][B][H_kv][rows][D],
or an fp16 [B][H_kv][L][D] tensor) and a list of *pages* in attention order, each page being
(arena, slot, tokens).  An AttentionPlan turns the page list into the kernel's device tables:
16-token tiles, chunks of tiles staged together (sized per tier so each chunk is ~9 KB of
compressed data) and split-K partitions balanced by an estimated cost.  A plan is reusable
across decode steps while the page list is unchanged; its launch only reads device pointers,
so it can be captured in a CUDA graph.
"""
import ctypes
import math

import numpy as np
import torch

from . import _lib

TIER_FP16, TIER_FP8SIM, TIER_INT8, TIER_INT4, TIER_INT2, TIER_1BIT = range(6)
TIER_NAMES = {"fp16": TIER_FP16, "fp8": TIER_FP8SIM, "int8": TIER_INT8, "int4": TIER_INT4, "int2": TIER_INT2,
              "one_bit": TIER_1BIT}
TIER_BITS = {TIER_FP16: 16, TIER_FP8SIM: 8, TIER_INT8: 8, TIER_INT4: 4, TIER_INT2: 2, TIER_1BIT: 1}
TIER_PER = {TIER_FP16: 1, TIER_FP8SIM: 1, TIER_INT8: 1, TIER_INT4: 2, TIER_INT2: 4, TIER_1BIT: 8}
MAX_ARENAS = 8
NUM_SMS = 148
# C-ABI entry points bound in this module (with structure-typed arguments)
BOUND_SYMBOLS = ("argus_decode_attention", "argus_decode_attention_workspace_size",
                 "argus_decode_attention_chunk_tiles", "argus_device_status")


class ArenaC(ctypes.Structure):
    _fields_ = [("tier", ctypes.c_int32), ("reserved", ctypes.c_int32), ("k", ctypes.c_void_p),
                ("v", ctypes.c_void_p), ("k_scale", ctypes.c_void_p), ("v_scale", ctypes.c_void_p),
                ("k_min", ctypes.c_void_p), ("v_min", ctypes.c_void_p), ("slot_stride", ctypes.c_int64),
                ("bh_stride", ctypes.c_int64), ("scale_slot_stride", ctypes.c_int64),
                ("scale_bh_stride", ctypes.c_int64)]


class ShapeC(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("heads_kv", ctypes.c_int32), ("group", ctypes.c_int32),
                ("q_len", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("n_splits", ctypes.c_int32),
                ("n_arenas", ctypes.c_int32), ("n_chunks", ctypes.c_int32), ("scale", ctypes.c_float),
                ("reserved", ctypes.c_int32)]


def _bind():
    L = _lib.lib()
    if not getattr(L, "_argus_attn_bound", False):
        L.argus_decode_attention.argtypes = [ctypes.POINTER(ShapeC), ctypes.POINTER(ArenaC), ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        L.argus_decode_attention.restype = ctypes.c_int
        L.argus_decode_attention_workspace_size.argtypes = [ctypes.POINTER(ShapeC)]
        L.argus_decode_attention_workspace_size.restype = ctypes.c_int64
        L.argus_decode_attention_chunk_tiles.argtypes = [ctypes.c_int, ctypes.c_int]
        L.argus_decode_attention_chunk_tiles.restype = ctypes.c_int
        L.argus_device_status.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
        L.argus_device_status.restype = ctypes.c_int
        L._argus_attn_bound = True
    return L


class KVArena:
    """One storage arena.  Tensors are kept referenced so their memory outlives the plan."""

    def __init__(self, tier, k, v, k_scale=None, v_scale=None, k_min=None, v_min=None, *, slot_stride,
                 bh_stride, scale_slot_stride=0, scale_bh_stride=0, page_tokens):
        self.tier = tier
        self.k, self.v = k, v
        self.k_scale, self.v_scale, self.k_min, self.v_min = k_scale, v_scale, k_min, v_min
        self.slot_stride, self.bh_stride = int(slot_stride), int(bh_stride)
        self.scale_slot_stride, self.scale_bh_stride = int(scale_slot_stride), int(scale_bh_stride)
        self.page_tokens = int(page_tokens)

    @classmethod
    def from_pools(cls, tier, k, v, k_scale=None, v_scale=None, k_min=None, v_min=None):
        """Pools shaped like the reference's: payload [slots, B, H, rows, D] (rows = P / per),
        scales/mins [slots, B, H, P, 1].  Each slot's [rows, D] block must be contiguous."""
        for t in (k, v):
            _lib.require_cuda(t, "pool")
            if t.stride(-1) != 1 or t.stride(-2) != t.shape[-1]:
                raise ValueError("pool pages must have contiguous [rows, D] blocks")
        es = k.element_size()
        rows = k.shape[-2]
        P = rows * TIER_PER[tier]
        if k.stride() != v.stride():
            raise ValueError("K and V pools must share a layout")
        kw = dict(slot_stride=k.stride(0) * es, bh_stride=k.stride(2) * es, page_tokens=P)
        if k.stride(1) != k.shape[2] * k.stride(2):
            raise ValueError("pool batch/head dims must be contiguous ([B][H] blocks)")
        if tier != TIER_FP16:
            if k_scale.stride() != v_scale.stride() or k_scale.stride(1) != k_scale.shape[2] * k_scale.stride(2):
                raise ValueError("scale pools must share a contiguous [B][H] layout")
            kw.update(scale_slot_stride=k_scale.stride(0), scale_bh_stride=k_scale.stride(2))
        return cls(tier, k, v, k_scale, v_scale, k_min, v_min, **kw)

    @classmethod
    def from_fp16(cls, k, v):
        """An fp16 [B, H, L, D] tensor pair (sinks, anchors, the staging buffer) as an arena whose
        slots are 16-token blocks."""
        _lib.require_cuda(k)
        if k.dtype != torch.float16 or v.dtype != torch.float16:
            raise TypeError("fp16 arenas take float16 tensors")
        if k.stride(-1) != 1 or k.stride(-2) != k.shape[-1] or k.stride() != v.stride():
            raise ValueError("fp16 arena tensors must have contiguous [L, D] rows and equal strides")
        if k.stride(0) != k.shape[1] * k.stride(1):
            raise ValueError("fp16 arena [B][H] blocks must be contiguous")
        D = k.shape[-1]
        return cls(TIER_FP16, k, v, slot_stride=16 * D * 2, bh_stride=k.stride(1) * 2, page_tokens=16)

    def c_struct(self):
        ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
        return ArenaC(self.tier, 0, ptr(self.k), ptr(self.v), ptr(self.k_scale), ptr(self.v_scale), ptr(self.k_min),
                      ptr(self.v_min), self.slot_stride, self.bh_stride, self.scale_slot_stride, self.scale_bh_stride)


def chunk_tiles(tier, head_dim):
    return _bind().argus_decode_attention_chunk_tiles(tier, head_dim)


def _tile_cost(tier, head_dim, ntok):
    """Estimated cost of one tile for split balancing: compressed bytes (K+V, scales) plus a
    per-token term for dequantization and the two contractions."""
    bits = TIER_BITS[tier]
    payload = 2 * ntok * head_dim * bits / 8
    meta = 0 if tier == TIER_FP16 else (2 * 2 * ntok * (2 if tier in (TIER_INT4, TIER_INT2) else 1))
    return payload + meta + 24.0 * ntok * head_dim / 128


class AttentionPlan:
    """Device tables for one page list.

    pages: sequence of (arena_index, slot, n_tokens) in attention order; n_tokens <= the
    arena's page size (partial pages only for fp16 arenas)."""

    def __init__(self, arenas, pages, *, batch, heads_kv, group, head_dim, q_len=1, n_splits=None, device=None):
        if not 0 < len(arenas) <= MAX_ARENAS:
            raise ValueError(f"1..{MAX_ARENAS} arenas supported")
        self.arenas = list(arenas)
        self.B, self.Hkv, self.G, self.D, self.qlen = int(batch), int(heads_kv), int(group), int(head_dim), int(q_len)
        self.device = device or self.arenas[0].k.device
        L = _bind()
        caps = {a.tier: L.argus_decode_attention_chunk_tiles(a.tier, self.D) for a in self.arenas}
        if min(caps.values()) <= 0:
            raise ValueError(f"head_dim {self.D} is not supported")
        # tiles
        tiles, tcost, tarena = [], [], []
        for ai, slot, ntok in pages:
            a = self.arenas[ai]
            if ntok <= 0:
                continue
            if a.tier != TIER_FP16 and ntok % 8:
                raise ValueError("quantized pages hold a multiple of 8 tokens")
            for t0 in range(0, ntok, 16):
                n = min(16, ntok - t0)
                tiles.append((slot, t0, ai, n))
                tcost.append(_tile_cost(a.tier, self.D, n))
                tarena.append(ai)
        self.n_tokens = int(sum(t[3] for t in tiles))
        # chunks: runs of one arena, at most the tier's chunk capacity
        chunks, ccost = [], []
        i = 0
        while i < len(tiles):
            ai = tarena[i]
            cap = caps[self.arenas[ai].tier]
            j = i
            while j < len(tiles) and j - i < cap and tarena[j] == ai:
                j += 1
            chunks.append((i, j - i, ai))
            ccost.append(sum(tcost[i:j]))
            i = j
        self.n_chunks = len(chunks)
        nqg = (self.G * self.qlen + 7) // 8
        groups = self.B * self.Hkv * nqg
        if n_splits is None:
            # about three CTAs per SM in one wave, at least one chunk per warp
            n_splits = max(1, min(math.ceil(3 * NUM_SMS / groups), max(1, self.n_chunks // 4)))
        n_splits = max(1, min(int(n_splits), max(1, self.n_chunks)))
        self.n_splits = n_splits
        # split boundaries at equal cumulative cost
        if self.n_chunks:
            cum = np.concatenate([[0.0], np.cumsum(ccost)])
            targets = cum[-1] * np.arange(n_splits + 1) / n_splits
            bounds = np.searchsorted(cum, targets, side="left").astype(np.int32)
            bounds[0], bounds[-1] = 0, self.n_chunks
            bounds = np.maximum.accumulate(bounds)
        else:
            bounds = np.zeros(n_splits + 1, np.int32)
        # device tables
        t = np.zeros((max(1, len(tiles)), 2), np.int32)
        for k, (slot, t0, ai, n) in enumerate(tiles):
            t[k, 0] = slot
            t[k, 1] = (t0 & 0xFFFF) | (ai << 16) | (n << 24)
        c = np.zeros((max(1, len(chunks)), 2), np.int32)
        for k, (t0, nt, ai) in enumerate(chunks):
            c[k, 0] = t0
            c[k, 1] = nt | (ai << 8)
        self.tiles_dev = torch.from_numpy(t).to(self.device)
        self.chunks_dev = torch.from_numpy(c).to(self.device)
        self.splits_dev = torch.from_numpy(bounds.astype(np.int32)).to(self.device)
        self._arena_c = (ArenaC * MAX_ARENAS)(*[a.c_struct() for a in self.arenas])
        self._shape = ShapeC(self.B, self.Hkv, self.G, self.qlen, self.D, n_splits, len(self.arenas), self.n_chunks,
                             1.0 / math.sqrt(self.D), 0)
        ws = L.argus_decode_attention_workspace_size(ctypes.byref(self._shape))
        self.workspace = torch.empty(max(ws, 16), dtype=torch.uint8, device=self.device) if ws > 0 else None
        self.compressed_bytes = self._algorithmic_bytes(tiles)

    def _algorithmic_bytes(self, tiles):
        """Compressed bytes one launch must read: K+V payload and per-token scales/mins over all
        (batch, kv_head) pairs."""
        total = 0
        for slot, t0, ai, n in tiles:
            tier = self.arenas[ai].tier
            total += 2 * n * self.D * TIER_BITS[tier] // 8
            if tier != TIER_FP16:
                total += 2 * 2 * n * (2 if tier in (TIER_INT4, TIER_INT2) else 1)
        return total * self.B * self.Hkv

    def run(self, q, scale=None, out=None, lse=None, stream=None):
        """q: [B, H_q, q_len, D] fp16 on the plan's device.  Returns out (and fills lse if given)."""
        _lib.require_cuda(q, "q")
        if q.dtype != torch.float16:
            raise TypeError("q must be float16")
        exp = (self.B, self.Hkv * self.G, self.qlen, self.D)
        if tuple(q.shape) != exp:
            raise ValueError(f"q shape {tuple(q.shape)} != {exp}")
        q = q.contiguous()
        if out is None:
            out = torch.empty_like(q)
        self._shape.scale = float(1.0 / math.sqrt(self.D) if scale is None else scale)
        st = stream if stream is not None else torch.cuda.current_stream(q.device).cuda_stream
        L = _bind()
        rc = L.argus_decode_attention(ctypes.byref(self._shape), self._arena_c, self.tiles_dev.data_ptr(),
                                      self.chunks_dev.data_ptr(), self.splits_dev.data_ptr(), q.data_ptr(),
                                      out.data_ptr(), lse.data_ptr() if lse is not None else None,
                                      self.workspace.data_ptr() if self.workspace is not None else None,
                                      ctypes.c_void_p(st))
        if rc != 0:
            raise _lib.ArgusError("argus_decode_attention", rc, L.argus_last_error().decode())
        return out


def device_status(stream=None):
    """Reads and clears the status word set by timed-out device waits (0 = ok)."""
    L = _bind()
    v = ctypes.c_int(0)
    st = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    rc = L.argus_device_status(ctypes.byref(v), ctypes.c_void_p(st))
    if rc != 0:
        raise _lib.ArgusError("argus_device_status", rc, L.argus_last_error().decode())
    return v.value


def smoke_check():
    """One small mixed-tier attention on cuda:0 checked against a float64 reference built from
    the CPU oracle's dequantization of the same pages."""
    import oracle
    from .core import quantization as Q

    torch.manual_seed(0)
    B, Hkv, G, D, P = 1, 2, 4, 128, 16
    dev = "cuda:0"
    kv = {name: (torch.randn(1, B, Hkv, P, D, device=dev).half(), torch.randn(1, B, Hkv, P, D, device=dev).half())
          for name in ("fp16", "int8", "int4", "one_bit")}
    arenas = [KVArena.from_pools(TIER_FP16, kv["fp16"][0], kv["fp16"][1])]
    refs = [(kv["fp16"][0][0].cpu().numpy(), kv["fp16"][1][0].cpu().numpy())]
    for name, tier in (("int8", TIER_INT8), ("int4", TIER_INT4), ("one_bit", TIER_1BIT)):
        k, v = kv[name]
        if tier == TIER_INT8:
            (kq, ks), (vq, vs) = Q.quantize_to_int8(k), Q.quantize_to_int8(v)
            arenas.append(KVArena.from_pools(tier, kq, vq, ks, vs))
            refs.append((oracle.dequantize_from_int8(kq[0].cpu().numpy(), ks[0].cpu().numpy()),
                         oracle.dequantize_from_int8(vq[0].cpu().numpy(), vs[0].cpu().numpy())))
        elif tier == TIER_INT4:
            (kp, ks, km), (vp, vs, vm) = Q.quantize_to_int4_packed(k), Q.quantize_to_int4_packed(v)
            arenas.append(KVArena.from_pools(tier, kp, vp, ks, vs, km, vm))
            refs.append((oracle.dequantize_from_int4_packed(kp[0].cpu().numpy(), ks[0].cpu().numpy(), km[0].cpu().numpy()),
                         oracle.dequantize_from_int4_packed(vp[0].cpu().numpy(), vs[0].cpu().numpy(), vm[0].cpu().numpy())))
        else:
            (kp, ks), (vp, vs) = Q.quantize_to_1bit_packed(k), Q.quantize_to_1bit_packed(v)
            arenas.append(KVArena.from_pools(tier, kp, vp, ks, vs))
            refs.append((oracle.dequantize_from_1bit_packed(kp[0].cpu().numpy(), ks[0].cpu().numpy()),
                         oracle.dequantize_from_1bit_packed(vp[0].cpu().numpy(), vs[0].cpu().numpy())))
    plan = AttentionPlan(arenas, [(i, 0, P) for i in range(len(arenas))], batch=B, heads_kv=Hkv, group=G,
                         head_dim=D, n_splits=2)
    q = torch.randn(B, Hkv * G, 1, D, device=dev).half()
    out = plan.run(q)
    K = np.concatenate([r[0] for r in refs], axis=2)
    V = np.concatenate([r[1] for r in refs], axis=2)
    ref = oracle.sdpa_f64(q.cpu().numpy(), K, V, 1.0 / math.sqrt(D))
    err = np.abs(out.cpu().numpy().astype(np.float64) - ref).max()
    assert err < 2e-3, f"decode attention smoke: max abs err {err}"
    assert device_status() == 0
