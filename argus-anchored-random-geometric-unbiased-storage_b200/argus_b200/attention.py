"""Host side of the fused mixed-tier decode attention (libargus_b200 argus_decode_attention).

KV storage is a set of *arenas* (at most eight per call):
  * record arenas, one per tier pool: a byte buffer [B*H_kv][slots][record] where a record holds
    one page of one (batch, kv_head): [K payload][V payload][K scales][V scales][K mins][V mins].
    Consecutive slots of one (b, h) are contiguous, so a run of small pages is staged into shared
    memory with a single TMA bulk copy.  The reference's page tensors (key_q, key_scales, ...) are
    strided views into the records (KVArena.view);
  * split fp16 arenas: a pair of [B, H_kv, L, D] fp16 tensors (sinks, anchors, the staging buffer).
A *page list* in attention order ((arena, slot, tokens) triples; attention is order-free, so the
list is best given in slot order) becomes an AttentionPlan: chunks of up to 16 tiles of 16 tokens
staged together (~9 KB of compressed data each) and split-K partitions balanced by estimated cost,
sized so the grid fills the GPU in one wave.  A plan is reusable across decode steps while the page
list is unchanged; its launch only reads device pointers, so it can be captured in a CUDA graph.
"""
import ctypes
import math

import numpy as np
import torch

from . import _lib

TIER_FP16, TIER_FP8SIM, TIER_INT8, TIER_INT4, TIER_INT2, TIER_1BIT, TIER_E4M3 = range(7)
LAYOUT_RECORD, LAYOUT_SPLIT_FP16 = 0, 1
# TIER_E4M3 is the true-e4m3 storage mode (codes of OCP FP8 E4M3 with an fp16 scale per token), a
# separately named non-parity tier: the reference's "fp8" tier is the int8-with-wrap simulation.
TIER_NAMES = {"fp16": TIER_FP16, "fp8": TIER_FP8SIM, "int8": TIER_INT8, "int4": TIER_INT4, "int2": TIER_INT2,
              "one_bit": TIER_1BIT, "e4m3": TIER_E4M3}
TIER_BITS = {TIER_FP16: 16, TIER_FP8SIM: 8, TIER_INT8: 8, TIER_INT4: 4, TIER_INT2: 2, TIER_1BIT: 1, TIER_E4M3: 8}
TIER_PER = {TIER_FP16: 1, TIER_FP8SIM: 1, TIER_INT8: 1, TIER_INT4: 2, TIER_INT2: 4, TIER_1BIT: 8, TIER_E4M3: 1}
TIER_PAYLOAD_DTYPE = {TIER_FP16: torch.float16, TIER_FP8SIM: torch.int8, TIER_INT8: torch.int8,
                      TIER_INT4: torch.uint8, TIER_INT2: torch.uint8, TIER_1BIT: torch.uint8,
                      TIER_E4M3: torch.uint8}
MAX_ARENAS = 8
NUM_SMS = 148


def ctas_per_sm(head_dim, sidecars=False):
    """Decode-attention CTAs resident per SM (the kernel's launch bounds and shared memory); launches
    over arenas with outlier sidecars run 3 per SM up to head_dim 128."""
    if head_dim >= 256:
        return 2
    return 3 if sidecars else 4

# C-ABI entry points bound in this module (with structure-typed arguments)
BOUND_SYMBOLS = ("argus_decode_attention", "argus_decode_attention_workspace_size",
                 "argus_decode_attention_chunk_tiles", "argus_record_bytes", "argus_device_status",
                 "argus_decode_attention_noalloc", "argus_decode_attention_noalloc_capacity")


class ArenaC(ctypes.Structure):
    _fields_ = [("tier", ctypes.c_int32), ("layout", ctypes.c_int32), ("k", ctypes.c_void_p),
                ("v", ctypes.c_void_p), ("bh_stride", ctypes.c_int64), ("record_bytes", ctypes.c_int32),
                ("page_tokens", ctypes.c_int32), ("outlier_dir", ctypes.c_void_p), ("dir_slots", ctypes.c_int32),
                ("reserved", ctypes.c_int32), ("slot_live", ctypes.c_void_p)]


class ChunkC(ctypes.Structure):
    _fields_ = [("slot0", ctypes.c_int32), ("tok0", ctypes.c_uint16), ("arena", ctypes.c_uint8),
                ("ntiles", ctypes.c_uint8), ("ntok_last", ctypes.c_uint8), ("reserved", ctypes.c_uint8 * 3)]


class ShapeC(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("heads_kv", ctypes.c_int32), ("group", ctypes.c_int32),
                ("q_len", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("n_splits", ctypes.c_int32),
                ("n_arenas", ctypes.c_int32), ("n_chunks", ctypes.c_int32), ("scale", ctypes.c_float),
                ("flags", ctypes.c_int32)]

ATTN_PRECISE_PV = 1


assert ctypes.sizeof(ChunkC) == 12


def _bind():
    L = _lib.lib()
    if not getattr(L, "_argus_attn_bound", False):
        L.argus_decode_attention.argtypes = [ctypes.POINTER(ShapeC), ctypes.POINTER(ArenaC), ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        L.argus_decode_attention.restype = ctypes.c_int
        L.argus_decode_attention_noalloc.argtypes = [ctypes.POINTER(ShapeC), ctypes.POINTER(ArenaC),
                                                     ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                     ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                     ctypes.c_void_p]
        L.argus_decode_attention_noalloc.restype = ctypes.c_int
        L.argus_decode_attention_noalloc_capacity.argtypes = []
        L.argus_decode_attention_noalloc_capacity.restype = ctypes.c_int64
        L.argus_decode_attention_workspace_size.argtypes = [ctypes.POINTER(ShapeC)]
        L.argus_decode_attention_workspace_size.restype = ctypes.c_int64
        L.argus_decode_attention_chunk_tiles.argtypes = [ctypes.c_int] * 4
        L.argus_decode_attention_chunk_tiles.restype = ctypes.c_int
        L.argus_record_bytes.argtypes = [ctypes.c_int] * 3
        L.argus_record_bytes.restype = ctypes.c_int
        L.argus_device_status.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
        L.argus_device_status.restype = ctypes.c_int
        L._argus_attn_bound = True
    return L


def record_bytes(tier, page_tokens, head_dim):
    return _bind().argus_record_bytes(tier, page_tokens, head_dim)


class KVArena:
    """One storage arena (see the module docstring).  Tensors are kept referenced so their memory
    outlives any plan that points at them."""

    def __init__(self, tier, layout, k, v=None, *, bh_stride, record_bytes=0, page_tokens, head_dim, batch,
                 heads, slots):
        self.tier, self.layout = tier, layout
        self.k, self.v = k, v
        self.bh_stride, self.record_bytes, self.page_tokens = int(bh_stride), int(record_bytes), int(page_tokens)
        self.D, self.B, self.H, self.slots = int(head_dim), int(batch), int(heads), int(slots)
        # outlier sidecars: directory [B*H, slots] of correction-block addresses (0 = none), and
        # the blocks of each slot kept referenced while the directory points at them
        self.outlier_dir = None
        self._outlier_blocks = {}
        # optional device occupancy [slots] uint8 (nonzero = live page), read by the kernel per tile
        self.slot_live = None

    # ---------------------------------------------------------------- record arenas
    @classmethod
    def allocate(cls, tier, batch, heads, slots, page_tokens, head_dim, device="cuda"):
        """A zero-filled record arena for `slots` pages of `page_tokens` tokens."""
        rec = record_bytes(tier, page_tokens, head_dim)
        if rec <= 0 or rec % 16:
            raise ValueError(f"no record layout for tier {tier}, page {page_tokens}, head_dim {head_dim}")
        buf = torch.zeros(batch * heads, slots, rec, dtype=torch.uint8, device=device)
        return cls(tier, LAYOUT_RECORD, buf, None, bh_stride=slots * rec, record_bytes=rec, page_tokens=page_tokens,
                   head_dim=head_dim, batch=batch, heads=heads, slots=slots)

    def _offsets(self):
        P, D, tier = self.page_tokens, self.D, self.tier
        pb = P * D * TIER_BITS[tier] // 8
        return {"k": 0, "v": pb, "ks": 2 * pb, "vs": 2 * pb + 2 * P, "km": 2 * pb + 4 * P, "vm": 2 * pb + 6 * P}

    def view(self, part, slot, n=None):
        """The reference-shaped tensor of one record component for page `slot` ([B, H, rows, D] payload
        or [B, H, P, 1] fp16 scales/mins), or of n consecutive pages with a leading page dim."""
        assert self.layout == LAYOUT_RECORD
        off = self._offsets()[part]
        rec, S, H, B, D, P = self.record_bytes, self.slots, self.H, self.B, self.D, self.page_tokens
        if part in ("k", "v"):
            dt = TIER_PAYLOAD_DTYPE[self.tier]
            es = torch.tensor([], dtype=dt).element_size()
            rows = P // TIER_PER[self.tier]
            base = self.k.view(dt) if es == 1 else self.k.view(torch.float16)
            size, stride = [B, H, rows, D], [H * S * rec // es, S * rec // es, D, 1]
        else:
            es = 2
            base = self.k.view(torch.float16)
            size, stride = [B, H, P, 1], [H * S * rec // 2, S * rec // 2, 1, 1]
        if n is not None:
            size, stride = [n] + size, [rec // es] + stride
        return torch.as_strided(base, size, stride, (slot * rec + off) // es)

    def write_pages(self, slot0, k, v, k_scale=None, v_scale=None, k_min=None, v_min=None):
        """Copies n pages ([n, B, H, rows, D] payloads, [n, B, H, P, 1] scales/mins) into slots
        slot0 .. slot0+n-1."""
        n = k.shape[0]
        self.view("k", slot0, n).copy_(k)
        self.view("v", slot0, n).copy_(v)
        if self.tier != TIER_FP16:
            self.view("ks", slot0, n).copy_(k_scale)
            self.view("vs", slot0, n).copy_(v_scale)
        if self.tier in (TIER_INT4, TIER_INT2):
            self.view("km", slot0, n).copy_(k_min)
            self.view("vm", slot0, n).copy_(v_min)

    # ---------------------------------------------------------------- split fp16 arenas
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
        B, H, L, D = k.shape
        return cls(TIER_FP16, LAYOUT_SPLIT_FP16, k, v, bh_stride=k.stride(1) * 2, page_tokens=16, head_dim=D,
                   batch=B, heads=H, slots=(L + 15) // 16)

    # ---------------------------------------------------------------- outlier sidecars
    def set_outliers(self, slot, blocks, block_addr):
        """Points the directory of page `slot` at its correction blocks (paged.outlier_corrections:
        a uint8 buffer and the [B*H] int64 block addresses), so the fused attention applies the
        page's sidecars while reading it compressed."""
        if self.layout != LAYOUT_RECORD or self.tier == TIER_FP16:
            raise ValueError("outlier sidecars belong to quantized record arenas")
        if self.outlier_dir is None:
            self.outlier_dir = torch.zeros(self.B * self.H, self.slots, dtype=torch.int64, device=self.k.device)
        self.outlier_dir[:, slot].copy_(block_addr)
        self._outlier_blocks[slot] = blocks

    def clear_outliers(self, slot=None):
        """Drops the sidecar corrections of page `slot` (of every page when slot is None)."""
        if self.outlier_dir is None:
            return
        if slot is None:
            self.outlier_dir = None
            self._outlier_blocks.clear()
        else:
            self.outlier_dir[:, slot].zero_()
            self._outlier_blocks.pop(slot, None)

    def c_struct(self):
        d, live = self.outlier_dir, self.slot_live
        return ArenaC(self.tier, self.layout, self.k.data_ptr(), self.v.data_ptr() if self.v is not None else None,
                      self.bh_stride, self.record_bytes, self.page_tokens, d.data_ptr() if d is not None else None,
                      self.slots if d is not None else 0, 0, live.data_ptr() if live is not None else None)


def chunk_capacity(arena, head_dim):
    return _bind().argus_decode_attention_chunk_tiles(arena.tier, arena.layout, arena.page_tokens, head_dim)


# Relative cost of one token of each tier in the fused kernel, measured on B200 with each tier alone
# over a 32K-token Llama-3-8B layer (B 8, 8 KV heads, D 128): a staged tile costs about the same
# whatever its bytes (the low-bit tiers are bound by instruction latency), except fp16, whose
# tiles stream at the HBM rate.
TIER_TOKEN_COST = {TIER_1BIT: 0.69, TIER_INT2: 0.93, TIER_INT4: 0.96, TIER_INT8: 1.06, TIER_FP8SIM: 1.06,
                   TIER_FP16: 2.0, TIER_E4M3: 1.06}

# CUDA graphs AttentionPlan.run_host keeps (one per pair of host buffers and scale).
RUN_HOST_GRAPHS = 4

# The kernel deals a split's chunks to its 4 warps by position: chunk i goes to warp pair i % 2, and
# within the pair to warp (i // 2) % 2.
CTA_WARPS = 4


def _tile_cost(tier, head_dim, ntok):
    """Estimated cost of ntok tokens of one tier, for balancing splits and warps."""
    return float(ntok) * head_dim / 128 * TIER_TOKEN_COST[tier]


def _balance_warps(part, cost):
    """Reorders one split's chunk list so that the kernel's positional dealing (position i to warp
    class i % CTA_WARPS) gives its warps nearly equal costs: the heaviest chunks first, each to the
    lightest class that still has a position free, then each class's chunks in their original
    (arena) order, so every warp still moves through the tiers in the same order."""
    n = len(part)
    cap = [len(range(c, n, CTA_WARPS)) for c in range(CTA_WARPS)]
    load = [0.0] * CTA_WARPS
    members = [[] for _ in range(CTA_WARPS)]
    for k in sorted(range(n), key=lambda k: -cost[part[k]]):
        c = min((c for c in range(CTA_WARPS) if len(members[c]) < cap[c]), key=lambda c: load[c])
        members[c].append(k)
        load[c] += cost[part[k]]
    for m in members:
        m.sort()
    return [part[members[i % CTA_WARPS][i // CTA_WARPS]] for i in range(n)]


def _deal_chunks(chunk_arena, cost, n_splits):
    """Orders the chunks for n_splits split-K slices and returns (order, bounds): slice s runs
    chunks order[bounds[s]:bounds[s+1]].

    Every slice takes a contiguous share of EVERY arena's chunks, and each of its warps meets its
    shares in the same arena order, so all CTAs move through the tiers together and the SMs'
    instruction caches hold one tier's code at a time.  Shares are cut by cost, and the rounding
    error of each cut is carried into the next arena's cut so the slices' total costs stay within
    about one chunk; within a slice the chunks are placed so its warps' costs are balanced
    (_balance_warps)."""
    n = len(cost)
    if n == 0:
        return [], np.zeros(n_splits + 1, np.int32)
    groups = {}
    for i, ai in enumerate(chunk_arena):
        groups.setdefault(ai, []).append(i)
    cuts = []
    carry = np.zeros(n_splits + 1)  # cost placed before each boundary minus its ideal share, so far
    for ai, idx in groups.items():
        cum = np.concatenate([[0.0], np.cumsum([cost[i] for i in idx])])
        ideal = cum[-1] * np.arange(n_splits + 1) / n_splits
        b = np.searchsorted(cum, ideal - carry, side="left")
        b = np.clip(b, 0, len(idx))
        b[0], b[-1] = 0, len(idx)
        b = np.maximum.accumulate(b)
        carry += cum[b] - ideal
        cuts.append((idx, b))
    order, bounds = [], [0]
    for s in range(n_splits):
        part = []
        for idx, b in cuts:
            part += idx[b[s]:b[s + 1]]
        order += _balance_warps(part, cost)
        bounds.append(len(order))
    return order, np.asarray(bounds, np.int32)


class AttentionPlan:
    """Device tables for one page list.

    pages: sequence of (arena_index, slot, n_tokens).  Record pages of <= 16 tokens must be full;
    longer record pages and split-fp16 slots may end short."""

    def __init__(self, arenas, pages, *, batch, heads_kv, group, head_dim, q_len=1, n_splits=None, device=None,
                 precise_pv=False, single_tile=()):
        """single_tile: indices of split fp16 arenas whose 16-token slots each get a chunk of their own,
        so that any slot's token count can be patched later (patch_tokens)."""
        if not 0 < len(arenas) <= MAX_ARENAS:
            raise ValueError(f"1..{MAX_ARENAS} arenas supported")
        self.arenas = list(arenas)
        self.B, self.Hkv, self.G, self.D, self.qlen = int(batch), int(heads_kv), int(group), int(head_dim), int(q_len)
        self.device = device or self.arenas[0].k.device
        caps = [chunk_capacity(a, self.D) for a in self.arenas]
        if min(caps) <= 0:
            raise ValueError(f"head_dim {self.D} is not supported")
        chunks, ccost, srcs = [], [], []  # srcs: per chunk, the index in `pages` of each tile
        cur = None  # open chunk: [slot0, tok0, arena, ntiles, ntok_last, next_slot]
        cur_src = []
        total_tokens = 0

        def close():
            nonlocal cur, cur_src
            if cur is not None:
                chunks.append(tuple(cur[:5]))
                srcs.append(cur_src)
                cur, cur_src = None, []

        for pi, (ai, slot, ntok) in enumerate(pages):
            ntok = int(ntok)
            if ntok <= 0:
                continue
            a = self.arenas[ai]
            total_tokens += ntok
            if a.layout == LAYOUT_RECORD and a.page_tokens <= 16:
                if ntok != a.page_tokens:
                    raise ValueError("record pages of <= 16 tokens must be full")
                if cur is not None and cur[2] == ai and cur[5] == slot and cur[3] < caps[ai]:
                    cur[3] += 1
                    cur[5] += 1
                else:
                    close()
                    cur = [slot, 0, ai, 1, ntok, slot + 1]
                cur_src.append(pi)
            elif a.layout == LAYOUT_RECORD:
                close()
                if a.tier != TIER_FP16 and ntok % 8:
                    raise ValueError("quantized pages hold a multiple of 8 tokens")
                ntiles_page = (ntok + 15) // 16
                for t0 in range(0, ntiles_page, caps[ai]):
                    nt = min(caps[ai], ntiles_page - t0)
                    last = ntok - 16 * (t0 + nt - 1)
                    chunks.append((slot, 16 * t0, ai, nt, min(16, last)))
                    srcs.append([pi] * nt)
            else:  # split fp16: slot = 16-token block
                if ntok > 16:
                    raise ValueError("split fp16 slots hold at most 16 tokens")
                if (cur is not None and cur[2] == ai and cur[5] == slot and cur[3] < caps[ai] and cur[4] == 16
                        and ai not in single_tile):
                    cur[3] += 1
                    cur[4] = ntok
                    cur[5] += 1
                else:
                    close()
                    cur = [slot, 0, ai, 1, ntok, slot + 1]
                cur_src.append(pi)
        close()
        self.n_tokens = total_tokens
        for slot, tok0, ai, nt, last in chunks:
            a = self.arenas[ai]
            toks = 16 * (nt - 1) + last if not (a.layout == LAYOUT_RECORD and a.page_tokens <= 16) else nt * last
            ccost.append(_tile_cost(a.tier, self.D, toks))
        self.n_chunks = len(chunks)
        nqg = (self.G * self.qlen + 7) // 8
        groups = self.B * self.Hkv * nqg
        if n_splits is None:
            # as many splits as fill one wave of CTAs, with at least ~2 chunks per warp
            side = any(a.outlier_dir is not None for a in self.arenas)
            wave = NUM_SMS * ctas_per_sm(self.D, side)
            n_splits = max(1, min(wave // groups, max(1, self.n_chunks // 8)))
            if groups * n_splits < NUM_SMS:
                # too little work for one CTA per SM at 8 chunks each: spread it down to 4 chunks a CTA
                n_splits = max(n_splits, min(wave // groups, max(1, self.n_chunks // 4)))
        n_splits = max(1, min(int(n_splits), max(1, self.n_chunks)))
        self.n_splits = n_splits
        order, bounds = _deal_chunks([c[2] for c in chunks], ccost, n_splits)
        chunks = [chunks[i] for i in order]
        srcs = [srcs[i] for i in order]
        arr = (ChunkC * max(1, len(chunks)))()
        for i, (slot, tok0, ai, nt, last) in enumerate(chunks):
            arr[i] = ChunkC(slot, tok0, ai, nt, last)
        raw = np.frombuffer(bytes(arr), dtype=np.uint8).copy()
        self.chunks_dev = torch.from_numpy(raw).to(self.device)
        self.splits_dev = torch.from_numpy(bounds.astype(np.int32)).to(self.device)
        self._arena_c = (ArenaC * MAX_ARENAS)(*[a.c_struct() for a in self.arenas])
        # the outlier directories the launch reads stay alive with the plan
        self._outlier_dirs = [a.outlier_dir for a in self.arenas]
        self.pages = list(pages)
        self._graphs = {}
        self._shape = ShapeC(self.B, self.Hkv, self.G, self.qlen, self.D, n_splits, len(self.arenas), self.n_chunks,
                             1.0 / math.sqrt(self.D), ATTN_PRECISE_PV if precise_pv else 0)
        ws = _bind().argus_decode_attention_workspace_size(ctypes.byref(self._shape))
        # zero-filled: the split-arrival counters at its front start at zero (launches leave them so)
        self.workspace = torch.zeros(max(ws, 16), dtype=torch.uint8, device=self.device) if ws > 0 else None
        self.chunks = chunks
        self.chunk_pages = srcs  # per chunk (in launch order), the index in `pages` of each of its tiles
        self.compressed_bytes = self._algorithmic_bytes(pages)

    def _algorithmic_bytes(self, pages):
        """Compressed bytes one launch must read: K+V payload and per-token scales/mins over all
        (batch, kv_head) pairs."""
        total = 0
        for ai, slot, n in pages:
            tier = self.arenas[ai].tier
            total += 2 * int(n) * self.D * TIER_BITS[tier] // 8
            if tier != TIER_FP16:
                total += 2 * 2 * int(n) * (2 if tier in (TIER_INT4, TIER_INT2) else 1)
        return total * self.B * self.Hkv

    def refresh_arenas(self):
        """Re-reads the arenas' device pointers (outlier directories, occupancy) into the launch."""
        self._arena_c = (ArenaC * MAX_ARENAS)(*[a.c_struct() for a in self.arenas])
        self._outlier_dirs = [a.outlier_dir for a in self.arenas]

    def patch_tokens(self, chunk, ntok):
        """Sets the token count of a single-tile chunk's tile (1..16) in the device chunk table."""
        slot, tok0, ai, nt, _ = self.chunks[chunk]
        if nt != 1 or not 1 <= ntok <= 16:
            raise ValueError("only single-tile chunks are patched")
        self.chunks[chunk] = (slot, tok0, ai, nt, int(ntok))
        self.chunks_dev[chunk * ctypes.sizeof(ChunkC) + 8] = int(ntok)  # ntok_last: byte 8 of argus_kv_chunk

    def tile_lse_shape(self):
        nqg = (self.G * self.qlen + 7) // 8
        return (self.B * self.Hkv * nqg, max(1, self.n_chunks), 16, 8)

    def run(self, q, scale=None, out=None, lse=None, stream=None, tile_lse=None):
        """q: [B, H_q, q_len, D] fp16 on the plan's device.  Returns out (and fills lse, and the
        per-tile log2-sum-exp tile_lse of shape tile_lse_shape(), if given)."""
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
        rc = L.argus_decode_attention(ctypes.byref(self._shape), self._arena_c, self.chunks_dev.data_ptr(),
                                      self.splits_dev.data_ptr(), q.data_ptr(), out.data_ptr(),
                                      lse.data_ptr() if lse is not None else None,
                                      tile_lse.data_ptr() if tile_lse is not None else None,
                                      self.workspace.data_ptr() if self.workspace is not None else None,
                                      ctypes.c_void_p(st))
        if rc != 0:
            raise _lib.ArgusError("argus_decode_attention", rc, L.argus_last_error().decode())
        return out


    def run_host(self, q_host, out_host, scale=None):
        """One decode step for a host-resident query and output (pinned CPU tensors of q's shape):
        copy q in, run the fused kernel, copy the output back, replayed as one CUDA graph captured on
        the first call for this pair of buffers and this scale (the RUN_HOST_GRAPHS most recently
        used pairs keep theirs).  Returns out_host once the copy-back has been queued on the
        current stream (synchronize before reading it)."""
        key = (q_host.data_ptr(), out_host.data_ptr(), scale)
        entry = self._graphs.pop(key, None)
        if entry is None:
            exp = (self.B, self.Hkv * self.G, self.qlen, self.D)
            if tuple(q_host.shape) != exp or tuple(out_host.shape) != exp:
                raise ValueError(f"host q/out must be {exp}")
            if q_host.dtype != torch.float16 or out_host.dtype != torch.float16:
                raise TypeError("host q/out must be float16")
            if q_host.is_cuda or out_host.is_cuda or not q_host.is_pinned() or not out_host.is_pinned():
                raise ValueError("host q/out must be pinned CPU tensors")
            q_dev = torch.empty(exp, dtype=torch.float16, device=self.device)
            out_dev = torch.empty_like(q_dev)
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                # one launch outside the capture sets the kernel's attributes
                q_dev.copy_(q_host, non_blocking=True)
                self.run(q_dev, scale=scale, out=out_dev)
            side.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side, capture_error_mode="relaxed"):
                q_dev.copy_(q_host, non_blocking=True)
                self.run(q_dev, scale=scale, out=out_dev)
                out_host.copy_(out_dev, non_blocking=True)
            entry = (graph, q_dev, out_dev, q_host, out_host)
            while len(self._graphs) >= RUN_HOST_GRAPHS:
                self._graphs.pop(next(iter(self._graphs)))  # least recently used
        self._graphs[key] = entry  # (re)inserted last: most recently used
        entry[0].replay()
        return out_host


def device_status(stream=None):
    """Reads and clears the status word set by timed-out device waits (0 = ok)."""
    L = _bind()
    v = ctypes.c_int(0)
    st = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    rc = L.argus_device_status(ctypes.byref(v), ctypes.c_void_p(st))
    if rc != 0:
        raise _lib.ArgusError("argus_device_status", rc, L.argus_last_error().decode())
    return v.value

