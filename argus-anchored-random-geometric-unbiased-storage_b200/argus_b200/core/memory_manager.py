"""Tiered paged KV cache manager with the reference's surface (argus_cache/core/memory_manager.py).

PagedDynamicKVCache keeps the reference's page lists, page-dict schema (key_q / key_packed /
key_proj, key_scales, key_min, key_out_indices, key_out_values, the value_* twins, pool_idx,
page_id, attention_sum, last_step_accessed, entropy, importance_score), policy (importance score,
locality EMA, stride predictor, resurrection) and event trace.  What changes is where the data
lives and what moves it:

  * every tier pool is a record arena (argus_b200.attention.KVArena): one record per (batch,
    kv_head, page) holding K and V payload, scales and mins, so the reference's page tensors are
    strided views into the records;
  * demotions run as single fused kernels (exact dequantization of the old tier, quantization into
    the new one, in place in the arenas) instead of a dozen torch ops per page;
  * inplace_paged_attention runs the fused mixed-tier decode-attention kernel over the compressed
    pages directly (GQA supported), with the per-page attention mass for the importance and
    resurrection policy coming from the same launch;
  * get_all_keys_values, _resurrect_page and speculate_and_prefetch dequantize with the page
    kernels; the prefetch runs on a side stream ordered with an event;
  * swap_out_to_host / swap_in_to_device move whole arenas between HBM and pinned host memory
    with asynchronous copies on a side stream.

Reference lines: ArgusConfig :17-48, argus_log :50-72, calculate_tensor_entropy :74-87,
isolate_outliers :89-113, PagedDynamicKVCache :115-1824 (methods cited below).
Only float16 K/V are supported (the tier codecs are fp16-exact).
"""
import ctypes
import math
import os
import time

import numpy as np
import torch

from .. import _lib
from .. import attention as A
from .. import paged
from . import jl as _jl


class ArgusConfig:
    """Tier budgets, outlier threshold and policy weights (core/memory_manager.py:17-48)."""

    def __init__(self, page_size=4096, max_active_pages=2, max_fp8_pages=2, max_int8_pages=2, max_int4_pages=2,
                 max_int2_pages=2, max_one_bit_pages=2, sink_tokens=4, threshold_sigma=3.0,
                 vram_oom_threshold_ratio=0.85, importance_alpha=0.5, importance_beta=0.3, importance_gamma=0.2,
                 resurrection_threshold=0.01):
        self.page_size = page_size
        self.max_active_pages = max_active_pages
        self.max_fp8_pages = max_fp8_pages
        self.max_int8_pages = max_int8_pages
        self.max_int4_pages = max_int4_pages
        self.max_int2_pages = max_int2_pages
        self.max_one_bit_pages = max_one_bit_pages
        self.sink_tokens = sink_tokens
        self.threshold_sigma = threshold_sigma
        self.vram_oom_threshold_ratio = vram_oom_threshold_ratio
        self.importance_alpha = importance_alpha
        self.importance_beta = importance_beta
        self.importance_gamma = importance_gamma
        self.resurrection_threshold = resurrection_threshold


def argus_log(level, message, file_name="memory_manager.py", line_no=None):
    """Coloured log line; ARGUS_LOG_LEVEL=quiet drops INFO (core/memory_manager.py:50-72)."""
    log_level = os.environ.get("ARGUS_LOG_LEVEL", "research").lower()
    if log_level == "quiet" and level == "INFO":
        return
    from datetime import datetime

    colour = {"INFO": "\033[1;32mINFO\033[0m", "WARNING": "\033[1;33mWARNING\033[0m",
              "ERROR": "\033[1;31mERROR\033[0m"}.get(level, f"\033[1;34m{level}\033[0m")
    where = f":{line_no}" if line_no is not None else ""
    print(f"{colour} {datetime.now().strftime('%m-%d %H:%M:%S')} {file_name}{where}] \033[1;36m[ARGUS]\033[0m {message}")


def calculate_tensor_entropy(tensor):
    """Entropy of |x| normalised to a distribution (core/memory_manager.py:74-87)."""
    if tensor is None or tensor.numel() == 0:
        return 0.0
    a = torch.abs(tensor).to(torch.float32)
    total = a.sum()
    if total == 0:
        return 0.0
    p = torch.clamp(a / total, min=1e-9)
    return -torch.sum(p * torch.log(p)).item()


def isolate_outliers(tensor, threshold_sigma=3.0):
    """NaN/Inf -> 0, then split |x| > fp16(mean|x| * sigma) (per row over the last dim) into an
    outlier tensor; returns (normal_vals, outlier_vals, outlier_mask) like
    core/memory_manager.py:89-113.  Runs as one libargus_b200 kernel."""
    _lib.require_cuda(tensor)
    if tensor.dtype != torch.float16:
        raise TypeError("isolate_outliers takes float16 tensors")
    x = tensor.contiguous()
    D = x.shape[-1]
    n = x.numel() // D if D else 0
    normal = torch.empty_like(x)
    outv = torch.empty_like(x)
    mask = torch.empty(x.shape, dtype=torch.bool, device=x.device)
    _lib.call("argus_isolate_outliers", _lib.ptr(x), n, D, float(threshold_sigma), _lib.ptr(normal),
              _lib.ptr(outv), _lib.ptr(mask), _lib.stream_handle(x.device))
    # sigma <= 0: normal is the cleansed tensor, outv zeros and the mask all False, as in the reference
    return normal, outv, mask


def _causal_sdpa(q, k, v, scale, with_lse=False):
    """Attention of q [B, H_q, q_len, D] over k, v [B, H_kv, L, D] with the bottom-right causal
    mask (query i sees keys j <= L - q_len + i), in fp32; fp16 output and, with with_lse, the
    natural-log LSE [B, H_q, q_len] in fp32."""
    B, Hq, ql, D = q.shape
    Hkv, L = k.shape[1], k.shape[-2]
    G = Hq // Hkv
    qf = q.float().view(B, Hkv, G, ql, D)
    s = torch.einsum("bhgqd,bhkd->bhgqk", qf, k.float()) * scale
    j = torch.arange(L, device=q.device)
    i = torch.arange(ql, device=q.device)
    s = s.masked_fill(j.view(1, -1) > (L - ql + i).view(-1, 1), float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    out = torch.einsum("bhgqk,bhkd->bhgqd", torch.exp(s - lse.unsqueeze(-1)), v.float())
    out = out.reshape(B, Hq, ql, D).half()
    if with_lse:
        return out, lse.reshape(B, Hq, ql).contiguous()
    return out


def _allocated_bytes(dev):
    """torch.cuda.memory_allocated(dev) without flattening the allocator's whole statistics dict
    (that flattening costs ~0.2 ms, and the check runs on every push)."""
    try:
        return int(torch._C._cuda_memoryStats(dev)["allocated_bytes"]["all"]["current"])
    except (AttributeError, KeyError, TypeError):
        return torch.cuda.memory_allocated(dev)


# tier name -> (page list attribute, arena tier, cascade key of the demotion into it)
_TIERS = {
    "fp8": ("fp8_pages", A.TIER_FP8SIM),
    "int8": ("int8_pages", A.TIER_INT8),
    "int4": ("int4_pages", A.TIER_INT4),
    "int2": ("int2_pages", A.TIER_INT2),
    "one_bit": ("one_bit_pages", A.TIER_1BIT),
}
_PAYLOAD_KEY = {"fp8": "q", "int8": "q", "int4": "packed", "int2": "packed", "one_bit": "packed"}
_DEPTH = {"fp8": 1, "int8": 2, "int4": 3, "int2": 4, "one_bit": 5, "jl": 6}


class PagedDynamicKVCache:
    """Seven-tier paged KV cache (core/memory_manager.py:115-1824)."""

    def __init__(self, page_size=4096, max_active_pages=2, max_fp8_pages=2, max_int8_pages=2, max_int4_pages=2,
                 max_int2_pages=2, max_one_bit_pages=2, sink_tokens=4, threshold_sigma=3.0, config=None,
                 fp8_format="simulated"):
        # "simulated": the reference's FP8 tier (int8 codes with wraparound, quantization.py:203-216);
        # "e4m3": true OCP E4M3 codes with an fp16 scale per token, a non-parity storage mode.  Fixed
        # once the pools are allocated (the first push).
        if fp8_format not in ("simulated", "e4m3"):
            raise ValueError("fp8_format must be 'simulated' or 'e4m3'")
        self.fp8_format = fp8_format
        if config is None:
            config = ArgusConfig(page_size=page_size, max_active_pages=max_active_pages, max_fp8_pages=max_fp8_pages,
                                 max_int8_pages=max_int8_pages, max_int4_pages=max_int4_pages,
                                 max_int2_pages=max_int2_pages, max_one_bit_pages=max_one_bit_pages,
                                 sink_tokens=sink_tokens, threshold_sigma=threshold_sigma)
        self.config = config
        self.page_size = config.page_size
        self.max_active_pages = config.max_active_pages
        self.max_fp8_pages = config.max_fp8_pages
        self.max_int8_pages = config.max_int8_pages
        self.max_int4_pages = config.max_int4_pages
        self.max_int2_pages = config.max_int2_pages
        self.max_one_bit_pages = config.max_one_bit_pages
        self.threshold_sigma = config.threshold_sigma
        assert self.page_size % 8 == 0, "Page size must be a multiple of 8 for 1-bit packing."

        self.generation_step = 0
        self._page_counter = 0
        self.event_log = []
        self.sink_tokens = config.sink_tokens
        self.sink_k = self.sink_v = None
        self.anchor_k = self.anchor_v = None
        self.active_pages, self.fp8_pages, self.int8_pages = [], [], []
        self.int4_pages, self.int2_pages, self.one_bit_pages, self.jl_pages = [], [], [], []
        self.w_proj = None
        self._jl_recon_operator = None
        self._pools_allocated = False
        self.prefetch_cache = {}
        self.prefetch_hits = 0
        self.prefetch_misses = 0
        self.prefetch_stream = None
        self._prefetch_event = None
        self.is_swapped_out = False
        self.num_resurrections = 0
        self.num_cpu_spills = 0
        self.total_dequant_time = 0.0
        self.num_dequants = 0
        self.total_demotions = 0
        self.dequant_latencies = []
        self.total_attention_calls = 0
        self.page_lifetimes = {}
        self.total_page_lifetimes = 0
        self.completed_page_lifetimes_count = 0
        self.resurrection_depths = []
        self.cascade_counts = {"fp16_to_fp8": 0, "fp8_to_int8": 0, "int8_to_int4": 0, "int4_to_int2": 0,
                               "int2_to_one_bit": 0, "one_bit_to_jl": 0}
        self.page_access_ema = {}
        self.page_access_history = {}
        self.arenas = {}
        self._host_arenas = {}
        self._plan = None
        self._plan_key = None
        self._plan_base_cache = None
        # occupancy of the pools' slots (see _attention_plan): host mirrors, what changed since the
        # last upload, and how many times the launch tables were built
        self._live_host = {}
        self._live_dirty = False
        self._tiers_dirty = set()
        self._tiers_dirty_all = False
        self._buf_live = None
        self._buf_live_host = None
        self._jl_ops = None
        self.plan_builds = 0
        self.fused_causal_page_steps = 0  # causal steps whose masked tail reached into the active pages
        # attend JL pages without rebuilding them (argus_b200.core.jl.JLAttention) when their shape
        # allows it (128-row blocks, i.e. 512-token pages, head_dim 128, <= 8 queries per kv head)
        self.fused_jl_attention = True
        self._jl_attention = None

    # ------------------------------------------------------------------- JL matrices
    def get_jl_projection_matrix(self, device, dtype):
        """Shared W [P/4, P]: QR of a seed-42 Gaussian drawn on the host (memory_manager.py:227-239)."""
        if self.w_proj is None or self.w_proj.device != torch.device(device) or self.w_proj.dtype != dtype:
            self.w_proj = _jl.projection_matrix(self.page_size, dtype=dtype, device=device)
        return self.w_proj

    def get_jl_reconstruction_operator(self, device, dtype, alpha=1e-3):
        """R = A^-1 W^T (W A^-1 W^T)^-1, built once in fp32 on the host (memory_manager.py:241-282)."""
        op = self._jl_recon_operator
        if op is None or op.device != torch.device(device) or op.dtype != dtype:
            W = self.get_jl_projection_matrix(device, dtype)
            self._jl_recon_operator = _jl.reconstruction_operator_inverse(W, alpha).to(dtype).to(device)
        return self._jl_recon_operator

    def log_event(self, event_type, page_id, **kwargs):
        """Appends to event_log and to ./tests/argus_attention_trace.jsonl (memory_manager.py:285-305)."""
        import json

        event = {"event": event_type, "page_id": page_id, "step": self.generation_step,
                 "timestamp": getattr(self, "generation_step", 0)}
        event.update(kwargs)
        self.event_log.append(event)
        try:
            os.makedirs("tests", exist_ok=True)
            with open("tests/argus_attention_trace.jsonl", "a") as f:
                f.write(json.dumps(event) + "\n")
        except Exception:
            pass

    @property
    def k_buffer(self):
        if not getattr(self, "buffer_length", 0):
            return None
        return self.static_k_buffer[..., :self.buffer_length, :]

    @property
    def v_buffer(self):
        if not getattr(self, "buffer_length", 0):
            return None
        return self.static_v_buffer[..., :self.buffer_length, :]

    # --------------------------------------------------------------------- storage
    def _ensure_pools_allocated(self, keys, values):
        """Record arenas for every tier (the static pools of memory_manager.py:319-381)."""
        B, H, _, D = keys.shape
        dev, dt = keys.device, keys.dtype
        if dt != torch.float16:
            raise TypeError("argus_b200's tier codecs are fp16-exact; K/V must be float16")
        _lib.require_cuda(keys, "keys")
        if (self._pools_allocated and self.static_k_buffer.shape[0] == B and self.static_k_buffer.shape[1] == H
                and self.static_k_buffer.shape[3] == D and self.static_k_buffer.device == dev):
            return
        P = self.page_size
        self.static_k_buffer = torch.zeros(B, H, P * 2, D, device=dev, dtype=dt)
        self.static_v_buffer = torch.zeros(B, H, P * 2, D, device=dev, dtype=dt)
        self.buffer_length = 0
        self.B, self.H, self.D = B, H, D
        self.arenas = {"fp16": A.KVArena.allocate(A.TIER_FP16, B, H, self.max_active_pages, P, D, dev)}
        if self.fp8_format not in ("simulated", "e4m3"):
            raise ValueError("fp8_format must be 'simulated' or 'e4m3'")
        for name, (attr, tier) in _TIERS.items():
            slots = getattr(self, f"max_{attr[:-6]}_pages")
            if name == "fp8" and self.fp8_format == "e4m3":
                tier = A.TIER_E4M3
            self.arenas[name] = A.KVArena.allocate(tier, B, H, max(1, slots), P, D, dev)
        # per pool: which slots hold live pages (host mirror, device array read by the kernel)
        self._live_host = {}
        for name, a in self.arenas.items():
            self._live_host[name] = np.zeros(a.slots, np.uint8)
            a.slot_live = torch.zeros(a.slots, dtype=torch.uint8, device=dev)
        self._pools_allocated = True
        self._invalidate()

    @property
    def active_pool_k(self):
        return self.arenas["fp16"].view("k", 0, self.max_active_pages)

    @property
    def active_pool_v(self):
        return self.arenas["fp16"].view("v", 0, self.max_active_pages)

    def _invalidate(self):
        self._plan = None
        self._plan_key = None
        self._plan_base_cache = None

    def _page_views(self, name, idx):
        """The reference-schema tensors of slot idx of tier `name` (views into the record arena)."""
        a = self.arenas[name]
        if name == "fp16":
            return {"key": a.view("k", idx), "value": a.view("v", idx)}
        pk = _PAYLOAD_KEY[name]
        d = {f"key_{pk}": a.view("k", idx), f"value_{pk}": a.view("v", idx), "key_scales": a.view("ks", idx),
             "value_scales": a.view("vs", idx)}
        if name in ("int4", "int2"):
            d["key_min"] = a.view("km", idx)
            d["value_min"] = a.view("vm", idx)
        return d

    # --------------------------------------------------------------------- ingest
    def push_new_tokens(self, keys, values, is_anchor=None):
        """Anchors, attention sinks, staging buffer, page formation and the tier cascade
        (memory_manager.py:383-489)."""
        self._check_and_prevent_oom()
        if is_anchor is not None:
            seq_len = keys.shape[-2]
            if is_anchor.dim() > 1:
                is_anchor = is_anchor.view(-1)
            if is_anchor.shape[0] != seq_len:
                is_anchor = is_anchor[:seq_len]
                if is_anchor.shape[0] < seq_len:
                    pad = torch.zeros(seq_len - is_anchor.shape[0], dtype=torch.bool, device=keys.device)
                    is_anchor = torch.cat([is_anchor, pad])
            anchor_idx = torch.where(is_anchor)[0]
            if len(anchor_idx) > 0:
                ak, av = keys[..., anchor_idx, :], values[..., anchor_idx, :]
                if self.anchor_k is None:
                    self.anchor_k, self.anchor_v = ak.clone(), av.clone()
                else:
                    self.anchor_k = torch.cat([self.anchor_k, ak], dim=-2)
                    self.anchor_v = torch.cat([self.anchor_v, av], dim=-2)
                keep = torch.where(~is_anchor)[0]
                keys, values = keys[..., keep, :], values[..., keep, :]
                self._invalidate()
                if keys.shape[-2] == 0:
                    return
        if self.sink_k is None and self.sink_tokens > 0:
            if keys.shape[-2] >= self.sink_tokens:
                self.sink_k = keys[..., :self.sink_tokens, :].clone()
                self.sink_v = values[..., :self.sink_tokens, :].clone()
                keys, values = keys[..., self.sink_tokens:, :], values[..., self.sink_tokens:, :]
            else:
                self.sink_k, self.sink_v = keys.clone(), values.clone()
                self._invalidate()
                return
        self._ensure_pools_allocated(keys, values)
        num_new = keys.shape[-2]
        if self.buffer_length + num_new > self.static_k_buffer.shape[-2]:
            new_size = max(self.static_k_buffer.shape[-2] * 2, self.buffer_length + num_new)
            B, H, _, D = keys.shape
            grow = new_size - self.static_k_buffer.shape[-2]
            z = torch.zeros(B, H, grow, D, device=keys.device, dtype=keys.dtype)
            self.static_k_buffer = torch.cat([self.static_k_buffer, z], dim=-2)
            self.static_v_buffer = torch.cat([self.static_v_buffer, z.clone()], dim=-2)
        self.static_k_buffer[..., self.buffer_length:self.buffer_length + num_new, :].copy_(keys)
        self.static_v_buffer[..., self.buffer_length:self.buffer_length + num_new, :].copy_(values)
        self.buffer_length += num_new
        # the attention plan reads the static buffer in place and tracks buffer_length itself
        P = self.page_size
        while self.buffer_length >= P:
            if len(self.active_pages) >= self.max_active_pages:
                self.manage_memory_lifecycle()
            idx = self._get_free_pool_idx(self.active_pages, self.max_active_pages)
            self._slot("fp16", idx, True)
            self.arenas["fp16"].view("k", idx).copy_(self.static_k_buffer[..., :P, :])
            self.arenas["fp16"].view("v", idx).copy_(self.static_v_buffer[..., :P, :])
            remaining = self.buffer_length - P
            if remaining > 0:
                self.static_k_buffer[..., :remaining, :].copy_(self.static_k_buffer[..., P:P + remaining, :].clone())
                self.static_v_buffer[..., :remaining, :].copy_(self.static_v_buffer[..., P:P + remaining, :].clone())
            self.buffer_length = remaining
            self._page_counter += 1
            views = self._page_views("fp16", idx)
            ent = calculate_tensor_entropy(views["key"])
            page = {"page_id": self._page_counter, "key": views["key"], "value": views["value"], "pool_idx": idx,
                    "attention_sum": 0.0, "last_step_accessed": self.generation_step, "entropy": ent,
                    "importance_score": 0.0}
            self._calculate_importance(page)
            self.active_pages.append(page)
            self.log_event("create", page["page_id"])
            self.page_lifetimes[page["page_id"]] = self.generation_step
            argus_log("INFO", f"Allocated Page {page['page_id']} (FP16) | Pool Slot: {idx} | Entropy: {ent:.4f}",
                      line_no=400)

    # --------------------------------------------------------------------- policy
    def _calculate_importance(self, page):
        """alpha*attention + beta*recency + gamma*entropy*factor + 0.5*EMA + stride bonus
        (memory_manager.py:491-539)."""
        cfg = self.config
        attention_sum = page.get("attention_sum", 0.0)
        last_step = page.get("last_step_accessed", 0)
        recency = 1.0 / (1.0 + float(self.generation_step - last_step))
        entropy = page.get("entropy", 0.0)
        page_id = page.get("page_id")
        accessed_now = 1.0 if self.generation_step == last_step else 0.0
        ema = 0.15 * accessed_now + 0.85 * self.page_access_ema.get(page_id, 0.0)
        self.page_access_ema[page_id] = ema
        hist = self.page_access_history.setdefault(page_id, [])
        if accessed_now > 0.0 and (not hist or hist[-1] != self.generation_step):
            hist.append(self.generation_step)
            if len(hist) > 5:
                hist.pop(0)
        stride_bonus = 0.0
        if len(hist) >= 3:
            strides = [hist[i] - hist[i - 1] for i in range(1, len(hist))]
            if len(set(strides)) == 1 and abs(hist[-1] + strides[0] - self.generation_step) <= 2:
                stride_bonus = 0.8
        factor = 1.3 if entropy > 10.0 else (0.6 if entropy < 5.0 else 1.0)
        score = (cfg.importance_alpha * attention_sum + cfg.importance_beta * recency
                 + cfg.importance_gamma * (entropy * factor)) + 0.5 * ema + stride_bonus
        page["importance_score"] = score
        return score

    def _get_free_pool_idx(self, pages_list, max_pages):
        used = {p["pool_idx"] for p in pages_list if "pool_idx" in p}
        for idx in range(max_pages):
            if idx not in used:
                return idx
        return 0

    def _check_and_prevent_oom(self):
        """Spill every compressed tier to host memory above the VRAM threshold (memory_manager.py:548-564)."""
        if torch.cuda.is_available():
            dev = torch.cuda.current_device()
            total = torch.cuda.get_device_properties(dev).total_memory
            alloc = _allocated_bytes(dev)
            ratio = float(alloc) / float(total)
            if ratio >= self.config.vram_oom_threshold_ratio:
                self.num_cpu_spills += 1
                argus_log("WARNING", f"VRAM pressure detected (allocated: {alloc / 1024 ** 3:.2f}GB / "
                          f"{total / 1024 ** 3:.2f}GB, ratio: {ratio * 100:.1f}%) -> spilling cold pages to CPU Host "
                          "RAM", line_no=431)
                self.swap_out_to_host()
        elif self.config.vram_oom_threshold_ratio <= 0.0:
            self.num_cpu_spills += 1
            self.swap_out_to_host()

    # --------------------------------------------------------------------- cascade
    def manage_memory_lifecycle(self):
        """Demote the least important active page (memory_manager.py:919-943)."""
        if len(self.active_pages) >= self.max_active_pages:
            self.active_pages.sort(key=lambda p: p.get("importance_score", 0.0))
            page = self.active_pages.pop(0)
            self._demote_active_to_fp8(page)
            if self.active_pages:
                keep = self.active_pages[-1]
                att = keep.get("attention_sum", 0.0)
                ent = keep.get("entropy", 0.0)
                rec = 1.0 / (1.0 + float(self.generation_step - keep.get("last_step_accessed", 0)))
                if att >= rec and att >= ent:
                    reason = "high attention recurrence"
                elif rec >= att and rec >= ent:
                    reason = "high recency bias"
                else:
                    reason = "high outlier magnitude"
                argus_log("INFO", f"Page {keep.get('page_id')} preserved in FP16 | Reason: {reason} "
                          f"(importance={keep.get('importance_score', 0.0):.2f})", line_no=734)

    def _carry(self, old):
        return {"page_id": old.get("page_id"), "attention_sum": old.get("attention_sum", 0.0),
                "last_step_accessed": old.get("last_step_accessed", self.generation_step),
                "entropy": old.get("entropy", 0.0), "importance_score": old.get("importance_score", 0.0)}

    def _demote_active_to_fp8(self, page):
        """Outlier isolation + simulated-FP8 quantization of an active page (memory_manager.py:944-987)."""
        self._slot("fp16", page["pool_idx"], False)
        k = page["key"].contiguous()
        v = page["value"].contiguous()
        k_norm, k_out, k_mask = isolate_outliers(k, self.threshold_sigma)
        v_norm, v_out, v_mask = isolate_outliers(v, self.threshold_sigma)
        k_idx, k_vals = paged.outliers_to_coo(k_mask, k_out)
        v_idx, v_vals = paged.outliers_to_coo(v_mask, v_out)
        if len(self.fp8_pages) >= self.max_fp8_pages:
            self.fp8_pages.sort(key=lambda p: p.get("importance_score", 0.0))
            self._demote_fp8_to_int8(self.fp8_pages.pop(0))
        idx = self._get_free_pool_idx(self.fp8_pages, self.max_fp8_pages)
        self._slot("fp8", idx, True)
        paged.quantize_page(self.arenas["fp8"], idx, k_norm, v_norm)
        entry = self._page_views("fp8", idx)
        entry.update({"key_out_indices": k_idx, "key_out_values": k_vals, "value_out_indices": v_idx,
                      "value_out_values": v_vals, "pool_idx": idx})
        entry.update(self._carry(page))
        entry["last_step_accessed"] = page.get("last_step_accessed", self.generation_step)
        self.fp8_pages.append(entry)
        self.log_event("demote", page.get("page_id"), tier_from="active", tier_to="fp8")
        self.total_demotions += 1
        self.cascade_counts["fp16_to_fp8"] += 1
        pid = page.get("page_id")
        if pid in self.page_lifetimes:
            self.total_page_lifetimes += self.generation_step - self.page_lifetimes.pop(pid)
            self.completed_page_lifetimes_count += 1
        argus_log("INFO", f"Demoting Page {pid} (FP16 -> FP8) | Reason: low attention prominence "
                  f"(importance={page.get('importance_score', 0.0):.2f})", line_no=800)

    def _demote_down(self, old, src, dst, next_demote, cascade_key, line_no):
        """Shared body of the FP8->INT8, INT8->INT4, INT4->INT2 and INT2->1-bit demotions
        (memory_manager.py:989-1123): make room in `dst` (recursively), then one fused kernel
        re-quantizes the page in place.  The V sidecar carries the K sidecar, as in the reference."""
        self._slot(src, old["pool_idx"], False)
        dst_attr = _TIERS[dst][0]
        lst = getattr(self, dst_attr)
        limit = getattr(self, f"max_{dst_attr[:-6]}_pages")
        if len(lst) >= limit:
            lst.sort(key=lambda p: p.get("importance_score", 0.0))
            next_demote(lst.pop(0))
        idx = self._get_free_pool_idx(lst, limit)
        self._slot(dst, idx, True)
        paged.requant_page(self.arenas[src], old["pool_idx"], self.arenas[dst], idx)
        entry = self._page_views(dst, idx)
        entry.update({"key_out_indices": old["key_out_indices"], "key_out_values": old["key_out_values"],
                      "value_out_indices": old["key_out_indices"], "value_out_values": old["key_out_values"],
                      "pool_idx": idx})
        entry.update(self._carry(old))
        lst.append(entry)
        self.log_event("demote", old.get("page_id"), tier_from=src, tier_to=dst)
        self.total_demotions += 1
        self.cascade_counts[cascade_key] += 1
        names = {"fp8": "FP8", "int8": "INT8", "int4": "INT4", "int2": "INT2", "one_bit": "1-Bit"}
        argus_log("INFO", f"Demoting Page {old.get('page_id')} ({names[src]} -> {names[dst]}) | Reason: cascading "
                  "compression cascade", line_no=line_no)

    def _demote_fp8_to_int8(self, old):
        self._demote_down(old, "fp8", "int8", self._demote_int8_to_int4, "fp8_to_int8", 830)

    def _demote_int8_to_int4(self, old):
        self._demote_down(old, "int8", "int4", self._demote_int4_to_int2, "int8_to_int4", 862)

    def _demote_int4_to_int2(self, old):
        self._demote_down(old, "int4", "int2", self._demote_int2_to_one_bit, "int4_to_int2", 894)

    def _demote_int2_to_one_bit(self, old):
        self._demote_down(old, "int2", "one_bit", self._demote_one_bit_to_jl, "int2_to_one_bit", 924)

    def _dequant_with_sidecars(self, name, page):
        """fp16 K, V of a page of tier `name` with its sidecars applied (new tensors)."""
        if name == "jl":
            R = self.get_jl_reconstruction_operator(page["key_proj"].device, page["key_proj"].dtype)
            return _jl.apply_left(R, page["key_proj"]), _jl.apply_left(R, page["value_proj"])
        k, v = paged.dequantize_page(self.arenas[name], page["pool_idx"])
        paged.scatter_coo(k, page.get("key_out_indices"), page.get("key_out_values"))
        paged.scatter_coo(v, page.get("value_out_indices"), page.get("value_out_values"))
        return k, v

    def _demote_one_bit_to_jl(self, old):
        """1-bit page -> fp16 (sidecars applied) -> sequence projection W @ X (memory_manager.py:1125-1155)."""
        self._slot("one_bit", old["pool_idx"], False)
        k_full, v_full = self._dequant_with_sidecars("one_bit", old)
        W = self.get_jl_projection_matrix(k_full.device, k_full.dtype)
        entry = {"key_proj": _jl.apply_left(W, k_full), "value_proj": _jl.apply_left(W, v_full)}
        entry.update(self._carry(old))
        self.jl_pages.append(entry)
        self.log_event("demote", old.get("page_id"), tier_from="one_bit", tier_to="jl")
        self.total_demotions += 1
        self.cascade_counts["one_bit_to_jl"] += 1
        argus_log("INFO", f"Demoting Page {old.get('page_id')} (1-Bit -> JL-Projection) | Reason: cascading "
                  "compression cascade", line_no=954)

    def _resurrect_page(self, page, tier):
        """Dequantize a compressed page back into the FP16 active pool (memory_manager.py:832-917)."""
        t0 = time.perf_counter()
        if tier not in _TIERS and tier != "jl":
            return
        k, v = self._dequant_with_sidecars(tier, page)
        attr = "jl_pages" if tier == "jl" else _TIERS[tier][0]
        # a page listed for resurrection may have been moved by an earlier resurrection's cascade in the
        # same call (the reference resurrects it anyway); its old slot then holds another page
        if tier in _TIERS and any(p is page for p in getattr(self, attr)):
            self._slot(tier, page["pool_idx"], False)
        setattr(self, attr, [p for p in getattr(self, attr) if p is not page])
        dt = (time.perf_counter() - t0) * 1000
        self.total_dequant_time += dt
        self.num_dequants += 1
        self.num_resurrections += 1
        self.dequant_latencies.append(dt)
        self.resurrection_depths.append(_DEPTH.get(tier, 1))
        self.page_lifetimes[page.get("page_id")] = self.generation_step
        rec = 1.0 / (1.0 + float(self.generation_step - page.get("last_step_accessed", 0)))
        reason = "high attention recurrence" if page.get("attention_sum", 0.0) >= rec else "high recency bias"
        argus_log("INFO", f"Page {page.get('page_id')} resurrected (importance={page.get('importance_score', 0.0):.2f})"
                  f" | Tier: {tier.upper()} -> FP16 Transient | Reason: {reason} | Dequant Latency: {dt:.3f}ms",
                  line_no=700)
        if len(self.active_pages) >= self.max_active_pages:
            self.active_pages.sort(key=lambda x: x.get("importance_score", 0.0))
            self._demote_active_to_fp8(self.active_pages.pop(0))
        idx = self._get_free_pool_idx(self.active_pages, self.max_active_pages)
        self._slot("fp16", idx, True)
        self.arenas["fp16"].view("k", idx).copy_(k)
        self.arenas["fp16"].view("v", idx).copy_(v)
        views = self._page_views("fp16", idx)
        entry = {"page_id": page.get("page_id"), "key": views["key"], "value": views["value"], "pool_idx": idx,
                 "attention_sum": page.get("attention_sum", 0.0), "last_step_accessed": self.generation_step,
                 "entropy": page.get("entropy", 0.0), "importance_score": page.get("importance_score", 0.0)}
        self._calculate_importance(entry)
        self.active_pages.append(entry)
        self.log_event("resurrect", entry["page_id"], tier=tier)

    # --------------------------------------------------------------------- readers
    def _compressed_order(self):
        return [("jl", self.jl_pages), ("one_bit", self.one_bit_pages), ("int2", self.int2_pages),
                ("int4", self.int4_pages), ("int8", self.int8_pages), ("fp8", self.fp8_pages)]

    def _wait_prefetch(self):
        if self._prefetch_event is not None:
            torch.cuda.current_stream().wait_event(self._prefetch_event)

    def get_all_keys_values(self):
        """Every tier rebuilt to fp16 and concatenated: sinks, anchors, JL, 1-bit, INT2, INT4, INT8,
        FP8, active pages, staging buffer (memory_manager.py:1157-1315)."""
        if self.is_swapped_out:
            self.swap_in_to_device()
        parts = []
        for name, lst in self._compressed_order():
            for page in lst:
                if id(page) in self.prefetch_cache:
                    self._wait_prefetch()
                    parts.append(("tensor", self.prefetch_cache[id(page)]))
                    self.prefetch_hits += 1
                else:
                    self.prefetch_misses += 1
                    parts.append((name, page))
        for page in self.active_pages:
            parts.append(("tensor", (page["key"], page["value"])))
        if self.k_buffer is not None and self.k_buffer.shape[-2] > 0:
            parts.append(("tensor", (self.k_buffer, self.v_buffer)))
        head = []
        if self.sink_k is not None:
            head.append(("tensor", (self.sink_k, self.sink_v)))
        if self.anchor_k is not None:
            head.append(("tensor", (self.anchor_k, self.anchor_v)))
        parts = head + parts
        if not parts:
            return None, None
        ref = next(x[1][0] if x[0] == "tensor" else None for x in parts)
        ref = ref if ref is not None else self.static_k_buffer
        B, H, D = ref.shape[0], ref.shape[1], ref.shape[-1]
        P = self.page_size
        lengths = [x[1][0].shape[-2] if x[0] == "tensor" else P for x in parts]
        L = sum(lengths)
        K = torch.empty(B, H, L, D, dtype=torch.float16, device=ref.device)
        V = torch.empty_like(K)
        off = 0
        for (kind, item), n in zip(parts, lengths):
            if kind == "tensor":
                K[:, :, off:off + n].copy_(item[0])
                V[:, :, off:off + n].copy_(item[1])
            elif kind == "jl":
                k, v = self._dequant_with_sidecars("jl", item)
                K[:, :, off:off + n].copy_(k)
                V[:, :, off:off + n].copy_(v)
            else:
                paged.dequantize_page(self.arenas[kind], item["pool_idx"], K, V, tok0=off)
                paged.scatter_coo(K, item.get("key_out_indices"), item.get("key_out_values"), tok0=off, page_tokens=P)
                paged.scatter_coo(V, item.get("value_out_indices"), item.get("value_out_values"), tok0=off,
                                  page_tokens=P)
            off += n
        return K, V

    def _attention_plan(self, q, tail=0):
        """Fused-kernel tables for the current cache, kept current at the cache's mutation points
        rather than rebuilt.  The chunk list covers every slot of the FP16 pool and of each tier's
        pool, and every 16-token block of the staging buffer's capacity (one chunk per block); which
        slots hold live pages is a per-arena device occupancy array (argus_kv_arena.slot_live) that
        page moves update a byte at a time (_slot), and the buffer's last live block gets its token
        count patched in the chunk table.  So a decode step across a page formation, a demotion or a
        resurrection uploads a few bytes and rebuilds nothing; the tables are rebuilt only when the
        cache's structure changes: the pools or the staging buffer are reallocated (first push, swap,
        buffer growth), the sinks or anchors change, or JL pages come or go.  The newest `tail`
        tokens of the staging buffer are left out (a causal step attends to them separately)."""
        B, Hq, qlen, D = q.shape
        nbuf = max(0, self.buffer_length - tail) if self.k_buffer is not None else 0
        cap = self.static_k_buffer.shape[-2] if self._pools_allocated else 0
        fused_jl = self._fused_jl(q)
        base_key = (B, Hq, qlen, D, tuple((n, a.slots) for n, a in self.arenas.items()) if self._pools_allocated else (),
                    self._scratch_version(fused_jl), fused_jl)
        key = (base_key, self.static_k_buffer.data_ptr() if cap else 0, cap)
        plan = self._plan
        if plan is None or self._plan_key != key:
            plan = self._build_plan(q, base_key, cap, fused_jl)
            self._plan, self._plan_key = plan, key
            self.plan_builds += 1
        self._sync_live(plan)
        self._sync_buffer(plan, nbuf)
        plan.jl = self._jl_operands(q) if fused_jl else None
        return plan

    def _fused_jl(self, q):
        """Whether JL pages are attended by the fused JL kernel (64- or 128-row blocks, i.e. 256- or
        512-token pages at the projection ratio 4, head_dim 64 or 128, <= 8 queries per kv head)
        rather than rebuilt into the scratch arena."""
        B, Hq, qlen, D = q.shape
        if not (self.fused_jl_attention and self.jl_pages) or self.page_size not in (256, 512) or D not in (64, 128):
            return False
        Hkv = self.H if self._pools_allocated else self.sink_k.shape[1]
        return (Hq // Hkv) * qlen <= 8 and self._pools_allocated

    def _jl_operands(self, q):
        """The fused JL kernel's operands (stacked Yk / Yv of the JL pages), rebuilt only when the JL
        pages change."""
        key = tuple(id(p) for p in self.jl_pages)
        if self._jl_ops is None or self._jl_ops[0] != key:
            R = self.get_jl_reconstruction_operator(q.device, torch.float16)
            if self._jl_attention is None or self._jl_attention[0] is not R:
                self._jl_attention = (R, _jl.JLAttention(R))
            ops = {"att": self._jl_attention[1], "pages": list(self.jl_pages),
                   "yk": torch.stack([pg["key_proj"] for pg in self.jl_pages], dim=2).contiguous(),
                   "yv": torch.stack([pg["value_proj"] for pg in self.jl_pages], dim=2).contiguous()}
            self._jl_ops = (key, ops)
        return self._jl_ops[1]

    def _build_plan(self, q, base_key, cap, fused_jl):
        B, Hq, qlen, D = q.shape
        base = self._plan_base(q, base_key, fused_jl)
        arenas, pages, page_seg = list(base["arenas"]), list(base["pages"]), list(base["page_seg"])
        segments = list(base["order"])
        buf_ai = -1
        nblk = (cap + 15) // 16
        if cap:
            buf_ai = len(arenas)
            buf = A.KVArena.from_fp16(self.static_k_buffer, self.static_v_buffer)
            self._buf_live = torch.zeros(nblk, dtype=torch.uint8, device=q.device)
            self._buf_live_host = np.zeros(nblk, np.uint8)
            buf.slot_live = self._buf_live
            arenas.append(buf)
            seg = len(segments)
            segments.append(("buffer", None, 0))
            for b in range(nblk):
                pages.append((buf_ai, b, min(16, cap - 16 * b)))
                page_seg.append(seg)
        Hkv = base["Hkv"]
        # attention is order-free: give each arena's pages in slot order so runs merge into chunks
        perm = sorted(range(len(pages)), key=lambda i: (pages[i][0], pages[i][1]))
        plan = A.AttentionPlan(arenas, [pages[i] for i in perm], batch=B, heads_kv=Hkv, group=Hq // Hkv,
                               head_dim=D, q_len=qlen, single_tile=(buf_ai,) if cap else ())
        # map (chunk, tile) of the launch -> segment
        cmap = torch.full((max(1, plan.n_chunks), 16), -1, dtype=torch.long)
        for c, src in enumerate(plan.chunk_pages):
            for i, pi in enumerate(src):
                cmap[c, i] = page_seg[perm[pi]]
        plan.tile_segment = cmap.to(q.device)
        plan.segments = segments
        plan.buf_ai = buf_ai
        # chunk of each buffer block, and the token count each block's chunk holds now
        plan.buffer_chunks = [-1] * nblk
        plan.buffer_ntok = [0] * nblk
        for c, (slot, _, ai, nt, last) in enumerate(plan.chunks):
            if ai == buf_ai:
                plan.buffer_chunks[slot] = c
                plan.buffer_ntok[slot] = last
        plan.buffer_tokens = -1
        self._live_dirty = True  # a fresh plan reads the occupancy of every arena
        return plan

    def _sync_buffer(self, plan, nbuf):
        """The staging buffer holds nbuf tokens: blocks below ceil(nbuf/16) live, the last one patched
        to its token count (a byte of the device chunk table), the others back to 16."""
        if plan.buf_ai < 0 or plan.buffer_tokens == nbuf:
            return
        nb = (nbuf + 15) // 16
        live = self._buf_live_host
        changed = False
        for b in range(len(live)):
            want = 1 if b < nb else 0
            if live[b] != want:
                live[b] = want
                changed = True
            if b < nb:
                ntok = 16 if b < nb - 1 else nbuf - 16 * (nb - 1)
                if plan.buffer_ntok[b] != ntok:
                    plan.patch_tokens(plan.buffer_chunks[b], ntok)
                    plan.buffer_ntok[b] = ntok
        if changed:
            self._buf_live.copy_(torch.from_numpy(live))
        plan.segments[-1] = ("buffer", None, nbuf)
        plan.buffer_tokens = nbuf

    def _slot(self, name, idx, live):
        """Page moves: slot idx of pool `name` ("fp16" or a tier) now holds a live page (or not)."""
        h = self._live_host.get(name)
        if h is None:
            return
        h[idx] = 1 if live else 0
        self._live_dirty = True
        self._tiers_dirty.add(name)

    def _sync_live(self, plan):
        """Uploads the pools' occupancy after page moves, refreshes the outlier directories of the
        tiers whose pages changed, and lets the plan re-read the arenas' pointers."""
        if not self._live_dirty:
            return
        for name, h in self._live_host.items():
            self.arenas[name].slot_live.copy_(torch.from_numpy(h))
        for name in self._tiers_dirty | (set(_TIERS) if self._tiers_dirty_all else set()):
            if name in _TIERS:
                self._attach_outliers(name)
        self._tiers_dirty = set()
        self._tiers_dirty_all = False
        plan.refresh_arenas()
        self._live_dirty = False

    def _plan_base(self, q, base_key, fused_jl):
        """The structure-dependent part of the attention tables (see _attention_plan), cached by key:
        the scratch fp16 arena (sinks, anchors, JL pages the fused JL kernel does not take) and every
        slot of the FP16 and tier pools."""
        if self._plan_base_cache is not None and self._plan_base_cache[0] == base_key:
            return self._plan_base_cache[1]
        B, Hq, qlen, D = q.shape
        P = self.page_size
        order = []  # (segment kind, page / (pool, slot) / None, tokens)
        if self.sink_k is not None:
            order.append(("sinks", None, self.sink_k.shape[-2]))
        if self.anchor_k is not None:
            order.append(("anchors", None, self.anchor_k.shape[-2]))
        Hkv = self.H if self._pools_allocated else (self.sink_k.shape[1])
        if not fused_jl:
            for page in self.jl_pages:
                order.append(("scratch:jl", page, P))
        if self._pools_allocated:
            for name in ["fp16"] + list(_TIERS):
                for slot in range(self.arenas[name].slots):
                    order.append(("slot", (name, slot), P))
        # scratch fp16 tensor: sinks, anchors and rebuilt JL pages, each padded to 16 tokens
        scratch_len = sum(-(-n // 16) * 16 for kind, _, n in order if kind in ("sinks", "anchors", "scratch:jl"))
        dev = q.device
        arenas, index, pages = [], {}, []
        scratch = None
        if scratch_len:
            sk = torch.empty(B, Hkv, scratch_len, D, dtype=torch.float16, device=dev)
            sv = torch.empty_like(sk)
            scratch = (sk, sv)
            index["scratch"] = len(arenas)
            arenas.append(A.KVArena.from_fp16(sk, sv))
        pos = 0
        page_seg = []  # per entry of `pages`: its segment
        for seg, (kind, page, n) in enumerate(order):
            if kind in ("sinks", "anchors", "scratch:jl"):
                sk, sv = scratch
                if kind == "sinks":
                    sk[:, :, pos:pos + n].copy_(self.sink_k)
                    sv[:, :, pos:pos + n].copy_(self.sink_v)
                elif kind == "anchors":
                    sk[:, :, pos:pos + n].copy_(self.anchor_k)
                    sv[:, :, pos:pos + n].copy_(self.anchor_v)
                else:
                    k, v = self._dequant_with_sidecars("jl", page)
                    sk[:, :, pos:pos + n].copy_(k)
                    sv[:, :, pos:pos + n].copy_(v)
                for t0 in range(0, n, 16):
                    pages.append((index["scratch"], (pos + t0) // 16, min(16, n - t0)))
                    page_seg.append(seg)
                pos += -(-n // 16) * 16
            else:
                name, slot = page
                if name not in index:
                    index[name] = len(arenas)
                    arenas.append(self.arenas[name])
                pages.append((index[name], slot, n))
                page_seg.append(seg)
        self._tiers_dirty_all = True  # the directories are rebuilt for the new plan
        base = {"order": order, "arenas": arenas, "pages": pages, "page_seg": page_seg, "Hkv": Hkv,
                "scratch": scratch}
        self._plan_base_cache = (base_key, base)
        return base

    def _attach_outliers(self, name):
        """Points tier `name`'s arena directory at the correction blocks of its pages' outlier
        sidecars, so the fused kernel applies them while reading the pages compressed.  A page's
        blocks are built once per (arena, slot) it occupies and kept in the page dict."""
        arena = self.arenas[name]
        arena.clear_outliers()
        for page in getattr(self, _TIERS[name][0]):
            ki, vi = page.get("key_out_indices"), page.get("value_out_indices")
            if (ki is None or ki.numel() == 0) and (vi is None or vi.numel() == 0):
                continue
            key = (arena.k.data_ptr(), page["pool_idx"])
            cached = page.get("_outlier_blocks")
            if cached is None or cached[0] != key:
                blocks, addr = paged.outlier_corrections(arena, page["pool_idx"], ki, page.get("key_out_values"), vi,
                                                         page.get("value_out_values"))
                cached = (key, blocks, addr)
                page["_outlier_blocks"] = cached
            arena.set_outliers(page["pool_idx"], cached[1], cached[2])

    def _scratch_version(self, fused_jl):
        """What the scratch arena is built from: the sinks, the anchors and (when the fused JL kernel
        does not take them) the JL pages.  Page moves between the pools do not change it."""
        return (self.sink_k.data_ptr() if self.sink_k is not None else 0,
                self.anchor_k.shape[-2] if self.anchor_k is not None else 0,
                () if fused_jl else tuple(id(p) for p in self.jl_pages))

    def attend(self, q, scale=None, causal=False):
        """softmax(q K^T * scale) V over every tier straight from the compressed pages, without the
        importance / resurrection side effects of inplace_paged_attention: what the HuggingFace path
        computes from get_all_keys_values + SDPA (models/attention_wrapper.py:87-88), without
        rebuilding the full K/V.  q: [B, H_q, q_len, D] fp16.  causal=False: every query attends
        to every cached token.  causal=True: the q_len queries are the newest q_len cached tokens
        and query i sees the tokens up to its own (the bottom-right causal mask)."""
        B, Hq, qlen, D = q.shape
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        if self.is_swapped_out:
            self.swap_in_to_device()
        if causal and qlen > 1:
            _lib.require_cuda(q, "q")
            if q.dtype != torch.float16:
                raise TypeError("q must be float16")
            return self._attend_causal(q, scale)
        if self.sink_k is None and self.anchor_k is None and not self.active_pages and self.k_buffer is None and \
                not any(lst for _, lst in self._compressed_order()):
            return torch.zeros_like(q)
        _lib.require_cuda(q, "q")
        if q.dtype != torch.float16:
            raise TypeError("q must be float16")
        plan = self._attention_plan(q)
        if plan.jl is None:
            return plan.run(q, scale=scale)
        lse = torch.empty(B, Hq, qlen, dtype=torch.float32, device=q.device)
        out = plan.run(q, scale=scale, lse=lse)
        out_j, lse_j = plan.jl["att"].run(q, plan.jl["yk"], plan.jl["yv"], scale=scale)
        return _jl.merge_attention(out, lse, out_j, lse_j)

    def newest_in_buffer(self, n):
        """True when the newest n cached tokens all sit in the fp16 staging buffer."""
        return self.k_buffer is not None and self.buffer_length >= n

    def causal_tail_pages(self, n):
        """The causal mask of a step of n tokens is bottom-right over the reference's concatenation
        order (..., FP8, active pages in list order, staging buffer): its last n entries are the
        masked ones.  Returns how many of the last active pages those entries reach into past the
        staging buffer (0: all in the buffer), or None when they reach past the active pages."""
        nbuf = self.buffer_length if self.k_buffer is not None else 0
        if nbuf >= n:
            return 0
        m = -(-(n - nbuf) // self.page_size)
        return m if m <= len(self.active_pages) else None

    def fused_causal_ok(self, n):
        """attend(q, causal=True) with n queries runs the fused kernel (no K/V rebuild)."""
        return self.causal_tail_pages(n) is not None

    def _attend_causal(self, q, scale):
        """attend(causal=True): the masked tail of the concatenation (the newest q_len entries, see
        causal_tail_pages) under the causal mask, everything before it through the fused kernel,
        joined by LSE.  The tail is the end of the staging buffer, or, when a page has just formed
        from the step's tokens, the last m active pages plus the whole buffer: those pages' slots
        are marked dead for the fused launch (slot occupancy) and attended with the tail instead.
        When the tail reaches past the active pages (a prefill into a fresh cache), K/V are rebuilt."""
        B, Hq, qlen, D = q.shape
        m = self.causal_tail_pages(qlen)
        if m is None:
            K, V = self.get_all_keys_values()
            return _causal_sdpa(q, K, V, scale)
        nbuf = self.buffer_length if self.k_buffer is not None else 0
        P = self.page_size
        tail_pages = self.active_pages[len(self.active_pages) - m:] if m else []
        if m:
            k_new = torch.cat([p["key"] for p in tail_pages] + [self.static_k_buffer[..., :nbuf, :]], dim=-2)
            v_new = torch.cat([p["value"] for p in tail_pages] + [self.static_v_buffer[..., :nbuf, :]], dim=-2)
        else:
            k_new = self.static_k_buffer[..., nbuf - qlen:nbuf, :]
            v_new = self.static_v_buffer[..., nbuf - qlen:nbuf, :]
        out_n, lse_n = _causal_sdpa(q, k_new, v_new, scale, with_lse=True)
        older = P * (len(self.active_pages) - m + sum(len(lst) for _, lst in self._compressed_order()))
        older += (nbuf - qlen) if not m else 0
        older += self.sink_k.shape[-2] if self.sink_k is not None else 0
        older += self.anchor_k.shape[-2] if self.anchor_k is not None else 0
        if older == 0:
            return out_n
        plan = self._attention_plan(q, tail=nbuf if m else qlen)
        lse = torch.empty(B, Hq, qlen, dtype=torch.float32, device=q.device)
        if m:
            self.fused_causal_page_steps += 1
            live = self._live_host["fp16"]
            saved = live.copy()
            for p in tail_pages:
                live[p["pool_idx"]] = 0
            self.arenas["fp16"].slot_live.copy_(torch.from_numpy(live))
            try:
                out = plan.run(q, scale=scale, lse=lse)
            finally:
                live[:] = saved
                self.arenas["fp16"].slot_live.copy_(torch.from_numpy(live))
        else:
            out = plan.run(q, scale=scale, lse=lse)
        if plan.jl is not None:
            out_j, lse_j = plan.jl["att"].run(q, plan.jl["yk"], plan.jl["yv"], scale=scale)
            lse_t = torch.empty_like(lse)
            out = _jl.merge_attention(out, lse, out_j, lse_j, lse=lse_t)
            lse = lse_t
        return _jl.merge_attention(out, lse, out_n, lse_n)

    def inplace_paged_attention(self, q, scale=None):
        """softmax(q K^T * scale) V over every tier, straight from the compressed pages, plus the
        per-page attention mass, importance update and resurrection (memory_manager.py:1317-1524).
        q: [B, H_q, q_len, D]; H_q may be any multiple of the KV heads (GQA)."""
        B, Hq, qlen, D = q.shape
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        self.total_attention_calls += 1
        if self.is_swapped_out:
            self.swap_in_to_device()
        for _, lst in self._compressed_order():
            for page in lst:
                if id(page) in self.prefetch_cache:
                    self.prefetch_hits += 1
                else:
                    self.prefetch_misses += 1
        if self.sink_k is None and self.anchor_k is None and not self.active_pages and self.k_buffer is None and \
                not any(lst for _, lst in self._compressed_order()):
            return torch.zeros_like(q)
        _lib.require_cuda(q, "q")
        if q.dtype != torch.float16:
            raise TypeError("q must be float16")
        plan = self._attention_plan(q)
        lse = torch.empty(B, Hq, qlen, dtype=torch.float32, device=q.device)
        tile_lse = torch.empty(plan.tile_lse_shape(), dtype=torch.float32, device=q.device)
        out = plan.run(q, scale=scale, lse=lse, tile_lse=tile_lse)
        block_lse = None
        if plan.jl is not None:
            # JL pages attended without rebuilding them, then joined with the other tiers by LSE
            jl_blocks = plan.jl["yk"].shape[2]
            block_lse = torch.empty(B * plan.Hkv, jl_blocks, 8, dtype=torch.float32, device=q.device)
            out_j, lse_j = plan.jl["att"].run(q, plan.jl["yk"], plan.jl["yv"], scale=scale, block_lse=block_lse)
            lse_tot = torch.empty_like(lse)
            out = _jl.merge_attention(out, lse, out_j, lse_j, lse=lse_tot)
            lse = lse_tot
        self.generation_step += 1
        # per-segment attention mass: mean over (b, h_q, q) of the segment's token probabilities
        nqg = tile_lse.shape[0] // (B * plan.Hkv)
        G = Hq // plan.Hkv
        lse2 = (lse * math.log2(math.e)).view(B, plan.Hkv, G * qlen)
        pad = nqg * 8 - G * qlen
        if pad:
            lse2 = torch.cat([lse2, torch.full((B, plan.Hkv, pad), float("inf"), device=q.device)], dim=-1)
        tl = tile_lse.view(B, plan.Hkv, nqg, -1, 16, 8)
        w = torch.exp2(tl - lse2.view(B, plan.Hkv, nqg, 1, 1, 8))
        valid = plan.tile_segment >= 0
        w = torch.where(valid.view(1, 1, 1, *valid.shape, 1), w, torch.zeros((), device=q.device))
        tile_mass = w.sum(dim=(0, 1, 2, 5)) / float(B * Hq * qlen)
        seg_mass = torch.zeros(len(plan.segments), device=q.device, dtype=torch.float32)
        seg_mass.index_add_(0, plan.tile_segment[valid], tile_mass[valid])
        jl_masses = []
        if block_lse is not None:
            nq = G * qlen
            wj = torch.exp(block_lse[:, :, :nq] - lse.view(B * plan.Hkv, 1, nq))
            jl_masses = (wj.sum(dim=(0, 2)) / float(B * Hq * qlen)).tolist()
        masses = seg_mass.tolist()
        # each page's mass from its pool slot (or, for JL pages, its own segment), in the reference's
        # page order: active pages, then JL, 1-bit, INT2, INT4, INT8, FP8
        by_seg = {}
        for (kind, where, n), m in zip(plan.segments, masses):
            if kind == "slot":
                by_seg[where] = m
            elif kind == "scratch:jl":
                by_seg[id(where)] = m
        if plan.jl is not None:
            for page, m in zip(plan.jl["pages"], jl_masses):
                by_seg[id(page)] = m
        resurrect = []
        compressed = {id(p): name for name, lst in self._compressed_order() for p in lst}
        ordered = [("fp16", p) for p in self.active_pages] + [(n, p) for n, lst in self._compressed_order() for p in lst]
        for name, page in ordered:
            block_w = by_seg.get(id(page) if name == "jl" else (name, page["pool_idx"]))
            if block_w is None:
                continue
            page["attention_sum"] = page.get("attention_sum", 0.0) + block_w
            if block_w > 0.0:
                page["last_step_accessed"] = self.generation_step
            self._calculate_importance(page)
            tier = compressed.get(id(page))
            if tier is not None and block_w > self.config.resurrection_threshold:
                resurrect.append((page, tier))
        for p, t in resurrect:
            self._resurrect_page(p, t)
        return out

    def speculate_and_prefetch(self, attn_weights=None):
        """Pre-dequantize the (up to 2) pages most likely to be read next, on a side stream
        (memory_manager.py:1526-1656).  Consumers wait on the prefetch event before reading."""
        self.prefetch_cache.clear()
        if self.is_swapped_out:
            return
        chosen = []
        if attn_weights is not None:
            try:
                weights = attn_weights.mean(dim=(0, 1))[-1]
                off = (self.sink_k.shape[-2] if self.sink_k is not None else 0) + \
                      (self.anchor_k.shape[-2] if self.anchor_k is not None else 0)
                ranked = []
                allp = [(name, p) for name, lst in self._compressed_order() for p in lst]
                for i, (tier, page) in enumerate(allp):
                    s, e = off + i * self.page_size, off + (i + 1) * self.page_size
                    ranked.append(((weights[s:e].mean().item() if e <= len(weights) else 0.0), page, tier))
                ranked.sort(key=lambda x: x[0], reverse=True)
                chosen = [(p, t) for _, p, t in ranked[:2]]
            except Exception:
                chosen = []
        if not chosen:
            for tier, lst in (("fp8", self.fp8_pages), ("int8", self.int8_pages), ("int4", self.int4_pages)):
                if lst:
                    chosen.append((lst[-1], tier))
        if not chosen or not torch.cuda.is_available():
            return
        if self.prefetch_stream is None:
            self.prefetch_stream = torch.cuda.Stream()
        main = torch.cuda.current_stream()
        self.prefetch_stream.wait_stream(main)
        with torch.cuda.stream(self.prefetch_stream):
            for page, tier in chosen:
                try:
                    k, v = self._dequant_with_sidecars(tier, page)
                    k.record_stream(main)
                    v.record_stream(main)
                    self.prefetch_cache[id(page)] = (k, v)
                except Exception:
                    pass
            self._prefetch_event = torch.cuda.Event()
            self._prefetch_event.record(self.prefetch_stream)

    # --------------------------------------------------------------------- host spill
    _SWAP_KEYS = ("key_out_indices", "key_out_values", "value_out_indices", "value_out_values")

    def swap_out_to_host(self):
        """Move every compressed tier (FP8 .. JL) to pinned host memory and release its HBM
        (memory_manager.py:1658-1684).  Arena copies run as asynchronous copies on a side stream;
        page dicts keep their schema as views into the host copies."""
        if self.is_swapped_out:
            return
        from .. import spill

        self._invalidate()
        if self._pools_allocated:
            self._host_arenas = spill.arenas_to_host([self.arenas[n] for n in _TIERS])
            for name, host in zip(_TIERS, self._host_arenas):
                self.arenas[name] = host
                for page in getattr(self, _TIERS[name][0]):
                    page.update(self._page_views(name, page["pool_idx"]))
        for _, lst in self._compressed_order():
            for page in lst:
                page.pop("_outlier_blocks", None)  # derived device data, rebuilt after swap-in
                for k in self._SWAP_KEYS + ("key_proj", "value_proj"):
                    if isinstance(page.get(k), torch.Tensor) and page[k].is_cuda:
                        page[k] = page[k].to("cpu")
        self.is_swapped_out = True

    def swap_in_to_device(self, device="cuda"):
        """Bring the spilled tiers back to HBM (memory_manager.py:1686-1713)."""
        if not self.is_swapped_out:
            return
        from .. import spill

        self._invalidate()
        target = torch.device(device if torch.cuda.is_available() else "cpu")
        if self._pools_allocated and self._host_arenas:
            dev_arenas = spill.arenas_to_device(self._host_arenas, target)
            for name, a in zip(_TIERS, dev_arenas):
                a.slot_live = torch.from_numpy(self._live_host[name]).to(target)
                self.arenas[name] = a
                for page in getattr(self, _TIERS[name][0]):
                    page.update(self._page_views(name, page["pool_idx"]))
            self._host_arenas = {}
        for _, lst in self._compressed_order():
            for page in lst:
                for k in self._SWAP_KEYS + ("key_proj", "value_proj"):
                    if isinstance(page.get(k), torch.Tensor) and not page[k].is_cuda:
                        page[k] = page[k].to(target)
        self.is_swapped_out = False

    # --------------------------------------------------------------------- accounting
    def get_vram_usage(self):
        """Bytes of cache state resident on the GPU (memory_manager.py:1715-1824)."""
        total = 0
        for t in (self.sink_k, self.sink_v, self.anchor_k, self.anchor_v):
            if t is not None:
                total += t.nelement() * 2
        for page in self.active_pages:
            total += page["key"].nelement() * 2 + page["value"].nelement() * 2
        if self.k_buffer is not None:
            total += self.k_buffer.nelement() * 2 + self.v_buffer.nelement() * 2
        if self.is_swapped_out:
            return total
        for name, lst in self._compressed_order():
            for page in lst:
                if name == "jl":
                    total += page["key_proj"].nelement() * 2 + page["value_proj"].nelement() * 2
                    continue
                pk = _PAYLOAD_KEY[name]
                total += page[f"key_{pk}"].nelement() + page[f"value_{pk}"].nelement()
                total += page["key_scales"].nelement() * 2 + page["value_scales"].nelement() * 2
                if name in ("int4", "int2"):
                    total += page["key_min"].nelement() * 2 + page["value_min"].nelement() * 2
                for pre in ("key", "value"):
                    if page.get(f"{pre}_out_indices") is not None:
                        total += page[f"{pre}_out_indices"].nelement() * 2 + page[f"{pre}_out_values"].nelement() * 2
        if self.w_proj is not None:
            total += self.w_proj.nelement() * 2
        return total

    def get_cache_telemetry(self):
        """(compression ratio, % bytes saved, pages, compressed bytes), memory_manager.py:566-674."""
        B, H, D = (getattr(self, "B", 1), getattr(self, "H", 1), getattr(self, "D", 16))
        per_page = B * H * self.page_size * D
        fp16_page = per_page * 2 * 2
        pages, comp = 0, 0
        for t in (self.sink_k, self.anchor_k):
            if t is not None:
                comp += t.element_size() * t.nelement() * 2
                pages += math.ceil(t.shape[-2] / self.page_size)
        pages += len(self.active_pages)
        comp += len(self.active_pages) * fp16_page
        rate = {"fp8": 1.0, "int8": 1.0, "int4": 0.5, "int2": 0.25, "one_bit": 0.125}
        for name, lst in self._compressed_order():
            for p in lst:
                pages += 1
                if name == "jl":
                    comp += p["key_proj"].element_size() * p["key_proj"].nelement() * 2
                    continue
                comp += int(per_page * 2 * rate[name])
                comp += p["key_scales"].element_size() * p["key_scales"].nelement() * 2
                if "key_min" in p:
                    comp += p["key_min"].element_size() * p["key_min"].nelement() * 2
                for pre in ("key", "value"):
                    for suf in ("out_indices", "out_values"):
                        t = p.get(f"{pre}_{suf}")
                        if t is not None:
                            comp += t.element_size() * t.nelement()
        if pages == 0:
            return 1.0, 0.0, 0, 0
        ratio = pages * fp16_page / max(1, comp)
        return ratio, (1.0 - 1.0 / ratio) * 100.0, pages, comp

    def print_telemetry_summary(self):
        """Text summary of the cache state (the reference prints a coloured panel)."""
        ratio, saved, pages, comp = self.get_cache_telemetry()
        print(f"[ARGUS] compression {ratio:.1f}x ({saved:.1f}% saved), {pages} pages, {comp} bytes | "
              f"active {len(self.active_pages)} fp8 {len(self.fp8_pages)} int8 {len(self.int8_pages)} int4 "
              f"{len(self.int4_pages)} int2 {len(self.int2_pages)} 1bit {len(self.one_bit_pages)} jl "
              f"{len(self.jl_pages)} | resurrections {self.num_resurrections} spills {self.num_cpu_spills} | "
              f"cascade {self.cascade_counts}")
