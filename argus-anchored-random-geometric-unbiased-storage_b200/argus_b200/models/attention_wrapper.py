"""HuggingFace cache adapter with the reference's surface (argus_cache/models/attention_wrapper.py:12-173).

One PagedDynamicKVCache per layer, created lazily on the first update() with the reference's
auto-adaptive tier budgets (low-precision key dtypes get shorter FP16/FP8 stages and longer
heavily-compressed ones, attention_wrapper.py:49-79).  update() pushes the new tokens (page
formation and the fused demotion cascade run on the GPU) and returns the full K/V rebuilt by the
page kernels, which is what transformers' attention consumes (attention_wrapper.py:87-88).

With fused_decode=True, update() returns placeholders instead and the "argus" attention
implementation (registered with transformers' AttentionInterface; load the model with
attn_implementation="argus") sends each decode step straight to the fused mixed-tier kernel over
the compressed pages, so the full K/V is never rebuilt (JL pages the fused JL kernel does not
take pass through the manager's fp16 scratch arena).  A step of several new tokens (speculative
or chunked decoding) takes the same route when those tokens are still in the staging buffer: the
kernel attends to everything older and the new tokens attend to one another under the causal
mask, joined by LSE; a step whose tokens just formed a page takes the same route, the newest active
pages joining the causal part.  A prefill whose tokens reach past the active pages (into tiers
compressed during the prefill itself) and padded batches rebuild K/V and run transformers' SDPA.
"""
import torch

from ..core.memory_manager import PagedDynamicKVCache

try:
    from transformers.cache_utils import Cache
except ImportError:  # transformers absent: a bare base class keeps the adapter importable
    class Cache:
        def __init__(self, *args, **kwargs):
            pass


class PagedDynamicQuantizedCache(Cache):
    def __init__(self, page_size=4096, max_active_pages=2, max_fp8_pages=2, max_int8_pages=2, max_int4_pages=2,
                 max_int2_pages=2, max_one_bit_pages=2, sink_tokens=4, threshold_sigma=3.0, fused_decode=False):
        try:
            super().__init__(layers=[])
        except TypeError:
            super().__init__()
        self.page_size = page_size
        self.max_active_pages = max_active_pages
        self.max_fp8_pages = max_fp8_pages
        self.max_int8_pages = max_int8_pages
        self.max_int4_pages = max_int4_pages
        self.max_int2_pages = max_int2_pages
        self.max_one_bit_pages = max_one_bit_pages
        self.sink_tokens = sink_tokens
        self.threshold_sigma = threshold_sigma
        self.fused_decode = fused_decode
        self.layer_caches = {}

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int, cache_kwargs=None):
        if layer_idx not in self.layer_caches:
            if key_states.dtype in (torch.float32, torch.float16, torch.bfloat16):
                budgets = (self.max_active_pages, self.max_fp8_pages, self.max_int8_pages, self.max_int4_pages,
                           self.max_int2_pages, self.max_one_bit_pages)
            else:
                budgets = (max(1, self.max_active_pages // 2), 1, self.max_int8_pages,
                           max(1, self.max_int4_pages * 2), max(1, self.max_int2_pages * 2),
                           max(1, self.max_one_bit_pages * 2))
            self.layer_caches[layer_idx] = PagedDynamicKVCache(
                page_size=self.page_size, max_active_pages=budgets[0], max_fp8_pages=budgets[1],
                max_int8_pages=budgets[2], max_int4_pages=budgets[3], max_int2_pages=budgets[4],
                max_one_bit_pages=budgets[5], sink_tokens=self.sink_tokens, threshold_sigma=self.threshold_sigma)
        cache = self.layer_caches[layer_idx]
        is_anchor = cache_kwargs.get("is_anchor") if cache_kwargs is not None else None
        cache.push_new_tokens(key_states, value_states, is_anchor=is_anchor)
        if self.fused_decode:
            # placeholders that carry the layer's cache to argus_attention_forward
            k = torch.empty(0, dtype=key_states.dtype, device=key_states.device)
            v = torch.empty(0, dtype=value_states.dtype, device=value_states.device)
            k._argus_layer_cache = cache
            v._argus_layer_cache = cache
            return k, v
        return cache.get_all_keys_values()

    def get_seq_length(self, layer_idx: int = 0) -> int:
        if layer_idx not in self.layer_caches:
            return 0
        c = self.layer_caches[layer_idx]
        n = 0
        if c.sink_k is not None:
            n += c.sink_k.shape[-2]
        if c.anchor_k is not None:
            n += c.anchor_k.shape[-2]
        pages = (len(c.active_pages) + len(c.fp8_pages) + len(c.int8_pages) + len(c.int4_pages) + len(c.int2_pages)
                 + len(c.one_bit_pages) + len(c.jl_pages))
        n += pages * c.page_size
        if c.k_buffer is not None:
            n += c.k_buffer.shape[-2]
        return n

    def get_mask_sizes(self, query_length, layer_idx: int = 0):
        """(kv_length, kv_offset) for transformers' mask builders: every cached token plus the new
        ones (older transformers pass cache_position instead of the query length)."""
        if torch.is_tensor(query_length):
            query_length = query_length.shape[0]
        return self.get_seq_length(layer_idx) + query_length, 0

    def get_usable_length(self, seq_len: int, layer_idx: int = 0) -> int:
        return self.get_seq_length(layer_idx)

    def get_vram_usage(self) -> int:
        return sum(c.get_vram_usage() for c in self.layer_caches.values())

    def speculate_and_prefetch(self, attn_weights=None):
        for c in self.layer_caches.values():
            c.speculate_and_prefetch(attn_weights)

    def swap_out_to_host(self):
        for c in self.layer_caches.values():
            c.swap_out_to_host()

    def swap_in_to_device(self, device="cuda"):
        for c in self.layer_caches.values():
            c.swap_in_to_device(device)

    @property
    def is_swapped_out(self) -> bool:
        return any(c.is_swapped_out for c in self.layer_caches.values()) if self.layer_caches else False

    def reset(self):
        self.layer_caches.clear()


def _bottom_right_causal(q_len, kv_len, device):
    """Boolean [q_len, kv_len] mask, True where query i (the (kv_len - q_len + i)-th token) may
    attend to key j."""
    j = torch.arange(kv_len, device=device)
    i = torch.arange(q_len, device=device)
    return j.view(1, -1) <= (kv_len - q_len + i).view(-1, 1)


def argus_attention_forward(module, query, key, value, attention_mask, dropout=0.0, scaling=None, is_causal=None,
                            **kwargs):
    """transformers attention function ("argus"): a decode step (no padding mask) over a
    PagedDynamicQuantizedCache(fused_decode=True) layer runs the fused mixed-tier kernel on the
    compressed pages (several query tokens: causal among themselves, see the module docstring);
    anything else rebuilds K/V and runs transformers' SDPA.  Returns ([B, q_len, H_q, D], None)
    as transformers' attention functions do."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    cache = getattr(key, "_argus_layer_cache", None)
    causal = getattr(module, "is_causal", True) if is_causal is None else is_causal
    ql = query.shape[2]
    if cache is None:
        if attention_mask is None and causal and 1 < ql < key.shape[-2]:
            attention_mask = _bottom_right_causal(ql, key.shape[-2], query.device)
        return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling,
                                      is_causal=is_causal, **kwargs)
    if attention_mask is None and dropout == 0.0 and query.dtype == torch.float16 and \
            (ql == 1 or (causal and cache.fused_causal_ok(ql))):
        out = cache.attend(query.contiguous(), scale=scaling, causal=ql > 1)
        return out.transpose(1, 2).contiguous(), None
    K, V = cache.get_all_keys_values()
    K, V = K.to(query.dtype), V.to(query.dtype)
    if attention_mask is None and causal and 1 < ql < K.shape[-2]:
        # SDPA's is_causal is top-left aligned; queries after a cached prefix need bottom-right
        attention_mask = _bottom_right_causal(ql, K.shape[-2], query.device)
    return sdpa_attention_forward(module, query, K, V, attention_mask, dropout=dropout, scaling=scaling,
                                  is_causal=is_causal, **kwargs)


def argus_mask(batch_size, q_length, kv_length, q_offset=0, kv_offset=0, mask_function=None, attention_mask=None,
               local_size=None, allow_is_causal_skip=True, **kwargs):
    """Mask builder registered with "argus": a plain causal mask without padding is left to the
    attention function (None), which knows the cached length and aligns the causal mask to its
    end; anything else is transformers' SDPA mask."""
    from transformers.masking_utils import causal_mask_function, sdpa_mask
    if mask_function is None:
        mask_function = causal_mask_function
    if mask_function is causal_mask_function and local_size is None and allow_is_causal_skip and \
            (attention_mask is None or bool(attention_mask.all())):
        return None
    return sdpa_mask(batch_size, q_length, kv_length, q_offset=q_offset, kv_offset=kv_offset,
                     mask_function=mask_function, attention_mask=attention_mask, local_size=local_size,
                     allow_is_causal_skip=allow_is_causal_skip, **kwargs)


def _register():
    try:
        from transformers.masking_utils import AttentionMaskInterface
        from transformers.modeling_utils import AttentionInterface
    except ImportError:
        return
    AttentionInterface.register("argus", argus_attention_forward)
    AttentionMaskInterface.register("argus", argus_mask)


_register()
