"""The "argus" transformers attention implementation on CPU: it is registered for attention and
masks, and with a cache other than PagedDynamicQuantizedCache(fused_decode=True) it is exactly
transformers' SDPA."""
import pytest
import torch


def test_argus_attention_registered_and_falls_back_to_sdpa():
    transformers = pytest.importorskip("transformers")
    from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    from argus_b200.models import attention_wrapper as W
    assert ALL_ATTENTION_FUNCTIONS["argus"] is W.argus_attention_forward
    assert "argus" in ALL_MASK_ATTENTION_FUNCTIONS
    cfg = transformers.LlamaConfig(vocab_size=64, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=128)
    torch.manual_seed(0)
    ref = transformers.LlamaForCausalLM(cfg).eval()
    cfg2 = transformers.LlamaConfig(**cfg.to_dict())
    cfg2._attn_implementation = "argus"
    ours = transformers.LlamaForCausalLM(cfg2).eval()
    ours.load_state_dict(ref.state_dict())
    ids = torch.randint(0, 64, (2, 12))
    mask = torch.ones_like(ids)
    mask[1, :3] = 0  # left padding
    with torch.no_grad():
        a = ref(ids, attention_mask=mask).logits
        b = ours(ids, attention_mask=mask).logits
    assert torch.equal(a, b)


def test_mask_sizes_count_cached_tokens():
    pytest.importorskip("transformers")
    from argus_b200.models.attention_wrapper import PagedDynamicQuantizedCache
    c = PagedDynamicQuantizedCache(page_size=16)
    assert c.get_mask_sizes(5, 0) == (5, 0)
    assert c.get_mask_sizes(torch.arange(3), 0) == (3, 0)


def test_argus_chunks_after_a_cached_prefix_match_sdpa():
    """Several new tokens after a cached prefix (chunked prefill / speculative steps) on a plain
    DynamicCache: the "argus" mask leaves the causal mask to the attention function, which aligns
    it to the end of the cache exactly as transformers' SDPA mask does."""
    transformers = pytest.importorskip("transformers")
    from transformers import DynamicCache

    from argus_b200.models import attention_wrapper  # noqa: F401
    cfg = transformers.LlamaConfig(vocab_size=64, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=128)
    torch.manual_seed(0)
    ref = transformers.LlamaForCausalLM(cfg).eval()
    cfg2 = transformers.LlamaConfig(**cfg.to_dict())
    cfg2._attn_implementation = "argus"
    ours = transformers.LlamaForCausalLM(cfg2).eval()
    ours.load_state_dict(ref.state_dict())
    ids = torch.randint(0, 64, (1, 17))
    ca, cb = DynamicCache(), DynamicCache()
    with torch.no_grad():
        for s, e in ((0, 9), (9, 12), (12, 17)):
            a = ref(ids[:, s:e], past_key_values=ca, use_cache=True).logits
            b = ours(ids[:, s:e], past_key_values=cb, use_cache=True).logits
            assert torch.allclose(a, b, atol=1e-5), (s, e, (a - b).abs().max())
