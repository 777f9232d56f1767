"""Decode attention for transformers without rebuilding K/V: PagedDynamicKVCache.attend() over the
reference's cascade runs (tests/golden/cascade.npz), and the "argus" attention implementation
with PagedDynamicQuantizedCache(fused_decode=True) against the materializing adapter.

Reference: the HuggingFace adapter returns get_all_keys_values() to transformers' attention
(argus_cache/models/attention_wrapper.py:87-88); attend() must give that attention (2e-3 max-abs
plus the fp16 output's half-ulp, as the other attention tests) and leave the cache as it was."""
import math
import os

import numpy as np
import pytest
import torch

from test_manager_gpu import RUNS, counts, host, replay

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", list(RUNS))
def test_attend_matches_reference_attention_without_side_effects(golden, name, tmp_path):
    import oracle
    z = golden("cascade")
    cache = replay(z, name, tmp_path)
    q = z[f"{name}/q"]
    before = (counts(cache), cache.generation_step, cache.total_attention_calls)
    out = host(cache.attend(torch.from_numpy(q).cuda())).astype(np.float64)
    ref = oracle.sdpa_f64(q, z[f"{name}/K"], z[f"{name}/V"], 1.0 / math.sqrt(q.shape[-1]))
    bar = 2e-3 + np.abs(ref) * 2.0 ** -11 + 4e-3 * (len(cache.jl_pages) > 0)
    assert (np.abs(out - ref) <= bar).all(), np.abs(out - ref).max()
    assert (counts(cache), cache.generation_step, cache.total_attention_calls) == before


def _models(num_layers, hidden, heads, kv_heads, head_dim):
    transformers = pytest.importorskip("transformers")
    from argus_b200.models import attention_wrapper  # noqa: F401  registers "argus"
    cfg = transformers.LlamaConfig(vocab_size=256, hidden_size=hidden, intermediate_size=2 * hidden,
                                   num_hidden_layers=num_layers, num_attention_heads=heads,
                                   num_key_value_heads=kv_heads, head_dim=head_dim, max_position_embeddings=1024)
    torch.manual_seed(0)
    ref = transformers.LlamaForCausalLM(cfg).cuda().half().eval()
    cfg2 = transformers.LlamaConfig(**cfg.to_dict())
    cfg2._attn_implementation = "argus"
    fused = transformers.LlamaForCausalLM(cfg2).cuda().half().eval()
    fused.load_state_dict(ref.state_dict())
    assert fused.config._attn_implementation == "argus"
    return ref, fused


def _cache(fused):
    from argus_b200.models.attention_wrapper import PagedDynamicQuantizedCache
    return PagedDynamicQuantizedCache(page_size=16, max_active_pages=1, max_fp8_pages=1, max_int8_pages=1,
                                      max_int4_pages=1, max_int2_pages=1, max_one_bit_pages=1, sink_tokens=4,
                                      fused_decode=fused)


@pytest.mark.parametrize("num_layers,hidden,heads,kv_heads,head_dim,atol", [
    (1, 256, 8, 2, 32, 1e-2),    # one layer: both caches receive identical K/V
    (1, 512, 4, 1, 128, 1e-2),
    (2, 256, 4, 2, 64, 5e-2),    # two layers: layer 1's K/V differ by the rounding of layer 0's attention
])
def test_fused_decode_matches_materializing_adapter(num_layers, hidden, heads, kv_heads, head_dim, atol, tmp_path,
                                                    monkeypatch):
    from argus_b200.core.memory_manager import PagedDynamicKVCache
    monkeypatch.setenv("ARGUS_LOG_LEVEL", "quiet")
    monkeypatch.chdir(tmp_path)
    ref_model, fused_model = _models(num_layers, hidden, heads, kv_heads, head_dim)
    ref_cache, fused_cache = _cache(False), _cache(True)
    g = torch.Generator(device="cuda").manual_seed(3)
    ids = torch.randint(0, 256, (1, 130), device="cuda", generator=g)
    steps = torch.randint(0, 256, (1, 24), device="cuda", generator=g)
    rebuilt = []
    real = PagedDynamicKVCache.get_all_keys_values

    def counting(self):
        rebuilt.append(1)
        return real(self)

    with torch.no_grad():
        a = ref_model(ids, past_key_values=ref_cache, use_cache=True).logits
        b = fused_model(ids, past_key_values=fused_cache, use_cache=True).logits
        assert (a.float() - b.float()).abs().max() <= 1e-3
        monkeypatch.setattr(PagedDynamicKVCache, "get_all_keys_values", counting)
        worst = 0.0
        for t in range(steps.shape[1]):
            tok = steps[:, t:t + 1]
            n_before = len(rebuilt)
            a = ref_model(tok, past_key_values=ref_cache, use_cache=True).logits
            assert len(rebuilt) > n_before
            n_before = len(rebuilt)
            b = fused_model(tok, past_key_values=fused_cache, use_cache=True).logits
            assert len(rebuilt) == n_before, "fused decode rebuilt K/V"
            worst = max(worst, float((a.float() - b.float()).abs().max()))
    c0 = fused_cache.layer_caches[0]
    assert len(c0.jl_pages) >= 1 and len(c0.one_bit_pages) == 1
    assert fused_cache.get_seq_length(0) == ref_cache.get_seq_length(0) == 154
    assert worst <= atol, worst


def test_attend_follows_single_token_appends(tmp_path, monkeypatch):
    """Decode-style pushes of one token: attend() stays on float64 attention over the rebuilt K/V
    (get_all_keys_values) through tile and page boundaries, and within a 16-token tile of the
    staging buffer it reuses its launch tables (the buffer tile's token count is patched)."""
    import oracle
    from argus_b200.core.memory_manager import PagedDynamicKVCache
    monkeypatch.setenv("ARGUS_LOG_LEVEL", "quiet")
    monkeypatch.chdir(tmp_path)
    B, H, G, D = 1, 2, 4, 64
    cache = PagedDynamicKVCache(page_size=32, max_active_pages=1, max_fp8_pages=1, max_int8_pages=1,
                                max_int4_pages=1, max_int2_pages=1, max_one_bit_pages=1, sink_tokens=4)
    g = torch.Generator().manual_seed(9)
    kv = lambda n: (torch.randn(B, H, n, D, generator=g) * 1.5).half().cuda()  # noqa: E731
    cache.push_new_tokens(kv(200), kv(200))
    plans = []
    for step in range(40):
        cache.push_new_tokens(kv(1), kv(1))
        q = (torch.randn(B, H * G, 1, D, generator=g) / 8).half()
        out = host(cache.attend(q.cuda())).astype(np.float64)
        K, V = cache.get_all_keys_values()
        ref = oracle.sdpa_f64(q.numpy(), host(K), host(V), 1.0 / math.sqrt(D))
        bar = 2e-3 + np.abs(ref) * 2.0 ** -11
        assert (np.abs(out - ref) <= bar).all(), (step, np.abs(out - ref).max())
        plans.append((id(cache._plan), cache.buffer_length))
    # consecutive steps inside one buffer tile share the launch tables
    same = sum(1 for (a, na), (b, nb) in zip(plans, plans[1:]) if (na - 1) // 16 == (nb - 1) // 16 and nb > na)
    reused = sum(1 for (a, na), (b, nb) in zip(plans, plans[1:])
                 if (na - 1) // 16 == (nb - 1) // 16 and nb > na and a == b)
    assert same > 20 and reused == same
    assert any(pg.get("key_out_indices") is not None and pg["key_out_indices"].numel()
               for _, lst in cache._compressed_order() for pg in lst)


def test_attend_causal_queries_of_the_newest_tokens(tmp_path, monkeypatch):
    """attend(causal=True) for steps of several tokens: query i sees the cached tokens up to its
    own (bottom-right causal mask over the rebuilt K/V), through page formation and demotions."""
    import oracle
    from argus_b200.core.memory_manager import PagedDynamicKVCache
    monkeypatch.setenv("ARGUS_LOG_LEVEL", "quiet")
    monkeypatch.chdir(tmp_path)
    B, H, G, D = 2, 2, 4, 64
    cache = PagedDynamicKVCache(page_size=32, max_active_pages=1, max_fp8_pages=1, max_int8_pages=1,
                                max_int4_pages=1, max_int2_pages=1, max_one_bit_pages=1, sink_tokens=4)
    g = torch.Generator().manual_seed(11)
    kv = lambda n: (torch.randn(B, H, n, D, generator=g) * 1.5).half().cuda()  # noqa: E731
    scale = 1.0 / math.sqrt(D)
    checked = 0
    for pushes in ([200, 3], [200, 5, 4], [30, 40], [6]):
        for n in pushes:
            cache.push_new_tokens(kv(n), kv(n))
        ql = pushes[-1]
        q = (torch.randn(B, H * G, ql, D, generator=g) / 8).half()
        out = host(cache.attend(q.cuda(), causal=True)).astype(np.float64)
        K, V = (host(t) for t in cache.get_all_keys_values())
        L = K.shape[-2]
        ref = np.stack([oracle.sdpa_f64(q.numpy()[:, :, i:i + 1], K[:, :, :L - ql + i + 1], V[:, :, :L - ql + i + 1],
                                        scale)[:, :, 0] for i in range(ql)], axis=2)
        bar = 2e-3 + np.abs(ref) * 2.0 ** -10
        assert (np.abs(out - ref) <= bar).all(), (pushes, np.abs(out - ref).max())
        checked += 1
        # a decode step after the causal one sees every cached token
        q1 = (torch.randn(B, H * G, 1, D, generator=g) / 8).half()
        out1 = host(cache.attend(q1.cuda())).astype(np.float64)
        ref1 = oracle.sdpa_f64(q1.numpy(), K, V, scale)
        assert (np.abs(out1 - ref1) <= 2e-3 + np.abs(ref1) * 2.0 ** -11).all()
    assert checked == 4


def test_fused_steps_of_several_tokens_match_materializing_adapter(tmp_path, monkeypatch):
    """Chunked decode (3 tokens a step) through the "argus" attention: steps whose tokens are in
    the staging buffer run fused without rebuilding K/V and match the materializing adapter."""
    from argus_b200.core.memory_manager import PagedDynamicKVCache
    monkeypatch.setenv("ARGUS_LOG_LEVEL", "quiet")
    monkeypatch.chdir(tmp_path)
    ref_model, fused_model = _models(1, 256, 8, 2, 32)
    ref_cache, fused_cache = _cache(False), _cache(True)
    g = torch.Generator(device="cuda").manual_seed(5)
    ids = torch.randint(0, 256, (1, 120), device="cuda", generator=g)
    steps = torch.randint(0, 256, (1, 24), device="cuda", generator=g)
    rebuilt = []
    real = PagedDynamicKVCache.get_all_keys_values

    def counting(self):
        rebuilt.append(1)
        return real(self)

    fused_steps, worst = 0, 0.0
    with torch.no_grad():
        a = ref_model(ids, past_key_values=ref_cache, use_cache=True).logits
        b = fused_model(ids, past_key_values=fused_cache, use_cache=True).logits
        assert (a.float() - b.float()).abs().max() <= 1e-3
        monkeypatch.setattr(PagedDynamicKVCache, "get_all_keys_values", counting)
        for t in range(0, steps.shape[1], 3):
            tok = steps[:, t:t + 3]
            a = ref_model(tok, past_key_values=ref_cache, use_cache=True).logits
            n_before = len(rebuilt)
            b = fused_model(tok, past_key_values=fused_cache, use_cache=True).logits
            fused_steps += len(rebuilt) == n_before
            worst = max(worst, float((a.float() - b.float()).abs().max()))
    assert fused_cache.get_seq_length(0) == ref_cache.get_seq_length(0) == 144
    assert fused_steps >= 4, fused_steps
    assert worst <= 1e-2, worst



def test_decode_steps_across_demotions_keep_the_launch_tables(tmp_path, monkeypatch):
    """The launch tables cover every pool slot and the staging buffer's capacity: single-token decode
    steps that cross new 16-token tiles, page formations, demotions down the cascade (no JL) and
    resurrections only update the device occupancy and a token count, so after the first step no
    table is rebuilt; attention stays within the bar of float64 attention over the rebuilt K/V and
    inplace_paged_attention keeps taking its per-page masses from the same launch."""
    import time

    import oracle
    from argus_b200.core.memory_manager import PagedDynamicKVCache
    monkeypatch.setenv("ARGUS_LOG_LEVEL", "quiet")
    monkeypatch.chdir(tmp_path)
    B, H, G, D = 1, 2, 4, 64
    # tiers with room enough that the cascade (and the resurrections' churn) stays above the JL archive,
    # which 16-token pages attend through the scratch arena and so would rebuild the tables
    cache = PagedDynamicKVCache(page_size=16, max_active_pages=4, max_fp8_pages=4, max_int8_pages=4,
                                max_int4_pages=4, max_int2_pages=4, max_one_bit_pages=16, sink_tokens=4)
    g = torch.Generator().manual_seed(13)
    kv = lambda n: (torch.randn(B, H, n, D, generator=g) * 1.5).half().cuda()  # noqa: E731
    cache.push_new_tokens(kv(100), kv(100))
    q0 = (torch.randn(B, H * G, 1, D, generator=g) / 8).half().cuda()
    cache.attend(q0)
    builds = cache.plan_builds
    demotions = cache.total_demotions
    times = []
    for step in range(60):
        cache.push_new_tokens(kv(1), kv(1))
        q = (torch.randn(B, H * G, 1, D, generator=g) / 8).half()
        # the reference K/V before the call: inplace_paged_attention may resurrect pages afterwards
        K, V = cache.get_all_keys_values()
        ref = oracle.sdpa_f64(q.numpy(), host(K), host(V), 1.0 / math.sqrt(D))
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = cache.attend(q.cuda()) if step % 2 else cache.inplace_paged_attention(q.cuda())
        torch.cuda.synchronize()
        times.append(time.perf_counter() - t0)
        got = host(out).astype(np.float64)
        bar = 2e-3 + np.abs(ref) * 2.0 ** -11
        assert (np.abs(got - ref) <= bar).all(), (step, np.abs(got - ref).max())
    assert not cache.jl_pages
    assert cache.total_demotions - demotions >= 3  # pages formed and moved down the cascade meanwhile
    assert cache.num_resurrections > 0
    assert cache.plan_builds == builds, (cache.plan_builds, builds)


def test_causal_steps_that_form_pages_run_fused(tmp_path, monkeypatch):
    """A step of several tokens whose tokens just formed a page (the masked tail of the concatenation
    reaches one or two active pages past the staging buffer): attend(causal=True) runs the fused kernel
    with those pages' slots left out and attends them with the step's causal part, matching float64
    attention over the rebuilt K/V under the bottom-right causal mask."""
    import oracle
    from argus_b200.core.memory_manager import PagedDynamicKVCache
    monkeypatch.setenv("ARGUS_LOG_LEVEL", "quiet")
    monkeypatch.chdir(tmp_path)
    B, H, G, D = 2, 2, 4, 64
    cache = PagedDynamicKVCache(page_size=16, max_active_pages=4, max_fp8_pages=2, max_int8_pages=2,
                                max_int4_pages=2, max_int2_pages=2, max_one_bit_pages=8, sink_tokens=4)
    g = torch.Generator().manual_seed(17)
    kv = lambda n: (torch.randn(B, H, n, D, generator=g) * 1.5).half().cuda()  # noqa: E731
    scale = 1.0 / math.sqrt(D)
    cache.push_new_tokens(kv(4 + 16 * 6 + 14), kv(4 + 16 * 6 + 14))  # sinks, 6 pages, 14 in the buffer
    fused_before = cache.fused_causal_page_steps
    for ql, want_pages in ((3, 1), (40, 2), (5, 0)):
        cache.push_new_tokens(kv(ql), kv(ql))
        assert cache.causal_tail_pages(ql) == want_pages, (ql, cache.buffer_length)
        q = (torch.randn(B, H * G, ql, D, generator=g) / 8).half()
        K, V = (host(t) for t in cache.get_all_keys_values())
        out = host(cache.attend(q.cuda(), causal=True)).astype(np.float64)
        L = K.shape[-2]
        ref = np.stack([oracle.sdpa_f64(q.numpy()[:, :, i:i + 1], K[:, :, :L - ql + i + 1], V[:, :, :L - ql + i + 1],
                                        scale)[:, :, 0] for i in range(ql)], axis=2)
        bar = 2e-3 + np.abs(ref) * 2.0 ** -10
        assert (np.abs(out - ref) <= bar).all(), (ql, np.abs(out - ref).max())
    assert cache.fused_causal_page_steps - fused_before == 2
    # the occupancy the launch borrowed is back: a decode step sees every cached token
    q1 = (torch.randn(B, H * G, 1, D, generator=g) / 8).half()
    K, V = (host(t) for t in cache.get_all_keys_values())
    out1 = host(cache.attend(q1.cuda())).astype(np.float64)
    ref1 = oracle.sdpa_f64(q1.numpy(), K, V, scale)
    assert (np.abs(out1 - ref1) <= 2e-3 + np.abs(ref1) * 2.0 ** -11).all()
