"""GPU replay of the reference's PagedDynamicKVCache runs (tests/golden/cascade.npz): the same pushes
must give the same tier occupancy, page ids, page payloads and sidecars (bit for bit), the same
get_all_keys_values output (bit for bit; JL-archived rows within fp16 matmul rounding), attention
within the attention bar, and the same resurrections."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

RUNS = {
    # name: (page_size, max pages per tier, sink tokens, sigma) as in make_golden.gen_cascade
    "t1": (8, 1, 8, 3.0),
    "t2": (16, 2, 4, 3.0),
}
TIERS = ("fp16", "fp8", "int8", "int4", "int2", "one_bit", "jl")
ATTR = {"fp16": "active_pages", "fp8": "fp8_pages", "int8": "int8_pages", "int4": "int4_pages", "int2": "int2_pages",
        "one_bit": "one_bit_pages", "jl": "jl_pages"}


def host(t):
    return t.detach().cpu().contiguous().numpy()


def replay(z, name, tmp_path):
    from argus_b200.core.memory_manager import PagedDynamicKVCache
    P, maxp, sinks, sigma = RUNS[name]
    os.environ["ARGUS_LOG_LEVEL"] = "quiet"
    cwd = os.getcwd()
    os.chdir(tmp_path)  # the manager appends its event trace under ./tests
    try:
        cache = PagedDynamicKVCache(page_size=P, max_active_pages=maxp, max_fp8_pages=maxp, max_int8_pages=maxp,
                                    max_int4_pages=maxp, max_int2_pages=maxp, max_one_bit_pages=maxp,
                                    sink_tokens=sinks, threshold_sigma=sigma)
        for i in range(int(z[f"{name}/n_pushes"])):
            cache.push_new_tokens(torch.from_numpy(z[f"{name}/push{i}/k"]).cuda(),
                                  torch.from_numpy(z[f"{name}/push{i}/v"]).cuda())
    finally:
        os.chdir(cwd)
    return cache


def counts(cache):
    return [len(getattr(cache, ATTR[t])) for t in TIERS]


@pytest.mark.parametrize("name", list(RUNS))
def test_cascade_replay_bit_exact(golden, name, tmp_path):
    z = golden("cascade")
    cache = replay(z, name, tmp_path)
    assert counts(cache) == list(z[f"{name}/tier_counts"])
    for tier in TIERS:
        pages = getattr(cache, ATTR[tier])
        assert [p["page_id"] for p in pages] == list(z[f"{name}/{tier}/page_ids"]), tier
        for j, page in enumerate(pages):
            for field, val in page.items():
                key = f"{name}/{tier}/{j}/{field}"
                if not isinstance(val, torch.Tensor) or key not in z:
                    continue
                got, ref = host(val), z[key]
                assert got.shape == ref.shape, (key, got.shape, ref.shape)
                if field in ("key_proj", "value_proj"):
                    np.testing.assert_allclose(got.astype(np.float32), ref.astype(np.float32), rtol=2e-3, atol=2e-3)
                elif got.dtype == np.float16:
                    assert (got.view(np.uint16) == ref.view(np.uint16)).all(), key
                else:
                    assert (got == ref).all(), key


@pytest.mark.parametrize("name", list(RUNS))
def test_get_all_keys_values(golden, name, tmp_path):
    z = golden("cascade")
    cache = replay(z, name, tmp_path)
    K, V = cache.get_all_keys_values()
    Kr, Vr = z[f"{name}/K"], z[f"{name}/V"]
    assert K.shape == Kr.shape and V.shape == Vr.shape
    P = RUNS[name][0]
    sinks = RUNS[name][2]
    n_jl = len(cache.jl_pages)
    jl = slice(sinks, sinks + n_jl * P)
    for got, ref in ((host(K), Kr), (host(V), Vr)):
        np.testing.assert_allclose(got[:, :, jl].astype(np.float32), ref[:, :, jl].astype(np.float32), atol=4e-3,
                                   rtol=4e-3)
        rest = np.ones(got.shape[2], bool)
        rest[jl] = False
        assert (got[:, :, rest].view(np.uint16) == ref[:, :, rest].view(np.uint16)).all()


@pytest.mark.parametrize("name", list(RUNS))
def test_inplace_attention_and_resurrection(golden, name, tmp_path):
    import math
    import oracle
    z = golden("cascade")
    cache = replay(z, name, tmp_path)
    q = z[f"{name}/q"]
    Kr, Vr = z[f"{name}/K"], z[f"{name}/V"]
    out = host(cache.inplace_paged_attention(torch.from_numpy(q).cuda())).astype(np.float64)
    ref = oracle.sdpa_f64(q, Kr, Vr, 1.0 / math.sqrt(q.shape[-1]))
    bar = 2e-3 + np.abs(ref) * 2.0 ** -11 + 4e-3 * (len(cache.jl_pages) > 0)
    assert (np.abs(out - ref) <= bar).all(), np.abs(out - ref).max()
    ref16 = z[f"{name}/attn"].astype(np.float64)
    assert (np.abs(out - ref16) <= bar + np.abs(ref - ref16)).all()
    assert counts(cache) == list(z[f"{name}/tier_counts_after_attn"])


def test_hf_adapter_matches_dynamic_cache_before_compression():
    """With pages larger than the prompt, every token stays in the fp16 staging buffer, so a model
    decoding through PagedDynamicQuantizedCache must produce the same logits as DynamicCache."""
    transformers = pytest.importorskip("transformers")
    from argus_b200.models.attention_wrapper import PagedDynamicQuantizedCache
    cfg = transformers.LlamaConfig(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256)
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(cfg).cuda().half().eval()
    ids = torch.randint(0, 128, (1, 24), device="cuda")
    with torch.no_grad():
        ref = model(ids, past_key_values=transformers.DynamicCache(), use_cache=True).logits
        ours = model(ids, past_key_values=PagedDynamicQuantizedCache(page_size=64, sink_tokens=4), use_cache=True).logits
    assert torch.allclose(ref.float(), ours.float(), atol=1e-3)


def test_hf_adapter_decodes_through_the_cascade():
    """A short generation with tiny pages runs every tier transition through the adapter."""
    transformers = pytest.importorskip("transformers")
    from argus_b200.models.attention_wrapper import PagedDynamicQuantizedCache
    cfg = transformers.LlamaConfig(vocab_size=128, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=512)
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(cfg).cuda().half().eval()
    cache = PagedDynamicQuantizedCache(page_size=16, max_active_pages=1, max_fp8_pages=1, max_int8_pages=1,
                                       max_int4_pages=1, max_int2_pages=1, max_one_bit_pages=1, sink_tokens=4)
    ids = torch.randint(0, 128, (1, 130), device="cuda")
    with torch.no_grad():
        out = model(ids, past_key_values=cache, use_cache=True)
        for _ in range(20):
            nxt = out.logits[:, -1:].argmax(-1)
            out = model(nxt, past_key_values=cache, use_cache=True)
    c0 = cache.layer_caches[0]
    assert len(c0.jl_pages) >= 1 and len(c0.one_bit_pages) == 1
    assert cache.get_seq_length(0) == 150
    assert torch.isfinite(out.logits).all()
