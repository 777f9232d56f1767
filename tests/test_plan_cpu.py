"""Host-side planning of the fused decode attention (no GPU): chunk formation from page lists,
chunk capacities per tier, split boundaries and record-view geometry."""
import numpy as np
import torch

from argus_b200 import attention as A


def arena(tier, slots, P=16, D=128, B=2, H=2):
    rec = A.record_bytes(tier, P, D)
    buf = torch.zeros(B * H, slots, rec, dtype=torch.uint8)
    return A.KVArena(tier, A.LAYOUT_RECORD, buf, None, bh_stride=slots * rec, record_bytes=rec, page_tokens=P,
                     head_dim=D, batch=B, heads=H, slots=slots)


def chunks_of(plan):
    return [tuple(c) for c in plan.chunks]


def test_record_sizes_and_capacity():
    D, P = 128, 16
    assert [A.record_bytes(t, P, D) for t in range(6)] == [8192, 4160, 4160, 2176, 1152, 576]
    caps = [A.chunk_capacity(arena(t, 4), D) for t in range(6)]
    assert caps == [1, 2, 2, 4, 7, 15]


def test_consecutive_slots_merge_up_to_capacity():
    a = arena(A.TIER_INT4, 10)
    plan = A.AttentionPlan([a], [(0, s, 16) for s in range(10)], batch=2, heads_kv=2, group=4, head_dim=128,
                           n_splits=1)
    assert chunks_of(plan) == [(0, 0, 0, 4, 16), (4, 0, 0, 4, 16), (8, 0, 0, 2, 16)]
    # a gap in slots starts a new chunk
    plan = A.AttentionPlan([a], [(0, s, 16) for s in (0, 1, 5, 6)], batch=2, heads_kv=2, group=4, head_dim=128,
                           n_splits=1)
    assert chunks_of(plan) == [(0, 0, 0, 2, 16), (5, 0, 0, 2, 16)]


def test_large_pages_tile_within_a_slot():
    a = arena(A.TIER_INT8, 2, P=80)
    plan = A.AttentionPlan([a], [(0, 0, 80), (0, 1, 80)], batch=2, heads_kv=2, group=4, head_dim=128, n_splits=1)
    cap = A.chunk_capacity(a, 128)
    assert cap == 2
    # (the plan may place the chunks in any order to balance its warps)
    assert sorted(chunks_of(plan)) == [(0, 0, 0, 2, 16), (0, 32, 0, 2, 16), (0, 64, 0, 1, 16),
                                       (1, 0, 0, 2, 16), (1, 32, 0, 2, 16), (1, 64, 0, 1, 16)]


def test_split_fp16_partial_closes_chunk():
    k = torch.zeros(2, 2, 40, 64, dtype=torch.float16)
    a = A.KVArena(A.TIER_FP16, A.LAYOUT_SPLIT_FP16, k, k.clone(), bh_stride=40 * 64 * 2, page_tokens=16, head_dim=64,
                  batch=2, heads=2, slots=3)
    plan = A.AttentionPlan([a], [(0, 0, 16), (0, 1, 16), (0, 2, 8)], batch=2, heads_kv=2, group=2, head_dim=64,
                           n_splits=1)
    assert chunks_of(plan) == [(0, 0, 0, 2, 16), (2, 0, 0, 1, 8)]


def test_splits_cover_chunks_in_order():
    arenas = [arena(t, 64) for t in (A.TIER_1BIT, A.TIER_INT2, A.TIER_INT4, A.TIER_FP16)]
    pages = [(i, s, 16) for i in range(4) for s in range(64)]
    plan = A.AttentionPlan(arenas, pages, batch=2, heads_kv=2, group=4, head_dim=128, n_splits=5)
    b = plan.splits_dev.numpy()
    assert b[0] == 0 and b[-1] == plan.n_chunks and (np.diff(b) >= 0).all() and len(b) == 6
    assert plan.n_tokens == 4 * 64 * 16
    # algorithmic bytes: per token K+V payload + scales/mins, over B*H
    per_tok = {A.TIER_1BIT: 2 * 16 + 4, A.TIER_INT2: 2 * 32 + 8, A.TIER_INT4: 2 * 64 + 8, A.TIER_FP16: 2 * 256}
    assert plan.compressed_bytes == sum(per_tok.values()) * 64 * 16 * 4


def test_splits_take_a_share_of_every_arena_in_the_same_order():
    arenas = [arena(t, 96) for t in (A.TIER_1BIT, A.TIER_INT2, A.TIER_INT4, A.TIER_INT8)]
    pages = [(i, s, 16) for i in range(4) for s in range(96)]
    plan = A.AttentionPlan(arenas, pages, batch=2, heads_kv=2, group=4, head_dim=128, n_splits=7)
    b = plan.splits_dev.numpy()
    costs = []
    for s in range(7):
        part = plan.chunks[b[s]:b[s + 1]]
        seq = [c[2] for c in part]
        for w in range(A.CTA_WARPS):  # each warp meets the arenas in the same order
            assert seq[w::A.CTA_WARPS] == sorted(seq[w::A.CTA_WARPS])
        assert set(seq) == {0, 1, 2, 3}  # a share of every arena
        costs.append(sum(A._tile_cost(arenas[c[2]].tier, 128, 16 * c[3]) for c in part))
    assert max(costs) - min(costs) <= max(A._tile_cost(t, 128, 16 * 16) for t in range(6))
    # every page's tiles are covered once, in page order within a chunk
    seen = sorted(pi for src in plan.chunk_pages for pi in src)
    assert seen == list(range(len(pages)))


def test_record_views_share_storage():
    a = arena(A.TIER_INT4, 3, P=16, D=64)
    ks = a.view("ks", 1)
    assert ks.shape == (2, 2, 16, 1)
    ks.fill_(1.5)
    kp = a.view("k", 1)
    assert kp.shape == (2, 2, 8, 64) and kp.dtype == torch.uint8
    kp.fill_(7)
    raw = a.k.view(2 * 2, 3, -1)
    rec = A.record_bytes(A.TIER_INT4, 16, 64)
    assert (raw[:, 1, :512] == 7).all() and (raw[:, 0] == 0).all() and (raw[:, 2] == 0).all()
    assert (raw[:, 1, 1024:1056].view(torch.float16) == 1.5).all() and rec == 1024 + 128


def test_warps_of_a_split_get_balanced_costs():
    """The kernel deals a split's chunks to its warps by position (i % 4); the plan places them so
    the warps' costs differ by at most one chunk's, on a layer with every tier (chunk capacities
    from 15 one-bit tiles down to one fp16 tile)."""
    tiers = [(A.TIER_1BIT, 512), (A.TIER_INT2, 512), (A.TIER_INT4, 512), (A.TIER_INT8, 256), (A.TIER_FP8SIM, 192),
             (A.TIER_FP16, 64)]
    arenas = [arena(t, n) for t, n in tiers]
    pages = [(i, s, 16) for i, (_, n) in enumerate(tiers) for s in range(n)]
    plan = A.AttentionPlan(arenas, pages, batch=1, heads_kv=1, group=8, head_dim=128, n_splits=9)
    b = plan.splits_dev.numpy()
    for s in range(9):
        part = plan.chunks[b[s]:b[s + 1]]
        cost = [A._tile_cost(arenas[c[2]].tier, 128, 16 * c[3]) for c in part]
        warps = [sum(cost[w::A.CTA_WARPS]) for w in range(A.CTA_WARPS)]
        assert max(warps) - min(warps) <= max(cost) + 1e-9, warps
