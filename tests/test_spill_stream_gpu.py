"""Attention over a spilled (pinned host) record arena streamed through device staging buffers
(StreamedArenaAttention) equals attention over the same arena resident in HBM, within the
attention bar, and the float64 reference; runs of every length, including a short last run."""
import math

import numpy as np
import pytest
import torch

import attn_util as U

pytestmark = pytest.mark.gpu
ATOL = 2e-3


@pytest.mark.parametrize("tier,chunk", [("one_bit", 16), ("int4", 7), ("int8", 40), ("fp16", 5)])
def test_streamed_spilled_tier_matches_resident(tier, chunk):
    from argus_b200 import attention as A
    from argus_b200 import spill
    B, Hkv, G, D, P, n = 2, 2, 4, 128, 16, 40
    rng = np.random.default_rng(3)
    pages = U.random_pages(rng, [(tier, n * P)], B, Hkv, D, P)
    arenas, plist = U.arenas_from_pages(pages)
    q = torch.from_numpy((rng.standard_normal((B, Hkv * G, 1, D)) / math.sqrt(D)).astype(np.float16)).cuda()
    plan = A.AttentionPlan(arenas, plist, batch=B, heads_kv=Hkv, group=G, head_dim=D)
    lse_ref = torch.empty(B, Hkv * G, 1, dtype=torch.float32, device="cuda")
    ref = plan.run(q, lse=lse_ref)
    host = spill.arenas_to_host(arenas)[0]
    st = spill.StreamedArenaAttention(host, group=G, chunk_slots=chunk)
    for _ in range(2):  # the staging buffers are reused across calls
        out, lse = st.run(q)
        torch.cuda.synchronize()
        assert A.device_status() == 0
        a, b = out.cpu().numpy().astype(np.float64), ref.cpu().numpy().astype(np.float64)
        assert (np.abs(a - b) <= ATOL + np.abs(b) * 2.0 ** -11).all(), np.abs(a - b).max()
        assert torch.allclose(lse, lse_ref, rtol=0, atol=1e-4)
    K, V = U.reference_kv(pages)
    f64 = U.f64_attention(q.cpu().numpy(), K, V)
    got = out.cpu().numpy().astype(np.float64)
    assert (np.abs(got - f64) <= ATOL + np.abs(f64) * 2.0 ** -11).all(), np.abs(got - f64).max()


# ------------------------------------------- a layer sharded by KV head with its oldest tier spilled
LB, LHKV, LG, LD, LP = 2, 4, 4, 128, 16
LTIERS = [("one_bit", 640), ("int2", 256), ("int4", 256), ("int8", 128), ("fp8", 96), ("fp16", 32)]
CHUNK, SPLITS = 12, 2  # runs of 12 slots (a short last run), fixed split count for every launch


def _layer(device):
    from argus_b200 import attention as A
    rng = np.random.default_rng(21)
    pages = U.random_pages(rng, LTIERS, LB, LHKV, LD, LP, outlier_frac=0.0)
    arenas, plist = U.arenas_from_pages(pages, device=device, sidecars=False)
    q = torch.from_numpy((rng.standard_normal((LB, LHKV * LG, 1, LD)) / math.sqrt(LD)).astype(np.float16)).to(device)
    return pages, arenas, plist, q


def _decode(arenas, plist, heads_kv, spilled_on_host):
    """Resident tiers in one launch, the 1-bit arena (arena 0) streamed in runs, joined by LSE."""
    from argus_b200 import attention as A
    from argus_b200 import spill
    res = arenas[1:]
    res_pages = [(ai - 1, s, n) for ai, s, n in plist if ai != 0]
    plan = A.AttentionPlan(res, res_pages, batch=LB, heads_kv=heads_kv, group=LG, head_dim=LD, n_splits=SPLITS)
    src = spill.arenas_to_host([arenas[0]])[0] if spilled_on_host else arenas[0]
    return spill.SpilledLayerDecode(plan, src, chunk_slots=CHUNK, n_splits=SPLITS)


def test_sharded_spilled_layer_equals_resident_unsharded_bit_for_bit():
    """Every rank's shard (2 and 4 ranks, run in turn on one GPU) with its 1-bit arena in pinned host
    memory and streamed gives, concatenated by head, the bits of the unsharded layer with that arena
    resident (the same runs and splits); the result is within the attention bar of float64
    attention over the oracle's rebuild."""
    from argus_b200 import attention as A
    from argus_b200 import sharding
    pages, arenas, plist, q = _layer("cuda")
    ref = _decode(arenas, plist, LHKV, spilled_on_host=False)(q)
    for world in (2, 4):
        parts = []
        for rank in range(world):
            shard = [sharding.shard_arena(a, world, rank) for a in arenas]
            step = _decode(shard, plist, LHKV // world, spilled_on_host=True)
            parts.append(step(sharding.shard_queries(q, LHKV, world, rank)))
        got = torch.cat(parts, dim=1)
        torch.cuda.synchronize()
        assert A.device_status() == 0
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), world
    K, V = U.reference_kv(pages)
    f64 = U.f64_attention(q.cpu().numpy(), K, V)
    r = ref.cpu().numpy().astype(np.float64)
    # two fp16 partial results joined: one more output half-ulp
    assert (np.abs(r - f64) <= ATOL + np.abs(f64) * 2.0 ** -10).all(), np.abs(r - f64).max()


def _rank_layer_main(rank, world, port, result_path):
    import datetime
    import os

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from argus_b200 import attention as A
        from argus_b200 import sharding
        pages, arenas, plist, q = _layer(dev)
        ref = _decode(arenas, plist, LHKV, spilled_on_host=False)(q)
        shard = [sharding.shard_arena(a, world, rank) for a in arenas]
        step = _decode(shard, plist, LHKV // world, spilled_on_host=True)
        gather = sharding.HeadShardedDecode(step.plan, LHKV)
        got = gather.gather(step(sharding.shard_queries(q, LHKV, world, rank)))
        torch.cuda.synchronize()
        ok = int(torch.equal(got.view(torch.int16), ref.view(torch.int16)) and A.device_status() == 0)
        t = torch.tensor([ok], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        if rank == 0:
            with open(result_path, "w") as f:
                f.write("ok" if int(t.item()) == 1 else "mismatch")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_spilled_layer_over_nccl_two_gpus(tmp_path):
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    path = str(tmp_path / "result.txt")
    mp.start_processes(_rank_layer_main, args=(2, port, path), nprocs=2, join=True, start_method="spawn")
    with open(path) as f:
        assert f.read() == "ok"
