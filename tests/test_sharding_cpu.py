"""KV-head sharding on CPU: head ranges, arena shards that keep the page table valid, and the
output all-gather across a world of 2 gloo ranks (each rank's local attention computed by the
float64 oracle), which must equal attention over all heads at once."""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from argus_b200 import attention as A
from argus_b200 import sharding


def test_head_range_and_query_shard():
    assert [sharding.head_range(8, 4, r) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        sharding.head_range(6, 4, 0)
    with pytest.raises(ValueError):
        sharding.head_range(8, 2, 2)
    q = torch.arange(2 * 8 * 1 * 4, dtype=torch.float32).view(2, 8, 1, 4)  # 8 query heads, 4 KV heads
    q1 = sharding.shard_queries(q, 4, 2, 1)
    assert torch.equal(q1, q[:, 4:8])


def _cpu_arena(tier, B, H, slots, P, D, seed):
    rec = A.record_bytes(tier, P, D)
    g = torch.Generator().manual_seed(seed)
    buf = torch.randint(0, 256, (B * H, slots, rec), generator=g, dtype=torch.uint8)
    return A.KVArena(tier, A.LAYOUT_RECORD, buf, None, bh_stride=slots * rec, record_bytes=rec, page_tokens=P,
                     head_dim=D, batch=B, heads=H, slots=slots)


@pytest.mark.parametrize("tier", [A.TIER_FP16, A.TIER_INT8, A.TIER_INT4, A.TIER_1BIT])
def test_shard_arena_keeps_every_page_view(tier):
    B, H, S, P, D = 2, 4, 3, 16, 64
    full = _cpu_arena(tier, B, H, S, P, D, seed=tier)
    parts = ["k", "v"] + (["ks", "vs"] if tier != A.TIER_FP16 else []) + (["km", "vm"] if tier == A.TIER_INT4 else [])
    for world in (2, 4):
        for rank in range(world):
            sh = sharding.shard_arena(full, world, rank)
            h0, h1 = sharding.head_range(H, world, rank)
            assert sh.H == h1 - h0 and sh.slots == S and sh.record_bytes == full.record_bytes
            for slot in range(S):
                for part in parts:
                    a, b = sh.view(part, slot), full.view(part, slot)[:, h0:h1]
                    if a.dtype == torch.float16:  # random bytes: compare bit patterns (NaNs included)
                        a, b = a.contiguous().view(torch.int16), b.contiguous().view(torch.int16)
                    assert torch.equal(a, b), (world, rank, part)


class _OraclePlan:
    """Stand-in for a rank's AttentionPlan on CPU: float64 attention over this rank's heads."""

    def __init__(self, K, V):
        self.K, self.V = K, V

    def run(self, q, scale=None, out=None):
        import oracle
        D = q.shape[-1]
        res = oracle.sdpa_f64(q.numpy(), self.K, self.V, 1.0 / math.sqrt(D) if scale is None else scale)
        res = torch.from_numpy(np.ascontiguousarray(res))
        if out is None:
            return res
        out.copy_(res)  # like AttentionPlan.run: the output lands in the caller's buffer
        return out


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        rng = np.random.default_rng(7)
        B, Hkv, G, L, D = 2, 4, 3, 40, 16
        K = rng.standard_normal((B, Hkv, L, D))
        V = rng.standard_normal((B, Hkv, L, D))
        q = torch.from_numpy(rng.standard_normal((B, Hkv * G, 1, D)))
        h0, h1 = sharding.head_range(Hkv, world, rank)
        step = sharding.HeadShardedDecode(_OraclePlan(K[:, h0:h1], V[:, h0:h1]), Hkv)
        out = step(q).clone()
        out2 = step(q)  # the gather buffers are reused
        if rank == 0:
            import oracle
            ref = oracle.sdpa_f64(q.numpy(), K, V, 1.0 / math.sqrt(D))
            ok = out.shape == (B, Hkv * G, 1, D) and np.allclose(out.numpy(), ref, rtol=0, atol=1e-12) \
                and torch.equal(out, out2)
            with open(result_path, "w") as f:
                f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


def test_head_sharded_gather_matches_full_attention_world2(tmp_path):
    path = str(tmp_path / "result.txt")
    mp.start_processes(_rank_main, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    with open(path) as f:
        assert f.read() == "ok"


def _rank_leaves_main(rank, world, port, result_path):
    """Both ranks run one sharded step; rank 1 then leaves between steps (no collective in flight)
    and rank 0's next step must end with an error within the process group's short timeout."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import time
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    rng = np.random.default_rng(3)
    B, Hkv, G, L, D = 1, 2, 2, 24, 16
    K = rng.standard_normal((B, Hkv, L, D))
    V = rng.standard_normal((B, Hkv, L, D))
    q = torch.from_numpy(rng.standard_normal((B, Hkv * G, 1, D)))
    h0, h1 = sharding.head_range(Hkv, world, rank)
    step = sharding.HeadShardedDecode(_OraclePlan(K[:, h0:h1], V[:, h0:h1]), Hkv)
    step(q)
    if rank == 1:
        return  # leaves without joining the next step
    t0 = time.monotonic()
    try:
        step(q)
        outcome = "completed"
    except Exception as e:  # gloo reports the lost peer or the timeout
        outcome = f"raised {type(e).__name__} after {time.monotonic() - t0:.1f} s"
    with open(result_path, "w") as f:
        f.write(outcome)


def test_a_rank_leaving_between_steps_ends_the_next_step_with_an_error(tmp_path):
    path = str(tmp_path / "result.txt")
    mp.start_processes(_rank_leaves_main, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    with open(path) as f:
        outcome = f.read()
    assert outcome.startswith("raised"), outcome
    assert float(outcome.split()[-2]) < 30.0
