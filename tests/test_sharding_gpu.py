"""KV-head sharding on GPUs: per-rank plans over shard_arena() copies reproduce the full cache's
attention bit for bit (same chunks per (batch, kv_head), one split), on one GPU by running every
rank's shard in turn, and on two GPUs through HeadShardedDecode's NCCL all-gather (skipped with
fewer than two GPUs)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import attn_util as U

pytestmark = pytest.mark.gpu

B, HKV, G, D, P = 2, 4, 4, 128, 16
TIERS = [("one_bit", 64), ("int2", 64), ("int4", 64), ("int8", 32), ("fp8", 32), ("fp16", 32)]


def build(device):
    from argus_b200 import attention as A
    rng = np.random.default_rng(11)
    pages = U.random_pages(rng, TIERS, B, HKV, D, P)
    arenas, plist = U.arenas_from_pages(pages, device=device)
    q = torch.from_numpy((rng.standard_normal((B, HKV * G, 1, D)) / np.sqrt(D)).astype(np.float16)).to(device)
    full = A.AttentionPlan(arenas, plist, batch=B, heads_kv=HKV, group=G, head_dim=D, n_splits=1)
    return arenas, plist, q, full


def rank_plan(arenas, plist, world, rank):
    from argus_b200 import attention as A
    from argus_b200 import sharding
    shards = [sharding.shard_arena(a, world, rank) for a in arenas]
    return A.AttentionPlan(shards, plist, batch=B, heads_kv=HKV // world, group=G, head_dim=D, n_splits=1)


@pytest.mark.parametrize("world", [2, 4])
def test_shards_reproduce_full_attention_on_one_gpu(world):
    from argus_b200 import sharding
    arenas, plist, q, full = build("cuda")
    ref = full.run(q)
    parts = []
    for rank in range(world):
        plan = rank_plan(arenas, plist, world, rank)
        parts.append(plan.run(sharding.shard_queries(q, HKV, world, rank)))
    got = torch.cat(parts, dim=1)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_path):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from argus_b200 import sharding
        arenas, plist, q, full = build(torch.device("cuda", rank))
        step = sharding.HeadShardedDecode(rank_plan(arenas, plist, world, rank), HKV)
        out = step(q)
        ref = full.run(q)
        torch.cuda.synchronize()
        ok = torch.tensor([1 if torch.equal(out.view(torch.int16), ref.view(torch.int16)) else 0], device=q.device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if rank == 0:
            with open(result_path, "w") as f:
                f.write("ok" if int(ok.item()) == 1 else "mismatch")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_head_sharded_decode_over_nccl_two_gpus(tmp_path):
    path = str(tmp_path / "result.txt")
    mp.start_processes(_rank_main, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    with open(path) as f:
        assert f.read() == "ok"


# ----------------------------------------------------------- all-gather fused into the kernel
def test_fused_gather_on_one_gpu_matches_plan_run_over_steps():
    """World of one (no process group): the fused-gather step writes into its own output pair, both
    halves in turn, and each step's output equals the plain launch bit for bit."""
    from argus_b200 import attention as A
    from argus_b200 import sharding
    arenas, plist, q, full = build("cuda")
    plan = A.AttentionPlan(arenas, plist, batch=B, heads_kv=HKV, group=G, head_dim=D, n_splits=3)
    step = sharding.FusedHeadShardedDecode(plan, HKV)
    try:
        rng = np.random.default_rng(5)
        for k in range(3):
            qk = torch.from_numpy((rng.standard_normal(q.shape) / np.sqrt(D)).astype(np.float16)).cuda()
            got = step(qk).clone()
            ref = plan.run(qk)
            torch.cuda.synchronize()
            assert A.device_status() == 0
            assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), k
    finally:
        step.close()


def test_fused_gather_wait_times_out_when_rows_never_arrive():
    """The wait kernel gives up after its poll limit when the counter never reaches the target (here a
    step that was never issued), records ARGUS_ERR_TIMEOUT and leaves the context usable."""
    import ctypes

    from argus_b200 import _lib
    from argus_b200 import attention as A
    from argus_b200 import sharding
    arenas, plist, q, full = build("cuda")
    step = sharding.FusedHeadShardedDecode(full, HKV, wait_polls=2000)
    try:
        L = sharding._bind()
        st = torch.cuda.current_stream().cuda_stream
        # one signal lands (its own), the target asks for three
        rc = L.argus_gather_wait(ctypes.byref(step._spec), 3 * step.per_step, 2000, ctypes.c_void_p(st))
        assert rc == 0
        torch.cuda.synchronize()
        assert A.device_status() == _lib.ERR_TIMEOUT
    finally:
        step.close()
    step = sharding.FusedHeadShardedDecode(full, HKV)  # a fresh step on the same context runs normally
    try:
        out = step(q)
        ref = full.run(q)
        torch.cuda.synchronize()
        assert A.device_status() == 0
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    finally:
        step.close()


def _rank_fused_main(rank, world, port, result_path):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    step = None
    try:
        from argus_b200 import sharding
        arenas, plist, q, full = build(torch.device("cuda", rank))
        step = sharding.FusedHeadShardedDecode(rank_plan(arenas, plist, world, rank), HKV)
        ok = 1
        rng = np.random.default_rng(9)  # the same queries on every rank
        for k in range(3):
            qk = torch.from_numpy((rng.standard_normal(q.shape) / np.sqrt(D)).astype(np.float16)).to(q.device)
            out = step(qk).clone()
            ref = full.run(qk)
            torch.cuda.synchronize()
            ok &= int(torch.equal(out.view(torch.int16), ref.view(torch.int16)))
        from argus_b200 import attention as A
        ok &= int(A.device_status() == 0)
        t = torch.tensor([ok], device=q.device)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        if rank == 0:
            with open(result_path, "w") as f:
                f.write("ok" if int(t.item()) == 1 else "mismatch")
    finally:
        if step is not None:
            step.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_gather_over_peer_memory_two_gpus(tmp_path):
    path = str(tmp_path / "result.txt")
    mp.start_processes(_rank_fused_main, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    with open(path) as f:
        assert f.read() == "ok"
