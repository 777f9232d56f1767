"""KV-head sharding of mixed-tier decode attention across GPUs (one process per GPU).

The tiered cache's page boundaries and tier assignment are the same for every (batch, kv_head)
(core/memory_manager.py:333-379 lays a page out as one [B, H_kv, P, D] block), so the cache splits
cleanly by KV head: rank r of G keeps heads [r*H_kv/G, (r+1)*H_kv/G) of every arena, runs the
fused kernel on its heads' query groups, and the only exchange is an all-gather of the per-head
outputs ([B, H_q/G, q_len, D] fp16 per rank) into [B, H_q, q_len, D].  With the batch grown in
proportion to the ranks (B = 8 x ranks for the Llama-3-8B layer), every GPU holds the same bytes
(H_kv/G heads x B sequences) and the step exercises the collective at every scale; batch sharding
needs no exchange at all.

Collectives go through torch.distributed: NCCL over NVLink on GPUs, gloo on CPU (tests).  Every
rank issues the same collectives in the same order.
"""
import torch
import torch.distributed as dist

from .attention import LAYOUT_RECORD, KVArena


def head_range(n_kv_heads, world, rank):
    """[h0, h1): the KV heads rank `rank` of `world` owns (equal contiguous blocks)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if n_kv_heads % world:
        raise ValueError(f"{n_kv_heads} KV heads do not split evenly over {world} ranks")
    per = n_kv_heads // world
    return rank * per, (rank + 1) * per


def shard_arena(arena: KVArena, world, rank):
    """A record arena holding only this rank's KV heads (a copy on the arena's device), with the same
    slots, page size and tier, so the page table of the full cache indexes it unchanged."""
    if arena.layout != LAYOUT_RECORD:
        raise ValueError("only record arenas are sharded; rebuild split fp16 tensors per rank")
    h0, h1 = head_range(arena.H, world, rank)
    rec, S = arena.record_bytes, arena.slots
    full = arena.k.view(arena.B, arena.H, S, rec)
    part = full[:, h0:h1].contiguous().view(arena.B * (h1 - h0), S, rec)
    return KVArena(arena.tier, arena.layout, part, None, bh_stride=S * rec, record_bytes=rec,
                   page_tokens=arena.page_tokens, head_dim=arena.D, batch=arena.B, heads=h1 - h0, slots=S)


def shard_queries(q, n_kv_heads, world, rank):
    """The query heads of this rank's KV heads: q [B, H_q, q_len, D] -> [B, H_q/G, q_len, D]."""
    group = q.shape[1] // n_kv_heads
    h0, h1 = head_range(n_kv_heads, world, rank)
    return q[:, h0 * group:h1 * group].contiguous()


class HeadShardedDecode:
    """Runs one decode step of a head-sharded cache: local fused attention, then the output gather.

    plan: this rank's AttentionPlan (built over its shard_arena()s).  The kernel writes its output
    straight into this rank's slot of a [world, B, H_q/G, q_len, D] gather buffer and the all-gather
    runs in place on that buffer (NCCL: no staging copy), so the step is one kernel, one collective
    and one head-order copy.  Buffers are allocated once per output shape and reused."""

    def __init__(self, plan, n_kv_heads, group=None):
        self.plan, self.group = plan, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n_kv_heads = int(n_kv_heads)
        head_range(self.n_kv_heads, self.world, self.rank)
        self._buf = None
        self._out = None

    def _buffers(self, local_shape, dtype, device):
        shape = (self.world,) + tuple(local_shape)
        if self._buf is None or self._buf.shape != shape or self._buf.device != device:
            self._buf = torch.empty(shape, dtype=dtype, device=device)
            B, hl, ql, D = local_shape
            self._out = torch.empty(B, self.world * hl, ql, D, dtype=dtype, device=device)
        return self._buf, self._out

    def gather(self, local):
        """[B, H_q/G, q_len, D] per rank -> [B, H_q, q_len, D], heads in rank order."""
        buf, out = self._buffers(local.shape, local.dtype, local.device)
        if local.data_ptr() != buf[self.rank].data_ptr():
            buf[self.rank].copy_(local)
        self.all_gather(buf)
        return self.to_head_order(buf, out)

    def all_gather(self, buf):
        """In-place all-gather of every rank's slot of buf."""
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(buf.view(-1), buf[self.rank].view(-1), group=self.group)
        else:
            parts = list(buf.unbind(0))
            mine = parts[self.rank].clone()
            dist.all_gather(parts, mine, group=self.group)

    def to_head_order(self, buf, out):
        B, hl, ql, D = buf.shape[1:]
        out.view(B, self.world, hl, ql, D).copy_(buf.permute(1, 0, 2, 3, 4))
        return out

    def local(self, q_full, scale=None):
        """This rank's attention, written into its slot of the gather buffer (returned)."""
        q_local = shard_queries(q_full, self.n_kv_heads, self.world, self.rank)
        buf, _ = self._buffers(q_local.shape, q_local.dtype, q_local.device)
        self.plan.run(q_local, scale=scale, out=buf[self.rank])
        return buf

    def __call__(self, q_full, scale=None):
        buf = self.local(q_full, scale=scale)
        self.all_gather(buf)
        return self.to_head_order(buf, self._out)
