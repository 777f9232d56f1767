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
import ctypes

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


# ---------------------------------------------------------------------------------------------
# The all-gather fused into the attention kernel (libargus_b200 argus_decode_attention_gather)

MAX_PEERS = 8
# C-ABI entry points bound in this module
BOUND_SYMBOLS = ("argus_decode_attention_gather", "argus_gather_arrivals_per_step", "argus_gather_wait",
                 "argus_peer_alloc", "argus_peer_open", "argus_peer_close", "argus_peer_free")
# polls of argus_gather_wait before it reports a timeout (~0.25 us apart: about one second)
WAIT_POLLS = 4_000_000


class PeerGatherC(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("heads_kv_total", ctypes.c_int32),
                ("parity", ctypes.c_int32), ("out", ctypes.c_void_p * MAX_PEERS),
                ("arrivals", ctypes.c_void_p * MAX_PEERS)]


def _bind():
    from .attention import ArenaC, ShapeC, _bind as bind_attention
    L = bind_attention()
    if not getattr(L, "_argus_gather_bound", False):
        L.argus_decode_attention_gather.argtypes = [ctypes.POINTER(ShapeC), ctypes.POINTER(ArenaC), ctypes.c_void_p,
                                                    ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(PeerGatherC),
                                                    ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                    ctypes.c_void_p]
        L.argus_gather_arrivals_per_step.argtypes = [ctypes.c_int]
        L.argus_gather_arrivals_per_step.restype = ctypes.c_int64
        L.argus_gather_wait.argtypes = [ctypes.POINTER(PeerGatherC), ctypes.c_uint64, ctypes.c_int64,
                                        ctypes.c_void_p]
        L.argus_peer_alloc.argtypes = [ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
        L.argus_peer_open.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
        L.argus_peer_close.argtypes = [ctypes.c_void_p]
        L.argus_peer_free.argtypes = [ctypes.c_void_p]
        for name in BOUND_SYMBOLS:
            if name != "argus_gather_arrivals_per_step":
                getattr(L, name).restype = ctypes.c_int
        L._argus_gather_bound = True
    return L


def _check(L, name, rc):
    from . import _lib
    if rc != 0:
        raise _lib.ArgusError(name, rc, L.argus_last_error().decode())


class _DeviceArray:
    """A device buffer owned elsewhere, seen by torch through __cuda_array_interface__."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


class FusedHeadShardedDecode:
    """One decode step of a head-sharded cache with the output all-gather inside the attention kernel.

    Every rank owns an output pair [2][B][H_q][q_len][D] fp16 and a 64-bit arrival counter in device
    memory it exports with CUDA IPC; the handles are exchanged once over the process group.  Step k
    writes half k % 2: the kernel that finishes a (batch, kv_head, query group) stores its rows in
    every rank's half at their place in the full layout (peer memory over NVLink); a one-thread kernel
    queued after it signals every rank (system-scope fence, release add) and holds this rank's stream
    until all ranks have signalled step k.  So a step is one attention launch and one wait launch, with
    no collective call, no staging copy and no head reordering.  A rank cannot get more than one
    step ahead of a slower peer (its own wait needs that peer's rows), so the pair of halves is
    enough for a caller that consumes each step's output on the same stream before the next step.

    plan: this rank's AttentionPlan over its shard_arena()s.  Without an initialised process group
    (or with a group of one) the step runs on this GPU alone through the same path."""

    def __init__(self, plan, n_kv_heads, group=None, wait_polls=WAIT_POLLS):
        self.plan, self.group, self.wait_polls = plan, group, int(wait_polls)
        dist_on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if dist_on else 1
        self.rank = dist.get_rank(group) if dist_on else 0
        if self.world > MAX_PEERS:
            raise ValueError(f"at most {MAX_PEERS} ranks")
        self.n_kv_heads = int(n_kv_heads)
        head_range(self.n_kv_heads, self.world, self.rank)
        if plan.Hkv * self.world != self.n_kv_heads:
            raise ValueError("the plan must hold n_kv_heads / world KV heads")
        L = _bind()
        self._L = L
        self.shape = (plan.B, self.n_kv_heads * plan.G, plan.qlen, plan.D)
        out_bytes = 2 * plan.B * self.n_kv_heads * plan.G * plan.qlen * plan.D * 2
        self._own, handles = [], []
        for nbytes in (out_bytes, 256):
            ptr, h = ctypes.c_void_p(), (ctypes.c_uint8 * 64)()
            _check(L, "argus_peer_alloc", L.argus_peer_alloc(nbytes, ctypes.byref(ptr), h))
            self._own.append(ptr.value)
            handles.append(bytes(h))
        if self.world > 1:
            everyone = [None] * self.world
            dist.all_gather_object(everyone, handles, group=group)
        else:
            everyone = [handles]
        self._opened = []
        spec = PeerGatherC(self.world, self.rank, self.n_kv_heads, 0)
        for r in range(self.world):
            if r == self.rank:
                spec.out[r], spec.arrivals[r] = self._own
                continue
            ptrs = []
            for h in everyone[r]:
                ptr = ctypes.c_void_p()
                _check(L, "argus_peer_open", L.argus_peer_open((ctypes.c_uint8 * 64).from_buffer_copy(h),
                                                               ctypes.byref(ptr)))
                self._opened.append(ptr.value)
                ptrs.append(ptr.value)
            spec.out[r], spec.arrivals[r] = ptrs
        self._spec = spec
        self.per_step = int(L.argus_gather_arrivals_per_step(self.world))
        self.steps = 0
        half = _DeviceArray(self._own[0], (2,) + self.shape, "<f2")
        self.out_pair = torch.as_tensor(half, device=plan.device)  # a view of the rank's output pair

    def local(self, q_full, scale=None, stream=None):
        """Queues this rank's attention for q_full [B, H_q, q_len, D]: its rows go to every rank."""
        import math
        from . import _lib
        _lib.require_cuda(q_full, "q")
        plan = self.plan
        if tuple(q_full.shape) != self.shape or q_full.dtype != torch.float16:
            raise ValueError(f"q must be float16 {self.shape}")
        q_full = q_full.contiguous()  # the kernel reads this rank's heads' rows in place
        plan._shape.scale = float(1.0 / math.sqrt(plan.D) if scale is None else scale)
        st = stream if stream is not None else torch.cuda.current_stream(q_full.device).cuda_stream
        self._spec.parity = self.steps & 1
        rc = self._L.argus_decode_attention_gather(
            ctypes.byref(plan._shape), plan._arena_c, plan.chunks_dev.data_ptr(), plan.splits_dev.data_ptr(),
            q_full.data_ptr(), ctypes.byref(self._spec), None, None,
            plan.workspace.data_ptr() if plan.workspace is not None else None, ctypes.c_void_p(st))
        _check(self._L, "argus_decode_attention_gather", rc)
        self._q_keep = q_full  # alive until the launch has read it
        return self.steps & 1

    def wait(self, stream=None):
        """Queues the wait for every rank's rows of the step just issued; returns its output half."""
        st = stream if stream is not None else torch.cuda.current_stream(self.plan.device).cuda_stream
        parity = self.steps & 1
        self.steps += 1
        rc = self._L.argus_gather_wait(ctypes.byref(self._spec), self.steps * self.per_step, self.wait_polls,
                                       ctypes.c_void_p(st))
        _check(self._L, "argus_gather_wait", rc)
        return self.out_pair[parity]

    def __call__(self, q_full, scale=None):
        """[B, H_q, q_len, D] on every rank -> the full output [B, H_q, q_len, D] (a view of this rank's
        output pair, valid until the step after next)."""
        self.local(q_full, scale=scale)
        return self.wait()

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (every rank calls it; it synchronises the
        device and, with several ranks, the process group first)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.plan.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        for ptr in self._opened:
            _check(self._L, "argus_peer_close", self._L.argus_peer_close(ctypes.c_void_p(ptr)))
        self._opened = []
        if self.world > 1:
            dist.barrier(group=self.group)  # no peer maps this rank's memory any more
        self.out_pair = None
        for ptr in self._own:
            _check(self._L, "argus_peer_free", self._L.argus_peer_free(ctypes.c_void_p(ptr)))
        self._own = None
