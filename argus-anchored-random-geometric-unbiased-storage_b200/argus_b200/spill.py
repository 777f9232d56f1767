"""Host spill and prefetch of record arenas: pinned host mirrors filled and drained with
asynchronous copies (libargus_b200 argus_memcpy_async, one cudaMemcpyAsync per arena) on a side
stream, ordered against the compute stream with CUDA events.

Replaces the synchronous, pageable per-tensor .to("cpu") / .to(device) moves of
swap_out_to_host / swap_in_to_device (core/memory_manager.py:1658-1713).
"""
import ctypes

import torch

from . import _lib
from .attention import KVArena

_streams = {}


def side_stream(device):
    device = torch.device(device)
    if device not in _streams:
        _streams[device] = torch.cuda.Stream(device=device)
    return _streams[device]


def _clone_meta(a, buf):
    return KVArena(a.tier, a.layout, buf, None, bh_stride=a.bh_stride, record_bytes=a.record_bytes,
                   page_tokens=a.page_tokens, head_dim=a.D, batch=a.B, heads=a.H, slots=a.slots)


def arenas_to_host(arenas, wait=True):
    """Pinned host copies of device record arenas (D2H on a side stream after the compute stream's
    pending writes).  With wait=True the host copies are complete on return."""
    if not arenas:
        return []
    dev = arenas[0].k.device
    st = side_stream(dev)
    st.wait_stream(torch.cuda.current_stream(dev))
    out = []
    for a in arenas:
        host = torch.empty(a.k.shape, dtype=torch.uint8, pin_memory=True)
        _lib.call("argus_memcpy_async", _lib.ptr(host), _lib.ptr(a.k), a.k.numel(), _lib.ptr_stream(st))
        a.k.record_stream(st)
        out.append(_clone_meta(a, host))
    ev = torch.cuda.Event()
    ev.record(st)
    if wait:
        ev.synchronize()
    return out


def arenas_to_device(host_arenas, device, event_out=None):
    """Device copies of pinned host arenas (H2D on a side stream); the compute stream waits on the
    copies before any later work reads them."""
    if not host_arenas:
        return []
    device = torch.device(device)
    st = side_stream(device)
    # the new buffers come from the compute stream's pool: a block it freed may still have reads or
    # writes queued there, so the copies start after the compute stream's pending work
    st.wait_stream(torch.cuda.current_stream(device))
    out = []
    for a in host_arenas:
        buf = torch.empty(a.k.shape, dtype=torch.uint8, device=device)
        buf.record_stream(st)
        _lib.call("argus_memcpy_async", _lib.ptr(buf), _lib.ptr(a.k), a.k.numel(), _lib.ptr_stream(st))
        out.append(_clone_meta(a, buf))
    ev = torch.cuda.Event()
    ev.record(st)
    torch.cuda.current_stream(device).wait_event(ev)
    if event_out is not None:
        event_out.append(ev)
    return out


class StreamedArenaAttention:
    """Attention over a record arena that stays in pinned host memory (a spilled tier), without
    bringing it all back first: runs of `chunk_slots` slots of every (batch, kv_head) are copied
    (one 2-D asynchronous copy per run) into two device staging arenas on a side stream while the
    previous run is attended on the compute stream; the runs' results are joined by their LSE in
    fp32.  The reference instead moves every spilled tensor back synchronously before attending
    (core/memory_manager.py:1163, 1686-1713)."""

    def __init__(self, host_arena: KVArena, *, group, chunk_slots=256, n_slots=None, device="cuda", n_splits=None):
        """host_arena: the spilled arena, in pinned host memory (a device arena is accepted too: the
        runs are then copied device to device, which computes the same result from resident memory).
        n_splits: split-K partitions of every run's launch (default: the plan's own choice)."""
        if not host_arena.k.is_cuda and not host_arena.k.is_pinned():
            raise ValueError("a host arena must live in pinned memory")
        from .attention import LAYOUT_RECORD
        if host_arena.layout != LAYOUT_RECORD:
            raise ValueError("only record arenas stream")
        self.h, self.G = host_arena, int(group)
        self.n = int(n_slots if n_slots is not None else host_arena.slots)
        self.chunk = max(1, min(int(chunk_slots), self.n))
        self.device = torch.device(device)
        a = host_arena
        self.bufs = [torch.empty(a.B * a.H, self.chunk, a.record_bytes, dtype=torch.uint8, device=self.device)
                     for _ in range(2)]
        self.arenas = [KVArena(a.tier, a.layout, b, None, bh_stride=self.chunk * a.record_bytes,
                               record_bytes=a.record_bytes, page_tokens=a.page_tokens, head_dim=a.D, batch=a.B,
                               heads=a.H, slots=self.chunk) for b in self.bufs]
        self._plans = {}
        self.n_splits = n_splits
        self.copied = [torch.cuda.Event() for _ in range(2)]
        self.released = [torch.cuda.Event() for _ in range(2)]
        # the staging buffers were allocated on the current stream (whose earlier work may still use
        # their blocks): the first copies into them wait for it through these events
        for ev in self.released:
            ev.record(torch.cuda.current_stream(self.device))

    def _plan(self, buf, ns, q_len):
        from .attention import AttentionPlan
        key = (buf, ns, q_len)
        if key not in self._plans:
            a = self.h
            self._plans[key] = AttentionPlan([self.arenas[buf]], [(0, j, a.page_tokens) for j in range(ns)], batch=a.B,
                                             heads_kv=a.H, group=self.G, head_dim=a.D, q_len=q_len,
                                             n_splits=self.n_splits)
        return self._plans[key]

    def _copy(self, run, s0, ns, stream):
        a = self.h
        rec = a.record_bytes
        _lib.call("argus_memcpy2d_async", _lib.ptr(self.bufs[run % 2]), self.chunk * rec,
                  ctypes.c_void_p(a.k.data_ptr() + s0 * rec), a.bh_stride, ns * rec, a.B * a.H, _lib.ptr_stream(stream))

    def run(self, q, scale=None):
        """q [B, H_q, q_len, D] fp16 (on the device) -> (out fp16, lse natural log fp32) over the spilled tier."""
        _lib.require_cuda(q, "q")
        q = q.contiguous()
        compute = torch.cuda.current_stream(q.device)
        copy = side_stream(q.device)
        runs = [(s0, min(self.chunk, self.n - s0)) for s0 in range(0, self.n, self.chunk)]
        rows = q.numel() // q.shape[-1]
        acc_o = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        acc_lse = torch.full(q.shape[:3], float("-inf"), dtype=torch.float32, device=q.device)
        out_i = torch.empty_like(q)
        lse_i = torch.empty(q.shape[:3], dtype=torch.float32, device=q.device)
        # the staging buffers are free once the previous call's attention has read them; work issued
        # on the compute stream before this call (the resident tiers) overlaps the first copies
        for ev in self.released:
            copy.wait_event(ev)
        for i, (s0, ns) in enumerate(runs[:2]):
            self._copy(i, s0, ns, copy)
            self.copied[i % 2].record(copy)
        for i, (s0, ns) in enumerate(runs):
            compute.wait_event(self.copied[i % 2])
            self._plan(i % 2, ns, q.shape[2]).run(q, scale=scale, out=out_i, lse=lse_i)
            _lib.call("argus_attention_accumulate", _lib.ptr(acc_o), _lib.ptr(acc_lse), _lib.ptr(out_i),
                      _lib.ptr(lse_i), rows, q.shape[-1], _lib.ptr_stream(compute))
            self.released[i % 2].record(compute)
            if i + 2 < len(runs):  # the buffer is free once this run's attention has read it
                copy.wait_event(self.released[i % 2])
                self._copy(i + 2, *runs[i + 2], copy)
                self.copied[i % 2].record(copy)
        return acc_o.to(torch.float16), acc_lse


class SpilledLayerDecode:
    """Decode attention over a layer whose oldest tier lives in pinned host memory: the resident
    tiers in one fused launch (with their log-sum-exp), the spilled arena streamed in runs on a side
    stream while the resident launch runs (StreamedArenaAttention), the two results joined by LSE.
    The reference instead swaps the whole spilled cache back before attending
    (core/memory_manager.py:1163, 1345, 1686-1713).

    resident_plan: AttentionPlan over the resident arenas; spilled: the spilled record arena (pinned
    host, or a device arena for a resident run of the same computation)."""

    def __init__(self, resident_plan, spilled, *, chunk_slots=512, n_splits=None):
        self.plan = resident_plan
        self.stream = StreamedArenaAttention(spilled, group=resident_plan.G, chunk_slots=chunk_slots,
                                             device=resident_plan.device, n_splits=n_splits)
        self._lse = None

    def __call__(self, q, scale=None, out=None):
        from .core import jl
        shape = q.shape[:3]
        if self._lse is None or tuple(self._lse.shape) != tuple(shape) or self._lse.device != q.device:
            self._lse = torch.empty(shape, dtype=torch.float32, device=q.device)
        o_r = self.plan.run(q, scale=scale, lse=self._lse)
        o_s, l_s = self.stream.run(q, scale=scale)
        return jl.merge_attention(o_r, self._lse, o_s, l_s, out=out)


def numa_local_cpus(device):
    """CPU ids close to the GPU (NVML's CPU affinity of the device; a read-only query), or None when
    unknown.  A process pinned to them allocates its pinned host buffers on the GPU's NUMA node
    (first touch)."""
    import os
    try:
        import pynvml
        idx = torch.device(device).index or 0
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        phys = int(vis.split(",")[idx]) if vis else idx
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByIndex(phys)
            words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = {64 * w + b for w, m in enumerate(words) for b in range(64) if (m >> b) & 1}
        return cpus & set(range(os.cpu_count())) or None
    except Exception:
        return None
