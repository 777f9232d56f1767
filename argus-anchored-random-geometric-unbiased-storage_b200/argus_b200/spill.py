"""Host spill and prefetch of record arenas: pinned host mirrors filled and drained with
asynchronous copies (libargus_b200 argus_memcpy_async, one cudaMemcpyAsync per arena) on a side
stream, ordered against the compute stream with CUDA events.

Replaces the synchronous, pageable per-tensor .to("cpu") / .to(device) moves of
swap_out_to_host / swap_in_to_device (core/memory_manager.py:1658-1713).
"""
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
