"""Tiered paged KV cache manager with the reference's surface (argus_cache/core/memory_manager.py).

This first part holds isolate_outliers; the PagedDynamicKVCache class follows.
"""
import torch

from .. import _lib


def isolate_outliers(tensor, threshold_sigma=3.0):
    """NaN/Inf -> 0, then split |x| > fp16(mean|x| * sigma) (per row over the last dim) into an
    outlier tensor; returns (normal_vals, outlier_vals, outlier_mask) like
    core/memory_manager.py:89-113.  Runs as one libargus_b200 kernel."""
    _lib.require_cuda(tensor)
    if tensor.dtype != torch.float16:
        raise TypeError("isolate_outliers takes float16 tensors")
    x = tensor.contiguous()
    D = x.shape[-1]
    n = x.numel() // D if D else 0
    normal = torch.empty_like(x)
    outv = torch.empty_like(x)
    mask = torch.empty(x.shape, dtype=torch.bool, device=x.device)
    _lib.call("argus_isolate_outliers", _lib.ptr(x), n, D, float(threshold_sigma), _lib.ptr(normal),
              _lib.ptr(outv), _lib.ptr(mask), _lib.stream_handle(x.device))
    # sigma <= 0: normal is the cleansed tensor, outv zeros and the mask all False, as in the reference
    return normal, outv, mask
