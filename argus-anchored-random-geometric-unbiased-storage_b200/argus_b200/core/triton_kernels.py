"""Pack/unpack entry points with the names and signatures of argus_cache/core/triton_kernels.py.

The reference module holds four Triton kernels plus a torch fallback; on CPU tensors the fallback
runs and defines the results (triton_kernels.py:177-189,217-239,264-308,334-386).  Here all four
run as hand-written sm_100a CUDA (libargus_b200) with the fallback's semantics: packing along the
sequence axis (adjacent token pairs / octets), per-token scales.  The reference's GPU Triton
kernels pack flat-adjacent elements instead (triton_kernels.py:27-37,89-109); that layout is not
reproduced, since its own CPU and GPU results disagree.

TRITON_AVAILABLE is kept for import compatibility; it is False because no Triton is used and it
gates nothing here.
"""
import torch

from .. import _lib
from . import quantization as _q

TRITON_AVAILABLE = False


def triton_pack_int4(tensor: torch.Tensor, seq_dim: int = -2):
    """uint8 codes -> two tokens per byte along seq_dim (low nibble = even token)."""
    _lib.require_cuda(tensor)
    if tensor.dtype != torch.uint8:
        tensor = tensor.to(torch.uint8)
    T = tensor.shape[seq_dim]
    assert T % 2 == 0, "Sequence length must be even for 4-bit packing."
    x, moved = _q._canon(tensor, seq_dim, -1)
    n, D = _q._rows(x)
    packed = torch.empty(x.shape[:-2] + (x.shape[-2] // 2, D), dtype=torch.uint8, device=x.device)
    _lib.call("argus_pack_int4_codes", _lib.ptr(x), n, D, _lib.ptr(packed), _lib.stream_handle(x.device))
    return _q._uncanon(packed, moved)


def triton_unpack_int4(packed: torch.Tensor, scales: torch.Tensor, min_vals: torch.Tensor, seq_dim: int = -2):
    """Unpack and dequantize: fp16(fp16(u * scale) + min)."""
    return _q.dequantize_from_int4_packed(packed, scales, min_vals, seq_dim=seq_dim)


def triton_pack_1bit(tensor: torch.Tensor, seq_dim: int = -2):
    """Sign bits (x >= 0) of a float16 tensor, eight tokens per byte along seq_dim."""
    _q._check(tensor)
    T = tensor.shape[seq_dim]
    assert T % 8 == 0, "Sequence length must be a multiple of 8 for 1-bit packing."
    x, moved = _q._canon(tensor, seq_dim, -1)
    n, D = _q._rows(x)
    packed = torch.empty(x.shape[:-2] + (x.shape[-2] // 8, D), dtype=torch.uint8, device=x.device)
    _lib.call("argus_pack_1bit_signs", _lib.ptr(x), n, D, _lib.ptr(packed), _lib.stream_handle(x.device))
    return _q._uncanon(packed, moved)


def triton_unpack_1bit(packed: torch.Tensor, scales: torch.Tensor, seq_dim: int = -2):
    """Unpack sign bits to (2b - 1) * scale."""
    return _q.dequantize_from_1bit_packed(packed, scales, seq_dim=seq_dim)
