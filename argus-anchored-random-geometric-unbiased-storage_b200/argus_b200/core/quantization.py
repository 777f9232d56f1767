"""Tier codecs with the reference's signatures, on CUDA tensors, computed by libargus_b200.

Mirrors argus_cache/core/quantization.py (argus_cache 0.1.8): same function names, argument
names and defaults, return tuples, dtypes and shapes; results are bit-identical to the
reference's CPU path (the CUDA kernels restate its fp16 arithmetic, including the int8 wrap of
the simulated-FP8 tier and torch's summation order for the 1-bit scale).

Reference lines per function:
  quantize_to_int8 / dequantize_from_int8                  core/quantization.py:3-28
  quantize_to_int4_packed / dequantize_from_int4_packed    core/quantization.py:30-67
  quantize_to_int2_packed / dequantize_from_int2_packed    core/quantization.py:69-171
  quantize_to_1bit_packed / dequantize_from_1bit_packed    core/quantization.py:173-201
  quantize_to_fp8_simulated / dequantize_from_fp8_simulated core/quantization.py:203-222
  quantize_to_jl_projection / dequantize_from_jl_projection core/quantization.py:224-290

Only fp16 tensors are accepted (the reference's tiers store fp16 scales for fp16 KV); packing
along a dim other than -2, or reducing over a dim other than -1, is done on a moved view.
"""
import torch

from .. import _lib
from . import jl as _jl


def _check(t, name="tensor"):
    _lib.require_cuda(t, name)
    if t.dtype != torch.float16:
        raise TypeError(f"argus_b200 codecs take float16 tensors; {name} is {t.dtype}")


def _canon(t, seq_dim, quant_dim):
    """View with (seq_dim, quant_dim) moved to (-2, -1), made contiguous."""
    nd = t.dim()
    sd, qd = seq_dim % nd, quant_dim % nd
    if (sd, qd) == (nd - 2, nd - 1):
        return t.contiguous(), None
    if sd == qd:
        raise ValueError("seq_dim and quant_dim must differ")
    return torch.movedim(t, (sd, qd), (-2, -1)).contiguous(), (sd, qd)


def _uncanon(t, moved):
    if moved is None:
        return t
    return torch.movedim(t, (-2, -1), moved)


def _rows(t):
    D = t.shape[-1]
    return (t.numel() // D if D else 0), D


# ------------------------------------------------------------------------- symmetric 8-bit
def _quant_sym8(fn, tensor, dim):
    _check(tensor)
    nd = tensor.dim()
    d = dim % nd
    x = tensor.contiguous() if d == nd - 1 else torch.movedim(tensor, d, -1).contiguous()
    n, D = _rows(x)
    q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    s = torch.empty(x.shape[:-1] + (1,), dtype=torch.float16, device=x.device)
    _lib.call(fn, _lib.ptr(x), n, D, _lib.ptr(q), _lib.ptr(s), _lib.stream_handle(x.device))
    if d != nd - 1:
        q, s = torch.movedim(q, -1, d), torch.movedim(s, -1, d)
    return q, s


def _dequant_sym8(fn, quantized, scales):
    _lib.require_cuda(quantized, "quantized")
    _check(scales, "scales")
    if scales.shape[-1] != 1 or quantized.shape[:-1] != scales.shape[:-1]:
        # general broadcasting (a scale along another dim) is done as the reference does it
        raise ValueError("scales must be [..., 1] per-token scales matching quantized[..., :]")
    q = quantized.contiguous().view(torch.int8)
    s = scales.contiguous()
    n, D = _rows(q)
    out = torch.empty(q.shape, dtype=torch.float16, device=q.device)
    _lib.call(fn, _lib.ptr(q), _lib.ptr(s), n, D, _lib.ptr(out), _lib.stream_handle(q.device))
    return out


def quantize_to_int8(tensor: torch.Tensor, dim: int = -1):
    """Symmetric per-token INT8; returns (int8 codes, fp16 scales [..., 1])."""
    return _quant_sym8("argus_quant_int8", tensor, dim)


def dequantize_from_int8(quantized: torch.Tensor, scales: torch.Tensor):
    """codes * scales in fp16."""
    return _dequant_sym8("argus_dequant_int8", quantized, scales)


def quantize_to_fp8_simulated(tensor: torch.Tensor, dim: int = -1):
    """Simulated FP8: amax/240 scale, codes clamped to +-240 and stored with int8 wraparound."""
    return _quant_sym8("argus_quant_fp8sim", tensor, dim)


def dequantize_from_fp8_simulated(quantized: torch.Tensor, scales: torch.Tensor):
    return _dequant_sym8("argus_dequant_fp8sim", quantized, scales)


def quantize_to_e4m3(tensor: torch.Tensor, dim: int = -1):
    """True e4m3 (a separately named non-parity mode; the reference's FP8 tier is the simulation
    above): s = fp16(amax / 448) per token, codes = e4m3(x / s) (nearest even, saturating, NaN -> 0),
    returned as uint8 codes and fp16 scales [..., 1]."""
    q, s = _quant_sym8("argus_quant_e4m3", tensor, dim)
    return q.view(torch.uint8), s


def dequantize_from_e4m3(quantized: torch.Tensor, scales: torch.Tensor):
    """fp16(e4m3(code) * s)."""
    return _dequant_sym8("argus_dequant_e4m3", quantized, scales)


# --------------------------------------------------------------- sequence-packed low bits
def _quant_packed(fn, per, tensor, seq_dim, quant_dim, with_min):
    _check(tensor)
    T = tensor.shape[seq_dim]
    assert T % per == 0, (
        f"Sequence dimension size ({T}) must be "
        + ("even for 4-bit packing." if per == 2 else f"a multiple of {per} for {8 // per}-way packing."))
    x, moved = _canon(tensor, seq_dim, quant_dim)
    n, D = _rows(x)
    packed = torch.empty(x.shape[:-2] + (x.shape[-2] // per, D), dtype=torch.uint8, device=x.device)
    s = torch.empty(x.shape[:-1] + (1,), dtype=torch.float16, device=x.device)
    args = [_lib.ptr(x), n, D, _lib.ptr(packed), _lib.ptr(s)]
    mn = None
    if with_min:
        mn = torch.empty_like(s)
        args.append(_lib.ptr(mn))
    _lib.call(fn, *args, _lib.stream_handle(x.device))
    out = [_uncanon(packed, moved), _uncanon(s, moved)]
    if with_min:
        out.append(_uncanon(mn, moved))
    return tuple(out)


def _dequant_packed(fn, per, packed, scales, min_vals, seq_dim):
    _lib.require_cuda(packed, "packed")
    _check(scales, "scales")
    p, moved = _canon(packed, seq_dim, -1)
    s, _ = _canon(scales, seq_dim, -1)
    args_m = []
    if min_vals is not None:
        _check(min_vals, "min_vals")
        m, _ = _canon(min_vals, seq_dim, -1)
        args_m = [_lib.ptr(m)]
    D = p.shape[-1]
    T = p.shape[-2] * per
    if s.shape[-2] != T:
        raise ValueError(f"scales cover {s.shape[-2]} tokens, packed data {T}")
    out = torch.empty(p.shape[:-2] + (T, D), dtype=torch.float16, device=p.device)
    n = out.numel() // D if D else 0
    _lib.call(fn, _lib.ptr(p), _lib.ptr(s), *args_m, n, D, _lib.ptr(out), _lib.stream_handle(p.device))
    return _uncanon(out, moved)


def quantize_to_int4_packed(tensor: torch.Tensor, seq_dim: int = -2, quant_dim: int = -1):
    """Asymmetric INT4, two tokens per byte along seq_dim; returns (packed, scales, min_vals)."""
    return _quant_packed("argus_quant_int4", 2, tensor, seq_dim, quant_dim, True)


def dequantize_from_int4_packed(packed: torch.Tensor, scales: torch.Tensor, min_vals: torch.Tensor,
                                seq_dim: int = -2):
    return _dequant_packed("argus_dequant_int4", 2, packed, scales, min_vals, seq_dim)


def quantize_to_int2_packed(tensor: torch.Tensor, seq_dim: int = -2, quant_dim: int = -1):
    """Asymmetric INT2, four tokens per byte along seq_dim; returns (packed, scales, min_vals)."""
    return _quant_packed("argus_quant_int2", 4, tensor, seq_dim, quant_dim, True)


def dequantize_from_int2_packed(packed: torch.Tensor, scales: torch.Tensor, min_vals: torch.Tensor,
                                seq_dim: int = -2):
    return _dequant_packed("argus_dequant_int2", 4, packed, scales, min_vals, seq_dim)


def quantize_to_1bit_packed(tensor: torch.Tensor, seq_dim: int = -2, quant_dim: int = -1):
    """Sign bits, eight tokens per byte along seq_dim, scale = mean|x|; returns (packed, scales)."""
    return _quant_packed("argus_quant_1bit", 8, tensor, seq_dim, quant_dim, False)


def dequantize_from_1bit_packed(packed: torch.Tensor, scales: torch.Tensor, seq_dim: int = -2):
    return _dequant_packed("argus_dequant_1bit", 8, packed, scales, None, seq_dim)


# ---------------------------------------------------------------------------- JL archive
def quantize_to_jl_projection(tensor: torch.Tensor, ratio: int = 4):
    """Projects the sequence axis N -> N // ratio with a fresh random orthogonal W.

    W is drawn exactly as the reference draws it -- torch.randn(N, M) float32 on the CPU from
    the global generator, QR on the CPU, transposed, cast to the tensor's dtype -- and the
    projection W @ X runs on the GPU.  Returns (compressed [..., M, D], w_proj [M, N])."""
    _check(tensor)
    n = tensor.shape[-2]
    m = n // ratio
    raw = torch.randn(n, m, dtype=torch.float32, device="cpu")
    q, _ = torch.linalg.qr(raw)
    w_proj = q.t().to(tensor.dtype).to(tensor.device)
    return _jl.apply_left(w_proj, tensor), w_proj


def dequantize_from_jl_projection(compressed: torch.Tensor, w_proj: torch.Tensor, recon_operator: torch.Tensor = None,
                                  alpha: float = 1e-3):
    """Rebuilds [..., N, D] as R @ compressed with the Laplacian-regularised operator
    R = A^-1 W^T (W A^-1 W^T)^-1, A = L + alpha I (built once on the host in fp32 when not given)."""
    _check(compressed, "compressed")
    if recon_operator is None:
        recon_operator = _jl.reconstruction_operator_solve(w_proj, alpha).to(compressed.device).to(compressed.dtype)
    return _jl.apply_left(recon_operator, compressed)
