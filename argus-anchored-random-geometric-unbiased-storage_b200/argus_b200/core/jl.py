"""JL sequence-projection archive: matrices (host, fp32/CPU as the reference builds them) and the
batched contraction C[b] = A @ X[b] on the GPU (libargus_b200 argus_jl_apply).

Reference lines: core/memory_manager.py:227-282 (W and R of the manager, ratio 4, seed 42),
core/quantization.py:224-290 (per-call W and the solve-form R).
"""
import ctypes
import math

import torch

from .. import _lib


def projection_matrix(page_size, dtype=torch.float16, device="cuda", seed=42, ratio=4):
    """The manager's shared W [N/ratio, N]: QR of a seed-42 Gaussian [N, N/ratio] transposed.

    The Gaussian is drawn on the CPU from a private generator seeded 42, which gives the same
    values as torch.manual_seed(42) + torch.randn on the CPU without resetting the global RNG;
    drawing on the host keeps one W for the GPU path and the CPU reference alike."""
    n, m = page_size, page_size // ratio
    g = torch.Generator(device="cpu").manual_seed(seed)
    raw = torch.randn(n, m, dtype=torch.float32, generator=g)
    q, _ = torch.linalg.qr(raw)
    return q.t().to(dtype).to(device)


def _laplacian(N, alpha):
    L = torch.zeros(N, N, dtype=torch.float32)
    L.diagonal().fill_(2.0)
    L.diagonal(-1).fill_(-1.0)
    L.diagonal(1).fill_(-1.0)
    L[0, 0] = 1.0
    L[N - 1, N - 1] = 1.0
    return L + alpha * torch.eye(N, dtype=torch.float32)


def reconstruction_operator_inverse(w_proj, alpha=1e-3):
    """R = A^-1 W^T (W A^-1 W^T)^-1 via explicit inverses, fp32 on the CPU
    (core/memory_manager.py:241-282)."""
    W = w_proj.detach().to("cpu", torch.float32)
    M, N = W.shape
    A_inv = torch.inverse(_laplacian(N, alpha))
    inv_term = torch.inverse(W @ A_inv @ W.t())
    return (A_inv @ W.t()) @ inv_term


def reconstruction_operator_solve(w_proj, alpha=1e-3):
    """Same operator via a linear solve, fp32 on the CPU (core/quantization.py:257-289)."""
    W = w_proj.detach().to("cpu", torch.float32)
    M, N = W.shape
    Y = torch.linalg.solve(_laplacian(N, alpha), W.t())
    return Y @ torch.inverse(W @ Y)


def apply_left(A, X):
    """A [M, K] @ X [..., K, N] -> [..., M, N] in fp16 with fp32 accumulation, on the GPU."""
    _lib.require_cuda(A, "operator")
    _lib.require_cuda(X, "pages")
    if A.dtype != torch.float16 or X.dtype != torch.float16:
        raise TypeError("JL contraction takes float16 operands")
    M, K = A.shape
    if X.shape[-2] != K:
        raise RuntimeError(f"shape mismatch: operator is {tuple(A.shape)}, pages are {tuple(X.shape)}")
    N = X.shape[-1]
    Ac = A.contiguous()
    Xc = X.contiguous()
    batch = Xc.numel() // (K * N) if K * N else 0
    out = torch.empty(X.shape[:-2] + (M, N), dtype=torch.float16, device=X.device)
    _lib.call("argus_jl_apply", _lib.ptr(Ac), _lib.ptr(Xc), batch, M, K, N, _lib.ptr(out),
              _lib.stream_handle(X.device))
    return out


# ------------------------------------------------------------------ attention over archived blocks
BOUND_SYMBOLS = ("argus_jl_operator_fragments", "argus_jl_attention_workspace_size", "argus_jl_attention",
                 "argus_attention_merge")


class JLShapeC(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("heads_kv", ctypes.c_int32), ("group", ctypes.c_int32),
                ("q_len", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("block_rows", ctypes.c_int32),
                ("block_tokens", ctypes.c_int32), ("n_blocks", ctypes.c_int32), ("n_splits", ctypes.c_int32),
                ("n_ctas", ctypes.c_int32), ("scale", ctypes.c_float), ("reserved", ctypes.c_int32),
                ("bh_stride", ctypes.c_int64), ("block_stride", ctypes.c_int64)]


_jl_bound = None


def _jl_bind():
    global _jl_bound
    if _jl_bound is None:
        L = _lib.lib()
        p = ctypes.c_void_p
        L.argus_jl_operator_fragments.argtypes = [p, ctypes.c_int, ctypes.c_int, p, p, p]
        L.argus_jl_operator_fragments.restype = ctypes.c_int
        L.argus_jl_attention_workspace_size.argtypes = [ctypes.POINTER(JLShapeC)]
        L.argus_jl_attention_workspace_size.restype = ctypes.c_int64
        L.argus_jl_attention.argtypes = [ctypes.POINTER(JLShapeC), p, p, p, p, p, p, p, p, p, p]
        L.argus_jl_attention.restype = ctypes.c_int
        L.argus_attention_merge.argtypes = [p, p, p, p, ctypes.c_int64, ctypes.c_int, p, p, p]
        L.argus_attention_merge.restype = ctypes.c_int
        _jl_bound = L
    return _jl_bound


def _check(name, rc):
    if rc != 0:
        raise _lib.ArgusError(name, rc, _lib.lib().argus_last_error().decode())


class JLAttention:
    """Decode attention over JL-archived blocks for one reconstruction operator R [N, MJ] (fp16):
    the same result as softmax attention over K = R @ Yk, V = R @ Yv of every block, computed
    without rebuilding them (libargus_b200 argus_jl_attention).  Blocks are
    yk, yv [B, H_kv, n_blocks, MJ, D] fp16."""

    def __init__(self, recon_operator):
        _lib.require_cuda(recon_operator, "reconstruction operator")
        R = recon_operator.to(torch.float16).contiguous()
        self.N, self.MJ = R.shape
        n = self.N * self.MJ * 2
        self.r_frag = torch.empty(n, dtype=torch.uint8, device=R.device)
        self.rt_frag = torch.empty(n, dtype=torch.uint8, device=R.device)
        _check("argus_jl_operator_fragments", _jl_bind().argus_jl_operator_fragments(
            R.data_ptr(), self.N, self.MJ, self.r_frag.data_ptr(), self.rt_frag.data_ptr(),
            _lib.stream_handle(R.device)))
        self._ws = {}

    def shape(self, q, yk, n_splits=None, scale=None, n_ctas=None):
        B, Hq, qlen, D = q.shape
        _, Hkv, nb, MJ, D2 = yk.shape
        if MJ != self.MJ or D2 != D:
            raise ValueError(f"blocks {tuple(yk.shape)} do not match operator rows {self.MJ} / head_dim {D}")
        if n_ctas is not None:
            n_splits = 1
        n_ctas = int(n_ctas or 0)
        if n_splits is None:
            # one CTA per SM, sharing all heads' blocks in equal contiguous ranges
            n_ctas = min(148, B * Hkv * nb)
            n_splits = 1
        n_splits = max(1, min(int(n_splits), max(1, nb)))
        return JLShapeC(B, Hkv, Hq // Hkv, qlen, D, MJ, self.N, nb, n_splits, n_ctas,
                        1.0 / math.sqrt(D) if scale is None else float(scale), 0, nb * MJ * D, MJ * D)

    def run(self, q, yk, yv, n_splits=None, scale=None, out=None, lse=None, block_lse=None, n_ctas=None):
        """q [B, H_q, q_len, D] fp16 -> out (fp16, same shape) and lse (natural log, fp32 [B, H_q, q_len])
        over the archived tokens only; block_lse ([B*H_kv, n_blocks, 8] fp32), if given, receives each
        block's natural-log LSE per query.  By default one CTA per SM shares all heads' blocks evenly;
        n_splits gives each (batch, kv_head) that many CTAs instead, n_ctas an explicit CTA count."""
        for t, name in ((q, "q"), (yk, "yk"), (yv, "yv")):
            _lib.require_cuda(t, name)
            if t.dtype != torch.float16:
                raise TypeError(f"{name} must be float16")
        if yk.shape != yv.shape:
            raise ValueError("yk and yv shapes differ")
        q, yk, yv = q.contiguous(), yk.contiguous(), yv.contiguous()
        s = self.shape(q, yk, n_splits, scale, n_ctas)
        if out is None:
            out = torch.empty_like(q)
        if lse is None:
            lse = torch.empty(q.shape[:3], dtype=torch.float32, device=q.device)
        L = _jl_bind()
        ws_bytes = L.argus_jl_attention_workspace_size(ctypes.byref(s))
        key = (s.batch, s.heads_kv, s.n_splits, s.n_ctas, q.device)
        ws = self._ws.get(key)
        if ws is None or ws.numel() < ws_bytes:
            ws = torch.zeros(max(ws_bytes, 16), dtype=torch.uint8, device=q.device)  # counters start at zero
            self._ws[key] = ws
        _check("argus_jl_attention", L.argus_jl_attention(
            ctypes.byref(s), yk.data_ptr(), yv.data_ptr(), self.r_frag.data_ptr(), self.rt_frag.data_ptr(),
            q.data_ptr(), out.data_ptr(), lse.data_ptr(), block_lse.data_ptr() if block_lse is not None else None,
            ws.data_ptr(), _lib.stream_handle(q.device)))
        return out, lse


def merge_attention(out_a, lse_a, out_b, lse_b, out=None, lse=None):
    """Joins two attention results over disjoint token sets (fp16 rows, natural-log LSE)."""
    for t in (out_a, lse_a, out_b, lse_b):
        _lib.require_cuda(t)
    D = out_a.shape[-1]
    rows = out_a.numel() // D
    if out is None:
        out = torch.empty_like(out_a)
    _check("argus_attention_merge", _jl_bind().argus_attention_merge(
        out_a.contiguous().data_ptr(), lse_a.contiguous().data_ptr(), out_b.contiguous().data_ptr(),
        lse_b.contiguous().data_ptr(), rows, D, out.data_ptr(), lse.data_ptr() if lse is not None else None,
        _lib.stream_handle(out_a.device)))
    return out
