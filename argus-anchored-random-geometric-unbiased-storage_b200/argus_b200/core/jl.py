"""JL sequence-projection archive: matrices (host, fp32/CPU as the reference builds them) and the
batched contraction C[b] = A @ X[b] on the GPU (libargus_b200 argus_jl_apply).

Reference lines: core/memory_manager.py:227-282 (W and R of the manager, ratio 4, seed 42),
core/quantization.py:224-290 (per-call W and the solve-form R).
"""
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
