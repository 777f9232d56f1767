"""GPU parity of decode attention over JL-archived blocks computed without rebuilding K and V
(argus_jl_attention), and of joining it with the other tiers (argus_attention_merge).

Reference: the reference rebuilds every block as fp16(R @ Y) (core/memory_manager.py:1176-1178) and
runs softmax attention over the rebuilt tokens; here that is float64 attention over the same fp16
rebuilt K/V.  Bar: 2e-3 max-abs plus the fp16 output's half-ulp (2^-11 |ref|), as for the other
tiers; the JL result also matches the materializing path (tensor-core R @ Y, then the fused
mixed-tier kernel) within the same bar."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ATOL = 2e-3


def within(out, ref):
    return np.abs(out - ref) <= ATOL + np.abs(ref) * 2.0 ** -11


def operator(N, ratio):
    from argus_b200.core import jl
    W = jl.projection_matrix(N, dtype=torch.float16, device="cpu", seed=42, ratio=ratio)
    return jl.reconstruction_operator_solve(W).to(torch.float16)  # [N, N/ratio]


def f64_attention(q, K, V, scale):
    """q [B, Hq, ql, D]; K, V [B, Hkv, L, D] (numpy) -> float64 softmax attention, GQA expanded."""
    B, Hq, ql, D = q.shape
    Hkv = K.shape[1]
    g = Hq // Hkv
    Kx = np.repeat(K.astype(np.float64), g, axis=1)
    Vx = np.repeat(V.astype(np.float64), g, axis=1)
    s = np.einsum("bhqd,bhkd->bhqk", q.astype(np.float64), Kx) * scale
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, Vx), None


def rebuild(R, Y):
    """fp16(R @ Y) per block, computed in float64 then rounded: Y [B, H, nb, MJ, D] -> [B, H, nb*N, D]."""
    R64 = R.double().numpy()
    Y64 = Y.double().numpy()
    K = np.einsum("nm,bhjmd->bhjnd", R64, Y64).astype(np.float16)
    B, H, nb, N, D = K.shape
    return K.reshape(B, H, nb * N, D)


CASES = [
    # B, Hkv, G, q_len, N (block tokens), ratio, n_blocks, splits
    (2, 2, 4, 1, 1024, 8, 3, 1),
    (1, 2, 4, 1, 1024, 8, 4, 2),
    (1, 1, 2, 2, 512, 4, 5, 2),
    (1, 2, 8, 1, 256, 2, 2, 1),   # 8 queries per kv head: one block per MMA
    (1, 1, 4, 1, 1024, 8, 6, 3),
]


@pytest.mark.parametrize("B,Hkv,G,ql,N,ratio,nb,splits", CASES)
def test_jl_attention_matches_rebuilt_attention(B, Hkv, G, ql, N, ratio, nb, splits):
    from argus_b200 import attention as A
    from argus_b200.core import jl
    MJ, D = N // ratio, 128
    R = operator(N, ratio)
    g = torch.Generator().manual_seed(N + nb + G)
    yk = torch.randn(B, Hkv, nb, MJ, D, generator=g).half()
    yv = torch.randn(B, Hkv, nb, MJ, D, generator=g).half()
    q = (torch.randn(B, Hkv * G, ql, D, generator=g) / math.sqrt(D) * 2.0).half()
    att = jl.JLAttention(R.cuda())
    block_lse = torch.empty(B * Hkv, nb, 8, dtype=torch.float32, device="cuda")
    out, lse = att.run(q.cuda(), yk.cuda(), yv.cuda(), n_splits=splits, block_lse=block_lse)
    torch.cuda.synchronize()
    assert A.device_status() == 0
    K, V = rebuild(R, yk), rebuild(R, yv)
    ref, _ = f64_attention(q.numpy(), K, V, 1.0 / math.sqrt(D))
    got = out.cpu().numpy().astype(np.float64)
    assert within(got, ref).all(), np.abs(got - ref).max()
    # LSE (natural log) of the scores over the archived tokens
    Kx = np.repeat(K.astype(np.float64), G, axis=1)
    s = np.einsum("bhqd,bhkd->bhqk", q.numpy().astype(np.float64), Kx) / math.sqrt(D)
    mx = s.max(-1)
    ref_lse = mx + np.log(np.exp(s - mx[..., None]).sum(-1))
    assert np.allclose(lse.cpu().numpy(), ref_lse, rtol=0, atol=2e-3)
    # per-block LSE (the per-page attention mass of the importance policy is exp(block - total))
    sb = s.reshape(B, Hkv, G, ql, nb, N)
    mb = sb.max(-1)
    ref_blk = mb + np.log(np.exp(sb - mb[..., None]).sum(-1))          # [B, Hkv, G, ql, nb]
    ref_blk = ref_blk.reshape(B * Hkv, G * ql, nb).transpose(0, 2, 1)  # [B*Hkv, nb, G*ql]
    got_blk = block_lse.cpu().numpy()[:, :, :G * ql]
    assert np.allclose(got_blk, ref_blk, rtol=0, atol=2e-3), np.abs(got_blk - ref_blk).max()
    # the materializing path: tensor-core rebuild, then the fused mixed-tier kernel
    Kg = jl.apply_left(R.cuda(), yk.cuda().reshape(B * Hkv * nb, MJ, D)).reshape(B, Hkv, nb * N, D)
    Vg = jl.apply_left(R.cuda(), yv.cuda().reshape(B * Hkv * nb, MJ, D)).reshape(B, Hkv, nb * N, D)
    arena = A.KVArena.from_fp16(Kg.contiguous(), Vg.contiguous())
    plan = A.AttentionPlan([arena], [(0, j, 16) for j in range(nb * N // 16)], batch=B, heads_kv=Hkv, group=G,
                           head_dim=D, q_len=ql)
    mat = plan.run(q.cuda()).cpu().numpy().astype(np.float64)
    assert within(got, mat).all(), np.abs(got - mat).max()


@pytest.mark.parametrize("B,Hkv,G,nb,n_ctas", [
    (2, 2, 4, 7, 5),      # CTA ranges that span two heads
    (1, 3, 4, 9, 4),
    (2, 2, 8, 3, 5),      # 8 queries per head
    (1, 2, 4, 6, None),   # the default: one CTA per block here
    (1, 1, 4, 40, 1),     # one CTA, two rounds: 32 blocks (128 rows, hi and lo MMAs) then 8 (stacked)
    (1, 2, 8, 20, 2),     # 8 queries: rounds of 16 blocks, a head continued across rounds
    (1, 2, 4, 20, 2),     # 80 rows in one round (hi and lo MMAs, three softmax warps)
])
def test_jl_attention_ctas_span_heads(B, Hkv, G, nb, n_ctas):
    """CTAs that take a contiguous range of all heads' blocks (crossing from one head to the next,
    in rounds of at most 128 (block, query) rows) give the same attention and per-block LSE as the
    rebuilt K/V, on two launches in a row (the arrival counters are left at zero)."""
    from argus_b200 import attention as A
    from argus_b200.core import jl
    N, ratio, D, ql = 512, 4, 128, 1
    MJ = N // ratio
    R = operator(N, ratio)
    g = torch.Generator().manual_seed(100 + nb + (n_ctas or 0))
    yk = torch.randn(B, Hkv, nb, MJ, D, generator=g).half()
    yv = torch.randn(B, Hkv, nb, MJ, D, generator=g).half()
    q = (torch.randn(B, Hkv * G, ql, D, generator=g) / math.sqrt(D) * 2.0).half()
    att = jl.JLAttention(R.cuda())
    K, V = rebuild(R, yk), rebuild(R, yv)
    ref, _ = f64_attention(q.numpy(), K, V, 1.0 / math.sqrt(D))
    Kx = np.repeat(K.astype(np.float64), G, axis=1)
    s = np.einsum("bhqd,bhkd->bhqk", q.numpy().astype(np.float64), Kx) / math.sqrt(D)
    sb = s.reshape(B, Hkv, G, ql, nb, N)
    mb = sb.max(-1)
    ref_blk = (mb + np.log(np.exp(sb - mb[..., None]).sum(-1))).reshape(B * Hkv, G * ql, nb).transpose(0, 2, 1)
    block_lse = torch.empty(B * Hkv, nb, 8, dtype=torch.float32, device="cuda")
    for _ in range(2):
        out, lse = att.run(q.cuda(), yk.cuda(), yv.cuda(), block_lse=block_lse, n_ctas=n_ctas)
        torch.cuda.synchronize()
        assert A.device_status() == 0
        got = out.cpu().numpy().astype(np.float64)
        assert within(got, ref).all(), np.abs(got - ref).max()
        assert np.allclose(block_lse.cpu().numpy()[:, :, :G * ql], ref_blk, rtol=0, atol=2e-3)


@pytest.mark.parametrize("D,N,ratio,G,nb,n_ctas", [
    (64, 512, 4, 4, 5, 3),     # head_dim 64, 128-row blocks
    (128, 256, 4, 4, 5, 3),    # 64-row blocks
    (64, 256, 4, 4, 5, 3),     # both
    (64, 256, 4, 8, 20, 2),    # 64-row blocks, 8 queries: rounds of 16 blocks (128 rows), then 4
    (64, 1024, 16, 4, 40, 1),  # one CTA over two rounds
])
def test_jl_attention_head_dims_and_block_rows(D, N, ratio, G, nb, n_ctas):
    """head_dim 64 and 64-row blocks (256-token pages at the reference's ratio 4) through the same
    kernel: attention and per-block LSE as the rebuilt K/V."""
    from argus_b200 import attention as A
    from argus_b200.core import jl
    B, Hkv, ql = 1, 2, 1
    MJ = N // ratio
    R = operator(N, ratio)
    g = torch.Generator().manual_seed(D + N + nb)
    yk = torch.randn(B, Hkv, nb, MJ, D, generator=g).half()
    yv = torch.randn(B, Hkv, nb, MJ, D, generator=g).half()
    q = (torch.randn(B, Hkv * G, ql, D, generator=g) / math.sqrt(D) * 2.0).half()
    att = jl.JLAttention(R.cuda())
    block_lse = torch.empty(B * Hkv, nb, 8, dtype=torch.float32, device="cuda")
    out, lse = att.run(q.cuda(), yk.cuda(), yv.cuda(), block_lse=block_lse, n_ctas=n_ctas)
    torch.cuda.synchronize()
    assert A.device_status() == 0
    K, V = rebuild(R, yk), rebuild(R, yv)
    ref, _ = f64_attention(q.numpy(), K, V, 1.0 / math.sqrt(D))
    got = out.cpu().numpy().astype(np.float64)
    assert within(got, ref).all(), np.abs(got - ref).max()
    Kx = np.repeat(K.astype(np.float64), G, axis=1)
    s = np.einsum("bhqd,bhkd->bhqk", q.numpy().astype(np.float64), Kx) / math.sqrt(D)
    mx = s.max(-1)
    assert np.allclose(lse.cpu().numpy(), mx + np.log(np.exp(s - mx[..., None]).sum(-1)), rtol=0, atol=2e-3)
    sb = s.reshape(B, Hkv, G, ql, nb, N)
    mb = sb.max(-1)
    ref_blk = (mb + np.log(np.exp(sb - mb[..., None]).sum(-1))).reshape(B * Hkv, G * ql, nb).transpose(0, 2, 1)
    assert np.allclose(block_lse.cpu().numpy()[:, :, :G * ql], ref_blk, rtol=0, atol=2e-3)


def test_merge_joins_jl_archive_with_other_tiers():
    from argus_b200 import attention as A
    from argus_b200.core import jl
    B, Hkv, G, N, ratio, nb, D, Lhot = 1, 2, 4, 512, 4, 2, 128, 96
    MJ = N // ratio
    R = operator(N, ratio)
    g = torch.Generator().manual_seed(5)
    yk = torch.randn(B, Hkv, nb, MJ, D, generator=g).half()
    yv = torch.randn(B, Hkv, nb, MJ, D, generator=g).half()
    kh = torch.randn(B, Hkv, Lhot, D, generator=g).half()
    vh = torch.randn(B, Hkv, Lhot, D, generator=g).half()
    q = (torch.randn(B, Hkv * G, 1, D, generator=g) / math.sqrt(D)).half()
    out_j, lse_j = jl.JLAttention(R.cuda()).run(q.cuda(), yk.cuda(), yv.cuda())
    arena = A.KVArena.from_fp16(kh.cuda(), vh.cuda())
    plan = A.AttentionPlan([arena], [(0, j, 16) for j in range(Lhot // 16)], batch=B, heads_kv=Hkv, group=G,
                           head_dim=D)
    lse_h = torch.empty(B, Hkv * G, 1, dtype=torch.float32, device="cuda")
    out_h = plan.run(q.cuda(), lse=lse_h)
    out = jl.merge_attention(out_j, lse_j, out_h, lse_h)
    torch.cuda.synchronize()
    K = np.concatenate([rebuild(R, yk), kh.numpy()], axis=2)
    V = np.concatenate([rebuild(R, yv), vh.numpy()], axis=2)
    ref, _ = f64_attention(q.numpy(), K, V, 1.0 / math.sqrt(D))
    got = out.cpu().numpy().astype(np.float64)
    # two fp16 partial results are joined: allow one more output half-ulp
    assert (np.abs(got - ref) <= ATOL + np.abs(ref) * 2.0 ** -10).all(), np.abs(got - ref).max()
