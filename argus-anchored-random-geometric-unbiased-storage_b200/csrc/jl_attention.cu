// Decode attention over the JL sequence-projection archive, without reconstructing K and V.
//
// The reference rebuilds each archived block as K = R . Yk, V = R . Yv (R = A^-1 W^T (W A^-1 W^T)^-1,
// core/memory_manager.py:241-282, 1176-1178) and runs softmax attention over the rebuilt tokens.
// Because the reconstruction is linear, the same attention is
//     s = R . (Yk . q^T)          scores of the block's N tokens      (N x MJ) . (MJ x Q)
//     w = R^T . p                 softmax weights folded back         (MJ x N) . (N x Q)
//     o += Yv^T . w               output contribution                 (D x MJ) . (MJ x Q)
// which costs 2*N*MJ*Q + 2*MJ*D*Q multiply-adds per block instead of 2*N*MJ*D (K and V rebuilt)
// plus the attention itself.  All contractions run on the tensor cores (mma.sync m16n8k16, fp32
// accumulation; u, p and w enter as fp16 hi + lo pairs).  R and R^T are stored once in MMA fragment
// order so every operand load is one coalesced 16-byte read per lane from L2.
//
// The CTAs (8 warps each) share the block pairs of all (batch, kv_head) in equal contiguous ranges,
// so every SM gets the same work whatever the head count; a range that spans two heads yields a
// partial for each, and the last CTA to finish a head merges its partials.  With at most 4 queries
// per kv head two archive blocks share the 8 query columns of every MMA.  Per block pair: warp w forms u rows 16w..16w+15,
// then streams token tiles w, w+8, ... through scores, online softmax (per column, log2 domain)
// and w accumulation; the warps' partial w merge in shared memory; warp w then adds Yv^T . w for
// dims 16w..16w+15.  Yk / Yv blocks arrive by TMA tensor copies in 128-byte swizzle (two 64-column
// halves of 128 rows x 128 bytes, 16-byte chunk c of row r stored at chunk c ^ (r % 8)) so the
// ldmatrix reads of both contractions are free of bank conflicts; each buffer is refilled as soon as
// it is consumed.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace argus {
namespace jla {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kD = 128;   // head_dim
constexpr int kMJ = 128;  // rows per archived block
constexpr int kCols = 8;  // query columns per MMA
constexpr long long kSpinLimit = 1ll << 26;
constexpr float kNoMax = -1.0e30f;
constexpr float kSlack = 8.0f;

__device__ int g_status = 0;

struct Params {
    CUtensorMap tmk;    // Yk as [B*Hkv][n_blocks][MJ][D], box 64 x MJ, 128-byte swizzle
    CUtensorMap tmv;    // Yv, same
    const __half* yk;   // block j of (b, h) at yk + bh * bh_stride + j * block_stride
    const __half* yv;
    const uint4* rf;    // R [N x MJ] in A-fragment order: [N/16][MJ/16][32 lanes]
    const uint4* rtf;   // R^T [MJ x N] in A-fragment order: [MJ/16][N/16][32 lanes]
    const __half* q;    // [B, Hkv*G, qlen, D]
    __half* out;
    float* lse;
    float* block_lse;   // optional [B*Hkv][n_blocks][8]: natural-log LSE of each block's scores
    float* part_o;      // [B*Hkv][S][8][D]  (S: partial slots per (b, h))
    float* part_lse;    // [B*Hkv][S][8]
    int* counters;      // [B*Hkv]
    int64_t bh_stride, block_stride;  // elements
    int B, Hkv, G, qlen, n_blocks, N, S;
    float scale_log2;
};

constexpr int kRowPad = kMJ + 8;  // u^T / w^T row stride in halves (272 bytes: conflict-free reads)

__host__ __device__ constexpr size_t smem_bytes(int pack) {
    return 1024                                 // alignment of the swizzled tiles
           + (size_t)2 * pack * kMJ * kD * 2    // Yk, Yv blocks
           + (size_t)2 * 2 * kCols * kRowPad * 2  // u^T and w^T, fp16 hi / lo
           + (size_t)kWarps * 32 * 33 * 4       // per-warp partial w (lane stride 33)
           + (size_t)(2 * kWarps * kCols + kWarps * kCols + 4 * kCols) * 4 + 64;
}

__device__ __forceinline__ uint32_t su32(const void* p) { return smem_u32(p); }
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
    uint32_t y;
    asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&a)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&a)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
                 : "r"(addr));
}
__device__ __forceinline__ uint32_t h2pack(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void split_hl(float v, __half& hi, __half& lo) {
    hi = __float2half_rn(v);
    lo = __float2half_rn(v - __half2float(hi));
}
__device__ __forceinline__ void mbar_init(uint32_t bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t phase) {
    for (long long i = 0; i < kSpinLimit; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(bar), "r"(phase)
            : "memory");
        if (ok) return true;
    }
    return false;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ uint4 ldg_nc(const uint4* p) {
    uint4 r;
    asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
        : "memory");
}

// Copies blocks j .. j+nb-1 of (b, h) into `dst` (per block two swizzled 64-column halves) and arms
// `bar` for the bytes.
__device__ __forceinline__ void issue_blocks(const CUtensorMap* map, int64_t bh, int j, int nb, __half* dst, uint32_t bar) {
    constexpr uint32_t bytes = kMJ * kD * 2;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(bar, bytes * nb);
    for (int i = 0; i < nb; ++i) {
        const uint32_t d = su32(dst + (size_t)i * kMJ * kD);
        tma_load_4d(d, map, 0, 0, j + i, (int)bh, bar);
        tma_load_4d(d + kMJ * 128, map, 64, 0, j + i, (int)bh, bar);
    }
}

// Shared-memory address of element (row r, column c) of a swizzled [MJ][D] block.
__device__ __forceinline__ uint32_t swz(uint32_t base, int r, int c) {
    return base + (uint32_t)((c >> 6) * (kMJ * 128) + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + (c & 7) * 2);
}

template <int PACK>
__global__ void __launch_bounds__(kThreads, 1) jl_attn_kernel(const __grid_constant__ Params p) {
    constexpr int KD = kD / 16, KM = kMJ / 16;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    __half* ykbuf = reinterpret_cast<__half*>(smem);               // [PACK][MJ][D] swizzled
    __half* yvbuf = ykbuf + PACK * kMJ * kD;                        // [PACK][MJ][D]
    __half* uT = yvbuf + PACK * kMJ * kD;                           // [2][8][MJ + pad]
    __half* wt = uT + 2 * kCols * kRowPad;                          // [2][8][MJ + pad]
    float* wpart = reinterpret_cast<float*>(wt + 2 * kCols * kRowPad);  // [warps][32 lanes][33]
    float* mw = wpart + kWarps * 32 * 33;                           // [warps][8]
    float* lw = mw + kWarps * kCols;                                // [warps][8]
    float* fw = lw + kWarps * kCols;                                // [warps][8] merge factors
    float* mrun = fw + kWarps * kCols;                              // [8]
    float* lrun = mrun + kCols;                                     // [8]
    float* alpha = lrun + kCols;                                    // [8]
    float* beta = alpha + kCols;                                    // [8]
    uint64_t* bars = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(beta + kCols) + 15) & ~(uintptr_t)15);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int NQ = p.G * p.qlen;
    const int qpb = PACK == 2 ? 4 : 8;  // query columns per block
    const uint32_t ykbar = su32(&bars[0]), yvbar = su32(&bars[1]);
    if (tid == 0) {
        mbar_init(ykbar);
        mbar_init(yvbar);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __shared__ int last;

    // The block pairs of all (batch, kv_head) groups, group after group, are dealt to the CTAs in
    // equal contiguous ranges: pair x goes to CTA floor(x C / T).  A CTA whose range crosses groups
    // finishes one group's segment (a partial) and starts the next.
    const int64_t groups = (int64_t)p.B * p.Hkv;
    const int64_t PP = (p.n_blocks + PACK - 1) / PACK, T = groups * PP;
    const int64_t C = gridDim.x, c = blockIdx.x;
    const int64_t x_end = ((c + 1) * T + C - 1) / C;
    bool ok = true;
    int it = 0;
    // parity of each buffer's issued copy not yet seen complete (-1: none); kept alike by every
    // thread, so that after a timed-out wait the CTA waits (bounded) for exactly the copies in flight
    int yk_pend = -1, yv_pend = -1;
    for (int64_t xs = (c * T + C - 1) / C; xs < x_end && ok;) {
    const int64_t bh = xs / PP;
    const int64_t xe = (x_end < (bh + 1) * PP) ? x_end : (bh + 1) * PP;
    const int j0 = (int)((xs - bh * PP) * PACK);
    const int j1 = (int)(((xe - bh * PP) * PACK < p.n_blocks) ? (xe - bh * PP) * PACK : p.n_blocks);
    const int64_t first_c = bh * PP * C / T, last_c = ((bh + 1) * PP - 1) * C / T;
    const int n_seg = (int)(last_c - first_c + 1), split = (int)(c - first_c);  // this group's partials
    xs = xe;
    const int b = (int)(bh / p.Hkv), h = (int)(bh - (int64_t)b * p.Hkv);

    // query fragments: column n of the U contraction is query n (block A) or n - 4 (block B)
    uint32_t qa[KD][2], qb[KD][2];
    {
        const int na = g, nb_ = g - 4;
        const bool la = na < (PACK == 2 ? 4 : 8) && na < NQ, lb = PACK == 2 && nb_ >= 0 && nb_ < NQ;
        const __half* qbase = p.q + (((int64_t)b * p.Hkv * p.G + (int64_t)h * p.G) * p.qlen) * kD;
#pragma unroll
        for (int kk = 0; kk < KD; ++kk) {
            const int d = 16 * kk + 2 * t;
            qa[kk][0] = la ? *reinterpret_cast<const uint32_t*>(qbase + (int64_t)na * kD + d) : 0u;
            qa[kk][1] = la ? *reinterpret_cast<const uint32_t*>(qbase + (int64_t)na * kD + d + 8) : 0u;
            qb[kk][0] = lb ? *reinterpret_cast<const uint32_t*>(qbase + (int64_t)nb_ * kD + d) : 0u;
            qb[kk][1] = lb ? *reinterpret_cast<const uint32_t*>(qbase + (int64_t)nb_ * kD + d + 8) : 0u;
        }
    }
    if (tid < kCols) {
        mrun[tid] = kNoMax;
        lrun[tid] = 0.f;
    }
    __syncthreads();
    if (j0 < j1) {
        if (tid == 0) {
            const int nb = (j1 - j0) < PACK ? (j1 - j0) : PACK;
            issue_blocks(&p.tmk, bh, j0, nb, ykbuf, ykbar);
            issue_blocks(&p.tmv, bh, j0, nb, yvbuf, yvbar);
        }
        yk_pend = yv_pend = it & 1;
    }

    float oacc[4] = {0.f, 0.f, 0.f, 0.f};  // dims 16*warp + g (+8), columns 2t, 2t+1
    for (int j = j0; j < j1 && ok; j += PACK, ++it) {
        const bool hasB = PACK == 2 && j + 1 < j1;
        ok = __syncthreads_and(mbar_wait(ykbar, (uint32_t)(it & 1)));
        if (!ok) break;
        yk_pend = -1;
        // ---- u = Yk . q^T: rows 16*warp .. +15, block A in columns 0..3 (or 0..7), block B in 4..7
        {
            float u[4] = {0.f, 0.f, 0.f, 0.f}, u2[4] = {0.f, 0.f, 0.f, 0.f};  // two independent chains
            const int row = 16 * warp + (lane & 7) + 8 * ((lane >> 3) & 1);
            const int colo = 8 * (lane >> 4);
            const uint32_t ka = su32(ykbuf), kb = su32(ykbuf + (size_t)kMJ * kD);
#pragma unroll
            for (int kk = 0; kk < KD; ++kk) {
                uint32_t a[4];
                ldsm_x4(swz(ka, row, 16 * kk + colo), a);
                mma16816((kk & 1) ? u2 : u, a, qa[kk][0], qa[kk][1]);
                if (hasB) {
                    ldsm_x4(swz(kb, row, 16 * kk + colo), a);
                    mma16816((kk & 1) ? u : u2, a, qb[kk][0], qb[kk][1]);
                }
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) u[c] += u2[c];
            const int m0 = 16 * warp + g;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int m = m0 + 8 * (c >> 1), n = 2 * t + (c & 1);
                __half hi, lo;
                split_hl(u[c], hi, lo);
                uT[n * kRowPad + m] = hi;
                uT[kCols * kRowPad + n * kRowPad + m] = lo;
            }
        }
        __syncthreads();
        if (j + PACK < j1) {  // Yk buffer consumed: bring the next pair
            if (tid == 0) {
                const int nb = (j1 - j - PACK) < PACK ? (j1 - j - PACK) : PACK;
                issue_blocks(&p.tmk, bh, j + PACK, nb, ykbuf, ykbar);
            }
            yk_pend = (it + 1) & 1;
        }
        // ---- scores, softmax and w over this warp's token tiles
        uint32_t ub[KM][2][2];
#pragma unroll
        for (int kk = 0; kk < KM; ++kk)
#pragma unroll
            for (int hl = 0; hl < 2; ++hl) {
                const __half* r = uT + hl * kCols * kRowPad + g * kRowPad + 16 * kk + 2 * t;
                ub[kk][hl][0] = *reinterpret_cast<const uint32_t*>(r);
                ub[kk][hl][1] = *reinterpret_cast<const uint32_t*>(r + 8);
            }
        // columns this thread's scores belong to: 2t, 2t+1; dead when the block or query is absent
        const int qn0 = (2 * t) % qpb, qn1 = (2 * t + 1) % qpb;
        const bool colB = PACK == 2 && t >= 2;
        const bool live0 = qn0 < NQ && (!colB || hasB), live1 = qn1 < NQ && (!colB || hasB);
        float ms[2] = {kNoMax, kNoMax}, ls[2] = {0.f, 0.f};
        float wacc[KM][4];
#pragma unroll
        for (int mt = 0; mt < KM; ++mt) wacc[mt][0] = wacc[mt][1] = wacc[mt][2] = wacc[mt][3] = 0.f;
        const int ntiles = p.N / 16;
        uint4 rcur[KM];  // R fragments of the current tile, loaded one tile ahead
#pragma unroll
        for (int kk = 0; kk < KM; ++kk) rcur[kk] = ldg_nc(p.rf + ((size_t)warp * KM + kk) * 32 + lane);
        for (int tt = warp; tt < ntiles; tt += kWarps) {
            uint4 rt[KM];  // R^T fragments of this tile: in flight while the scores and softmax run
            const uint4* rtf = p.rtf + (size_t)tt * 32 + lane;
#pragma unroll
            for (int mt = 0; mt < KM; ++mt) rt[mt] = ldg_nc(rtf + (size_t)mt * ntiles * 32);
            float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
            float sc[4] = {0.f, 0.f, 0.f, 0.f}, sd[4] = {0.f, 0.f, 0.f, 0.f};  // four independent chains
#pragma unroll
            for (int kk = 0; kk < KM; ++kk) {
                const uint32_t a[4] = {rcur[kk].x, rcur[kk].y, rcur[kk].z, rcur[kk].w};
                mma16816((kk & 1) ? sc : sa, a, ub[kk][0][0], ub[kk][0][1]);
                mma16816((kk & 1) ? sd : sb, a, ub[kk][1][0], ub[kk][1][1]);
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) { sa[c] += sc[c]; sb[c] += sd[c]; }
            if (tt + kWarps < ntiles) {
#pragma unroll
                for (int kk = 0; kk < KM; ++kk) rcur[kk] = ldg_nc(p.rf + ((size_t)(tt + kWarps) * KM + kk) * 32 + lane);
            }
            float x[4];
            x[0] = live0 ? (sa[0] + sb[0]) * p.scale_log2 : -INFINITY;
            x[1] = live1 ? (sa[1] + sb[1]) * p.scale_log2 : -INFINITY;
            x[2] = live0 ? (sa[2] + sb[2]) * p.scale_log2 : -INFINITY;
            x[3] = live1 ? (sa[3] + sb[3]) * p.scale_log2 : -INFINITY;
            const bool over = (fmaxf(x[0], x[2]) > ms[0] + kSlack) | (fmaxf(x[1], x[3]) > ms[1] + kSlack);
            if (__any_sync(0xffffffffu, over)) {
                float mx0 = fmaxf(x[0], x[2]), mx1 = fmaxf(x[1], x[3]);
#pragma unroll
                for (int off = 4; off < 32; off <<= 1) {
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
                }
                const float n0 = fmaxf(ms[0], mx0), n1 = fmaxf(ms[1], mx1);
                const float f0 = exp2f(ms[0] - n0), f1 = exp2f(ms[1] - n1);
                // w rows are MJ, columns are the score columns: c0/c2 -> column 2t, c1/c3 -> 2t+1
#pragma unroll
                for (int mt = 0; mt < KM; ++mt) { wacc[mt][0] *= f0; wacc[mt][2] *= f0; wacc[mt][1] *= f1; wacc[mt][3] *= f1; }
                ls[0] *= f0; ls[1] *= f1;
                ms[0] = n0; ms[1] = n1;
            }
            const float p0 = exp2f(x[0] - ms[0]), p1 = exp2f(x[1] - ms[1]);
            const float p2 = exp2f(x[2] - ms[0]), p3 = exp2f(x[3] - ms[1]);
            ls[0] += p0 + p2;
            ls[1] += p1 + p3;
            const __half2 h01 = __floats2half2_rn(p0, p1), h23 = __floats2half2_rn(p2, p3);
            const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
            const uint32_t b01 = movmatrix_t(*reinterpret_cast<const uint32_t*>(&h01));
            const uint32_t b23 = movmatrix_t(*reinterpret_cast<const uint32_t*>(&h23));
            const uint32_t c01 = movmatrix_t(h2pack(p0 - f01.x, p1 - f01.y));
            const uint32_t c23 = movmatrix_t(h2pack(p2 - f23.x, p3 - f23.y));
#pragma unroll
            for (int mt = 0; mt < KM; ++mt) {
                const uint32_t a[4] = {rt[mt].x, rt[mt].y, rt[mt].z, rt[mt].w};
                mma16816(wacc[mt], a, b01, b23);
            }
#pragma unroll
            for (int mt = 0; mt < KM; ++mt) {
                const uint32_t a[4] = {rt[mt].x, rt[mt].y, rt[mt].z, rt[mt].w};
                mma16816(wacc[mt], a, c01, c23);
            }
        }
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            ls[0] += __shfl_xor_sync(0xffffffffu, ls[0], off);
            ls[1] += __shfl_xor_sync(0xffffffffu, ls[1], off);
        }
        if (g == 0) {
            mw[warp * kCols + 2 * t] = ms[0];
            mw[warp * kCols + 2 * t + 1] = ms[1];
            lw[warp * kCols + 2 * t] = ls[0];
            lw[warp * kCols + 2 * t + 1] = ls[1];
        }
        {
            float* wp = wpart + ((size_t)warp * 32 + lane) * 33;
#pragma unroll
            for (int mt = 0; mt < KM; ++mt)
#pragma unroll
                for (int c = 0; c < 4; ++c) wp[4 * mt + c] = wacc[mt][c];
        }
        __syncthreads();
        // ---- merge the warps' w, fold into the running (per column) softmax state
        if (tid < kCols) {
            const int n = tid;
            float mb = kNoMax;
            for (int w = 0; w < kWarps; ++w) mb = fmaxf(mb, mw[w * kCols + n]);
            float lb = 0.f;
            for (int w = 0; w < kWarps; ++w) lb += exp2f(mw[w * kCols + n] - mb) * lw[w * kCols + n];
            if (p.block_lse) {  // column n belongs to block j (+1 for the upper columns when packed)
                const int blk = j + ((PACK == 2 && n >= 4) ? 1 : 0), qn = n % qpb;
                if (qn < NQ && blk < j1)
                    p.block_lse[(bh * p.n_blocks + blk) * kCols + qn] =
                        lb > 0.f ? (mb + log2f(lb)) * 0.69314718055994530942f : -INFINITY;
            }
            const float mo = mrun[n], mn = fmaxf(mo, mb);
            const float a = exp2f(mo - mn), be = exp2f(mb - mn);
            lrun[n] = a * lrun[n] + be * lb;
            mrun[n] = mn;
            alpha[n] = a;
            for (int w = 0; w < kWarps; ++w) fw[w * kCols + n] = exp2f(mw[w * kCols + n] - mb) * be;
        }
        __syncthreads();
        for (int pos = tid; pos < kMJ * kCols; pos += kThreads) {
            const int ln = pos & 31, idx = pos >> 5;  // (lane, value index) of the per-warp fragments
            const int mt = idx >> 2, c = idx & 3;
            const int m = 16 * mt + (ln >> 2) + 8 * (c >> 1), n = 2 * (ln & 3) + (c & 1);
            float wv = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) wv += fw[w * kCols + n] * wpart[((size_t)w * 32 + ln) * 33 + idx];
            __half hi, lo;
            split_hl(wv, hi, lo);
            wt[n * kRowPad + m] = hi;
            wt[kCols * kRowPad + n * kRowPad + m] = lo;
        }
        __syncthreads();
        ok = __syncthreads_and(mbar_wait(yvbar, (uint32_t)(it & 1)));
        if (!ok) break;
        yv_pend = -1;
        // ---- o += Yv^T . w for dims 16*warp .. +15
        {
            const float a0 = alpha[2 * t], a1 = alpha[2 * t + 1];
            oacc[0] *= a0; oacc[2] *= a0; oacc[1] *= a1; oacc[3] *= a1;
            float olo[4] = {0.f, 0.f, 0.f, 0.f};  // the lo parts of w: an independent chain
            const int mrow = (lane & 7) + 8 * (lane >> 4), dcol = 16 * warp + 8 * ((lane >> 3) & 1);
            const bool inA = PACK == 1 || g < 4;
#pragma unroll
            for (int kk = 0; kk < KM; ++kk) {
                const __half* wr = wt + g * kRowPad + 16 * kk + 2 * t;
                const uint32_t wh0 = *reinterpret_cast<const uint32_t*>(wr), wh1 = *reinterpret_cast<const uint32_t*>(wr + 8);
                const uint32_t wl0 = *reinterpret_cast<const uint32_t*>(wr + kCols * kRowPad);
                const uint32_t wl1 = *reinterpret_cast<const uint32_t*>(wr + kCols * kRowPad + 8);
                uint32_t a[4];
                ldsm_x4_t(swz(su32(yvbuf), 16 * kk + mrow, dcol), a);
                mma16816(oacc, a, inA ? wh0 : 0u, inA ? wh1 : 0u);
                mma16816(olo, a, inA ? wl0 : 0u, inA ? wl1 : 0u);
                if (hasB) {
                    ldsm_x4_t(swz(su32(yvbuf + (size_t)kMJ * kD), 16 * kk + mrow, dcol), a);
                    mma16816(oacc, a, inA ? 0u : wh0, inA ? 0u : wh1);
                    mma16816(olo, a, inA ? 0u : wl0, inA ? 0u : wl1);
                }
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) oacc[c] += olo[c];
        }
        __syncthreads();
        if (j + PACK < j1) {  // Yv buffer consumed
            if (tid == 0) {
                const int nb = (j1 - j - PACK) < PACK ? (j1 - j - PACK) : PACK;
                issue_blocks(&p.tmv, bh, j + PACK, nb, yvbuf, yvbar);
            }
            yv_pend = (it + 1) & 1;
        }
    }
    if (!ok) {
        if (tid == 0) atomicExch(&g_status, (int)ARGUS_ERR_TIMEOUT);
        // let copies in flight land before the CTA exits (bounded)
        if (yk_pend >= 0) (void)mbar_wait(ykbar, (uint32_t)yk_pend);
        if (yv_pend >= 0) (void)mbar_wait(yvbar, (uint32_t)yv_pend);
        break;
    }
    __syncthreads();

    // ---- per query: merge block columns (n and n + 4 when two blocks share the MMA), write partials
    float o0 = oacc[0], o1 = oacc[1], o2 = oacc[2], o3 = oacc[3];
    float M0 = mrun[2 * t], M1 = mrun[2 * t + 1], L0 = lrun[2 * t], L1 = lrun[2 * t + 1];
    if (PACK == 2) {
        const float po0 = __shfl_xor_sync(0xffffffffu, o0, 2), po1 = __shfl_xor_sync(0xffffffffu, o1, 2);
        const float po2 = __shfl_xor_sync(0xffffffffu, o2, 2), po3 = __shfl_xor_sync(0xffffffffu, o3, 2);
        const int pt = t ^ 2;
        const float PM0 = mrun[2 * pt], PM1 = mrun[2 * pt + 1], PL0 = lrun[2 * pt], PL1 = lrun[2 * pt + 1];
        const float N0 = fmaxf(M0, PM0), N1 = fmaxf(M1, PM1);
        const float x0 = exp2f(M0 - N0), y0 = exp2f(PM0 - N0), x1 = exp2f(M1 - N1), y1 = exp2f(PM1 - N1);
        o0 = x0 * o0 + y0 * po0; o2 = x0 * o2 + y0 * po2;
        o1 = x1 * o1 + y1 * po1; o3 = x1 * o3 + y1 * po3;
        L0 = x0 * L0 + y0 * PL0; L1 = x1 * L1 + y1 * PL1;
        M0 = N0; M1 = N1;
    }
    const bool writer = PACK == 1 || t < 2;
    const int d0 = 16 * warp + g;
    if (writer) {
        const int n0 = 2 * t, n1 = 2 * t + 1;  // query index (t < 2 when packed)
        float* po = p.part_o + ((bh * p.S + split) * kCols) * kD;  // p.S: partial slots per group
        po[n0 * kD + d0] = L0 > 0.f ? o0 / L0 : 0.f;
        po[n0 * kD + d0 + 8] = L0 > 0.f ? o2 / L0 : 0.f;
        po[n1 * kD + d0] = L1 > 0.f ? o1 / L1 : 0.f;
        po[n1 * kD + d0 + 8] = L1 > 0.f ? o3 / L1 : 0.f;
        if (warp == 0 && g == 0) {
            p.part_lse[(bh * p.S + split) * kCols + n0] = L0 > 0.f ? M0 + log2f(L0) : -INFINITY;
            p.part_lse[(bh * p.S + split) * kCols + n1] = L1 > 0.f ? M1 + log2f(L1) : -INFINITY;
        }
    }
    // ---- the last segment CTA of this (b, h) merges its partials
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const int prev = atomicAdd(&p.counters[bh], 1);
        last = prev == n_seg - 1;
        if (last) p.counters[bh] = 0;
    }
    __syncthreads();
    if (last) {
    __threadfence();
    for (int e = tid; e < NQ * kD; e += kThreads) {
        const int n = e / kD, d = e - n * kD;
        const float* pl = p.part_lse + bh * p.S * kCols + n;
        float M = -INFINITY;
        for (int s = 0; s < n_seg; ++s) M = fmaxf(M, __ldcg(pl + s * kCols));
        float W = 0.f, acc = 0.f;
        if (M != -INFINITY) {
            for (int s = 0; s < n_seg; ++s) {
                const float wgt = exp2f(__ldcg(pl + s * kCols) - M);
                W += wgt;
                acc += wgt * __ldcg(p.part_o + ((bh * p.S + s) * kCols + n) * kD + d);
            }
        }
        const int gi = n / p.qlen, qi = n - gi * p.qlen;
        const int64_t row = ((int64_t)b * p.Hkv * p.G + (int64_t)h * p.G + gi) * p.qlen + qi;
        p.out[row * kD + d] = __float2half_rn(W > 0.f ? acc / W : 0.f);
        if (p.lse && d == 0) p.lse[row] = (W > 0.f) ? (M + log2f(W)) * 0.69314718055994530942f : -INFINITY;
    }
    }
    __syncthreads();  // shared state is reset for the next segment
    }
}

// R [N x MJ] fp16 row-major -> A-fragment orders of R (tokens x MJ) and R^T (MJ x tokens).
__global__ void operator_fragments_kernel(const __half* __restrict__ R, int N, int MJ, uint4* __restrict__ rf,
                                          uint4* __restrict__ rtf) {
    const int64_t total = (int64_t)(N / 16) * (MJ / 16) * 32;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31);
        const int64_t tile = i >> 5;
        const int g = lane >> 2, t = lane & 3;
        auto at = [&](int r, int c) { return R[(int64_t)r * MJ + c]; };
        auto pk = [](__half lo, __half hi) {
            return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
        };
        {  // R: tile (tt, kk) row-major over [N/16][MJ/16]
            const int tt = (int)(tile / (MJ / 16)), kk = (int)(tile % (MJ / 16));
            const int r0 = 16 * tt + g, c0 = 16 * kk + 2 * t;
            rf[i] = make_uint4(pk(at(r0, c0), at(r0, c0 + 1)), pk(at(r0 + 8, c0), at(r0 + 8, c0 + 1)),
                               pk(at(r0, c0 + 8), at(r0, c0 + 9)), pk(at(r0 + 8, c0 + 8), at(r0 + 8, c0 + 9)));
        }
        {  // R^T: tile (mt, tt) over [MJ/16][N/16]; element (row m, col token) = R[token][m]
            const int mt = (int)(tile / (N / 16)), tt = (int)(tile % (N / 16));
            const int m0 = 16 * mt + g, k0 = 16 * tt + 2 * t;
            rtf[i] = make_uint4(pk(at(k0, m0), at(k0 + 1, m0)), pk(at(k0, m0 + 8), at(k0 + 1, m0 + 8)),
                                pk(at(k0 + 8, m0), at(k0 + 9, m0)), pk(at(k0 + 8, m0 + 8), at(k0 + 9, m0 + 8)));
        }
    }
}

// Merges two attention results over disjoint token sets (rows of D values + natural-log LSE).
__global__ void merge_kernel(const __half* __restrict__ oa, const float* __restrict__ la, const __half* __restrict__ ob,
                             const float* __restrict__ lb, int64_t rows, int D, __half* __restrict__ out,
                             float* __restrict__ lse) {
    const int64_t total = rows * D;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / D;
        const float A = la[r], Bv = lb[r], M = fmaxf(A, Bv);
        float wa = 0.f, wb = 0.f;
        if (M != -INFINITY) { wa = __expf(A - M); wb = __expf(Bv - M); }
        const float W = wa + wb;
        const float v = W > 0.f ? (wa * __half2float(oa[i]) + wb * __half2float(ob[i])) / W : 0.f;
        out[i] = __float2half_rn(v);
        if (lse && i % D == 0) lse[r] = W > 0.f ? M + __logf(W) : -INFINITY;
    }
}

// acc <- join(acc, b) in fp32, in place: acc_o [rows][D] fp32, acc_lse natural log (-inf: empty).
__global__ void accumulate_kernel(float* __restrict__ acc_o, float* __restrict__ acc_lse, const __half* __restrict__ ob,
                                  const float* __restrict__ lb, int64_t rows, int D) {
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const float A = acc_lse[r], Bv = lb[r], M = fmaxf(A, Bv);
        float wa = 0.f, wb = 0.f;
        if (M != -INFINITY) { wa = __expf(A - M); wb = __expf(Bv - M); }
        const float W = wa + wb;
        for (int d = threadIdx.x; d < D; d += blockDim.x) {
            const float v = W > 0.f ? (wa * acc_o[r * D + d] + wb * __half2float(ob[r * D + d])) / W : 0.f;
            acc_o[r * D + d] = v;
        }
        __syncthreads();
        if (threadIdx.x == 0) acc_lse[r] = W > 0.f ? M + __logf(W) : -INFINITY;
    }
}

}  // namespace jla
}  // namespace argus

using namespace argus;

int argus_jla_take_status(int* status, cudaStream_t st) {
    int v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(&v, jla::g_status, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(jla::g_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return argus_set_cuda_error(e);
    *status = v;
    return ARGUS_OK;
}

extern "C" {

int argus_jl_operator_fragments(const uint16_t* R, int n_tokens, int n_rows, void* r_frag, void* rt_frag,
                                argus_stream_t stream) {
    if (!R || !r_frag || !rt_frag) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    if (n_tokens <= 0 || n_rows <= 0 || n_tokens % 16 || n_rows % 16)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "block tokens and rows must be positive multiples of 16");
    if (!argus_aligned(r_frag, 16) || !argus_aligned(rt_frag, 16))
        return argus_set_error(ARGUS_ERR_MISALIGNED, "fragment buffers must be 16-byte aligned");
    const int64_t total = (int64_t)(n_tokens / 16) * (n_rows / 16) * 32;
    jla::operator_fragments_kernel<<<argus_grid_cap((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const __half*>(R), n_tokens, n_rows, static_cast<uint4*>(r_frag), static_cast<uint4*>(rt_frag));
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

// Yk / Yv as a 4-D tensor [B*Hkv][n_blocks][MJ][D] of fp16, box 64 x MJ x 1 x 1, 128-byte swizzle.
int make_block_map(CUtensorMap* map, const void* base, const argus_jl_attn_shape* s) {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_encode) return argus_set_error(ARGUS_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled is not available");
    const cuuint64_t dims[4] = {(cuuint64_t)s->head_dim, (cuuint64_t)s->block_rows, (cuuint64_t)s->n_blocks,
                                (cuuint64_t)s->batch * (cuuint64_t)s->heads_kv};
    const cuuint64_t strides[3] = {(cuuint64_t)s->head_dim * 2, (cuuint64_t)s->block_stride * 2,
                                   (cuuint64_t)s->bh_stride * 2};
    const cuuint32_t box[4] = {64, (cuuint32_t)s->block_rows, 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "tensor map for the JL blocks was refused");
    return ARGUS_OK;
}

}  // namespace

namespace {
// CTAs of a launch and the partial slots each (batch, kv_head) needs (see argus_jl_attn_shape.n_ctas).
int64_t jl_ctas(const argus_jl_attn_shape* s) {
    return s->n_ctas > 0 ? (int64_t)s->n_ctas : (int64_t)s->batch * s->heads_kv * s->n_splits;
}
int64_t jl_slots(const argus_jl_attn_shape* s) {
    const int64_t groups = (int64_t)s->batch * s->heads_kv;
    return (jl_ctas(s) + groups - 1) / groups + 1;
}
}  // namespace

int64_t argus_jl_attention_workspace_size(const argus_jl_attn_shape* s) {
    if (!s || s->batch <= 0 || s->heads_kv <= 0 || s->n_splits <= 0 || s->n_ctas < 0) return 0;
    const int64_t groups = (int64_t)s->batch * s->heads_kv;
    return ((groups * 4 + 255) & ~255LL) + groups * jl_slots(s) * jla::kCols * (int64_t)(jla::kD + 1) * 4 + 256;
}

int argus_jl_attention(const argus_jl_attn_shape* s, const uint16_t* yk, const uint16_t* yv, const void* r_frag,
                       const void* rt_frag, const uint16_t* q, uint16_t* out, float* lse, float* block_lse,
                       void* workspace, argus_stream_t stream) {
    if (!s || !yk || !yv || !r_frag || !rt_frag || !q || !out || !workspace)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    if (s->batch <= 0 || s->heads_kv <= 0 || s->group <= 0 || s->q_len <= 0 || s->n_blocks < 0 || s->n_splits <= 0)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "non-positive size");
    if (s->head_dim != jla::kD || s->block_rows != jla::kMJ)
        return argus_set_error(ARGUS_ERR_UNSUPPORTED, "JL attention supports head_dim 128 and 128-row blocks");
    if (s->block_tokens <= 0 || s->block_tokens % (16 * jla::kWarps))
        return argus_set_error(ARGUS_ERR_UNSUPPORTED, "block tokens must be a multiple of 128");
    const int NQ = s->group * s->q_len;
    if (NQ > jla::kCols) return argus_set_error(ARGUS_ERR_UNSUPPORTED, "at most 8 queries per kv head");
    if (s->n_splits > (s->n_blocks > 0 ? s->n_blocks : 1))
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "more splits than blocks");
    if (s->n_ctas < 0) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "negative CTA count");
    if (!argus_aligned(yk, 16) || !argus_aligned(yv, 16) || !argus_aligned(workspace, 16) ||
        (s->bh_stride * 2) % 16 || (s->block_stride * 2) % 16)
        return argus_set_error(ARGUS_ERR_MISALIGNED, "blocks must start on 16-byte boundaries");
    if (s->n_blocks == 0) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "no archived blocks");
    jla::Params p;
    int rc = make_block_map(&p.tmk, yk, s);
    if (rc == ARGUS_OK) rc = make_block_map(&p.tmv, yv, s);
    if (rc != ARGUS_OK) return rc;
    p.yk = reinterpret_cast<const __half*>(yk);
    p.yv = reinterpret_cast<const __half*>(yv);
    p.rf = static_cast<const uint4*>(r_frag);
    p.rtf = static_cast<const uint4*>(rt_frag);
    p.q = reinterpret_cast<const __half*>(q);
    p.out = reinterpret_cast<__half*>(out);
    p.lse = lse;
    p.block_lse = block_lse;
    const int64_t groups = (int64_t)s->batch * s->heads_kv;
    p.counters = static_cast<int*>(workspace);
    p.part_lse = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + ((groups * 4 + 255) & ~255LL));
    p.part_o = p.part_lse + groups * jl_slots(s) * jla::kCols;
    p.bh_stride = s->bh_stride;
    p.block_stride = s->block_stride;
    p.B = s->batch; p.Hkv = s->heads_kv; p.G = s->group; p.qlen = s->q_len;
    p.n_blocks = s->n_blocks; p.N = s->block_tokens; p.S = (int)jl_slots(s);
    p.scale_log2 = s->scale * 1.4426950408889634f;
    cudaStream_t st = (cudaStream_t)stream;
    const bool pack = NQ <= 4;
    const int64_t pairs = groups * ((s->n_blocks + (pack ? 1 : 0)) / (pack ? 2 : 1));
    const int64_t ctas = jl_ctas(s);
    if (ctas > pairs || ctas > 0x7fffffff)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "more CTAs than block pairs");
    const size_t smem = jla::smem_bytes(pack ? 2 : 1);
    auto kern = pack ? jla::jl_attn_kernel<2> : jla::jl_attn_kernel<1>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return argus_set_cuda_error(e);
    kern<<<(unsigned)ctas, jla::kThreads, smem, st>>>(p);
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

int argus_attention_accumulate(float* acc_o, float* acc_lse, const uint16_t* out_b, const float* lse_b, int64_t rows,
                               int head_dim, argus_stream_t stream) {
    if (!acc_o || !acc_lse || !out_b || !lse_b) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    if (rows < 0 || head_dim <= 0) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad size");
    if (rows == 0) return ARGUS_OK;
    jla::accumulate_kernel<<<argus_grid_cap(rows), 128, 0, (cudaStream_t)stream>>>(
        acc_o, acc_lse, reinterpret_cast<const __half*>(out_b), lse_b, rows, head_dim);
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

int argus_attention_merge(const uint16_t* out_a, const float* lse_a, const uint16_t* out_b, const float* lse_b,
                          int64_t rows, int head_dim, uint16_t* out, float* lse, argus_stream_t stream) {
    if (!out_a || !lse_a || !out_b || !lse_b || !out) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    if (rows < 0 || head_dim <= 0) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad size");
    if (rows == 0) return ARGUS_OK;
    jla::merge_kernel<<<argus_grid_cap((rows * head_dim + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const __half*>(out_a), lse_a, reinterpret_cast<const __half*>(out_b), lse_b, rows, head_dim,
        reinterpret_cast<__half*>(out), lse);
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

}  // extern "C"
