// Mixed-tier paged decode attention for sm_100a, fused with the dequantization of every tier.
//
// Replaces the dequantize -> concatenate -> dense softmax path of
// PagedDynamicKVCache.inplace_paged_attention (core/memory_manager.py:1317-1447) and the
// reconstruct-then-SDPA path (get_all_keys_values + transformers' attention).
//
// Work decomposition: one CTA per (split, batch*kv_head, query group of 8).  The CTA's four warps
// each stream their own chunks of compressed tiles (<= 16 tokens each) from HBM into a private
// two-stage shared-memory ring with cp.async.bulk (TMA bulk copies) completed on an mbarrier.
// A warp rebuilds each staged tile in registers and feeds it to mma.sync m16n8k16.  V is rebuilt as
// the exact fp16 values the reference's dequantizers produce (fp16(fp16(u*s) + min), fp16(q*s), +-s).
// Scores are linear in K, so the key side keeps a per-token affine step out of the fragments and
// applies it to the 16 x 8 score tile in fp32 instead: INT8 / FP8-sim keys enter the MMA as their
// codes (1152 + q, exact in fp16) and the score is s * (S - 1152 * sum(q)); INT4 / INT2 keys enter as
// fp16(u*s) (the reference's first rounding, exact) and min * sum(q) is added to the score.  The
// scores therefore skip the reference's fp16 rounding of q*s and of fp16(u*s) + min (a relative
// 2^-11 change per key value, inside the attention tolerance).
//   S^T[16 tokens x 8 queries] = K[16 x D] . Q^T        (tokens on M, queries on N)
//   O^T[D x 8 queries]        += V^T[D x 16] . P^T      (P = unnormalised softmax weights as an
//                                                        fp16 hi + lo pair, two MMAs)
// A token/dim permutation lets each thread turn whole packed bytes into fragments:
//   K (A operand) thread (g, t) holds tokens 2g, 2g+1 and dims t*D/4 .. t*D/4 + D/4 - 1;
//   V (A operand) thread (g, t) holds tokens 4t .. 4t+3 and dims g*D/8 .. g*D/8 + D/8 - 1.
// The score tile is moved into the PV operand layout with movmatrix (8x8 transpose).  Online
// softmax runs in the log2 domain; warps merge in shared memory; the last CTA of each (batch,
// kv_head, query group) to finish merges the split-K partials by log-sum-exp inside this kernel.
#include <mutex>

#include <cuda_fp8.h>

#include "common.cuh"

namespace argus {
namespace da {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kPairWarps = 2;                 // warps sharing one staging ring
constexpr int kPairs = kWarps / kPairWarps;
constexpr int kStages = 3;                    // ring slots per warp pair
constexpr int kMaxTiles = 16;
constexpr int kQ = 8;                       // queries per CTA (mma N)
constexpr long long kSpinLimit = 1ll << 26; // bounded mbarrier waits

__device__ int g_status = 0;

// One ring slot: a whole fp16 tile (16 tokens of K and V, 64 D bytes) plus 4 D, at least 8.5 KB
// (so 4 CTAs of two 3-slot rings fit in an SM's shared memory up to D = 128).
__host__ __device__ constexpr int stage_bytes(int D) { return 68 * D > 8704 ? 68 * D : 8704; }
// CTAs per SM the launch bounds and shared memory are sized for
__host__ __device__ constexpr int ctas_per_sm(int D) { return D >= 256 ? 2 : 4; }
// Shared memory past the last stage that fragment loads of short (8-token) pages may touch.
__host__ __device__ constexpr int stage_slack(int D) { return 16 * D; }
__host__ __device__ constexpr int tier_bits(int tier) {
    return tier == ARGUS_TIER_FP16 ? 16 : (tier == ARGUS_TIER_INT4 ? 4 : (tier == ARGUS_TIER_INT2 ? 2 : (tier == ARGUS_TIER_1BIT ? 1 : 8)));
}
__host__ __device__ constexpr int tier_log2per(int tier) {
    return tier == ARGUS_TIER_INT4 ? 1 : (tier == ARGUS_TIER_INT2 ? 2 : (tier == ARGUS_TIER_1BIT ? 3 : 0));
}
__host__ __device__ constexpr bool tier_scaled(int tier) { return tier != ARGUS_TIER_FP16; }
__host__ __device__ constexpr bool tier_min(int tier) { return tier == ARGUS_TIER_INT4 || tier == ARGUS_TIER_INT2; }
// bytes of one packed row (`per` tokens x D)
__host__ __device__ constexpr int row_bytes(int tier, int D) { return tier == ARGUS_TIER_FP16 ? 2 * D : D; }
// payload bytes of `tokens` tokens of K (or V)
__host__ __device__ constexpr int payload_bytes(int tier, int tokens, int D) { return tokens * D * tier_bits(tier) / 8; }
// bytes of one record: [K][V][K scales][V scales][K mins][V mins]
__host__ __device__ constexpr int record_bytes(int tier, int P, int D) {
    return 2 * payload_bytes(tier, P, D) + (tier_scaled(tier) ? 4 * P : 0) + (tier_min(tier) ? 4 * P : 0);
}
// staged bytes of one 16-token tile when tiles are not whole records
__host__ __device__ constexpr int tile_stage_bytes(int tier, int D) {
    return 2 * payload_bytes(tier, 16, D) + (tier_scaled(tier) ? 64 : 0) + (tier_min(tier) ? 64 : 0);
}
__host__ __device__ constexpr bool whole_records(int layout, int P) { return layout == ARGUS_LAYOUT_RECORD && P <= 16; }
__host__ __device__ constexpr int chunk_tiles(int tier, int layout, int P, int D) {
    return whole_records(layout, P)
               ? ((stage_bytes(D) / record_bytes(tier, P, D)) > kMaxTiles ? kMaxTiles : (stage_bytes(D) / record_bytes(tier, P, D)))
               : ((stage_bytes(D) / tile_stage_bytes(tier, D)) > kMaxTiles ? kMaxTiles : (stage_bytes(D) / tile_stage_bytes(tier, D)));
}

struct Params {
    argus_kv_arena arenas[ARGUS_MAX_ARENAS];
    const argus_kv_chunk* chunks;
    const int32_t* split_chunk0;
    const __half* q;
    __half* out;
    float* lse;
    float* part_o;    // [B*Hkv*NQG][S][8][D]
    float* part_lse;  // [B*Hkv*NQG][S][8]
    int* counters;    // [B*Hkv*NQG] split arrivals; zero between launches
    float* tile_lse;  // optional [B*Hkv*NQG][n_chunks][16][8]: log2-sum-exp of each tile's scores
    int B, Hkv, G, qlen, S, nqg, n_chunks;
    float scale_log2;
    argus_peer_gather gat;  // gat.world > 0: outputs go to every rank (argus_decode_attention_gather)
};

// Where the pieces of tile i of a staged chunk sit in shared memory (uniform across the warp).
struct ChunkView {
    int k_off, v_off, ks_off, vs_off, km_off, vm_off;
    int pstride, sstride;  // bytes between consecutive tiles: payload, scales
    int ntok_full;         // tokens in every tile but the last
};

template <int D>
__device__ __forceinline__ ChunkView chunk_view(const argus_kv_arena& ar, int n) {
    ChunkView cv;
    const int tier = ar.tier;
    if (whole_records(ar.layout, ar.page_tokens)) {
        const int P = ar.page_tokens;
        const int pb = payload_bytes(tier, P, D);
        cv.k_off = 0;
        cv.v_off = pb;
        cv.ks_off = 2 * pb;
        cv.vs_off = 2 * pb + 2 * P;
        cv.km_off = 2 * pb + 4 * P;
        cv.vm_off = 2 * pb + 6 * P;
        cv.pstride = cv.sstride = ar.record_bytes;
        cv.ntok_full = P;
    } else {
        const int pb = payload_bytes(tier, 16, D);
        cv.k_off = 0;
        cv.v_off = n * pb;
        cv.ks_off = 2 * n * pb;
        cv.vs_off = cv.ks_off + 32 * n;
        cv.km_off = cv.ks_off + 64 * n;
        cv.vm_off = cv.ks_off + 96 * n;
        cv.pstride = pb;
        cv.sstride = 32;
        cv.ntok_full = 16;
    }
    return cv;
}

// ------------------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}
// Bounded wait: false after `polls` polls (the caller records a timeout and stops).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, long long polls = kSpinLimit) {
    for (long long i = 0; i < polls; ++i)
        if (mbar_try_wait(bar, phase)) return true;
    return false;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
// two e4m3 codes (low 16 bits of x, low byte first) -> their exact fp16 values as an f16x2
__device__ __forceinline__ uint32_t e4m3x2_f16x2(uint32_t x) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(x & 0xffffu), __NV_E4M3);
    return (uint32_t)h.x | ((uint32_t)h.y << 16);
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}
__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t m, uint32_t o) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(m), "r"(o));  // (a & m) | o
    return r;
}
__device__ __forceinline__ uint32_t lop_and_xor(uint32_t a, uint32_t m, uint32_t x) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(r) : "r"(a), "r"(m), "r"(x));  // (a & m) ^ x
    return r;
}
__device__ __forceinline__ uint32_t hsub2u(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Loads BYTES (a multiple of 4) of shared memory into u32 registers with the widest vectors.
template <int BYTES>
__device__ __forceinline__ void lds(const unsigned char* p, uint32_t* r) {
    if constexpr (BYTES % 16 == 0) {
#pragma unroll
        for (int i = 0; i < BYTES / 16; ++i) {
            uint4 v = *reinterpret_cast<const uint4*>(p + 16 * i);
            r[4 * i] = v.x; r[4 * i + 1] = v.y; r[4 * i + 2] = v.z; r[4 * i + 3] = v.w;
        }
    } else if constexpr (BYTES % 8 == 0) {
#pragma unroll
        for (int i = 0; i < BYTES / 8; ++i) {
            uint2 v = *reinterpret_cast<const uint2*>(p + 8 * i);
            r[2 * i] = v.x; r[2 * i + 1] = v.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < BYTES / 4; ++i) r[i] = *reinterpret_cast<const uint32_t*>(p + 4 * i);
    }
}

// Loads BYTES (>= 2, even) into u32 registers; a 2-byte span lands zero-extended in r[0].
template <int BYTES>
__device__ __forceinline__ void lds_small(const unsigned char* p, uint32_t* r) {
    if constexpr (BYTES >= 4) {
        lds<BYTES>(p, r);
    } else {
        r[0] = *reinterpret_cast<const uint16_t*>(p);
    }
}

constexpr uint32_t kMagic1024 = 0x64006400u;  // fp16 1024.0 in both halves: 1024 + u for u in 0..1023
constexpr uint32_t kMagic1152 = 0x64806480u;  // 1024 + 128 (bias of sign-flipped int8 codes)

// A code u masked in place at mantissa bit p of an fp16 half whose exponent field is 25 - p reads
// as 2^(10-p) + u exactly (u < 2^(10-p)), so packed codes need no shift before the dequantization.
__host__ __device__ constexpr uint32_t magic_at(int p) { return (uint32_t)(25 - p) << 10; }
__host__ __device__ constexpr uint32_t magic2(int p_lo, int p_hi) { return magic_at(p_lo) | (magic_at(p_hi) << 16); }

// x * y (mod 2^32) kept as an integer multiply, so left shifts by a per-thread amount run on the
// FMA pipe instead of the busier ALU pipe.
__device__ __forceinline__ uint32_t imul(uint32_t x, uint32_t y) {
    uint32_t r;
    asm("mul.lo.u32 %0, %1, %2;" : "=r"(r) : "r"(x), "r"(y));
    return r;
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
// (~a & m) ^ c: the sign bit of c flipped where the bit of a is clear (1-bit tier: b ? s : -s)
__device__ __forceinline__ uint32_t lop_sign(uint32_t a, uint32_t m, uint32_t c) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xA6;" : "=r"(r) : "r"(a), "r"(m), "r"(c));
    return r;
}

// Exact dequantization of unsigned codes held as (2^(10-p) + u) in fp16 halves (magic_at(p)):
// fp16(fp16(u*s) + mn).  r = fma(2^(10-p) + u, s*2^-k, -2^(10-p)*s*2^-k) is fp16(u*s)*2^-k with a
// single rounding (both operands are exact: s*2^-k is s or a normal number, the addend is s scaled
// up by 2^(10-p) >= 16 or, for k = 10, a normal number), then fma(r, 2^k, mn) = fp16(fp16(u*s) + mn).
// k = 0 for s < 64, k = 10 above, so every finite scale, subnormal ones included, is exact.
__device__ __forceinline__ uint32_t deq_u(uint32_t biased, __half2 b, __half2 c, __half2 f, __half2 mn) {
    return h2u(__hfma2(__hfma2(u2h(biased), b, c), f, mn));
}

// Per-token dequantization parameters of one operand, as half2 pairs over two tokens.
struct TokScale {
    __half2 s[2];   // scale
    __half2 b[2];   // s * 2^-k
    __half2 c[2];   // -2^(10-p) * s * 2^-k   (p: mantissa bit the token's codes sit at)
    __half2 f[2];   // 2^k
    __half2 mn[2];  // min
    // key side only: score = (S + kz * sum(q)) * kw * scale, S the MMA over the key fragments
    float kz[2], kw[2];
};

// Fills b, c, f from s and the codes' base 2^(10-p) per half: k = 10 where s >= 64 (so the addend
// cannot overflow fp16), else 0.
__device__ __forceinline__ void scale_terms(TokScale& t, int i, __half2 base) {
    const __half2 big = __hge2(t.s[i], __float2half2_rn(64.0f));  // 1.0 where s >= 64
    const __half2 kf = __hfma2(big, __float2half2_rn(1023.0f), __float2half2_rn(1.0f));  // 2^k: 1 or 1024
    const __half2 ik = __hfma2(big, __float2half2_rn(-0.9990234375f), __float2half2_rn(1.0f));  // 2^-k
    t.f[i] = kf;
    t.b[i] = __hmul2(t.s[i], ik);
    t.c[i] = __hmul2(__hneg2(t.s[i]), __hmul2(base, ik));
}

// ------------------------------------------------------------------------ K fragments (QK^T)
// a[c][0..3] for k-chunk c: (token 2g, dims 4c and 4c+2), (token 2g+1, same), (token 2g, dims 4c+1
// and 4c+3), (token 2g+1, same), dims relative to this thread's span t*D/4 (the query fragments use
// the same pairing).  Pairing dims two bytes apart lets a 32-bit word of packed codes feed two
// fragments with a mask each.  Values are the reference's fp16 dequantization, bit for bit.
// ts.s[0] is token 2g broadcast, ts.s[1] token 2g+1.
template <int D, int TIER>
__device__ __forceinline__ void k_frags(const unsigned char* kp, int g4, int t4, const TokScale& ts,
                                        uint32_t (&a)[D / 16][4]) {
    constexpr int KC = D / 16;
    if constexpr (TIER == ARGUS_TIER_FP16) {
        uint32_t ra[D / 8], rb[D / 8];
        lds<D / 2>(kp + (2 * g4) * D * 2 + t4 * (D / 2), ra);
        lds<D / 2>(kp + (2 * g4 + 1) * D * 2 + t4 * (D / 2), rb);
#pragma unroll
        for (int c = 0; c < KC; ++c) {
            a[c][0] = prmt(ra[2 * c], ra[2 * c + 1], 0x5410);
            a[c][2] = prmt(ra[2 * c], ra[2 * c + 1], 0x7632);
            a[c][1] = prmt(rb[2 * c], rb[2 * c + 1], 0x5410);
            a[c][3] = prmt(rb[2 * c], rb[2 * c + 1], 0x7632);
        }
    } else if constexpr (TIER == ARGUS_TIER_INT8 || TIER == ARGUS_TIER_FP8SIM) {
        uint32_t ra[KC], rb[KC];
        lds<D / 4>(kp + (2 * g4) * D + t4 * (D / 4), ra);
        lds<D / 4>(kp + (2 * g4 + 1) * D + t4 * (D / 4), rb);
#pragma unroll
        for (int c = 0; c < KC; ++c) {
            const uint32_t wa = ra[c] ^ 0x80808080u, wb = rb[c] ^ 0x80808080u;
            // 1024 + (q + 128) = 1152 + q, exact; the scale and the bias are applied to the scores
            a[c][0] = prmt(wa, kMagic1024, 0x7270);
            a[c][2] = prmt(wa, kMagic1024, 0x7371);
            a[c][1] = prmt(wb, kMagic1024, 0x7270);
            a[c][3] = prmt(wb, kMagic1024, 0x7371);
        }
    } else if constexpr (TIER == ARGUS_TIER_E4M3) {
        // e4m3 code pairs (bytes 0, 2 and 1, 3) to their exact fp16 values; the token's scale is
        // applied to the score tile
        uint32_t ra[KC], rb[KC];
        lds<D / 4>(kp + (2 * g4) * D + t4 * (D / 4), ra);
        lds<D / 4>(kp + (2 * g4 + 1) * D + t4 * (D / 4), rb);
#pragma unroll
        for (int c = 0; c < KC; ++c) {
            a[c][0] = e4m3x2_f16x2(prmt(ra[c], 0u, 0x3120));
            a[c][2] = e4m3x2_f16x2(prmt(ra[c], 0u, 0x3120) >> 16);
            a[c][1] = e4m3x2_f16x2(prmt(rb[c], 0u, 0x3120));
            a[c][3] = e4m3x2_f16x2(prmt(rb[c], 0u, 0x3120) >> 16);
        }
    } else if constexpr (TIER == ARGUS_TIER_INT4 || TIER == ARGUS_TIER_INT2) {
        // codes of token 2g at mantissa bit pA of each byte, of token 2g+1 at pB
        uint32_t r[KC], mA, mB, gA, gB;
        if constexpr (TIER == ARGUS_TIER_INT4) {
            lds<D / 4>(kp + g4 * D + t4 * (D / 4), r);
            mA = 0x000F000Fu; mB = 0x00F000F0u; gA = magic2(0, 0); gB = magic2(4, 4);
        } else {
            lds<D / 4>(kp + (g4 >> 1) * D + t4 * (D / 4), r);
            const int pA = 4 * (g4 & 1);
            mA = 0x00030003u << pA; mB = mA << 2;
            gA = (g4 & 1) ? magic2(4, 4) : magic2(0, 0);
            gB = (g4 & 1) ? magic2(6, 6) : magic2(2, 2);
        }
#pragma unroll
        for (int c = 0; c < KC; ++c) {
            const uint32_t r8 = r[c] >> 8;  // bytes 1 and 3 moved to 0 and 2
            // fp16(u * s) * 2^-k, one rounding (see deq_u); the min is added to the scores
            a[c][0] = h2u(__hfma2(u2h(lop_and_or(r[c], mA, gA)), ts.b[0], ts.c[0]));
            a[c][1] = h2u(__hfma2(u2h(lop_and_or(r[c], mB, gB)), ts.b[1], ts.c[1]));
            a[c][2] = h2u(__hfma2(u2h(lop_and_or(r8, mA, gA)), ts.b[0], ts.c[0]));
            a[c][3] = h2u(__hfma2(u2h(lop_and_or(r8, mB, gB)), ts.b[1], ts.c[1]));
        }
    } else {  // 1-bit: b ? +s : -s, the sign bit taken from the packed bit moved to bit 15 / 31
        uint32_t r[KC];
        lds<D / 4>(kp + (g4 >> 2) * D + t4 * (D / 4), r);
        const int k = 2 * (g4 & 3);  // bit of token 2g; token 2g+1 at k + 1
        const uint32_t pA = 1u << (15 - k), pB = 1u << (14 - k), pC = 1u << (7 - k), pD = 1u << (6 - k);
        const uint32_t sA = h2u(ts.s[0]), sB = h2u(ts.s[1]);
#pragma unroll
        for (int c = 0; c < KC; ++c) {
            a[c][0] = lop_sign(imul(r[c], pA), 0x80008000u, sA);  // bytes 0, 2
            a[c][1] = lop_sign(imul(r[c], pB), 0x80008000u, sB);
            a[c][2] = lop_sign(imul(r[c], pC), 0x80008000u, sA);  // bytes 1, 3
            a[c][3] = lop_sign(imul(r[c], pD), 0x80008000u, sB);
        }
    }
}

// ------------------------------------------------------------------------ V fragments (PV)
// a[t][0..3] for m-tile t: (dim 2t, tokens 4u,4u+2), (dim 2t+1, tokens 4u,4u+2),
// (dim 2t, tokens 4u+1,4u+3), (dim 2t+1, tokens 4u+1,4u+3); u = t4, dims relative to g*D/8.
// ts.s[0] = (s_4u, s_4u+2), ts.s[1] = (s_4u+1, s_4u+3).  Exact fp16 dequantized values.
template <int D, int TIER>
__device__ __forceinline__ void v_frags(const unsigned char* vp, int g4, int t4, const TokScale& ts,
                                        uint32_t (&a)[D / 16][4]) {
    constexpr int KC = D / 16;
    constexpr int W = (D / 8 + 3) / 4;
    if constexpr (TIER == ARGUS_TIER_FP16) {
        uint32_t r0[KC], r1[KC], r2[KC], r3[KC];
        const unsigned char* base = vp + (4 * t4) * D * 2 + g4 * (D / 4);
        lds_small<D / 4>(base, r0);
        lds_small<D / 4>(base + D * 2, r1);
        lds_small<D / 4>(base + 2 * D * 2, r2);
        lds_small<D / 4>(base + 3 * D * 2, r3);
#pragma unroll
        for (int t = 0; t < KC; ++t) {
            a[t][0] = prmt(r0[t], r2[t], 0x5410);
            a[t][1] = prmt(r0[t], r2[t], 0x7632);
            a[t][2] = prmt(r1[t], r3[t], 0x5410);
            a[t][3] = prmt(r1[t], r3[t], 0x7632);
        }
    } else if constexpr (TIER == ARGUS_TIER_INT8 || TIER == ARGUS_TIER_FP8SIM) {
        uint32_t r0[W], r1[W], r2[W], r3[W];
        const unsigned char* base = vp + (4 * t4) * D + g4 * (D / 8);
        lds_small<D / 8>(base, r0);
        lds_small<D / 8>(base + D, r1);
        lds_small<D / 8>(base + 2 * D, r2);
        lds_small<D / 8>(base + 3 * D, r3);
#pragma unroll
        for (int t = 0; t < KC; ++t) {
            const int w = t >> 1, e0 = 2 * (t & 1);
            const uint32_t sel = e0 | ((4 + e0) << 4) | ((e0 + 1) << 8) | ((5 + e0) << 12);
            const uint32_t y02 = prmt(r0[w], r2[w], sel) ^ 0x80808080u;  // (tok 4u d0, tok 4u+2 d0, .. d1, .. d1)
            const uint32_t y13 = prmt(r1[w], r3[w], sel) ^ 0x80808080u;
            a[t][0] = h2u(__hmul2_rn(u2h(hsub2u(prmt(y02, kMagic1024, 0x7170), kMagic1152)), ts.s[0]));
            a[t][1] = h2u(__hmul2_rn(u2h(hsub2u(prmt(y02, kMagic1024, 0x7372), kMagic1152)), ts.s[0]));
            a[t][2] = h2u(__hmul2_rn(u2h(hsub2u(prmt(y13, kMagic1024, 0x7170), kMagic1152)), ts.s[1]));
            a[t][3] = h2u(__hmul2_rn(u2h(hsub2u(prmt(y13, kMagic1024, 0x7372), kMagic1152)), ts.s[1]));
        }
    } else if constexpr (TIER == ARGUS_TIER_E4M3) {
        uint32_t r0[W], r1[W], r2[W], r3[W];
        const unsigned char* base = vp + (4 * t4) * D + g4 * (D / 8);
        lds_small<D / 8>(base, r0);
        lds_small<D / 8>(base + D, r1);
        lds_small<D / 8>(base + 2 * D, r2);
        lds_small<D / 8>(base + 3 * D, r3);
#pragma unroll
        for (int t = 0; t < KC; ++t) {
            const int w = t >> 1, e0 = 2 * (t & 1);
            const uint32_t sel = e0 | ((4 + e0) << 4) | ((e0 + 1) << 8) | ((5 + e0) << 12);
            const uint32_t y02 = prmt(r0[w], r2[w], sel);  // (tok 4u d0, tok 4u+2 d0, .. d1, .. d1)
            const uint32_t y13 = prmt(r1[w], r3[w], sel);
            a[t][0] = h2u(__hmul2_rn(u2h(e4m3x2_f16x2(y02)), ts.s[0]));
            a[t][1] = h2u(__hmul2_rn(u2h(e4m3x2_f16x2(y02 >> 16)), ts.s[0]));
            a[t][2] = h2u(__hmul2_rn(u2h(e4m3x2_f16x2(y13)), ts.s[1]));
            a[t][3] = h2u(__hmul2_rn(u2h(e4m3x2_f16x2(y13 >> 16)), ts.s[1]));
        }
    } else if constexpr (TIER == ARGUS_TIER_INT4) {
        uint32_t ra[W], rb[W];
        const unsigned char* base = vp + (2 * t4) * D + g4 * (D / 8);
        lds_small<D / 8>(base, ra);   // pair row 2u: tokens 4u (lo), 4u+1 (hi)
        lds_small<D / 8>(base + D, rb);  // pair row 2u+1: tokens 4u+2 (lo), 4u+3 (hi)
#pragma unroll
        for (int t = 0; t < KC; ++t) {
            const int w = t >> 1, e0 = 2 * (t & 1);
            const uint32_t y0 = prmt(ra[w], rb[w], e0 | ((4 + e0) << 8));              // (A.d0, -, B.d0, -)
            const uint32_t y1 = prmt(ra[w], rb[w], (e0 + 1) | ((5 + e0) << 8));        // (A.d1, -, B.d1, -)
            // low nibbles: tokens 4u, 4u+2; high nibbles (read in place): tokens 4u+1, 4u+3
            a[t][0] = deq_u(lop_and_or(y0, 0x000F000Fu, magic2(0, 0)), ts.b[0], ts.c[0], ts.f[0], ts.mn[0]);
            a[t][2] = deq_u(lop_and_or(y0, 0x00F000F0u, magic2(4, 4)), ts.b[1], ts.c[1], ts.f[1], ts.mn[1]);
            a[t][1] = deq_u(lop_and_or(y1, 0x000F000Fu, magic2(0, 0)), ts.b[0], ts.c[0], ts.f[0], ts.mn[0]);
            a[t][3] = deq_u(lop_and_or(y1, 0x00F000F0u, magic2(4, 4)), ts.b[1], ts.c[1], ts.f[1], ts.mn[1]);
        }
    } else if constexpr (TIER == ARGUS_TIER_INT2) {
        uint32_t r[W];
        lds_small<D / 8>(vp + t4 * D + g4 * (D / 8), r);  // tokens 4u+i in bits 2i..2i+1
#pragma unroll
        for (int t = 0; t < KC; ++t) {
            const int w = t >> 1, e0 = 2 * (t & 1);
            const uint32_t y0 = prmt(r[w], 0u, e0 | (e0 << 8));              // the byte of dim d0 in both halves
            const uint32_t y1 = prmt(r[w], 0u, (e0 + 1) | ((e0 + 1) << 8));  // dim d1
            // codes read in place: token 4u (bits 0-1) | 4u+2 (bits 4-5); 4u+1 (2-3) | 4u+3 (6-7)
            a[t][0] = deq_u(lop_and_or(y0, 0x00300003u, magic2(0, 4)), ts.b[0], ts.c[0], ts.f[0], ts.mn[0]);
            a[t][2] = deq_u(lop_and_or(y0, 0x00C0000Cu, magic2(2, 6)), ts.b[1], ts.c[1], ts.f[1], ts.mn[1]);
            a[t][1] = deq_u(lop_and_or(y1, 0x00300003u, magic2(0, 4)), ts.b[0], ts.c[0], ts.f[0], ts.mn[0]);
            a[t][3] = deq_u(lop_and_or(y1, 0x00C0000Cu, magic2(2, 6)), ts.b[1], ts.c[1], ts.f[1], ts.mn[1]);
        }
    } else {  // 1-bit: tokens 4u+i sit in bit k0+i of row u/2, k0 = 4(u&1)
        uint32_t r[W];
        lds_small<D / 8>(vp + (t4 >> 1) * D + g4 * (D / 8), r);
        const int k0 = 4 * (t4 & 1);
        const uint32_t pA = 1u << (15 - k0), pB = 1u << (14 - k0);
        const uint32_t s02 = h2u(ts.s[0]), s13 = h2u(ts.s[1]);
#pragma unroll
        for (int t = 0; t < KC; ++t) {
            const int w = t >> 1, e0 = 2 * (t & 1);
            const uint32_t rs = r[w] >> 2;  // bit k0+2 moved to k0
            const uint32_t y0 = prmt(r[w], rs, e0 | ((4 + e0) << 8));
            const uint32_t y1 = prmt(r[w], rs, (e0 + 1) | ((5 + e0) << 8));
            a[t][0] = lop_sign(imul(y0, pA), 0x80008000u, s02);  // tokens 4u, 4u+2
            a[t][2] = lop_sign(imul(y0, pB), 0x80008000u, s13);  // tokens 4u+1, 4u+3
            a[t][1] = lop_sign(imul(y1, pA), 0x80008000u, s02);
            a[t][3] = lop_sign(imul(y1, pB), 0x80008000u, s13);
        }
    }
}

struct SoftmaxState {
    float m[2];  // reference max (log2 domain) for queries 2t, 2t+1; weights are 2^(x - m)
    float l[2];  // this thread's partial sum of weights
};
// Reference max before any score: finite, so that 2^(x - m) of masked (-inf) scores is 0, far below
// any score fp16 inputs can produce, and 2^(kNoMax - score) underflows to 0 at the first rescale.
constexpr float kNoMax = -1.0e30f;

// Lazy rescaling: the reference max only moves when a score exceeds it by more than this (log2
// units), so weights stay <= 2^8 (exact range for fp16 P) and rescales of O are rare.
#ifndef ARGUS_DA_RESCALE_SLACK
#define ARGUS_DA_RESCALE_SLACK 8.0f
#endif
constexpr float kRescaleSlack = ARGUS_DA_RESCALE_SLACK;

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ __half2 load_h2(const __half* p) { return *reinterpret_cast<const __half2*>(p); }

// Pointers of one staged tile.
struct TilePtr {
    const unsigned char* k;
    const unsigned char* v;
    const __half *ks, *vs, *km, *vm;
    int ntok;
};

template <int TIER>
__device__ __forceinline__ void load_tok_scales(const TilePtr& tp, int g4, int t4, TokScale& tk, TokScale& tv) {
    // key-side score terms (see TokScale): fp16 and 1-bit keys enter the MMA as their values
    tk.kz[0] = tk.kz[1] = 0.f;
    tk.kw[0] = tk.kw[1] = 1.f;
    if constexpr (TIER != ARGUS_TIER_FP16) {
        const __half2 k2 = load_h2(tp.ks + 2 * g4);
        tk.s[0] = __low2half2(k2);
        tk.s[1] = __high2half2(k2);
        if constexpr (TIER == ARGUS_TIER_INT8 || TIER == ARGUS_TIER_FP8SIM) {
            // codes 1152 + q: score = s * (S - 1152 * sum(q))
            tk.kz[0] = tk.kz[1] = -1152.f;
            tk.kw[0] = __low2float(k2);
            tk.kw[1] = __high2float(k2);
        } else if constexpr (TIER == ARGUS_TIER_E4M3) {  // e4m3 values: score = s * S
            tk.kw[0] = __low2float(k2);
            tk.kw[1] = __high2float(k2);
        }
        const uint2 v4 = *reinterpret_cast<const uint2*>(tp.vs + 4 * t4);
        tv.s[0] = u2h(prmt(v4.x, v4.y, 0x5410));
        tv.s[1] = u2h(prmt(v4.x, v4.y, 0x7632));
        if constexpr (tier_min(TIER)) {
            const __half2 m2 = load_h2(tp.km + 2 * g4);
            tk.mn[0] = __low2half2(m2);
            tk.mn[1] = __high2half2(m2);
            const uint2 w4 = *reinterpret_cast<const uint2*>(tp.vm + 4 * t4);
            tv.mn[0] = u2h(prmt(w4.x, w4.y, 0x5410));
            tv.mn[1] = u2h(prmt(w4.x, w4.y, 0x7632));
            // code bases 2^(10-p) of each token's in-place codes (see k_frags / v_frags)
            const __half2 b1024 = __float2half2_rn(1024.0f), b256 = __float2half2_rn(256.0f);
            const __half2 b64 = __float2half2_rn(64.0f), b16 = __float2half2_rn(16.0f);
            __half2 bk0, bk1, bv0, bv1;
            if constexpr (TIER == ARGUS_TIER_INT4) {
                bk0 = b1024; bk1 = b64; bv0 = b1024; bv1 = b64;
            } else {
                const bool odd = (g4 & 1) != 0;
                bk0 = odd ? b64 : b1024; bk1 = odd ? b16 : b256;
                bv0 = __halves2half2(__float2half_rn(1024.0f), __float2half_rn(64.0f));
                bv1 = __halves2half2(__float2half_rn(256.0f), __float2half_rn(16.0f));
            }
            const __half2 smax = __hmax2(__hmax2(tk.s[0], tk.s[1]), __hmax2(tv.s[0], tv.s[1]));
            if (__all_sync(0xffffffffu, __hblt2(smax, __float2half2_rn(64.0f)))) {
                // every scale of the tile is below 64: k = 0 (b = s, f = 1)
                const __half2 one = __float2half2_rn(1.0f);
                tk.b[0] = tk.s[0]; tk.c[0] = __hmul2(tk.s[0], __hneg2(bk0)); tk.f[0] = one;
                tk.b[1] = tk.s[1]; tk.c[1] = __hmul2(tk.s[1], __hneg2(bk1)); tk.f[1] = one;
                tv.b[0] = tv.s[0]; tv.c[0] = __hmul2(tv.s[0], __hneg2(bv0)); tv.f[0] = one;
                tv.b[1] = tv.s[1]; tv.c[1] = __hmul2(tv.s[1], __hneg2(bv1)); tv.f[1] = one;
                // key values fp16(u * s): score = S + min * sum(q)
                tk.kz[0] = __low2float(m2);
                tk.kz[1] = __high2float(m2);
            } else {
                scale_terms(tk, 0, bk0); scale_terms(tk, 1, bk1);
                scale_terms(tv, 0, bv0); scale_terms(tv, 1, bv1);
                // key values fp16(u * s) * 2^-k: score = (S + min * 2^-k * sum(q)) * 2^k
                tk.kw[0] = __low2float(tk.f[0]);
                tk.kw[1] = __low2float(tk.f[1]);
                tk.kz[0] = __low2float(m2) / tk.kw[0];
                tk.kz[1] = __high2float(m2) / tk.kw[1];
            }
        }
    }
}

// Query fragments live in shared memory (read again for every tile, which keeps 2*D/16 registers
// free): lane l's words j are at word ((j / V) * 32 + l) * V + j % V with V = 4 (2 for D = 16), so
// each vector load of a warp is conflict-free.
template <int D>
__device__ __forceinline__ void load_qfrags(uint32_t qs, int lane, uint32_t (&qf)[D / 16][2]) {
    constexpr int W = 2 * (D / 16);
    if constexpr (W % 4 == 0) {
#pragma unroll
        for (int v = 0; v < W / 4; ++v) {
            uint32_t r0, r1, r2, r3;
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                         : "r"(qs + (uint32_t)((v * 32 + lane) * 16)));
            qf[2 * v][0] = r0; qf[2 * v][1] = r1; qf[2 * v + 1][0] = r2; qf[2 * v + 1][1] = r3;
        }
    } else {
        uint32_t r0, r1;
        asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(qs + (uint32_t)(lane * 8)));
        qf[0][0] = r0; qf[0][1] = r1;
    }
}

// Scores of one tile in the log2 domain: x[0..3] = (token 2g, query 2t), (2g, 2t+1), (2g+1, 2t),
// (2g+1, 2t+1); tokens past the tile's end are -inf.
// qsum: sums over d of queries 2t and 2t+1 (fp32), for the key-side score terms.
template <int D, int TIER>
__device__ __forceinline__ void tile_scores(const TilePtr& tp, int g4, int t4, const TokScale& tk,
                                            uint32_t qs, float scale_log2, float2 qsum, float (&x)[4]) {
    constexpr int KC = D / 16;
    uint32_t a[KC][4];
    k_frags<D, TIER>(tp.k, g4, t4, tk, a);
    uint32_t qf[KC][2];
    load_qfrags<D>(qs, threadIdx.x & 31, qf);
    // the first chain starts from the key-side offsets kz * sum(q) (zero for fp16 and 1-bit keys)
    float s[4] = {tk.kz[0] * qsum.x, tk.kz[0] * qsum.y, tk.kz[1] * qsum.x, tk.kz[1] * qsum.y};
    float s2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < KC; c += 2) {
        mma16816(s, a[c], qf[c][0], qf[c][1]);
        if (c + 1 < KC) mma16816(s2, a[c + 1], qf[c + 1][0], qf[c + 1][1]);
    }
    const bool va = 2 * g4 < tp.ntok, vb = 2 * g4 + 1 < tp.ntok;
    const float w0 = tk.kw[0] * scale_log2, w1 = tk.kw[1] * scale_log2;
    x[0] = va ? (s[0] + s2[0]) * w0 : -INFINITY;
    x[1] = va ? (s[1] + s2[1]) * w0 : -INFINITY;
    x[2] = vb ? (s[2] + s2[2]) * w1 : -INFINITY;
    x[3] = vb ? (s[3] + s2[3]) * w1 : -INFINITY;
}

// V^T fragments of one tile (tokens past the tile's end zeroed: they may hold non-finite garbage).
template <int D, int TIER>
__device__ __forceinline__ void tile_vfrags(const TilePtr& tp, int g4, int t4, const TokScale& tv, uint32_t (&av)[D / 16][4]) {
    constexpr int KC = D / 16;
    v_frags<D, TIER>(tp.v, g4, t4, tv, av);
    if (tp.ntok < 16) {
        const int nt = tp.ntok;
        const uint32_t m01 = (4 * t4 < nt ? 0x0000FFFFu : 0u) | (4 * t4 + 2 < nt ? 0xFFFF0000u : 0u);
        const uint32_t m23 = (4 * t4 + 1 < nt ? 0x0000FFFFu : 0u) | (4 * t4 + 3 < nt ? 0xFFFF0000u : 0u);
#pragma unroll
        for (int t = 0; t < KC; ++t) { av[t][0] &= m01; av[t][1] &= m01; av[t][2] &= m23; av[t][3] &= m23; }
    }
}

// O^T += V^T . P^T for one tile, P given as the two movmatrix-transposed fp16 fragments.
template <int D, bool PRECISE>
__device__ __forceinline__ void tile_pv(const uint32_t (&av)[D / 16][4], uint32_t b01, uint32_t b23, uint32_t c01,
                                        uint32_t c23, float (&o)[D / 16][4]) {
    constexpr int KC = D / 16;
#pragma unroll
    for (int t = 0; t < KC; ++t) {
        mma16816(o[t], av[t], b01, b23);
        if constexpr (PRECISE) mma16816(o[t], av[t], c01, c23);
    }
}

// Online softmax over NT tiles' scores at once: one max reduction and at most one rescale.  The
// weights go to the PV contraction as two fp16 fragments, p = hi + lo (lo = fp16(p - hi)), so the
// product keeps ~22 bits of the fp32 weight instead of fp16's 11.
template <int KC, int NT, bool PRECISE, bool MASS>
__device__ __forceinline__ void softmax_update(const float (&x)[NT][4], SoftmaxState& st, float (&o)[KC][4],
                                               uint32_t (&b01)[NT], uint32_t (&b23)[NT], uint32_t (&c01)[NT],
                                               uint32_t (&c23)[NT], float* mass_out) {
    // The tile's maxima are reduced across the 8 token lanes only when some lane holds a score above
    // the reference max plus the slack; otherwise the reference max stands and no O rescale is due.
    const float t0 = st.m[0] + kRescaleSlack, t1 = st.m[1] + kRescaleSlack;
    bool over = false;
#pragma unroll
    for (int i = 0; i < NT; ++i) over |= (fmaxf(x[i][0], x[i][2]) > t0) | (fmaxf(x[i][1], x[i][3]) > t1);
    if (__any_sync(0xffffffffu, over)) {
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int i = 0; i < NT; ++i) { mx0 = fmaxf(mx0, fmaxf(x[i][0], x[i][2])); mx1 = fmaxf(mx1, fmaxf(x[i][1], x[i][3])); }
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
        }
        const float n0 = fmaxf(st.m[0], mx0), n1 = fmaxf(st.m[1], mx1);
        const float f0 = ex2(st.m[0] - n0), f1 = ex2(st.m[1] - n1);  // kNoMax - finite -> 0
#pragma unroll
        for (int t = 0; t < KC; ++t) { o[t][0] *= f0; o[t][2] *= f0; o[t][1] *= f1; o[t][3] *= f1; }
        st.l[0] *= f0; st.l[1] *= f1;
        st.m[0] = n0; st.m[1] = n1;
    }
    const float m0 = st.m[0], m1 = st.m[1];
#pragma unroll
    for (int i = 0; i < NT; ++i) {
        const float p0 = ex2(x[i][0] - m0), p1 = ex2(x[i][1] - m1);
        const float p2 = ex2(x[i][2] - m0), p3 = ex2(x[i][3] - m1);
        st.l[0] += p0 + p2;
        st.l[1] += p1 + p3;
        if constexpr (MASS) {
            // this tile's log2-sum-exp per query: sum over the 16 tokens, relative to the reference max
            float s0 = p0 + p2, s1 = p1 + p3;
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                s0 += __shfl_xor_sync(0xffffffffu, s0, off);
                s1 += __shfl_xor_sync(0xffffffffu, s1, off);
            }
            if ((threadIdx.x & 31) < 4) {
                const int t = threadIdx.x & 3;
                mass_out[i * kQ + 2 * t] = (s0 > 0.f) ? __log2f(s0) + m0 : -INFINITY;
                mass_out[i * kQ + 2 * t + 1] = (s1 > 0.f) ? __log2f(s1) + m1 : -INFINITY;
            }
        }
        const __half2 h01 = __floats2half2_rn(p0, p1), h23 = __floats2half2_rn(p2, p3);
        const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
        b01[i] = movmatrix_t(h2u(h01));  // mma rows 0..7 (tokens 2g)
        b23[i] = movmatrix_t(h2u(h23));  // mma rows 8..15 (tokens 2g+1)
        if constexpr (PRECISE) {
            c01[i] = movmatrix_t(pack_half2(p0 - f01.x, p1 - f01.y));
            c23[i] = movmatrix_t(pack_half2(p2 - f23.x, p3 - f23.y));
        }
    }
}

// ------------------------------------------------------------------------------ outlier sidecars
// The reference overwrites each sidecar position of a dequantized page with the sidecar's fp16 value
// before attending.  Here the page stays compressed and the kernel adds the difference: the tile's
// scores get delta . q over its key outliers and its output gets delta^T . p over its value
// outliers, delta = sidecar value minus dequantized value (argus_outlier_corrections).
//
// Head dims up to 128 scatter the tile's deltas into a dense fp16 16 x D tile in the warp's shared
// memory (zero between uses, stored in MMA fragment order) and run it through the same tensor-core
// MMAs as the tile itself, so the cost hardly depends on how many outliers a tile has; deltas that
// fp16 does not hold exactly take a second pass with the remainder.  These kernels run 3 CTAs per SM to make room
// for the tiles.  Head dim 256 walks each lane's own entries (keys by the token pair whose scores
// the lane holds, values by the dims of the outputs it holds), using a 512-byte buffer per warp.
__host__ __device__ constexpr bool side_dense(int D) { return D <= 128; }
__host__ __device__ constexpr int side_ctas_per_sm(int D) { return side_dense(D) ? 3 : ctas_per_sm(D); }
__host__ __device__ constexpr int side_warp_bytes(int D) { return side_dense(D) ? 32 * D : 16 * kQ * 4; }

// The corrections of one tile: the page's block (header and entries; null when it has none), the
// tile's key and value entry ranges, its index within the page and the page's tile count, this
// lane's first two key and value entries (entries k0 + lane, k0 + 32 + lane, and likewise for the
// values; loaded as the tile starts); buf: the warp's shared-memory buffer.
struct OutlierTile {
    const uint32_t* hdr;
    const uint2* ent;
    int k0, k1, v0, v1;
    int ti, nt;
    uint2 ke[2], ve[2];
    unsigned char* buf;
};

// The dense delta tile is stored in MMA fragment order: lane l's 4 KC words are the A fragments
// a[c][0..3] (c = 0 .. KC-1) that k_frags / v_frags of an fp16 tile would give lane l, its 16-byte
// groups rotated by (l mod KC) so that the fragment loads are free of bank conflicts.
template <int D>
__device__ __forceinline__ int frag_half(int lane, int c, int r, int half) {
    constexpr int KC = D / 16;
    return ((lane * KC + (c ^ (lane & (KC - 1)))) * 4 + r) * 2 + half;
}
// (token, dim) of a K tile -> its half in the fragment-ordered tile (k_frags: lane 4 (tok/2) +
// d/(D/4) holds dims 4c + {0,2} in a[c][0 (even tok) / 1 (odd)], dims 4c + {1,3} in a[c][2 / 3])
template <int D>
__device__ __forceinline__ int k_half(int tok, int d) {
    const int dd = d % (D / 4), w = dd & 3;
    return frag_half<D>(4 * (tok >> 1) + d / (D / 4), dd >> 2, ((w & 1) << 1) | (tok & 1), w >> 1);
}
// (token, dim) of a V tile -> its half (v_frags: lane 4 (d/(D/8)) + tok/4 holds, for t = (d mod D/8)/2,
// tokens 4u+{0,2} in a[t][0 (even d) / 1 (odd d)], tokens 4u+{1,3} in a[t][2 / 3])
template <int D>
__device__ __forceinline__ int v_half(int tok, int d) {
    const int dd = d % (D / 8), w = tok & 3;
    return frag_half<D>(4 * (d / (D / 8)) + (tok >> 2), dd >> 1, ((w & 1) << 1) | (dd & 1), w >> 1);
}
template <int D>
__device__ __forceinline__ void load_delta_frags(const unsigned char* buf, uint32_t (&a)[D / 16][4]) {
    constexpr int KC = D / 16;
    const int lane = threadIdx.x & 31;
    const uint4* b4 = reinterpret_cast<const uint4*>(buf);
#pragma unroll
    for (int c = 0; c < KC; ++c) {
        const uint4 v = b4[lane * KC + (c ^ (lane & (KC - 1)))];
        a[c][0] = v.x; a[c][1] = v.y; a[c][2] = v.z; a[c][3] = v.w;
    }
}

// This lane's share of a tile's key or value entries, ready to store: positions (halves of the
// fragment-ordered tile, -1 = none) and fp16 hi | lo << 16 of each delta.
struct DeltaSlots {
    int pos[2];
    uint32_t hl[2];
};

template <int D>
__device__ __forceinline__ void delta_slot(uint2 raw, bool key, int tb, int ntok, int& pos, uint32_t& hl) {
    const int tok = (int)(raw.x & 0xffffu) - tb, d = (int)(raw.x >> 16);
    pos = -1;
    hl = 0u;
    if (tok < 0 || tok >= ntok || d >= D) return;
    const float delta = __uint_as_float(raw.y);
    const __half hi = __float2half_rn(delta);
    const __half lo = __float2half_rn(delta - __half2float(hi));
    pos = key ? k_half<D>(tok, d) : v_half<D>(tok, d);
    hl = (uint32_t)__half_as_ushort(hi) | ((uint32_t)__half_as_ushort(lo) << 16);
}

// Prepares this lane's slots; returns (warp-uniform) whether any delta has a nonzero fp16 remainder.
template <int D>
__device__ __forceinline__ bool delta_slots(const OutlierTile& ot, bool key, int ntok, DeltaSlots& ds) {
    const int lane = threadIdx.x & 31;
    const int e0 = key ? ot.k0 : ot.v0, e1 = key ? ot.k1 : ot.v1;
    bool rem = false;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        ds.pos[u] = -1;
        ds.hl[u] = 0u;
        if (e0 + 32 * u + lane < e1) {
            delta_slot<D>(key ? ot.ke[u] : ot.ve[u], key, 16 * ot.ti, ntok, ds.pos[u], ds.hl[u]);
            rem |= (ds.hl[u] >> 16) != 0u;
        }
    }
    for (int e = e0 + 64 + lane; e < e1; e += 32) {  // tiles with more than 64 entries
        int pos;
        uint32_t hl;
        delta_slot<D>(__ldg(ot.ent + e), key, 16 * ot.ti, ntok, pos, hl);
        rem |= (hl >> 16) != 0u;
    }
    return __any_sync(0xffffffffu, rem);
}

// Stores pass 0: hi, 1: lo, 2: zero of the slots (and of any entries past the first 64).
template <int D>
__device__ __forceinline__ void store_deltas(const OutlierTile& ot, bool key, int ntok, const DeltaSlots& ds, int pass) {
    unsigned short* buf = reinterpret_cast<unsigned short*>(ot.buf);
#pragma unroll
    for (int u = 0; u < 2; ++u)
        if (ds.pos[u] >= 0) buf[ds.pos[u]] = pass == 2 ? (unsigned short)0 : (unsigned short)(ds.hl[u] >> (16 * pass));
    const int e0 = key ? ot.k0 : ot.v0, e1 = key ? ot.k1 : ot.v1;
    for (int e = e0 + 64 + (threadIdx.x & 31); e < e1; e += 32) {
        int pos;
        uint32_t hl;
        delta_slot<D>(__ldg(ot.ent + e), key, 16 * ot.ti, ntok, pos, hl);
        if (pos >= 0) buf[pos] = pass == 2 ? (unsigned short)0 : (unsigned short)(hl >> (16 * pass));
    }
    __syncwarp();
}

// x[.] += scale_log2 * (delta tile) . Q^T for the key outliers of the tile.
template <int D>
__device__ __forceinline__ void dense_k_outliers(const OutlierTile& ot, uint32_t qs, float scale_log2, int ntok,
                                                 float (&x)[4]) {
    if (ot.k0 >= ot.k1) return;
    constexpr int KC = D / 16;
    DeltaSlots ds;
    const bool rem = delta_slots<D>(ot, true, ntok, ds);
    uint32_t qf[KC][2];
    load_qfrags<D>(qs, threadIdx.x & 31, qf);
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    for (int pass = 0; pass < 2; ++pass) {
        store_deltas<D>(ot, true, ntok, ds, pass);
        uint32_t a[KC][4];
        load_delta_frags<D>(ot.buf, a);
#pragma unroll
        for (int c = 0; c < KC; ++c) mma16816(s, a[c], qf[c][0], qf[c][1]);
        __syncwarp();  // every lane has its fragments before the tile is rewritten
        if (!rem) break;
    }
    store_deltas<D>(ot, true, ntok, ds, 2);
    x[0] += s[0] * scale_log2;
    x[1] += s[1] * scale_log2;
    x[2] += s[2] * scale_log2;
    x[3] += s[3] * scale_log2;
}

// O^T += (delta tile)^T . P^T for the value outliers of the tile, P the tile's fp16 weights.
template <int D, bool PRECISE>
__device__ __forceinline__ void dense_v_outliers(const OutlierTile& ot, int ntok, uint32_t b01, uint32_t b23,
                                                 uint32_t c01, uint32_t c23, float (&o)[D / 16][4]) {
    if (ot.v0 >= ot.v1) return;
    constexpr int KC = D / 16;
    DeltaSlots ds;
    const bool rem = delta_slots<D>(ot, false, ntok, ds);
    for (int pass = 0; pass < 2; ++pass) {
        store_deltas<D>(ot, false, ntok, ds, pass);
        uint32_t av[KC][4];
        load_delta_frags<D>(ot.buf, av);
#pragma unroll
        for (int t = 0; t < KC; ++t) {
            mma16816(o[t], av[t], b01, b23);
            if constexpr (PRECISE) mma16816(o[t], av[t], c01, c23);
        }
        __syncwarp();
        if (!rem) break;
    }
    store_deltas<D>(ot, false, ntok, ds, 2);
}

// q[n][d] of the CTA's query group from the Q^T fragments in shared memory (load_qfrags layout:
// lane 4n + d/(D/4) holds dims 4c, 4c+2 in word 2c and 4c+1, 4c+3 in word 2c+1 of its block).
template <int D>
__device__ __forceinline__ float q_at(uint32_t qs, int n, int d) {
    constexpr int KC = D / 16;
    constexpr int V = (2 * KC) % 4 == 0 ? 4 : 2;
    const int src = 4 * n + d / (D / 4), dd = d % (D / 4);
    const int j = 2 * (dd >> 2) + (dd & 1), half = (dd >> 1) & 1;
    const uint32_t addr = qs + (uint32_t)((((j / V) * 32 + src) * V + (j % V)) * 4 + 2 * half);
    unsigned short h;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(addr));
    return __half2float(__ushort_as_half(h));
}

template <int D>
__device__ __forceinline__ void k_entry(uint2 raw, int tok0, int g4, int t4, uint32_t qs, float scale_log2, int ntok,
                                        float (&x)[4]) {
    const int odd = (int)(raw.x & 0xffffu) - tok0, d = (int)(raw.x >> 16);
    if (odd < 0 || odd > 1 || 2 * g4 + odd >= ntok || d >= D) return;
    const float c = __uint_as_float(raw.y) * scale_log2;
    const float q0 = q_at<D>(qs, 2 * t4, d), q1 = q_at<D>(qs, 2 * t4 + 1, d);
    if (odd) { x[2] = fmaf(c, q0, x[2]); x[3] = fmaf(c, q1, x[3]); }
    else     { x[0] = fmaf(c, q0, x[0]); x[1] = fmaf(c, q1, x[1]); }
}

// Walk form of the key corrections: x[.] (scores of tokens 2g4, 2g4+1 for queries 2t4, 2t4+1) +=
// scale_log2 * delta * q[n][d] over the entries of this lane's token pair, four loads in flight.
template <int D>
__device__ __forceinline__ void walk_k_outliers(const OutlierTile& ot, int g4, int t4, uint32_t qs, float scale_log2,
                                                int ntok, float (&x)[4]) {
    if (ot.k0 >= ot.k1) return;
    const int j = 8 * ot.ti + g4;
    int e = (int)__ldg(ot.hdr + j);
    const int e1 = (int)__ldg(ot.hdr + j + 1);
    const int tok0 = 16 * ot.ti + 2 * g4;
    for (; e < e1; e += 4) {
        uint2 rr[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) rr[u] = (e + u < e1) ? __ldg(ot.ent + e + u) : make_uint2(0xffffu, 0u);
#pragma unroll
        for (int u = 0; u < 4; ++u) k_entry<D>(rr[u], tok0, g4, t4, qs, scale_log2, ntok, x);
    }
}

// Walk form of the value corrections: O^T[d][2t4 .. 2t4+1] += p[.][tok] * delta over the entries of
// this lane's dim group (dims g4 D/8 ..), p = 2^(x - m) staged as fp16 in the warp's buffer.  A
// lane's entries are sorted by dim, so a static walk over its output registers picks them up.
template <int D>
__device__ __forceinline__ void walk_v_outliers(const OutlierTile& ot, int g4, int t4, int ntok, const SoftmaxState& st,
                                                const float (&x)[4], float (&o)[D / 16][4]) {
    if (ot.v0 >= ot.v1) return;
    const uint32_t* voff = ot.hdr + 8 * ot.nt + 1;
    int e = (int)__ldg(voff + 8 * ot.ti + g4);
    const int e1 = (int)__ldg(voff + 8 * ot.ti + g4 + 1);
    __half* ph = reinterpret_cast<__half*>(ot.buf);  // [16 tokens][8 queries] fp16 weights (<= 2^8)
    *reinterpret_cast<__half2*>(ph + (2 * g4) * kQ + 2 * t4) =
        __floats2half2_rn(exp2f(x[0] - st.m[0]), exp2f(x[1] - st.m[1]));
    *reinterpret_cast<__half2*>(ph + (2 * g4 + 1) * kQ + 2 * t4) =
        __floats2half2_rn(exp2f(x[2] - st.m[0]), exp2f(x[3] - st.m[1]));
    __syncwarp();
    const int dlo = g4 * (D / 8), tb = 16 * ot.ti;
    uint2 n0 = make_uint2(0u, 0xffffffffu), n1 = n0;
    if (e < e1) n0 = __ldg(ot.ent + e);
    if (e + 1 < e1) n1 = __ldg(ot.ent + e + 1);
#pragma unroll
    for (int t = 0; t < D / 16; ++t) {
        while (e < e1 && (int)(n0.x >> 16) < dlo + 2 * (t + 1)) {
            const int tok = (int)(n0.x & 0xffffu) - tb, d = (int)(n0.x >> 16);
            if (tok >= 0 && tok < ntok && d >= dlo + 2 * t) {
                const float delta = __uint_as_float(n0.y);
                const float2 pf = __half22float2(*reinterpret_cast<const __half2*>(ph + tok * kQ + 2 * t4));
                if (d & 1) { o[t][2] = fmaf(pf.x, delta, o[t][2]); o[t][3] = fmaf(pf.y, delta, o[t][3]); }
                else       { o[t][0] = fmaf(pf.x, delta, o[t][0]); o[t][1] = fmaf(pf.y, delta, o[t][1]); }
            }
            ++e;
            n0 = n1;
            if (e + 1 < e1) n1 = __ldg(ot.ent + e + 1);
        }
    }
    __syncwarp();  // the buffer is rewritten by the next tile
}

// The corrections of tile i of a chunk from the chunk's per-lane prefetch (lane i holds tile i's block
// address and entry ranges); also starts the loads of this lane's first two key and value entries.
__device__ __forceinline__ OutlierTile outlier_tile(unsigned long long blk, int k0, int k1, int v0, int v1, int i,
                                                    int ti, int nt, unsigned char* buf) {
    OutlierTile ot;
    const unsigned long long b = __shfl_sync(0xffffffffu, blk, i);
    ot.hdr = reinterpret_cast<const uint32_t*>(b);
    ot.ent = b ? reinterpret_cast<const uint2*>(ot.hdr + 2 * (8 * nt + 1)) : nullptr;
    ot.k0 = __shfl_sync(0xffffffffu, k0, i);
    ot.k1 = __shfl_sync(0xffffffffu, k1, i);
    ot.v0 = __shfl_sync(0xffffffffu, v0, i);
    ot.v1 = __shfl_sync(0xffffffffu, v1, i);
    ot.ti = ti;
    ot.nt = nt;
    ot.buf = buf;
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        ot.ke[u] = (ot.k0 + 32 * u + lane < ot.k1) ? __ldg(ot.ent + ot.k0 + 32 * u + lane) : make_uint2(0u, 0u);
        ot.ve[u] = (ot.v0 + 32 * u + lane < ot.v1) ? __ldg(ot.ent + ot.v0 + 32 * u + lane) : make_uint2(0u, 0u);
    }
    return ot;
}

// A tile of a slot that holds no live page: nothing attends to it; its per-tile mass reads -inf.
template <bool MASS>
__device__ __forceinline__ void skip_tile(float* mass_out) {
    if constexpr (MASS) {
        if ((threadIdx.x & 31) < kQ) mass_out[threadIdx.x & 31] = -INFINITY;
    }
}

// Processes one staged tile: scores, online softmax, PV (OUT: with the page's outlier corrections).
template <int D, int TIER, bool PRECISE, bool MASS, bool OUT>
__device__ __forceinline__ void process_tile(const TilePtr& tp, int g4, int t4, uint32_t qs, float scale_log2, float2 qsum,
                                             SoftmaxState& st, float (&o)[D / 16][4], float* mass_out,
                                             const OutlierTile& ot) {
    TokScale tk[1], tv[1];
    float x[1][4];
    load_tok_scales<TIER>(tp, g4, t4, tk[0], tv[0]);
    tile_scores<D, TIER>(tp, g4, t4, tk[0], qs, scale_log2, qsum, x[0]);
    if constexpr (OUT) {
        if constexpr (side_dense(D)) dense_k_outliers<D>(ot, qs, scale_log2, tp.ntok, x[0]);
        else walk_k_outliers<D>(ot, g4, t4, qs, scale_log2, tp.ntok, x[0]);
    }
    // the V fragments do not depend on the scores: built here, their dequantization overlaps the
    // score MMAs' latency and the softmax's exponentials
    uint32_t av[D / 16][4];
    tile_vfrags<D, TIER>(tp, g4, t4, tv[0], av);
    uint32_t b01[1], b23[1], c01[1], c23[1];
    softmax_update<D / 16, 1, PRECISE, MASS>(x, st, o, b01, b23, c01, c23, mass_out);
    if constexpr (OUT) {
        if constexpr (side_dense(D)) dense_v_outliers<D, PRECISE>(ot, tp.ntok, b01[0], b23[0], c01[0], c23[0], o);
        else walk_v_outliers<D>(ot, g4, t4, tp.ntok, st, x[0], o);
    }
    tile_pv<D, PRECISE>(av, b01[0], b23[0], c01[0], c23[0], o);
}

// Gather mode: shared memory past the merge buffers where a group's output rows are staged as fp16
// [kQ][D] before they go to the ranks.
template <int D>
__device__ __forceinline__ __half* gather_stage(unsigned char* smem) {
    return reinterpret_cast<__half*>(smem + (size_t)kPairs * kStages * stage_bytes(D) - (size_t)kQ * D * 2);
}

// Gather mode: copies the staged rows of group (b, h, qg) into every rank's output buffer at their
// rows of the full layout (16-byte stores, peers through their IPC mappings).  No fence here: the
// arrival signal comes from gather_signal_wait_kernel, queued after this kernel on the same stream.
template <int D>
__device__ __forceinline__ void gather_rows(const Params& p, int b, int h, int qg, const __half* ost) {
    constexpr int V = D / 8;  // 16-byte vectors per row
    const int NQ = p.G * p.qlen;
    const int hg = p.gat.rank * p.Hkv + h;
    const int64_t half_elems = (int64_t)p.B * p.gat.heads_kv_total * p.G * p.qlen * D;
    for (int e = threadIdx.x; e < p.gat.world * kQ * V; e += kThreads) {
        const int r = e / (kQ * V), rem = e - r * (kQ * V);
        const int n = rem / V, v = rem - n * V;
        const int ng = qg * kQ + n;
        if (ng >= NQ) continue;
        const int gi = ng / p.qlen, qi = ng - gi * p.qlen;
        const int64_t row = (((int64_t)b * p.gat.heads_kv_total + hg) * p.G + gi) * p.qlen + qi;
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(p.gat.out[r]) + p.gat.parity * half_elems + row * D);
        dst[v] = reinterpret_cast<const uint4*>(ost + n * D)[v];
    }
}

// Merges the split partials of one (batch, kv_head, query group): out = sum_s 2^(lse_s - LSE) O_s,
// LSE = log2 sum_s 2^lse_s.  Run by the group's last CTA to finish (all its threads); the other
// CTAs' partials are read through L2.  The per-(split, query) weights are formed once in shared
// memory (wbuf: S*8 + 16 floats), then every output element sums its S partials eight at a time.
template <int D>
__device__ __forceinline__ void combine_group(const Params& p, int64_t grp, int b, int h, int qg, float* wbuf,
                                              __half* ost) {
    const int NQ = p.G * p.qlen, S = p.S;
    float* Ms = wbuf;           // [kQ] max lse per query
    float* Ws = wbuf + kQ;      // [kQ] sum of weights per query
    float* w = wbuf + 2 * kQ;   // [S][kQ] weights 2^(lse_s - M)
    const float* pl = p.part_lse + grp * S * kQ;
    for (int i = threadIdx.x; i < S * kQ; i += kThreads) w[i] = __ldcg(pl + i);
    __syncthreads();
    if (threadIdx.x < kQ) {
        float M = -INFINITY;
        for (int s = 0; s < S; ++s) M = fmaxf(M, w[s * kQ + threadIdx.x]);
        Ms[threadIdx.x] = M;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < S * kQ; i += kThreads) {
        const float M = Ms[i % kQ];
        w[i] = (M == -INFINITY) ? 0.f : exp2f(w[i] - M);  // an empty split (-inf) weighs 0
    }
    __syncthreads();
    if (threadIdx.x < kQ) {
        float W = 0.f;
        for (int s = 0; s < S; ++s) W += w[s * kQ + threadIdx.x];
        Ws[threadIdx.x] = W;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < kQ * D; e += kThreads) {
        const int n = e / D, d = e - n * D;
        const int ng = qg * kQ + n;
        if (ng >= NQ) continue;
        const float* po = p.part_o + (grp * S * kQ + n) * (int64_t)D + d;  // split s at + s * kQ * D
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        int s = 0;
        for (; s + 8 <= S; s += 8) {
#pragma unroll
            for (int u = 0; u < 8; ++u) acc[u] += w[(s + u) * kQ + n] * __ldcg(po + (int64_t)(s + u) * kQ * D);
        }
        for (; s < S; ++s) acc[0] += w[s * kQ + n] * __ldcg(po + (int64_t)s * kQ * D);
        const float sum = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
        const float W = Ws[n], M = Ms[n];
        const int gi = ng / p.qlen, qi = ng - gi * p.qlen;
        const int64_t row = ((int64_t)b * p.Hkv * p.G + (int64_t)h * p.G + gi) * p.qlen + qi;
        const __half val = __float2half_rn(W > 0.f ? sum / W : 0.f);
        if (p.gat.world > 0) ost[n * D + d] = val;
        else p.out[row * D + d] = val;
        if (p.lse && d == 0) p.lse[row] = (W > 0.f) ? (M + log2f(W)) * 0.69314718055994530942f : -INFINITY;
    }
    if (p.gat.world > 0) {
        __syncthreads();
        gather_rows<D>(p, b, h, qg, ost);
    }
}

// SIDE: some arena carries outlier sidecars (a separate instantiation, so launches without them run
// the plain kernel's register allocation).
template <int D, bool PRECISE, bool MASS, bool SIDE>
__global__ void __launch_bounds__(kThreads, SIDE ? side_ctas_per_sm(D) : ctas_per_sm(D))
    decode_attn_kernel(const __grid_constant__ Params p) {
    constexpr int KC = D / 16;
    constexpr int STAGE = stage_bytes(D);
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t mbar[kPairs][kStages];
    // pair chunk most recently issued into each slot.  A slot's consumers alternate between the
    // two warps, so a warp may reach chunk j + kStages before its partner's chunk j (same slot) has
    // even landed; an mbarrier parity test would then match the previous, completed phase.  Waiters
    // first see their chunk issued here, then test the parity.
    __shared__ int issued[kPairs][kStages];
    __shared__ float qsum_s[kQ];  // sum over d of each query of the group (key-side score terms)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g4 = lane >> 2, t4 = lane & 3;
    const int split = blockIdx.x, bh = blockIdx.y, qg = blockIdx.z;
    const int b = bh / p.Hkv, h = bh - b * p.Hkv;
    const int NQ = p.G * p.qlen;
    const int pair = warp / kPairWarps, wip = warp - pair * kPairWarps;
    unsigned char* wbuf = smem + (size_t)pair * kStages * STAGE;

    SoftmaxState st;
    st.m[0] = st.m[1] = kNoMax;
    st.l[0] = st.l[1] = 0.f;
    float o[KC][4];
#pragma unroll
    for (int t = 0; t < KC; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;

    // The split's chunks are dealt to the warp pairs round-robin; pair chunk j sits in ring slot
    // j % kStages and is processed by warp j % kPairWarps of the pair.  The warp that finishes a
    // slot refills it with pair chunk j + kStages (which its partner will process).
    const int c_begin = p.split_chunk0[split], c_end = p.split_chunk0[split + 1];
    const int first = c_begin + pair;
    const int n_pair = first < c_end ? (c_end - first + kPairs - 1) / kPairs : 0;

    // Issue the bulk copies of pair chunk j into slot j % kStages (one lane).
    auto issue = [&](int j) {
        const argus_kv_chunk ch = p.chunks[first + j * kPairs];
        const argus_kv_arena& ar = p.arenas[ch.arena];
        const int tier = ar.tier, n = ch.ntiles, P = ar.page_tokens;
        unsigned char* dst = wbuf + (j % kStages) * STAGE;
        uint64_t* bar = &mbar[pair][j % kStages];
        const unsigned char* blk = static_cast<const unsigned char*>(ar.k) + (int64_t)bh * ar.bh_stride;
        fence_proxy_async();
        if (whole_records(ar.layout, P)) {
            // n consecutive records of this (b, h): one contiguous copy
            const uint32_t bytes = (uint32_t)n * (uint32_t)ar.record_bytes;
            mbar_expect_tx(bar, bytes);
            bulk_g2s(dst, blk + (int64_t)ch.slot0 * ar.record_bytes, bytes, bar);
        } else {
            const int ntok = 16 * (n - 1) + ch.ntok_last;
            const int lp = tier_log2per(tier);
            const int rb = row_bytes(tier, D);
            const uint32_t pbytes = (uint32_t)(((ntok + (1 << lp) - 1) >> lp) * rb);
            const int pb16 = payload_bytes(tier, 16, D);
            const uint32_t sbytes = (uint32_t)((ntok * 2 + 15) & ~15);
            uint32_t total = 2 * pbytes;
            if (tier_scaled(tier)) total += 2 * sbytes * (tier_min(tier) ? 2 : 1);
            mbar_expect_tx(bar, total);
            if (ar.layout == ARGUS_LAYOUT_SPLIT_FP16) {
                const int64_t off = (int64_t)bh * ar.bh_stride + (int64_t)ch.slot0 * 32 * D;
                bulk_g2s(dst, static_cast<const unsigned char*>(ar.k) + off, pbytes, bar);
                bulk_g2s(dst + n * pb16, static_cast<const unsigned char*>(ar.v) + off, pbytes, bar);
            } else {
                const unsigned char* rec = blk + (int64_t)ch.slot0 * ar.record_bytes;
                const int pbP = payload_bytes(tier, P, D);
                const int64_t roff = (int64_t)(ch.tok0 >> lp) * rb;
                bulk_g2s(dst, rec + roff, pbytes, bar);
                bulk_g2s(dst + n * pb16, rec + pbP + roff, pbytes, bar);
                if (tier_scaled(tier)) {
                    const unsigned char* sc = rec + 2 * pbP + 2 * ch.tok0;
                    unsigned char* sd = dst + 2 * n * pb16;
                    bulk_g2s(sd, sc, sbytes, bar);
                    bulk_g2s(sd + 32 * n, sc + 2 * P, sbytes, bar);
                    if (tier_min(tier)) {
                        bulk_g2s(sd + 64 * n, sc + 4 * P, sbytes, bar);
                        bulk_g2s(sd + 96 * n, sc + 6 * P, sbytes, bar);
                    }
                }
            }
        }
        __threadfence_block();  // the arrive above is visible before the slot's issued mark
        *reinterpret_cast<volatile int*>(&issued[pair][j % kStages]) = j;
    };

    // The pair's leading lane sets up its ring and starts the first copies before anything else, so
    // their DRAM latency overlaps the query setup.
    if (wip == 0 && lane == 0) {
#pragma unroll
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&mbar[pair][s], 1);
            issued[pair][s] = -1;
        }
        fence_mbar_init();
        for (int j = 0; j < kStages && j < n_pair; ++j) issue(j);
    }

    // ---- Q^T fragments (query qg*8 + g4, dims t4*D/4 ..), written once by warp 0 into the shared
    // memory past the last ring slot (load_qfrags layout), read back for every tile
    uint32_t* qsw = reinterpret_cast<uint32_t*>(smem + (size_t)kPairs * kStages * STAGE);
    const uint32_t qs = smem_u32(qsw);
    // SIDE: each warp's outlier-correction buffer, past the query fragments
    unsigned char* sbuf = SIDE ? smem + (size_t)kPairs * kStages * STAGE + stage_slack(D) + warp * side_warp_bytes(D)
                               : nullptr;
    if constexpr (SIDE && side_dense(D)) {
        // dense delta tiles start (and are left after every use) all zero
        for (int i = lane; i < side_warp_bytes(D) / 16; i += 32)
            reinterpret_cast<uint4*>(sbuf)[i] = make_uint4(0u, 0u, 0u, 0u);
        __syncwarp();
    }
    if (warp == 0) {
        constexpr int V = (2 * KC) % 4 == 0 ? 4 : 2;
        const int n = qg * kQ + g4;
        const bool live = n < NQ;
        const __half* qrow = p.q;
        if (live) {
            // gather mode reads the full query [B][H_q total][q_len][D]: this rank's heads start at rank * Hkv
            const int gi = n / p.qlen, qi = n - gi * p.qlen;
            const int hq = p.gat.world > 0 ? p.gat.heads_kv_total : p.Hkv;
            const int hh = p.gat.world > 0 ? p.gat.rank * p.Hkv + h : h;
            qrow = p.q + (((int64_t)b * hq * p.G + (int64_t)hh * p.G + gi) * p.qlen + qi) * D + t4 * (D / 4);
        }
        float qsum = 0.f;
#pragma unroll
        for (int c = 0; c < KC; ++c) {
            uint32_t f0 = 0u, f1 = 0u;
            if (live) {
                const uint32_t q01 = *reinterpret_cast<const uint32_t*>(qrow + 4 * c);
                const uint32_t q23 = *reinterpret_cast<const uint32_t*>(qrow + 4 * c + 2);
                f0 = prmt(q01, q23, 0x5410);  // dims 4c, 4c+2
                f1 = prmt(q01, q23, 0x7632);  // dims 4c+1, 4c+3
                const float2 a01 = __half22float2(u2h(q01)), a23 = __half22float2(u2h(q23));
                qsum += (a01.x + a01.y) + (a23.x + a23.y);
            }
            const int j0 = 2 * c, j1 = 2 * c + 1;
            qsw[((j0 / V) * 32 + lane) * V + j0 % V] = f0;
            qsw[((j1 / V) * 32 + lane) * V + j1 % V] = f1;
        }
        // lanes 4n .. 4n+3 hold query n's four dim ranges
        qsum += __shfl_xor_sync(0xffffffffu, qsum, 1);
        qsum += __shfl_xor_sync(0xffffffffu, qsum, 2);
        if (t4 == 0) qsum_s[g4] = qsum;
    }

    __syncthreads();  // rings initialised, first copies issued, query fragments in place
    const float2 qsum = make_float2(qsum_s[2 * t4], qsum_s[2 * t4 + 1]);

    bool failed = false;
    argus_kv_chunk nch;  // descriptor of this warp's next chunk, loaded one chunk ahead
    if (wip < n_pair) nch = p.chunks[first + wip * kPairs];
    for (int j = wip; j < n_pair; j += kPairWarps) {
        const argus_kv_chunk ch = nch;
        if (j + kPairWarps < n_pair) nch = p.chunks[first + (j + kPairWarps) * kPairs];
        const int stage = j % kStages;
        // outlier corrections of the chunk's tiles, fetched before the wait: lane i < ntiles holds tile
        // i's block address and key / value entry ranges (odir: the directory row of this (b, h))
        const unsigned long long* odir = nullptr;
        unsigned long long cblk = 0ull;
        int ck0 = 0, ck1 = 0, cv0 = 0, cv1 = 0, cnt = 1;
        bool cwhole = true;
        if constexpr (SIDE) {
            const argus_kv_arena& oa = p.arenas[ch.arena];
            if (oa.outlier_dir) {
                odir = reinterpret_cast<const unsigned long long*>(oa.outlier_dir) + (int64_t)bh * oa.dir_slots;
                cwhole = whole_records(oa.layout, oa.page_tokens);
                cnt = cwhole ? 1 : (oa.page_tokens + 15) >> 4;
                if (lane < ch.ntiles) {
                    const int ti = cwhole ? 0 : (ch.tok0 >> 4) + lane;
                    cblk = __ldg(odir + (cwhole ? ch.slot0 + lane : ch.slot0));
                    if (cblk) {
                        const uint32_t* h = reinterpret_cast<const uint32_t*>(cblk);
                        ck0 = (int)__ldg(h + 8 * ti);
                        ck1 = (int)__ldg(h + 8 * ti + 8);
                        cv0 = (int)__ldg(h + 8 * cnt + 1 + 8 * ti);
                        cv1 = (int)__ldg(h + 8 * cnt + 1 + 8 * ti + 8);
                    }
                }
            }
        }
        // tiles of slots that hold no live page (slot_live) are skipped: bit i of live_mask is tile i
        unsigned live_mask = 0xffffffffu;
        {
            const argus_kv_arena& la = p.arenas[ch.arena];
            if (la.slot_live) {
                const bool wr = whole_records(la.layout, la.page_tokens);
                const bool mine = wr ? lane < ch.ntiles : lane == 0;
                const bool alive = mine && __ldg(la.slot_live + ch.slot0 + (wr ? lane : 0)) != 0;
                live_mask = wr ? __ballot_sync(0xffffffffu, alive) : (__any_sync(0xffffffffu, alive) ? 0xffffffffu : 0u);
            }
        }
        {
            // bounded: chunk j is issued by whichever warp finishes chunk j - kStages.  Both waits are
            // voted over the warp, so its lanes leave the loop together.
            long long spin = 0;
            while (*reinterpret_cast<volatile int*>(&issued[pair][stage]) != j && spin < kSpinLimit) ++spin;
            if (__any_sync(0xffffffffu, spin >= kSpinLimit)) {
                failed = true;
                break;
            }
            __threadfence_block();
        }
        if (!__all_sync(0xffffffffu, mbar_wait(&mbar[pair][stage], (uint32_t)((j / kStages) & 1)))) {
            failed = true;
            break;
        }
        const argus_kv_arena& ar = p.arenas[ch.arena];
        const int n = ch.ntiles;
        const unsigned char* sb = wbuf + stage * STAGE;
        float* mass_base = nullptr;
        if constexpr (MASS)
            mass_base = p.tile_lse + (((int64_t)bh * p.nqg + qg) * p.n_chunks + (first + j * kPairs)) * 16 * kQ;
        const bool rec16 = ar.layout == ARGUS_LAYOUT_RECORD && ar.page_tokens == 16;
        switch (ar.tier) {
#define ARGUS_TILE_LOOPS(T, OUT)                                                                                  \
        if (rec16) {                                                                                              \
            /* one full 16-token page per record: compile-time offsets */                                        \
            constexpr int RB = record_bytes(T, 16, D), PB = payload_bytes(T, 16, D);                              \
            for (int i = 0; i < n; ++i) {                                                                         \
                if (!((live_mask >> i) & 1u)) {                                                                   \
                    skip_tile<MASS>(mass_base ? mass_base + i * kQ : nullptr);                                    \
                    continue;                                                                                     \
                }                                                                                                 \
                const unsigned char* r = sb + i * RB;                                                             \
                TilePtr tp;                                                                                       \
                tp.k = r;                                                                                         \
                tp.v = r + PB;                                                                                    \
                tp.ks = reinterpret_cast<const __half*>(r + 2 * PB);                                              \
                tp.vs = reinterpret_cast<const __half*>(r + 2 * PB + 32);                                         \
                tp.km = reinterpret_cast<const __half*>(r + 2 * PB + 64);                                         \
                tp.vm = reinterpret_cast<const __half*>(r + 2 * PB + 96);                                         \
                tp.ntok = 16;                                                                                     \
                OutlierTile ot;                                                                                   \
                if constexpr (OUT) ot = outlier_tile(cblk, ck0, ck1, cv0, cv1, i, 0, 1, sbuf);                  \
                process_tile<D, T, PRECISE, MASS, OUT>(tp, g4, t4, qs, p.scale_log2, qsum, st, o,                       \
                                                       mass_base ? mass_base + i * kQ : nullptr, ot);             \
            }                                                                                                     \
        } else {                                                                                                  \
            const ChunkView cv = chunk_view<D>(ar, n);                                                            \
            for (int i = 0; i < n; ++i) {                                                                         \
                if (!((live_mask >> i) & 1u)) {                                                                   \
                    skip_tile<MASS>(mass_base ? mass_base + i * kQ : nullptr);                                    \
                    continue;                                                                                     \
                }                                                                                                 \
                TilePtr tp;                                                                                       \
                const int po = i * cv.pstride, so = i * cv.sstride;                                               \
                tp.k = sb + cv.k_off + po;                                                                        \
                tp.v = sb + cv.v_off + po;                                                                        \
                tp.ks = reinterpret_cast<const __half*>(sb + cv.ks_off + so);                                     \
                tp.vs = reinterpret_cast<const __half*>(sb + cv.vs_off + so);                                     \
                tp.km = reinterpret_cast<const __half*>(sb + cv.km_off + so);                                     \
                tp.vm = reinterpret_cast<const __half*>(sb + cv.vm_off + so);                                     \
                tp.ntok = (i == n - 1) ? ch.ntok_last : cv.ntok_full;                                             \
                OutlierTile ot;                                                                                   \
                if constexpr (OUT) /* whole records: tile i is page slot0 + i; else tokens tok0 + 16 i .. */    \
                    ot = outlier_tile(cblk, ck0, ck1, cv0, cv1, i, cwhole ? 0 : (ch.tok0 >> 4) + i, cnt, sbuf);   \
                process_tile<D, T, PRECISE, MASS, OUT>(tp, g4, t4, qs, p.scale_log2, qsum, st, o,                       \
                                                       mass_base ? mass_base + i * kQ : nullptr, ot);             \
            }                                                                                                     \
        }
#define ARGUS_TILE_CASE(T)                                                                                        \
    case T: {                                                                                                     \
        if (SIDE && odir) {                                                                                       \
            ARGUS_TILE_LOOPS(T, SIDE)                                                                             \
        } else {                                                                                                  \
            ARGUS_TILE_LOOPS(T, false)                                                                            \
        }                                                                                                         \
        break;                                                                                                    \
    }
            case ARGUS_TIER_FP16: {  // fp16 arenas carry no sidecars
                ARGUS_TILE_LOOPS(ARGUS_TIER_FP16, false)
                break;
            }
            case ARGUS_TIER_FP8SIM:  // same dequantization as INT8: fp16(q * s)
            ARGUS_TILE_CASE(ARGUS_TIER_INT8)
            ARGUS_TILE_CASE(ARGUS_TIER_INT4)
            ARGUS_TILE_CASE(ARGUS_TIER_INT2)
            ARGUS_TILE_CASE(ARGUS_TIER_1BIT)
            ARGUS_TILE_CASE(ARGUS_TIER_E4M3)
#undef ARGUS_TILE_CASE
#undef ARGUS_TILE_LOOPS
            default: break;
        }
        __syncwarp();
        if (lane == 0 && j + kStages < n_pair) issue(j + kStages);
        __syncwarp();
    }
    if (failed) {
        if (lane == 0) atomicExch(&g_status, (int)ARGUS_ERR_TIMEOUT);
        // let copies still in flight land before the shared memory is released (bounded again): each
        // slot's last issued chunk j' completes phase j' / kStages of the slot's barrier
        for (int s = 0; s < kStages; ++s) {
            const int jl = *reinterpret_cast<volatile int*>(&issued[pair][s]);
            if (jl >= 0) (void)mbar_wait(&mbar[pair][s], (uint32_t)((jl / kStages) & 1));
        }
    }

    // ---- finish this warp: reduce l over the 8 token lanes
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        st.l[0] += __shfl_xor_sync(0xffffffffu, st.l[0], off);
        st.l[1] += __shfl_xor_sync(0xffffffffu, st.l[1], off);
    }
    __syncthreads();  // all warps are done with their stages: reuse shared memory for the merge

    // merge buffer: per warp m[8], l[8], O[8][D]
    float* mw = reinterpret_cast<float*>(smem);
    float* lw = mw + kWarps * kQ;
    float* ow = lw + kWarps * kQ;
    if (g4 == 0) {
        mw[warp * kQ + 2 * t4] = st.m[0];
        mw[warp * kQ + 2 * t4 + 1] = st.m[1];
        lw[warp * kQ + 2 * t4] = st.l[0];
        lw[warp * kQ + 2 * t4 + 1] = st.l[1];
    }
    {
        const int dbase = g4 * (D / 8);
        float* o0 = ow + ((size_t)warp * kQ + 2 * t4) * D + dbase;
        float* o1 = o0 + D;
#pragma unroll
        for (int t = 0; t < KC; ++t) {
            o0[2 * t] = o[t][0];
            o0[2 * t + 1] = o[t][2];
            o1[2 * t] = o[t][1];
            o1[2 * t + 1] = o[t][3];
        }
    }
    __syncthreads();

    const int64_t grp = ((int64_t)bh * p.nqg + qg);
    for (int e = threadIdx.x; e < kQ * D; e += kThreads) {
        const int n = e / D, d = e - n * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mw[w * kQ + n]);
        float L = 0.f, acc = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                const float f = exp2f(mw[w * kQ + n] - M);
                L += f * lw[w * kQ + n];
                acc += f * ow[((size_t)w * kQ + n) * D + d];
            }
        }
        const int ng = qg * kQ + n;
        if (p.S == 1) {
            if (ng < NQ) {
                const int gi = ng / p.qlen, qi = ng - gi * p.qlen;
                const int64_t row = ((int64_t)b * p.Hkv * p.G + (int64_t)h * p.G + gi) * p.qlen + qi;
                const __half val = __float2half_rn(L > 0.f ? acc / L : 0.f);
                if (p.gat.world > 0) gather_stage<D>(smem)[n * D + d] = val;
                else p.out[row * D + d] = val;
                if (p.lse && d == 0) p.lse[row] = (L > 0.f) ? (M + log2f(L)) * 0.69314718055994530942f : -INFINITY;
            }
        } else {
            float* po = p.part_o + ((grp * p.S + split) * kQ + n) * D;
            po[d] = L > 0.f ? acc / L : 0.f;
            if (d == 0) p.part_lse[(grp * p.S + split) * kQ + n] = (L > 0.f) ? M + log2f(L) : -INFINITY;
        }
    }
    if (p.S == 1 && p.gat.world > 0) {
        __syncthreads();
        gather_rows<D>(p, b, h, qg, gather_stage<D>(smem));
    }
    if (p.S > 1) {
        // the group's last CTA to arrive merges the splits (and resets the counter for the next launch)
        __shared__ int last;
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            const int prev = atomicAdd(&p.counters[grp], 1);
            last = (prev == p.S - 1);
            if (last) p.counters[grp] = 0;
        }
        __syncthreads();
        if (last) {
            __threadfence();
            combine_group<D>(p, grp, b, h, qg, reinterpret_cast<float*>(smem), gather_stage<D>(smem));
        }
    }
}

// Self-test of the bounded waits (argus_selftest_wait_timeout): the CTA waits, through the same
// mbar_wait the ring consumers use, on an mbarrier that no copy and no thread ever completes, gives
// up after `polls` polls and records ARGUS_ERR_TIMEOUT in the status word as a ring consumer does.
__device__ int g_selftest_gave_up = 0;

__global__ void wait_timeout_selftest_kernel(long long polls) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    const bool done = mbar_wait(&bar, 0u, polls);
    if (threadIdx.x == 0) {
        if (!done) atomicExch(&g_status, (int)ARGUS_ERR_TIMEOUT);
        g_selftest_gave_up = done ? 0 : 1;
    }
}

// One thread signals every rank, then waits (bounded, ~0.25 us between polls) until this rank's
// arrival counter reaches target.  The attention kernel before it on the stream stored this rank's
// rows into every rank's buffer: stream order puts those stores before the system-scope fence and
// the release adds here, so a rank whose acquire load sees every signal of a step also sees every
// row of it, and so do the kernels queued after this one.
__global__ void gather_signal_wait_kernel(argus_peer_gather g, unsigned long long target, long long polls) {
    if (threadIdx.x != 0) return;
    __threadfence_system();
    for (int r = 0; r < g.world; ++r)
        asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(g.arrivals[r]), "l"(1ull) : "memory");
    const unsigned long long* arrivals = static_cast<const unsigned long long*>(g.arrivals[g.rank]);
    for (long long i = 0;; ++i) {
        unsigned long long v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(arrivals) : "memory");
        if (v >= target) return;
        if (i >= polls) {
            atomicExch(&g_status, (int)ARGUS_ERR_TIMEOUT);
            return;
        }
        __nanosleep(256);
    }
}

template <int D>
int launch(const Params& prm, int n_splits, bool precise, cudaStream_t st) {
    bool side = false;
    for (int i = 0; i < ARGUS_MAX_ARENAS; ++i) side |= prm.arenas[i].outlier_dir != nullptr;
    // kernels with outlier sidecars also hold one correction buffer per warp
    const size_t smem = (size_t)kPairs * kStages * stage_bytes(D) + stage_slack(D) + (side ? kWarps * side_warp_bytes(D) : 0);
    static_assert((size_t)kWarps * kQ * (D + 2) * 4 + (size_t)kQ * D * 2 <= (size_t)kPairs * kStages * stage_bytes(D),
                  "merge buffer and gather staging must fit in the stage memory");
    const bool mass = prm.tile_lse != nullptr;
    auto kern = side ? (precise ? (mass ? decode_attn_kernel<D, true, true, true> : decode_attn_kernel<D, true, false, true>)
                                : (mass ? decode_attn_kernel<D, false, true, true> : decode_attn_kernel<D, false, false, true>))
                     : (precise ? (mass ? decode_attn_kernel<D, true, true, false> : decode_attn_kernel<D, true, false, false>)
                                : (mass ? decode_attn_kernel<D, false, true, false> : decode_attn_kernel<D, false, false, false>));
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return argus_set_cuda_error(e);
    // all of the unified L1/shared array as shared memory, so ctas_per_sm(D) CTAs fit
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return argus_set_cuda_error(e);
    dim3 grid(n_splits, prm.B * prm.Hkv, prm.nqg);
    kern<<<grid, kThreads, smem, st>>>(prm);
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

}  // namespace da
}  // namespace argus

using namespace argus;

namespace {
bool valid_head_dim(int D) { return D == 16 || D == 32 || D == 64 || D == 128 || D == 256; }
}  // namespace

extern "C" {

int argus_record_bytes(int tier, int page_tokens, int head_dim) {
    if (tier < ARGUS_TIER_FP16 || tier > ARGUS_TIER_E4M3 || page_tokens <= 0 || head_dim <= 0) return 0;
    return da::record_bytes(tier, page_tokens, head_dim);
}

int argus_decode_attention_chunk_tiles(int tier, int layout, int page_tokens, int head_dim) {
    if (tier < ARGUS_TIER_FP16 || tier > ARGUS_TIER_E4M3 || !valid_head_dim(head_dim) || page_tokens <= 0) return 0;
    if (layout != ARGUS_LAYOUT_RECORD && layout != ARGUS_LAYOUT_SPLIT_FP16) return 0;
    return da::chunk_tiles(tier, layout, page_tokens, head_dim);
}

int64_t argus_decode_attention_workspace_size(const argus_attn_shape* s) {
    if (!s || s->n_splits <= 1) return 0;
    const int64_t nqg = (s->group * (int64_t)s->q_len + da::kQ - 1) / da::kQ;
    const int64_t groups = (int64_t)s->batch * s->heads_kv * nqg;
    // [counters: groups ints, padded to 256 B][part_lse][part_o], plus alignment slack
    return ((groups * 4 + 255) & ~255LL) + groups * s->n_splits * da::kQ * ((int64_t)s->head_dim + 1) * (int64_t)sizeof(float) + 256;
}

}  // extern "C"

namespace {

// Checks every argument of a decode-attention call but the split-K workspace and fills the launch
// parameters.  Returns ARGUS_OK or an error status (argus_last_error has the text); nothing is
// queued on the device either way.
int prepare_attention(const argus_attn_shape* s, const argus_kv_arena* arenas, const argus_kv_chunk* chunks,
                      const int32_t* split_chunk0, const uint16_t* q, uint16_t* out, float* lse, float* tile_lse,
                      da::Params& prm) {
    if (!s || !arenas || !split_chunk0 || !q || !out)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    if (s->batch <= 0 || s->heads_kv <= 0 || s->group <= 0 || s->q_len <= 0 || s->n_splits <= 0)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "non-positive size");
    if (s->n_arenas <= 0 || s->n_arenas > ARGUS_MAX_ARENAS)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "arena count out of range");
    if (s->n_chunks > 0 && !chunks) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null chunk table");
    if ((int64_t)s->batch * s->heads_kv > 65535) return argus_set_error(ARGUS_ERR_UNSUPPORTED, "B*H_kv above 65535");
    const int D = s->head_dim;
    if (!valid_head_dim(D)) return argus_set_error(ARGUS_ERR_UNSUPPORTED, "head_dim must be 16, 32, 64, 128 or 256");
    if (!argus_aligned(q, 16) || !argus_aligned(out, 16)) return argus_set_error(ARGUS_ERR_MISALIGNED, "q/out alignment");
    memset(&prm, 0, sizeof(prm));
    for (int i = 0; i < s->n_arenas; ++i) {
        const argus_kv_arena& a = arenas[i];
        if (a.tier < ARGUS_TIER_FP16 || a.tier > ARGUS_TIER_E4M3)
            return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad arena tier");
        if (!a.k || !argus_aligned(a.k, 16) || (a.bh_stride % 16))
            return argus_set_error(ARGUS_ERR_MISALIGNED, "arena base and (b,h) stride must be 16-byte aligned");
        if (a.page_tokens <= 0 || a.page_tokens > 65535)
            return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad page_tokens");
        if (a.layout == ARGUS_LAYOUT_RECORD) {
            if (a.tier != ARGUS_TIER_FP16 && (a.page_tokens % 8))
                return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "quantized pages hold a multiple of 8 tokens");
            if (a.record_bytes != da::record_bytes(a.tier, a.page_tokens, D))
                return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "record_bytes does not match tier/page/head_dim");
            if (a.record_bytes % 16) return argus_set_error(ARGUS_ERR_MISALIGNED, "record size not a multiple of 16");
        } else if (a.layout == ARGUS_LAYOUT_SPLIT_FP16) {
            if (a.tier != ARGUS_TIER_FP16 || !a.v || !argus_aligned(a.v, 16) || a.page_tokens != 16)
                return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "split layout is fp16 K/V tensors in 16-token slots");
        } else {
            return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad arena layout");
        }
        if (a.outlier_dir) {
            if (a.layout != ARGUS_LAYOUT_RECORD || a.tier == ARGUS_TIER_FP16)
                return argus_set_error(ARGUS_ERR_UNSUPPORTED, "outlier sidecars belong to quantized record arenas");
            if (a.dir_slots <= 0 || !argus_aligned(a.outlier_dir, 8))
                return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "outlier directory needs dir_slots > 0, 8-byte alignment");
        }
        prm.arenas[i] = a;
    }
    prm.chunks = chunks;
    prm.split_chunk0 = split_chunk0;
    prm.q = reinterpret_cast<const __half*>(q);
    prm.out = reinterpret_cast<__half*>(out);
    prm.lse = lse;
    prm.B = s->batch;
    prm.Hkv = s->heads_kv;
    prm.G = s->group;
    prm.qlen = s->q_len;
    prm.S = s->n_splits;
    prm.n_chunks = s->n_chunks;
    prm.tile_lse = tile_lse;
    prm.nqg = (s->group * s->q_len + da::kQ - 1) / da::kQ;
    if (prm.nqg > 65535) return argus_set_error(ARGUS_ERR_UNSUPPORTED, "too many query groups");
    prm.scale_log2 = s->scale * 1.4426950408889634f;
    if ((int64_t)(s->n_splits + 2) * da::kQ * 4 > (int64_t)da::kPairs * da::kStages * da::stage_bytes(D))
        return argus_set_error(ARGUS_ERR_UNSUPPORTED, "too many splits for the split merge");
    return ARGUS_OK;
}

// Launches a prepared call with its split-K workspace (unused when n_splits == 1).
int launch_prepared(const argus_attn_shape* s, da::Params& prm, void* workspace, argus_stream_t stream) {
    const int D = s->head_dim;
    if (s->n_splits > 1) {
        if (!workspace || !argus_aligned(workspace, 16))
            return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "split-K needs a 16-byte aligned workspace");
        const int64_t groups = (int64_t)prm.B * prm.Hkv * prm.nqg;
        prm.counters = reinterpret_cast<int*>(workspace);
        prm.part_lse = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + ((groups * 4 + 255) & ~255LL));
        prm.part_o = prm.part_lse + groups * s->n_splits * da::kQ;
    }
    cudaStream_t st = (cudaStream_t)stream;
    const bool precise = (s->flags & ARGUS_ATTN_PRECISE_PV) != 0;
    switch (D) {
        case 16: return da::launch<16>(prm, s->n_splits, precise, st);
        case 32: return da::launch<32>(prm, s->n_splits, precise, st);
        case 64: return da::launch<64>(prm, s->n_splits, precise, st);
        case 128: return da::launch<128>(prm, s->n_splits, precise, st);
        default: return da::launch<256>(prm, s->n_splits, precise, st);
    }
}

}  // namespace

extern "C" {

int argus_decode_attention(const argus_attn_shape* s, const argus_kv_arena* arenas, const argus_kv_chunk* chunks,
                           const int32_t* split_chunk0, const uint16_t* q, uint16_t* out, float* lse, float* tile_lse,
                           void* workspace, argus_stream_t stream) {
    da::Params prm;
    const int rc = prepare_attention(s, arenas, chunks, split_chunk0, q, out, lse, tile_lse, prm);
    if (rc != ARGUS_OK) return rc;
    return launch_prepared(s, prm, workspace, stream);
}

int64_t argus_gather_arrivals_per_step(int world) { return world > 0 ? world : 0; }

int argus_decode_attention_gather(const argus_attn_shape* s, const argus_kv_arena* arenas, const argus_kv_chunk* chunks,
                                  const int32_t* split_chunk0, const uint16_t* q, const argus_peer_gather* g, float* lse,
                                  float* tile_lse, void* workspace, argus_stream_t stream) {
    if (!s || !g) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    if (g->world < 1 || g->world > ARGUS_MAX_PEERS || g->rank < 0 || g->rank >= g->world)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "world / rank out of range");
    if ((int64_t)g->heads_kv_total != (int64_t)s->heads_kv * g->world)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "heads_kv_total must be heads_kv * world");
    if (g->parity != 0 && g->parity != 1) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "parity must be 0 or 1");
    for (int r = 0; r < g->world; ++r) {
        if (!g->out[r] || !g->arrivals[r]) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null peer buffer");
        if (!argus_aligned(g->out[r], 16) || !argus_aligned(g->arrivals[r], 8))
            return argus_set_error(ARGUS_ERR_MISALIGNED, "peer output 16-byte / counter 8-byte alignment");
    }
    const int D = s->head_dim;
    if (valid_head_dim(D) && (int64_t)(s->n_splits + 2) * da::kQ * 4 + (int64_t)da::kQ * D * 2 >
                                 (int64_t)da::kPairs * da::kStages * da::stage_bytes(D))
        return argus_set_error(ARGUS_ERR_UNSUPPORTED, "too many splits for the split merge with gather staging");
    da::Params prm;
    // the local half of this rank's own buffer stands in for `out` in the common checks
    const int rc = prepare_attention(s, arenas, chunks, split_chunk0, q, static_cast<uint16_t*>(g->out[g->rank]), lse,
                                     tile_lse, prm);
    if (rc != ARGUS_OK) return rc;
    prm.gat = *g;
    return launch_prepared(s, prm, workspace, stream);
}

int argus_gather_wait(const argus_peer_gather* g, uint64_t target, int64_t max_polls, argus_stream_t stream) {
    if (!g || g->world < 1 || g->world > ARGUS_MAX_PEERS || g->rank < 0 || g->rank >= g->world)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad gather spec");
    for (int r = 0; r < g->world; ++r)
        if (!g->arrivals[r] || !argus_aligned(g->arrivals[r], 8))
            return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad arrival counter");
    if (max_polls <= 0) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "max_polls must be positive");
    da::gather_signal_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(*g, (unsigned long long)target,
                                                                     (long long)max_polls);
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

int argus_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle) {
    if (bytes <= 0 || !ptr || !ipc_handle) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad argument");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, (size_t)bytes);
    if (e != cudaSuccess) return argus_set_cuda_error(e);
    e = cudaMemset(p, 0, (size_t)bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return argus_set_cuda_error(e);
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");
    memcpy(ipc_handle, &h, sizeof(h));
    *ptr = p;
    return ARGUS_OK;
}

int argus_peer_open(const void* ipc_handle, void** ptr) {
    if (!ipc_handle || !ptr) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? ARGUS_OK : argus_set_cuda_error(e);
}

int argus_peer_close(void* ptr) {
    if (!ptr) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? ARGUS_OK : argus_set_cuda_error(e);
}

int argus_peer_free(void* ptr) {
    if (!ptr) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    const cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? ARGUS_OK : argus_set_cuda_error(e);
}

int argus_selftest_wait_timeout(int64_t polls, int* gave_up, argus_stream_t stream) {
    if (!gave_up) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null result");
    if (polls <= 0 || polls > (int64_t)1 << 20) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "polls out of range");
    cudaStream_t st = (cudaStream_t)stream;
    da::wait_timeout_selftest_kernel<<<1, 32, 0, st>>>((long long)polls);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbolAsync(gave_up, da::g_selftest_gave_up, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    return e == cudaSuccess ? ARGUS_OK : argus_set_cuda_error(e);
}

int argus_device_status(int* status, argus_stream_t stream) {
    if (!status) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null status");
    int v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(&v, da::g_status, sizeof(int), 0, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(da::g_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e != cudaSuccess) return argus_set_cuda_error(e);
    int jl = 0, jla = 0, side = 0;
    int rc = argus_jl_take_status(&jl, (cudaStream_t)stream);
    if (rc == ARGUS_OK) rc = argus_jla_take_status(&jla, (cudaStream_t)stream);
    if (rc == ARGUS_OK) rc = argus_side_take_status(&side, (cudaStream_t)stream);
    if (rc != ARGUS_OK) return rc;
    *status = v != 0 ? v : (jl != 0 ? jl : (jla != 0 ? jla : side));
    return ARGUS_OK;
}

}  // extern "C"

// --------------------------------------------------------------------------- allocation-free entry
// Split-K scratch for argus_decode_attention_noalloc: a fixed array in the module's own device
// memory, so callers that cannot allocate device memory (see the header) still get split-K.
#define ARGUS_NOALLOC_SCRATCH_BYTES (8u << 20)

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[ARGUS_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device, looked up once per device.  Host code
// must not pass the symbol itself to a kernel: in host code it names a host-side stand-in.
int noalloc_scratch(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return argus_set_cuda_error(e);
    if (dev < 0 || dev >= kMaxDevices) return argus_set_error(ARGUS_ERR_UNSUPPORTED, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return argus_set_cuda_error(e);
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return ARGUS_OK;
}

}  // namespace

extern "C" int64_t argus_decode_attention_noalloc_capacity(void) { return ARGUS_NOALLOC_SCRATCH_BYTES; }

extern "C" int argus_decode_attention_noalloc(const argus_attn_shape* s, const argus_kv_arena* arenas,
                                              const argus_kv_chunk* chunks, const int32_t* split_chunk0,
                                              const uint16_t* q, uint16_t* out, float* lse, float* tile_lse,
                                              argus_stream_t stream) {
    if (!s) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null shape");
    const int64_t need = argus_decode_attention_workspace_size(s);
    if (need > (int64_t)ARGUS_NOALLOC_SCRATCH_BYTES)
        return argus_set_error(ARGUS_ERR_CAPACITY,
                               "split-K partials exceed the 8 MiB built-in scratch: use fewer splits or "
                               "argus_decode_attention with a caller workspace");
    // every other argument is checked before anything touches the shared scratch, so a refused call
    // leaves the counters of a call still in flight alone
    da::Params prm;
    const int prc = prepare_attention(s, arenas, chunks, split_chunk0, q, out, lse, tile_lse, prm);
    if (prc != ARGUS_OK) return prc;
    void* scratch = nullptr;
    if (need > 0) {
        const int rc = noalloc_scratch(&scratch);
        if (rc) return rc;
        // the split-arrival counters at the front of the scratch start at zero (a previous call may
        // have used the array with another layout)
        const int64_t groups = (int64_t)s->batch * s->heads_kv * ((s->group * (int64_t)s->q_len + da::kQ - 1) / da::kQ);
        const cudaError_t e = cudaMemsetAsync(scratch, 0, (size_t)((groups * 4 + 255) & ~255LL), (cudaStream_t)stream);
        if (e != cudaSuccess) return argus_set_cuda_error(e);
    }
    return launch_prepared(s, prm, scratch, stream);
}
