// Decode attention over the JL sequence-projection archive, without reconstructing K and V.
//
// The reference rebuilds each archived block as K = R . Yk, V = R . Yv (R = A^-1 W^T (W A^-1 W^T)^-1,
// core/memory_manager.py:241-282, 1176-1178) and runs softmax attention over the rebuilt tokens.
// Because the reconstruction is linear, the same attention is, per block and query,
//     u = Yk . q^T                 (MJ)        the query seen through the block's key rows
//     s = R . u                    (N)         scores of the block's N tokens
//     w = R^T . softmax(s)         (MJ)        softmax weights folded back onto the rows
//     o = Yv^T . w                 (D)         output contribution
// and every block of a kv head shares the one operator R [N x MJ].  So one CTA stacks the (block,
// query) pairs of its blocks as the 128 rows of a tensor-memory tile and streams R past them once:
//
//   U phase   Yk blocks arrive by TMA (128-byte swizzle); the warps form u with mma.sync, stage U^T
//             (rows = block-query pairs, fp16 hi + lo) in shared memory, and warps 0-3 move their
//             rows into tensor memory (the A operand of the scores).
//   SW phase  for each pair of 64-token chunks of R: S = U^T . R_pair^T (tcgen05.mma, A from tensor
//             memory, M 128, N 128, fp32: one MMA group forms the scores of both chunks, since an
//             MMA costs about the same at N 64 as at N 128); per chunk c, warps 0-3 (one row per
//             thread) run the online softmax of their row in the log2 domain and write P_c (fp16)
//             over the first half of S_c; W += P_c . R_c (tcgen05.mma, A = P_c from tensor memory,
//             M 128, N = MJ, fp32).  One thread issues the MMAs and the copies of the operator
//             pairs (R of 128 tokens, R^T of both chunks, laid out as K-major operands in 128-byte
//             swizzle by argus_jl_operator_fragments); the first Yv blocks stream in meanwhile.
//   O phase   the W rows, scaled to a common max per (kv head, query), go to shared memory (hi + lo);
//             Yv blocks arrive by TMA and the warps add Yv^T . w with mma.sync.
//
// R is read from L2 once per CTA and round instead of once per block pair, the two large
// contractions run on the 5th-generation tensor cores, and their A operands never leave tensor
// memory.  CTAs take equal contiguous ranges of all (batch, kv_head) blocks; a range is processed
// in rounds of at most 128 / (queries per kv head) blocks; a range that spans heads yields one
// partial per head and the last CTA to finish a head merges its partials.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace argus {
namespace jla {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kD = 128;      // largest head_dim (64 or 128); strides of the partial outputs
constexpr int kMJ = 128;     // largest rows per archived block (64 or 128)
constexpr int kRows = 128;   // (block, query) rows per round = tensor-memory lanes
constexpr int kChunk = 64;   // operator tokens per softmax step
constexpr int kPairTok = 2 * kChunk;  // operator tokens per score MMA group and operator copy
constexpr int kCols = 8;     // query columns of the CUDA-core MMAs (queries per kv head <= 8)
constexpr int kSlots = 4;    // 32 KB shared-memory slots
constexpr uint32_t kSlotBytes = (uint32_t)kMJ * kD * 2;          // room for one Yk / Yv block
constexpr long long kWaitTries = 1ll << 21;  // x kWaitHintNs: about two seconds
constexpr uint32_t kWaitHintNs = 1000;
constexpr float kNoMax = -1.0e30f;
constexpr float kSlack = 8.0f;  // a row's reference max is raised only when a score passes it by 2^8
// tensor memory: four S / P buffers (64 columns each, filled in pairs; P, fp16, overwrites the
// first 32 columns of its S), W (128 fp32 columns), U^T hi and lo (64 columns each: two fp16 per
// column)
constexpr int kSBufs = 4;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemW = kSBufs * kChunk;        // 256
constexpr uint32_t kTmemUhi = kTmemW + kMJ;         // 384
constexpr uint32_t kTmemUlo = kTmemUhi + kMJ / 2;   // 448
static_assert(kTmemUlo + kMJ / 2 <= kTmemCols, "tensor memory");

__device__ int g_status = 0;

struct Params {
    CUtensorMap tmk;    // Yk as [B*Hkv][n_blocks][MJ][D], box 64 x MJ, 128-byte swizzle
    CUtensorMap tmv;    // Yv, same
    const unsigned char* rop;   // R pairs: [N/128][128 x MJ fp16], B operand of S (N = tokens, K = MJ)
    const unsigned char* rtop;  // R^T chunks: [N/64][64 x MJ fp16], B operand of W (N = MJ, K = tokens)
    const __half* q;    // [B, Hkv*G, qlen, D]
    __half* out;
    float* lse;
    float* block_lse;   // optional [B*Hkv][n_blocks][8]: natural-log LSE of each block's scores
    float* part_o;      // [B*Hkv][S][8][D]  (S: partial slots per (b, h))
    float* part_lse;    // [B*Hkv][S][8]
    int* counters;      // [B*Hkv]
    int B, Hkv, G, qlen, n_blocks, N, S;
    float scale_log2;
};

// Shared memory (offsets from a 1024-byte aligned base)
constexpr uint32_t kOffU = 0;                                   // U^T staging hi | lo (64 KB) = slots 4, 5
constexpr uint32_t kOffSlot = 65536;                            // slots 0 .. 3 (32 KB each)
constexpr uint32_t kOffRow = kOffSlot + kSlots * kSlotBytes;    // mrow, lrow, frow [128] fp32
constexpr uint32_t kOffSeg = kOffRow + 3 * kRows * 4;           // segM, segL, segA [128] fp32
constexpr uint32_t kOffOpen = kOffSeg + 3 * kRows * 4;          // openM, openL [8] fp32
constexpr uint32_t kOffBar = kOffOpen + 2 * kCols * 4;          // mbarriers
// slot full (6), operator pair full / empty (2 + 2), S full (4), P full (4), W done (2)
constexpr int kBarFull = 0, kBarRF = 6, kBarRE = 8, kBarS = 10, kBarP = 14, kBarW = 18, kNumBars = 20;
constexpr uint32_t kOffCnt = kOffBar + kNumBars * 8;            // per-slot release counters [6]
constexpr uint32_t kOffMisc = kOffCnt + 8 * 4;                  // tensor-memory base, last flag, chunk counts
constexpr size_t kSmemBytes = 1024 + kOffMisc + 16;
static_assert(kSmemBytes <= 232448, "shared memory");
// a CTA allocates all 512 tensor-memory columns, so no second CTA may share its SM
static_assert(kSmemBytes > 232448 / 2, "one CTA per SM");

// Slot roles.  U phase: Yk block i in slot i % 4, U^T staged in slots 4-5.  SW phase: operator pair
// k in slots 2 (k % 2) and 2 (k % 2) + 1 while the first two Yv blocks come into slots 4 and 5.
// O phase: W' hi | lo in slots 0-1, Yv block i in slot oslot(i % 4) (4, 5, 2, 3).
__host__ __device__ constexpr uint32_t oslot(int k) { return k < 2 ? 4u + (uint32_t)k : (uint32_t)k; }
constexpr int kNumSlots = 6;

__device__ __forceinline__ uint32_t su32(const void* p) { return smem_u32(p); }
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
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
__device__ __forceinline__ void split_hl(float v, __half& hi, __half& lo) {
    hi = __float2half_rn(v);
    lo = __float2half_rn(v - __half2float(hi));
}
// two fp32 -> fp16x2 (hi) and the fp16x2 of their remainders (lo)
__device__ __forceinline__ void split_hl2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 f = __half22float2(h);
    const __half2 l = __floats2half2_rn(a - f.x, b - f.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
// Bounded wait: each try_wait suspends the thread (up to kWaitHintNs) until the phase completes, so
// waiting warps leave the issue slots to the warps that share their scheduler.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t phase) {
    for (long long i = 0; i < kWaitTries; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(bar), "r"(phase), "n"(kWaitHintNs)
            : "memory");
        if (ok) return true;
    }
    return false;
}
// the same wait, decided for the whole warp (tensor-memory accesses that follow are warp-collective)
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t phase) {
    return __all_sync(0xffffffffu, mbar_wait(bar, phase));
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
        : "memory");
}

// Copies block j of (b, h) into `dst` (D / 64 swizzled 64-column halves of MJ rows) and arms `bar`.
template <int D, int MJ>
__device__ __forceinline__ void issue_block(const CUtensorMap* map, int64_t bh, int j, uint32_t dst, uint32_t bar) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(bar, (uint32_t)MJ * D * 2);
    tma_load_4d(dst, map, 0, 0, j, (int)bh, bar);
    if (D > 64) tma_load_4d(dst + MJ * 128, map, 64, 0, j, (int)bh, bar);
}
// bytes of R^T_c (64 operator tokens x MJ rows) and of an R pair (128 tokens x MJ rows)
template <int MJ>
__host__ __device__ constexpr uint32_t op_chunk_bytes() { return (uint32_t)kChunk * MJ * 2; }
template <int MJ>
__host__ __device__ constexpr uint32_t op_pair_bytes() { return (uint32_t)kPairTok * MJ * 2; }
// Copies operator pair k (R of chunks 2k, 2k+1, then R^T of both) into `dst` and arms `bar`.
template <int MJ>
__device__ __forceinline__ void issue_op_pair(const Params& p, int k, uint32_t dst, uint32_t bar) {
    constexpr uint32_t RB = op_pair_bytes<MJ>(), TB = 2 * op_chunk_bytes<MJ>();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(bar, RB + TB);
    bulk_g2s(dst, p.rop + (size_t)k * RB, RB, bar);
    bulk_g2s(dst + RB, p.rtop + (size_t)k * TB, TB, bar);
}

// Shared-memory address of element (row r, column c) of a swizzled [MJ][D] Y block.
template <int MJ>
__device__ __forceinline__ uint32_t swz(uint32_t base, int r, int c) {
    return base + (uint32_t)((c >> 6) * (MJ * 128) + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + (c & 7) * 2);
}
// K-major operand in 128-byte swizzle (the layout a TMA copy with SWIZZLE_128B writes): K in blocks of
// 64 fp16, each block `rows` x 128 bytes, 16-byte chunk c of row r at chunk c ^ (r % 8), 8-row groups
// 1024 bytes apart.  Byte offset of element (row, k) of a tile with `rows` rows.
__host__ __device__ __forceinline__ uint32_t sw128(int row, int k, int rows) {
    return (uint32_t)((k >> 6) * rows * 128 + row * 128 + ((((k & 63) >> 3) ^ (row & 7)) << 4) + (k & 7) * 2);
}
// Row-major [row][128] fp16 staging (U^T, W'): 256-byte rows, 16-byte chunk c of row r at c ^ (r % 8).
__device__ __forceinline__ uint32_t rowsw(int r, int k) {
    return (uint32_t)(r * 256 + ((((k >> 3) ^ (r & 7))) << 4) + (k & 7) * 2);
}

// tcgen05 shared-memory matrix descriptor of a K-major 128-byte-swizzled operand (version 1, stride
// 1024 bytes between 8-row groups; a K step of 16 fp16 advances the start address by 32 bytes inside
// the 1024-byte aligned swizzle atom) and kind::f16 instruction descriptor (fp32 accumulator, fp16 A
// and B, both K-major).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)((1024u >> 4) & 0x3FFFu) << 32) |
           (1ull << 46) | (2ull << 61);
}
__host__ __device__ constexpr uint32_t idesc(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void umma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(id), "r"(acc));
}
// the same with A (M 128 x K 16, two fp16 per column) in tensor memory
__device__ __forceinline__ void umma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
        "r"(a), "l"(b), "r"(id), "r"(acc));
}
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
#define JLA_TMEM_LD32(addr, v)                                                                                   \
    asm volatile(                                                                                                \
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"         \
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                               \
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),         \
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),  \
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]),             \
          "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),             \
          "=r"(v[30]), "=r"(v[31])                                                                               \
        : "r"(addr))
#define JLA_TMEM_ST32(addr, v)                                                                                   \
    asm volatile(                                                                                                \
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"  \
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(addr),                         \
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),      \
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),          \
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),         \
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])                       \
        : "memory")
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <int D, int MJ>
__global__ void __launch_bounds__(kThreads, 1) jl_attn_tc_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = su32(sm);
    float* mrow = reinterpret_cast<float*>(sm + kOffRow);
    float* lrow = mrow + kRows;
    float* frow = lrow + kRows;
    float* segM = reinterpret_cast<float*>(sm + kOffSeg);
    float* segL = segM + kRows;
    float* segA = segL + kRows;
    float* openM = reinterpret_cast<float*>(sm + kOffOpen);
    float* openL = openM + kCols;
    int* cnt = reinterpret_cast<int*>(sm + kOffCnt);              // slot release counters
    uint32_t* misc = reinterpret_cast<uint32_t*>(sm + kOffMisc);  // [0] tensor-memory base, [1] last flag, [2] [3] chunk counts
    auto bar = [&](int i) { return sbase + kOffBar + 8u * (uint32_t)i; };
    auto slot = [&](uint32_t s) { return s < 4 ? sbase + kOffSlot + s * kSlotBytes : sbase + kOffU + (s - 4) * kSlotBytes; };
    const uint32_t uhi = slot(4), ulo = slot(5);  // U^T staging
    const uint32_t whi = slot(0), wlo = slot(1);  // W' (O phase)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int NQ = p.G * p.qlen;
    const int bpr = kRows / NQ;  // blocks per round
    const int nchunks = p.N / kChunk;
    const int npairs = nchunks / 2;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(misc)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        for (int i = 0; i < kNumBars; ++i) mbar_init(bar(i), (i >= kBarP && i < kBarW) ? 4u : 1u);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (tid < kCols) { openM[tid] = kNoMax; openL[tid] = 0.f; }
    if (tid < kNumSlots) cnt[tid] = 0;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = misc[0];
    const uint32_t trow = tmem + ((uint32_t)(32 * (warp & 3)) << 16);  // this warp's lane quarter

    // Equal contiguous ranges of all (b, h) blocks: block x goes to CTA floor(x C / T).
    const int64_t T = (int64_t)p.B * p.Hkv * p.n_blocks, C = gridDim.x, c = blockIdx.x;
    const int64_t x_begin = (c * T + C - 1) / C, x_end = ((c + 1) * T + C - 1) / C;

    // Slot loads in flight, kept alike by every thread: pend bit s = a copy into slot s not yet seen
    // complete, whose completion has parity (ph >> s) & 1.
    uint32_t ph = 0, pend = 0;
    bool ok = true;
    int64_t gchunk = 0;    // operator chunks of earlier rounds (phases of the S, P, W barriers)
    int64_t gpair = 0;     // operator pairs of earlier rounds (phases of the pair barriers)
    int64_t cur_bh = -1;   // the (b, h) whose partial output the o accumulators hold
    float oacc[4] = {0.f, 0.f, 0.f, 0.f};  // dims 16*warp + g (+8), query columns 2t, 2t+1

    // A warp done with slot s: the last of the eight to get here copies block x of `map` into it.
    auto release = [&](int s, bool refill, const CUtensorMap* map, int64_t x) {
        if (!refill) return;
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            if (atomicAdd(&cnt[s], 1) == kWarps - 1) {
                cnt[s] = 0;
                issue_block<D, MJ>(map, x / p.n_blocks, (int)(x % p.n_blocks), slot((uint32_t)s), bar(kBarFull + s));
            }
        }
        pend |= 1u << s;
    };
    // waits for the copy into slot s (decided for the whole warp)
    auto arrive_slot = [&](int s) {
        const bool r = mbar_wait_warp(bar(kBarFull + s), (ph >> s) & 1u);
        if (r) {
            ph ^= 1u << s;
            pend &= ~(1u << s);
        }
        return r;
    };

    // Writes the partial of (b, h) `bh` (openM / openL: its max and normalizer per query) and, in
    // the last CTA to finish it, merges all its partials into out / lse.
    auto flush = [&](int64_t bh) {
        const int64_t first_c = bh * p.n_blocks * C / T, last_c = ((bh + 1) * p.n_blocks - 1) * C / T;
        const int n_seg = (int)(last_c - first_c + 1), split = (int)(c - first_c);
        const int d0 = 16 * warp + g;
        float* po = p.part_o + ((bh * p.S + split) * kCols) * kD;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int n = 2 * t + k;
            if (n < NQ && d0 < D) {
                const float L = openL[n];
                po[n * kD + d0] = L > 0.f ? oacc[k] / L : 0.f;
                po[n * kD + d0 + 8] = L > 0.f ? oacc[2 + k] / L : 0.f;
                if (warp == 0 && g == 0)
                    p.part_lse[(bh * p.S + split) * kCols + n] = L > 0.f ? openM[n] + log2f(L) : -INFINITY;
            }
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const int prev = atomicAdd(&p.counters[bh], 1);
            misc[1] = prev == n_seg - 1;
            if (prev == n_seg - 1) p.counters[bh] = 0;
        }
        __syncthreads();
        if (misc[1]) {
            __threadfence();
            const int64_t b = bh / p.Hkv, h = bh - b * p.Hkv;
            for (int e = tid; e < NQ * D; e += kThreads) {
                const int n = e / D, d = e - n * D;
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
                const int64_t row = ((b * p.Hkv + h) * p.G + gi) * p.qlen + qi;
                p.out[row * D + d] = __float2half_rn(W > 0.f ? acc / W : 0.f);
                if (p.lse && d == 0) p.lse[row] = (W > 0.f) ? (M + log2f(W)) * 0.69314718055994530942f : -INFINITY;
            }
        }
        __syncthreads();
    };

    for (int64_t xr = x_begin; xr < x_end && ok; xr += bpr) {
        const int nb = (int)((x_end - xr) < bpr ? (x_end - xr) : bpr);
        const int rows = nb * NQ;
        // ================================================================ U phase
        for (int i = 0; i < nb && i < 4; ++i) {
            const int64_t x = xr + i;
            if (tid == 0) issue_block<D, MJ>(&p.tmk, x / p.n_blocks, (int)(x % p.n_blocks), slot(i), bar(kBarFull + i));
            pend |= 1u << i;
        }
        bool wok = true;
        {
            int64_t qbh = -1;
            uint32_t qa[D / 16][2];
            for (int i = 0; i < nb; ++i) {
                const int s = i % 4;
                wok = arrive_slot(s);
                if (!wok) break;
                const int64_t x = xr + i, bh = x / p.n_blocks;
                if (bh != qbh) {  // query fragments of this (b, h): column n = query n
                    qbh = bh;
                    const int64_t b = bh / p.Hkv, h = bh - b * p.Hkv;
                    const __half* qb = p.q + ((b * p.Hkv + h) * p.G) * p.qlen * D;
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk) {
                        const int d = 16 * kk + 2 * t;
                        qa[kk][0] = g < NQ ? *reinterpret_cast<const uint32_t*>(qb + (int64_t)g * D + d) : 0u;
                        qa[kk][1] = g < NQ ? *reinterpret_cast<const uint32_t*>(qb + (int64_t)g * D + d + 8) : 0u;
                    }
                }
                // u = Yk . q^T for block rows 16*warp .. +15 -> U^T rows i*NQ + n (warps past the
                // block's MJ rows only pass the slot on)
                const bool urows = 16 * warp < MJ;
                float u[4] = {0.f, 0.f, 0.f, 0.f}, u2[4] = {0.f, 0.f, 0.f, 0.f};
                const int row = 16 * warp + (lane & 7) + 8 * ((lane >> 3) & 1), colo = 8 * (lane >> 4);
                if (urows) {
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk) {
                        uint32_t a[4];
                        ldsm_x4(swz<MJ>(slot((uint32_t)s), row, 16 * kk + colo), a);
                        mma16816((kk & 1) ? u2 : u, a, qa[kk][0], qa[kk][1]);
                    }
                }
                release(s, i + 4 < nb, &p.tmk, x + 4);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int mj = 16 * warp + g + 8 * (k >> 1), n = 2 * t + (k & 1);
                    if (urows && n < NQ) {
                        __half hi, lo;
                        split_hl(u[k] + u2[k], hi, lo);
                        const uint32_t off = rowsw(i * NQ + n, mj);
                        asm volatile("st.shared.b16 [%0], %1;" ::"r"(uhi + off), "h"(__half_as_ushort(hi)) : "memory");
                        asm volatile("st.shared.b16 [%0], %1;" ::"r"(ulo + off), "h"(__half_as_ushort(lo)) : "memory");
                    }
                }
            }
        }
        ok = __syncthreads_and(wok) != 0;
        if (!ok) break;
        // U^T rows -> tensor memory (the A operands of the scores: hi and lo, one MMA each); rows
        // past this round's (block, query) pairs are zero, so their scores stay finite.  (Stacking
        // hi and lo of a round of at most 64 rows in the two lane halves, for one MMA per K step,
        // measured slower: its lo scores have to cross to the softmax warps through the shared
        // memory that otherwise takes the first Yv blocks during the scores.)
        if (warp < 4) {
            const int r = 32 * warp + lane;
#pragma unroll
            for (int hl = 0; hl < 2; ++hl) {
                const int src = r;
                const uint32_t sbase_u = hl ? ulo : uhi;
#pragma unroll
                for (int h2 = 0; h2 < MJ / 64; ++h2) {
                    uint32_t v[32];
#pragma unroll
                    for (int kc = 0; kc < 8; ++kc) {
                        uint4 x = make_uint4(0u, 0u, 0u, 0u);
                        if (src < rows)
                            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                                         : "=r"(x.x), "=r"(x.y), "=r"(x.z), "=r"(x.w)
                                         : "r"(sbase_u + rowsw(src, 64 * h2 + 8 * kc)));
                        v[4 * kc] = x.x; v[4 * kc + 1] = x.y; v[4 * kc + 2] = x.z; v[4 * kc + 3] = x.w;
                    }
                    JLA_TMEM_ST32(trow + (hl ? kTmemUlo : kTmemUhi) + 32 * h2, v);
                }
            }
            tmem_wait_st();
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();

        // ================================================================ SW phase
        // the first two Yv blocks come in while the scores run (slots 4, 5: the staging is done)
        for (int i = 0; i < nb && i < 2; ++i) {
            const int64_t x = xr + i;
            const uint32_t sl = oslot(i);
            if (tid == 0) issue_block<D, MJ>(&p.tmv, x / p.n_blocks, (int)(x % p.n_blocks), slot(sl), bar(kBarFull + (int)sl));
            pend |= 1u << sl;
        }
        // Warps 0-3 run the softmax of the lane quarters that hold this round's rows (the others
        // sit out); warp 6 issues the MMAs and warp 7 copies the operator pairs.
        const int nact = rows >= 96 ? 4 : (rows + 31) / 32;
        if (warp == 7) {
            if (lane == 0) {  // copies the operator pairs: pair k+2 into the slots of pair k once its Ws are done
                int loaded = 0;
                auto load = [&](int k) {
                    const int e = (int)((gpair + k) & 1);
                    issue_op_pair<MJ>(p, k, slot(2u * (uint32_t)e), bar(kBarRF + e));
                    loaded = k + 1;
                };
                for (int k = 0; k < 2 && k < npairs; ++k) load(k);
                for (int k = 0; k + 2 < npairs; ++k) {
                    const int64_t gp = gpair + k;
                    wok = mbar_wait(bar(kBarRE + (int)(gp & 1)), (uint32_t)((gp >> 1) & 1));
                    if (!wok) break;
                    load(k + 2);
                }
                misc[3] = (uint32_t)loaded;
            }
            __syncwarp();
        } else if (warp == 6) {
            if (lane == 0) {  // issues the MMAs
                tc_fence_after();
                const uint32_t id_s = idesc(kRows, kPairTok), id_w = idesc(kRows, MJ);
                int last_bar = -1;
                uint32_t last_par = 0;
                int landed = 0;  // operator pairs seen arrived
                // S of chunks 2k, 2k+1 = U^T . R_pair^T into the adjacent S buffers gc % 4, +1 (gc even)
                auto s_mma = [&](int k) {
                    const int64_t gp = gpair + k, gc = gchunk + 2 * k;
                    if (!mbar_wait(bar(kBarRF + (int)(gp & 1)), (uint32_t)((gp >> 1) & 1))) return false;
                    landed = k + 1;
                    tc_fence_after();
                    const uint32_t d = tmem + (uint32_t)(gc % kSBufs) * kChunk, rsm = slot(2u * (uint32_t)(gp & 1));
#pragma unroll
                    for (int ks = 0; ks < MJ / 16; ++ks) {
                        const uint64_t bd = sdesc(rsm + (uint32_t)(ks >> 2) * (kPairTok * 128) + (uint32_t)(ks & 3) * 32);
                        umma_ts(d, tmem + kTmemUhi + 8 * ks, bd, id_s, ks > 0 ? 1u : 0u);
                        umma_ts(d, tmem + kTmemUlo + 8 * ks, bd, id_s, 1u);
                    }
                    umma_commit(bar(kBarS + (int)(gc % kSBufs)));
                    umma_commit(bar(kBarS + (int)((gc + 1) % kSBufs)));
                    last_bar = kBarS + (int)((gc + 1) % kSBufs);
                    last_par = (uint32_t)(((gc + 1) / kSBufs) & 1);
                    return true;
                };
                for (int k = 0; k < 2 && k < npairs && wok; ++k) wok = s_mma(k);
                // W_cc goes in as soon as P_cc is written; after the second W of pair k the S of
                // pair k+2 goes into the same two buffers (the MMAs run in issue order, so the
                // scores overwrite P_{2k}, P_{2k+1} after both W have read them)
                for (int cc = 0; cc < nchunks && wok; ++cc) {
                    const int64_t gc = gchunk + cc, gp = gpair + cc / 2;
                    wok = mbar_wait(bar(kBarP + (int)(gc % kSBufs)), (uint32_t)((gc / kSBufs) & 1));
                    if (!wok) break;
                    tc_fence_after();
                    // W += P_cc . R_cc  (A = P_cc in tensor memory; B = R^T_cc, K-major: rows MJ, K = tokens)
                    const uint32_t rtsm = slot(2u * (uint32_t)(gp & 1)) + op_pair_bytes<MJ>() +
                                          (uint32_t)(cc & 1) * op_chunk_bytes<MJ>();
                    const uint32_t pt = tmem + (uint32_t)(gc % kSBufs) * kChunk;
#pragma unroll
                    for (int ks = 0; ks < kChunk / 16; ++ks)
                        umma_ts(tmem + kTmemW, pt + 8 * ks, sdesc(rtsm + (uint32_t)ks * 32), id_w,
                                (cc > 0 || ks > 0) ? 1u : 0u);
                    umma_commit(bar(kBarW + (int)(gc & 1)));
                    last_bar = kBarW + (int)(gc & 1);
                    last_par = (uint32_t)((gc >> 1) & 1);
                    if (cc & 1) {
                        umma_commit(bar(kBarRE + (int)(gp & 1)));
                        if (cc / 2 + 2 < npairs) wok = s_mma(cc / 2 + 2);
                    }
                }
                if (!wok && last_bar >= 0) (void)mbar_wait(bar(last_bar), last_par);  // MMAs in flight finish
                misc[2] = (uint32_t)landed;
            }
            __syncwarp();
        } else if (warp < nact) {  // online softmax of row r
            const int r = 32 * warp + lane;
            float m = kNoMax, l = 0.f;
            for (int cc = 0; cc < nchunks; ++cc) {
                const int64_t gc = gchunk + cc;
                // S_cc complete; its pair was issued after W_{cc-4} and W_{cc-3}, so after the last
                // reader of the P this buffer held
                wok = mbar_wait_warp(bar(kBarS + (int)(gc % kSBufs)), (uint32_t)((gc / kSBufs) & 1));
                if (!wok) break;
                tc_fence_after();
                const uint32_t sb = trow + (uint32_t)(gc % kSBufs) * kChunk;
                uint32_t v[kChunk];
                JLA_TMEM_LD32(sb, v);
                JLA_TMEM_LD32(sb + 32, (v + 32));
                tmem_wait_ld();
                float cm = kNoMax;
#pragma unroll
                for (int j = 0; j < kChunk; ++j) {
                    const float x = __uint_as_float(v[j]) * p.scale_log2;
                    v[j] = __float_as_uint(x);
                    cm = fmaxf(cm, x);
                }
                const bool bump = cm > m + kSlack;
                const float mnew = bump ? cm : m;
                const float alpha = ex2(m - mnew);  // 0 on the first chunk (m = kNoMax)
                l *= alpha;
                m = mnew;
                uint32_t pp[kChunk / 2];
#pragma unroll
                for (int j = 0; j < kChunk / 2; ++j) {
                    const float e0 = ex2(__uint_as_float(v[2 * j]) - m), e1 = ex2(__uint_as_float(v[2 * j + 1]) - m);
                    l += e0 + e1;
                    const __half2 h = __floats2half2_rn(e0, e1);
                    pp[j] = *reinterpret_cast<const uint32_t*>(&h);
                }
                if (cc > 0 && __any_sync(0xffffffffu, bump)) {  // W_{cc-1} done, then rescaled to the new max
                    wok = mbar_wait_warp(bar(kBarW + (int)((gc - 1) & 1)), (uint32_t)(((gc - 1) >> 1) & 1));
                    if (!wok) break;
                    tc_fence_after();
#pragma unroll
                    for (int j0 = 0; j0 < MJ; j0 += 32) {
                        uint32_t w[32];
                        JLA_TMEM_LD32(trow + kTmemW + j0, w);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(__uint_as_float(w[j]) * alpha);
                        JLA_TMEM_ST32(trow + kTmemW + j0, w);
                    }
                }
                JLA_TMEM_ST32(sb, pp);  // P_cc (fp16) over the first 32 columns of its S
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(kBarP + (int)(gc % kSBufs)), warp == 0 ? 1u + 4u - (uint32_t)nact : 1u);
            }
            mrow[r] = m;
            lrow[r] = l;
        }
        ok = __syncthreads_and(wok) != 0;
        if (!ok && tid == 7 * 32) {  // operator copies still in flight land before the CTA goes on (bounded)
            for (int k = (int)misc[2]; k < (int)misc[3]; ++k) {
                const int64_t gp = gpair + k;
                (void)mbar_wait(bar(kBarRF + (int)(gp & 1)), (uint32_t)((gp >> 1) & 1));
            }
        }
        if (ok) {  // the last W (and with it every MMA of the round)
            const int64_t gl = gchunk + nchunks - 1;
            ok = __syncthreads_and(mbar_wait(bar(kBarW + (int)(gl & 1)), (uint32_t)((gl >> 1) & 1))) != 0;
        }
        gchunk += nchunks;
        gpair += npairs;
        if (!ok) break;
        tc_fence_after();
        // the operator slots are free again: slots 2, 3 take the third and fourth Yv blocks
        for (int i = 2; i < nb && i < 4; ++i) {
            const int64_t x = xr + i;
            const uint32_t sl = oslot(i);
            if (tid == 0) issue_block<D, MJ>(&p.tmv, x / p.n_blocks, (int)(x % p.n_blocks), slot(sl), bar(kBarFull + (int)sl));
            pend |= 1u << sl;
        }

        // ================================================================ O phase
        // per (segment = run of one (b, h)'s blocks, query), one warp each with its lanes over the
        // segment's blocks: the common max, the normalizer and the factor of each row; the first
        // segment continues the open head when it is the same (b, h)
        const int64_t bh0 = xr / p.n_blocks;
        const int nseg = (int)((xr + nb - 1) / p.n_blocks - bh0) + 1;
        const bool cont = bh0 == cur_bh;
        for (int sq = warp; sq < nseg * NQ; sq += kWarps) {
            const int s = sq / NQ, n = sq - s * NQ;
            const int64_t hb = (bh0 + s) * p.n_blocks;
            const int i0 = (int)(hb - xr > 0 ? hb - xr : 0);
            const int i1 = (int)(hb + p.n_blocks - xr < nb ? hb + p.n_blocks - xr : nb);
            float M = kNoMax, prevM = kNoMax, prevL = 0.f;
            for (int i = i0 + lane; i < i1; i += 32) M = fmaxf(M, mrow[i * NQ + n]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            if (s == 0 && cont) {
                prevM = openM[n];
                prevL = openL[n];
                M = fmaxf(M, prevM);
            }
            const float a = exp2f(prevM - M);
            float L = 0.f;
            for (int i = i0 + lane; i < i1; i += 32) {
                const float f = exp2f(mrow[i * NQ + n] - M);
                frow[i * NQ + n] = f;
                L += f * lrow[i * NQ + n];
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
            if (lane == 0) {
                segM[sq] = M;
                segL[sq] = a * prevL + L;
                segA[sq] = a;
            }
        }
        __syncthreads();
        {  // W rows, scaled, -> W' [row][MJ] fp16 hi | lo (16-byte chunks XOR-swizzled by row); warps
           // w and w + 4 share lane quarter w, each half of the columns
            const int r = 32 * (warp & 3) + lane;
            const bool live = r < rows;
            const float f = live ? frow[r] : 0.f;
            const int jb = (warp >> 2) * (MJ / 2);
#pragma unroll
            for (int j0 = jb; j0 < jb + MJ / 2; j0 += 32) {
                uint32_t w[32];
                JLA_TMEM_LD32(trow + kTmemW + j0, w);
                tmem_wait_ld();
                if (live) {
#pragma unroll
                    for (int kc = 0; kc < 4; ++kc) {
                        uint32_t h[4], lo[4];
#pragma unroll
                        for (int jj = 0; jj < 4; ++jj)
                            split_hl2(f * __uint_as_float(w[8 * kc + 2 * jj]), f * __uint_as_float(w[8 * kc + 2 * jj + 1]),
                                      h[jj], lo[jj]);
                        const uint32_t off = rowsw(r, j0 + 8 * kc);
                        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(whi + off), "r"(h[0]), "r"(h[1]),
                                     "r"(h[2]), "r"(h[3])
                                     : "memory");
                        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(wlo + off), "r"(lo[0]), "r"(lo[1]),
                                     "r"(lo[2]), "r"(lo[3])
                                     : "memory");
                    }
                }
            }
            if (live && p.block_lse && warp < 4) {
                const int i = r / NQ, n = r - i * NQ;
                p.block_lse[(xr + i) * kCols + n] =
                    lrow[r] > 0.f ? (mrow[r] + log2f(lrow[r])) * 0.69314718055994530942f : -INFINITY;
            }
        }
        tc_fence_before();
        __syncthreads();
        wok = true;
        for (int i = 0; i < nb; ++i) {
            const int s = (int)oslot(i % 4);
            wok = arrive_slot(s);
            if (!wok) break;
            const int64_t x = xr + i, bh = x / p.n_blocks;
            if (bh != cur_bh || i == 0) {  // every warp reaches this block: a CTA-wide step
                const int seg = (int)(bh - bh0);
                if (bh != cur_bh) {
                    if (cur_bh >= 0) flush(cur_bh);
                    oacc[0] = oacc[1] = oacc[2] = oacc[3] = 0.f;
                    cur_bh = bh;
                } else {  // the open head goes on: rescale its running output to the new max
                    const float a0 = 2 * t < NQ ? segA[2 * t] : 0.f, a1 = 2 * t + 1 < NQ ? segA[2 * t + 1] : 0.f;
                    oacc[0] *= a0; oacc[2] *= a0; oacc[1] *= a1; oacc[3] *= a1;
                }
                __syncthreads();
                if (tid < NQ) {
                    openM[tid] = segM[seg * NQ + tid];
                    openL[tid] = segL[seg * NQ + tid];
                }
                __syncthreads();
            }
            // o += Yv^T . w' for dims 16*warp .. +15 (columns: the block's queries)
            if (16 * warp < D) {
                const int mr = (lane & 7) + 8 * (lane >> 4), dcol = 16 * warp + 8 * ((lane >> 3) & 1);
                const bool lq = g < NQ;
                const int r = i * NQ + g;
                float olo[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int kk = 0; kk < MJ / 16; ++kk) {
                    uint32_t wh0 = 0u, wh1 = 0u, wl0 = 0u, wl1 = 0u;
                    if (lq) {
                        const uint32_t o0 = rowsw(r, 16 * kk + 2 * t), o1 = rowsw(r, 16 * kk + 8 + 2 * t);
                        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(wh0) : "r"(whi + o0));
                        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(wh1) : "r"(whi + o1));
                        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(wl0) : "r"(wlo + o0));
                        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(wl1) : "r"(wlo + o1));
                    }
                    uint32_t a[4];
                    ldsm_x4_t(swz<MJ>(slot((uint32_t)s), 16 * kk + mr, dcol), a);
                    mma16816(oacc, a, wh0, wh1);
                    mma16816(olo, a, wl0, wl1);
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) oacc[k] += olo[k];
            }
            release(s, i + 4 < nb, &p.tmv, x + 4);
        }
        ok = __syncthreads_and(wok) != 0;
    }
    if (ok && cur_bh >= 0) flush(cur_bh);
    if (!ok) {
        if (tid == 0) atomicExch(&g_status, (int)ARGUS_ERR_TIMEOUT);
        // copies in flight land before the CTA exits (bounded)
        for (int s = 0; s < kNumSlots; ++s)
            if (pend >> s & 1) (void)mbar_wait(bar(kBarFull + s), (ph >> s) & 1u);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// R [N x MJ] fp16 row-major -> the operator pieces the kernel copies: for each 128-token pair R_pair
// (rows = tokens, K = MJ) and for each 64-token chunk c R^T_c (rows = MJ, K = the chunk's tokens),
// each a K-major operand in 128-byte swizzle, ready for a plain bulk copy into a 1024-byte aligned
// shared-memory slot.
__global__ void operator_chunks_kernel(const __half* __restrict__ R, int N, int MJ, __half* __restrict__ rop,
                                       __half* __restrict__ rtop) {
    const int64_t total = (int64_t)N * MJ;
    const uint32_t chunk_elems = (uint32_t)kChunk * MJ, pair_elems = (uint32_t)kPairTok * MJ;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int tok = (int)(i / MJ), m = (int)(i - (int64_t)tok * MJ);
        const int cidx = tok / kChunk, tl = tok - cidx * kChunk;
        const int pidx = tok / kPairTok, tp = tok - pidx * kPairTok;
        const __half v = R[i];
        rop[(int64_t)pidx * pair_elems + sw128(tp, m, kPairTok) / 2] = v;
        rtop[(int64_t)cidx * chunk_elems + sw128(m, tl, MJ) / 2] = v;
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
    if (n_tokens <= 0 || n_rows <= 0 || n_tokens % jla::kPairTok || n_rows % 64)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT,
                               "block tokens must be a positive multiple of 128 and rows of 64");
    if (!argus_aligned(r_frag, 16) || !argus_aligned(rt_frag, 16))
        return argus_set_error(ARGUS_ERR_MISALIGNED, "operator buffers must be 16-byte aligned");
    const int64_t total = (int64_t)n_tokens * n_rows;
    jla::operator_chunks_kernel<<<argus_grid_cap((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const __half*>(R), n_tokens, n_rows, static_cast<__half*>(r_frag), static_cast<__half*>(rt_frag));
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
    if ((s->head_dim != 64 && s->head_dim != 128) || (s->block_rows != 64 && s->block_rows != 128))
        return argus_set_error(ARGUS_ERR_UNSUPPORTED, "JL attention supports head_dim 64 or 128 and 64- or 128-row blocks");
    if (s->block_tokens <= 0 || s->block_tokens % jla::kPairTok)
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
    p.rop = static_cast<const unsigned char*>(r_frag);
    p.rtop = static_cast<const unsigned char*>(rt_frag);
    p.q = reinterpret_cast<const __half*>(q);
    p.out = reinterpret_cast<__half*>(out);
    p.lse = lse;
    p.block_lse = block_lse;
    const int64_t groups = (int64_t)s->batch * s->heads_kv;
    p.counters = static_cast<int*>(workspace);
    p.part_lse = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + ((groups * 4 + 255) & ~255LL));
    p.part_o = p.part_lse + groups * jl_slots(s) * jla::kCols;
    p.B = s->batch; p.Hkv = s->heads_kv; p.G = s->group; p.qlen = s->q_len;
    p.n_blocks = s->n_blocks; p.N = s->block_tokens; p.S = (int)jl_slots(s);
    p.scale_log2 = s->scale * 1.4426950408889634f;
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t blocks = groups * s->n_blocks;
    const int64_t ctas = jl_ctas(s);
    if (ctas > blocks || ctas > 0x7fffffff)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "more CTAs than blocks");
    const size_t smem = jla::kSmemBytes;
    auto kern = s->head_dim == 128 ? (s->block_rows == 128 ? jla::jl_attn_tc_kernel<128, 128> : jla::jl_attn_tc_kernel<128, 64>)
                                   : (s->block_rows == 128 ? jla::jl_attn_tc_kernel<64, 128> : jla::jl_attn_tc_kernel<64, 64>);
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
