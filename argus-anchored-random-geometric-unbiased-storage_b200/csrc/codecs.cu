// Quantize/pack and unpack/dequantize kernels for ARGUS's storage tiers, bit-exact against the
// reference's CPU arithmetic (argus_cache 0.1.8, core/quantization.py, core/triton_kernels.py CPU
// path, core/memory_manager.py:89-113, :944-1155).
//
// Arithmetic model: every torch op on fp16 data is an fp32 op rounded to fp16 (rh); divisions use
// the IEEE-rounded fp32 divide so rh(x / s) equals the reference's fp16 quotient.  The per-token
// reductions (amax, min, max) are order-free; mean|x| (1-bit scale, outlier threshold) follows
// ATen's cascade_sum order: 8 fp32 lanes, 4 interleaved accumulators, 4 cascade levels, lanes
// combined 0..7 in order, then / D in fp32.
//
// Row layouts.  A tensor is a set of groups of `group_rows` token rows of D values (a flat
// [n_rows][D] tensor is one group; a page of a record arena is B*H_kv groups, one per (b, h),
// `group_stride` bytes apart).  Packed tiers store `per` consecutive rows of a group in one
// D-byte packed row; scales/mins are one fp16 per row.  The kernels stage a tile of rows of one
// group in shared memory (decoded from any tier), reduce each row with 8 lanes, then emit 4 output
// bytes per thread, so one kernel both quantizes fp16 and re-quantizes a page from one tier into
// another (the fused demotion of the cascade).
#include <cuda_fp8.h>

#include "common.cuh"

namespace argus {

// Q_E4M3 is the true-e4m3 storage mode, a separately named non-parity tier (the reference's FP8 is
// the int8-with-wrap simulation, Q_FP8SIM): s = fp16(amax / 448), code = e4m3(x / s) from the IEEE
// fp32 quotient (round to nearest even, saturating at 448, NaN -> 0), value = fp16(e4m3(code) * s).
enum QuantMode { Q_INT8 = 0, Q_FP8SIM = 1, Q_INT4 = 2, Q_INT2 = 3, Q_SIGN1 = 4, Q_OUTLIER = 5, Q_FP16 = 6, Q_E4M3 = 7 };

__host__ __device__ constexpr int mode_per(int m) { return m == Q_INT4 ? 2 : (m == Q_INT2 ? 4 : (m == Q_SIGN1 ? 8 : 1)); }
__host__ __device__ constexpr int tier_mode(int tier) {
    return tier == ARGUS_TIER_FP16 ? Q_FP16
         : tier == ARGUS_TIER_FP8SIM ? Q_FP8SIM
         : tier == ARGUS_TIER_INT8 ? Q_INT8
         : tier == ARGUS_TIER_INT4 ? Q_INT4
         : tier == ARGUS_TIER_INT2 ? Q_INT2
         : tier == ARGUS_TIER_E4M3 ? Q_E4M3 : Q_SIGN1;
}

// Addressing of one operand: row t of group g sits at
//   payload + g*group_stride + ((row0 + t) / per) * row_bytes      (bytes)
//   scales/mins + g*sgroup_stride + row0 + t                       (fp16 elements)
struct Rows {
    unsigned char* payload;
    __half* scales;
    __half* mins;
    int64_t group_stride;
    int64_t sgroup_stride;
    int row0;
};

constexpr int kQuantThreads = 256;
constexpr int kRowLanes = 8;  // threads that cooperate on one row's statistics

// One lane's share of ATen's cascade_sum over a row of D = 8 * count fp32 values: lane l sums
// elements 8c + l.  row_sum splits the `count` 8-wide chunks over 4 interleaved accumulators
// (chunk c -> accumulator c % 4); multi_row_sum feeds each through a 4-level cascade with
// 2^level_power chunks per level step; leftover chunks go to accumulator 0; accumulators 1..3 are
// then added to accumulator 0 in order.
template <bool ABS>
__device__ __forceinline__ float cascade_lane_sum(const __half* row, int count, int lane) {
    constexpr int ILP = 4, LEVELS = 4;
    auto ld = [](__half h) { return ABS ? fabsf(__half2float(h)) : __half2float(h); };
    float acc[LEVELS][ILP];
#pragma unroll
    for (int a = 0; a < LEVELS; ++a)
#pragma unroll
        for (int k = 0; k < ILP; ++k) acc[a][k] = 0.0f;
    const int size_ilp = count / ILP;
    int cl2 = 1;
    if (size_ilp > 2) { cl2 = 32 - __clz(size_ilp - 1); }
    int level_power = cl2 / LEVELS;
    if (level_power < 4) level_power = 4;
    const int level_step = 1 << level_power;
    const int level_mask = level_step - 1;
    int i = 0;
    while (i + level_step <= size_ilp) {
        for (int j = 0; j < level_step; ++j, ++i)
#pragma unroll
            for (int k = 0; k < ILP; ++k) acc[0][k] = __fadd_rn(acc[0][k], ld(row[(i * ILP + k) * 8 + lane]));
#pragma unroll
        for (int j = 1; j < LEVELS; ++j) {
#pragma unroll
            for (int k = 0; k < ILP; ++k) { acc[j][k] = __fadd_rn(acc[j][k], acc[j - 1][k]); acc[j - 1][k] = 0.0f; }
            if ((i & (level_mask << (j * level_power))) != 0) break;
        }
    }
    for (; i < size_ilp; ++i)
#pragma unroll
        for (int k = 0; k < ILP; ++k) acc[0][k] = __fadd_rn(acc[0][k], ld(row[(i * ILP + k) * 8 + lane]));
#pragma unroll
    for (int j = 1; j < LEVELS; ++j)
#pragma unroll
        for (int k = 0; k < ILP; ++k) acc[0][k] = __fadd_rn(acc[0][k], acc[j][k]);
    for (int t = size_ilp * ILP; t < count; ++t) acc[0][0] = __fadd_rn(acc[0][0], ld(row[t * 8 + lane]));
#pragma unroll
    for (int k = 1; k < ILP; ++k) acc[0][0] = __fadd_rn(acc[0][0], acc[0][k]);
    return acc[0][0];
}

// Combines the 8 lane sums of a row group in lane order: ((0 + L0) + L1) + ... + L7.
__device__ __forceinline__ float cascade_combine(float mine) {
    float total = 0.0f;
#pragma unroll
    for (int l = 0; l < kRowLanes; ++l) {
        float v = __shfl_sync(0xffffffffu, mine, (threadIdx.x & 31 & ~7) + l);
        total = __fadd_rn(total, v);
    }
    return total;
}

// fl32(x / s) for fp16 values x and s, s finite and > 0: the quotient from the correctly rounded
// reciprocal r = RN(1/s) and one FMA correction (Markstein's final division step, P. Markstein,
// IBM J. Res. Dev. 34(1), 1990).  For fp16 operands no intermediate overflows or underflows fp32,
// and argus_selftest_fp16_quotients checks it against the IEEE-rounded divide for every such pair.
__device__ __forceinline__ float quot_rn(float x, float s, float r) {
    const float q0 = __fmul_rn(x, r);
    const float e = __fmaf_rn(-s, q0, x);
    return __fmaf_rn(e, r, q0);
}
// The per-row divisor of a quantizer: the reciprocal when the fast quotient applies (0 otherwise).
__device__ __forceinline__ float quot_recip(float s) {
    return (s > 0.0f && s <= 65504.0f) ? __frcp_rn(s) : 0.0f;
}
__device__ __forceinline__ float quot(float x, float s, float r) {
    return r != 0.0f ? quot_rn(x, s, r) : __fdiv_rn(x, s);
}

// NaN/Inf cleaned to +0 (isolate_outliers' cleanse step).
__device__ __forceinline__ __half clean_nan_inf(__half h) {
    unsigned short b = __half_as_ushort(h);
    return ((b & 0x7c00u) == 0x7c00u) ? __ushort_as_half(0) : h;
}

// ------------------------------------------------------------------------------ decoding
// Decodes 8 consecutive columns (c8*8 ..) of the `per` rows held by packed row `pr` of group g
// (rows pr*per .. relative to row0) into out[i][0..7] for i < per.  Exact reference dequantization.
template <int SRC>
__device__ __forceinline__ void decode8(const Rows& s, int64_t g, int pr, int c8, int D, __half (&out)[8][8]) {
    constexpr int per = mode_per(SRC);
    const int t0 = pr * per;  // first row of the packed row, relative to row0
    if constexpr (SRC == Q_FP16) {
        const unsigned char* rp = s.payload + g * s.group_stride + (int64_t)(s.row0 + t0) * D * 2;
        *reinterpret_cast<uint4*>(out[0]) = *reinterpret_cast<const uint4*>(rp + c8 * 16);
    } else {
        const unsigned char* rp = s.payload + g * s.group_stride + (int64_t)((s.row0 + t0) / per) * D;
        const uint2 raw = *reinterpret_cast<const uint2*>(rp + c8 * 8);
        const uint8_t* b = reinterpret_cast<const uint8_t*>(&raw);
        const __half* sp = s.scales + g * s.sgroup_stride + s.row0 + t0;
        if constexpr (SRC == Q_INT8 || SRC == Q_FP8SIM) {
            // code pairs to fp16 without conversions: the sign-flipped byte under the exponent of
            // 1024 reads as 1024 + q + 128, so subtracting 1152 leaves q exactly; then fp16(q * s)
            const __half2 s2 = __half2half2(sp[0]);
            const uint32_t w[2] = {raw.x ^ 0x80808080u, raw.y ^ 0x80808080u};
            const __half2 bias = __float2half2_rn(1152.0f);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t hv = __byte_perm(w[e >> 1], 0x64646464u, (e & 1) ? 0x5342 : 0x5140);
                const __half2 v = __hmul2_rn(__hsub2(*reinterpret_cast<const __half2*>(&hv), bias), s2);
                out[0][2 * e] = __low2half(v);
                out[0][2 * e + 1] = __high2half(v);
            }
        } else if constexpr (SRC == Q_E4M3) {
            // e4m3 pairs to fp16 (exact), then fp16(v * s)
            const __half2 s2 = __half2half2(sp[0]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const __nv_fp8x2_storage_t pr = (__nv_fp8x2_storage_t)(((e < 2) ? raw.x : raw.y) >> (16 * (e & 1)));
                const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(pr, __NV_E4M3);
                const __half2 v = __hmul2_rn(*reinterpret_cast<const __half2*>(&hr), s2);
                out[0][2 * e] = __low2half(v);
                out[0][2 * e + 1] = __high2half(v);
            }
        } else if constexpr (SRC == Q_INT4 || SRC == Q_INT2) {
            constexpr int BITS = 8 / per;
            constexpr uint32_t m = (1u << BITS) - 1u;
            const __half* mp = s.mins + g * s.sgroup_stride + s.row0 + t0;
            // columns 2e, 2e+1 as the low bytes of two halves; row i's codes shifted down, masked and
            // put under the exponent of 1024 read as 1024 + u, so subtracting 1024 leaves u exactly
            uint32_t pairs[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) pairs[e] = __byte_perm((e < 2) ? raw.x : raw.y, 0u, (e & 1) ? 0x4342 : 0x4140);
            const __half2 base = __float2half2_rn(1024.0f);
#pragma unroll
            for (int i = 0; i < per; ++i) {
                const __half2 s2 = __half2half2(sp[i]), m2 = __half2half2(mp[i]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const uint32_t hv = ((pairs[e] >> (BITS * i)) & (m | (m << 16))) | 0x64006400u;
                    const __half2 u = __hsub2(*reinterpret_cast<const __half2*>(&hv), base);
                    const __half2 v = __hadd2_rn(__hmul2_rn(u, s2), m2);
                    out[i][2 * e] = __low2half(v);
                    out[i][2 * e + 1] = __high2half(v);
                }
            }
        } else {  // 1-bit: exactly +s or -s
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const __half sv = sp[i], nv = __hneg(sv);
#pragma unroll
                for (int e = 0; e < 8; ++e) out[i][e] = ((b[e] >> i) & 1u) ? sv : nv;
            }
        }
    }
}

// ------------------------------------------------------------------------------ quantizer
// Stages rows [t0, t0 + rows) of group g (decoded from SRC), then quantizes them to MODE.
template <int MODE, int SRC>
__global__ void __launch_bounds__(kQuantThreads)
quant_kernel(Rows src, Rows dst, int64_t n_groups, int group_rows, int D, int tile_rows, float sigma,
             __half* __restrict__ outv, uint8_t* __restrict__ mask) {
    constexpr int per = mode_per(MODE);
    constexpr int sper = mode_per(SRC);
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int stride = D + 8;  // halfs; +16 B keeps 16 B alignment and staggers banks by row
    __half* tile = reinterpret_cast<__half*>(smem_raw);
    float* st_a = reinterpret_cast<float*>(smem_raw + (size_t)tile_rows * stride * sizeof(__half));
    float* st_b = st_a + tile_rows;
    float* st_r = st_b + tile_rows;  // reciprocal of the scale for the fast quotient (0: IEEE divide)

    const int tiles_per_group = (group_rows + tile_rows - 1) / tile_rows;
    const int64_t n_tiles = n_groups * tiles_per_group;
    const int c8n = D / 8;
    for (int64_t tix = blockIdx.x; tix < n_tiles; tix += gridDim.x) {
        const int64_t g = tix / tiles_per_group;
        const int t0 = (int)(tix - g * tiles_per_group) * tile_rows;
        const int rows = min(tile_rows, group_rows - t0);
        // 1. stage the tile, decoded to fp16
        const int prows = rows / sper;
        for (int w = threadIdx.x; w < prows * c8n; w += kQuantThreads) {
            const int pr = w / c8n, c8 = w - pr * c8n;
            __half v[8][8];
            decode8<SRC>(src, g, t0 / sper + pr, c8, D, v);
#pragma unroll
            for (int i = 0; i < sper; ++i) {
                if (MODE == Q_OUTLIER) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[i][e] = clean_nan_inf(v[i][e]);
                }
                *reinterpret_cast<uint4*>(tile + (pr * sper + i) * stride + c8 * 8) = *reinterpret_cast<uint4*>(v[i]);
            }
        }
        __syncthreads();
        // 2. per-row statistics, 8 lanes per row
        const int lane8 = threadIdx.x & 7;
        for (int rb = threadIdx.x >> 3; rb < ((rows + 3) & ~3); rb += kQuantThreads / kRowLanes) {
            const bool live = rb < rows;
            const __half* row = tile + (live ? rb : 0) * stride;
            float a = 0.0f, b = 0.0f;
            if (MODE == Q_INT8 || MODE == Q_FP8SIM || MODE == Q_E4M3) {
                bool nan = false;
                float m = 0.0f;
                for (int c = lane8; c < D; c += 8) {
                    float v = fabsf(h2f(row[c]));
                    nan |= (v != v);
                    m = fmaxf(m, v);
                }
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) {
                    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                    nan |= __shfl_xor_sync(0xffffffffu, (int)nan, o) != 0;
                }
                const float div = (MODE == Q_INT8) ? 127.0f : (MODE == Q_E4M3 ? 448.0f : 240.0f);
                a = nan ? __int_as_float(0x7fc00000) : rh(__fdiv_rn(m, div));  // s = fp16(amax / div)
            } else if (MODE == Q_INT4 || MODE == Q_INT2) {
                bool nan = false;
                float lo = INFINITY, hi = -INFINITY;
                for (int c = lane8; c < D; c += 8) {
                    float v = h2f(row[c]);
                    nan |= (v != v);
                    lo = fminf(lo, v);
                    hi = fmaxf(hi, v);
                }
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) {
                    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
                    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
                    nan |= __shfl_xor_sync(0xffffffffu, (int)nan, o) != 0;
                }
                const float qmax = (MODE == Q_INT4) ? 15.0f : 3.0f;
                if (nan) {
                    a = b = __int_as_float(0x7fc00000);
                } else {
                    a = rh(__fdiv_rn(rh(__fsub_rn(hi, lo)), qmax));  // s = fp16(fp16(max-min)/qmax)
                    b = lo;
                }
            } else if (MODE == Q_SIGN1 || MODE == Q_OUTLIER) {  // mean|x| in ATen order
                const float lane_sum = cascade_lane_sum<true>(row, D / 8, lane8);
                const float total = cascade_combine(lane_sum);
                const float mean = rh(__fdiv_rn(total, (float)D));  // fp16(sum / D)
                a = (MODE == Q_SIGN1) ? mean : rh(__fmul_rn(mean, sigma));  // outliers: fp16(mean * sigma)
            }
            if (live && lane8 == 0) {
                st_a[rb] = a;
                st_b[rb] = b;
                st_r[rb] = quot_recip(a);
            }
        }
        __syncthreads();
        // 3. outputs: 4 consecutive columns x `per` rows per thread
        const int quads = D / 4;
        const int prw = rows / per;
        for (int w = threadIdx.x; w < prw * quads; w += kQuantThreads) {
            const int pr = w / quads, cq = w - pr * quads;
            if (MODE == Q_FP16) {
                // plain fp16 store (a page decoded into an fp16 page)
                unsigned char* dp = dst.payload + g * dst.group_stride + (int64_t)(dst.row0 + t0 + pr) * D * 2;
                *reinterpret_cast<uint2*>(dp + cq * 8) = *reinterpret_cast<const uint2*>(tile + pr * stride + cq * 4);
                continue;
            }
            uint32_t word = 0;
#pragma unroll
            for (int i = 0; i < per; ++i) {
                const int r = pr * per + i;
                const __half* hp = tile + r * stride + cq * 4;
                const float a = st_a[r], b = st_b[r], ra = st_r[r];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float v = h2f(hp[e]);
                    uint32_t code;
                    if (MODE == Q_INT8 || MODE == Q_FP8SIM) {
                        const float lo = (MODE == Q_INT8) ? -128.0f : -240.0f;
                        const float hi = (MODE == Q_INT8) ? 127.0f : 240.0f;
                        code = w8(clamp_nan(round_even(rh(quot(v, a, ra))), lo, hi));
                        word |= code << (8 * e);
                    } else if (MODE == Q_E4M3) {
                        const float qv = __fdiv_rn(v, a);  // keeps the sign of -0
                        code = (qv != qv) ? 0u : (uint32_t)__nv_cvt_float_to_fp8(qv, __NV_SATFINITE, __NV_E4M3);
                        word |= code << (8 * e);
                    } else if (MODE == Q_INT4 || MODE == Q_INT2) {
                        const float qmax = (MODE == Q_INT4) ? 15.0f : 3.0f;
                        code = w8(clamp_nan(round_even(rh(quot(rh(__fsub_rn(v, b)), a, ra))), 0.0f, qmax));
                        word |= code << (8 * e + (MODE == Q_INT4 ? 4 : 2) * i);
                    } else if (MODE == Q_SIGN1) {
                        code = (v >= 0.0f) ? 1u : 0u;  // false for NaN, true for -0
                        word |= code << (8 * e + i);
                    } else {  // Q_OUTLIER
                        const bool m = fabsf(v) > a;
                        word |= (m ? 1u : 0u) << (8 * e);
                    }
                }
            }
            if (MODE == Q_OUTLIER) {
                // flat layout only: normal -> dst.payload (fp16), outliers -> outv, mask -> mask
                const int64_t base = (g * group_rows + t0 + pr) * (int64_t)D + cq * 4;
                *reinterpret_cast<uint32_t*>(mask + base) = word;
                const __half* hp = tile + pr * stride + cq * 4;
                __half nv[4], ov[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const bool m = (word >> (8 * e)) & 1u;
                    nv[e] = m ? __ushort_as_half(0) : hp[e];
                    ov[e] = m ? hp[e] : __ushort_as_half(0);
                }
                *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(dst.payload) + base) = *reinterpret_cast<uint2*>(nv);
                *reinterpret_cast<uint2*>(outv + base) = *reinterpret_cast<uint2*>(ov);
            } else {
                unsigned char* dp = dst.payload + g * dst.group_stride + (int64_t)((dst.row0 + t0) / per + pr) * D;
                *reinterpret_cast<uint32_t*>(dp + cq * 4) = word;
            }
        }
        // 4. per-row scales / mins
        if (MODE != Q_OUTLIER && MODE != Q_FP16) {
            for (int r = threadIdx.x; r < rows; r += kQuantThreads) {
                if (dst.scales) dst.scales[g * dst.sgroup_stride + dst.row0 + t0 + r] = f2h(st_a[r]);
                if (MODE == Q_INT4 || MODE == Q_INT2) dst.mins[g * dst.sgroup_stride + dst.row0 + t0 + r] = f2h(st_b[r]);
            }
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------ register-only packing from fp16
// The order-free tiers (INT8, FP8-sim: amax; INT4, INT2: min/max) packed straight from fp16 rows
// without a shared-memory tile: 8 lanes take one packed row (the `per` token rows that share an
// output byte row), each lane D/8 consecutive columns of every row; the row statistics are reduced
// across the 8 lanes with shuffles and each lane writes its D/8 output bytes.  Per-element
// arithmetic is the same as quant_kernel's.
template <int BYTES>
__device__ __forceinline__ void ld_bytes(const unsigned char* p, uint32_t (&r)[BYTES / 4]) {
    if constexpr (BYTES % 16 == 0) {
#pragma unroll
        for (int i = 0; i < BYTES / 16; ++i) {
            const uint4 v = __ldcs(reinterpret_cast<const uint4*>(p) + i);
            r[4 * i] = v.x; r[4 * i + 1] = v.y; r[4 * i + 2] = v.z; r[4 * i + 3] = v.w;
        }
    } else if constexpr (BYTES == 8) {
        const uint2 v = __ldcs(reinterpret_cast<const uint2*>(p));
        r[0] = v.x; r[1] = v.y;
    } else {
        r[0] = __ldcs(reinterpret_cast<const unsigned int*>(p));
    }
}
template <int BYTES>
__device__ __forceinline__ void st_bytes(unsigned char* p, const uint32_t* r) {
    if constexpr (BYTES % 16 == 0) {
#pragma unroll
        for (int i = 0; i < BYTES / 16; ++i)
            reinterpret_cast<uint4*>(p)[i] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
    } else if constexpr (BYTES == 8) {
        *reinterpret_cast<uint2*>(p) = make_uint2(r[0], r[1]);
    } else if constexpr (BYTES == 4) {
        *reinterpret_cast<uint32_t*>(p) = r[0];
    } else {
        *reinterpret_cast<uint16_t*>(p) = (uint16_t)r[0];
    }
}

template <int MODE, int D>
__global__ void __launch_bounds__(256) pack_rows_kernel(Rows src, Rows dst, int64_t n_groups, int group_rows) {
    constexpr int per = mode_per(MODE);
    constexpr int C = D / 8;                     // columns per lane
    constexpr int LW = (C * 2 + 3) / 4;          // u32 words of one row's columns
    constexpr int OW = (C + 3) / 4;              // u32 words of the lane's output bytes
    const int lane8 = threadIdx.x & 7;
    const int64_t prg = group_rows / per;        // packed rows per group
    const int64_t total = n_groups * prg;
    for (int64_t pr = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3; pr < total;
         pr += ((int64_t)gridDim.x * blockDim.x) >> 3) {
        const int64_t g = n_groups == 1 ? 0 : pr / prg;  // one group (flat tensors): no division
        const int prl = (int)(pr - g * prg);
        uint32_t raw[per][LW];
#pragma unroll
        for (int i = 0; i < per; ++i)
            ld_bytes<C * 2>(src.payload + g * src.group_stride + (int64_t)(src.row0 + prl * per + i) * D * 2 + lane8 * C * 2,
                            raw[i]);
        float sa[per], sb[per], sr[per];
#pragma unroll
        for (int i = 0; i < per; ++i) {
            bool nan = false;
            float m = 0.0f, lo = INFINITY, hi = -INFINITY;
            if constexpr (C % 2 == 0) {
                // column pairs in half2 lanes (exact: min, max and |x| do not round); the
                // NaN-propagating max marks rows holding a NaN
                const __half2* hv2 = reinterpret_cast<const __half2*>(raw[i]);
                if constexpr (MODE == Q_INT8 || MODE == Q_FP8SIM) {
                    __half2 a2 = __habs2(hv2[0]);
#pragma unroll
                    for (int k = 1; k < C / 2; ++k) a2 = __hmax2_nan(a2, __habs2(hv2[k]));
                    const float2 af = __half22float2(a2);
                    nan = (af.x != af.x) || (af.y != af.y);
                    m = fmaxf(af.x, af.y);
                } else {
                    __half2 l2 = hv2[0], u2 = hv2[0];
#pragma unroll
                    for (int k = 1; k < C / 2; ++k) {
                        l2 = __hmin2(l2, hv2[k]);
                        u2 = __hmax2_nan(u2, hv2[k]);
                    }
                    const float2 lf = __half22float2(l2), uf = __half22float2(u2);
                    nan = (uf.x != uf.x) || (uf.y != uf.y);
                    lo = fminf(lf.x, lf.y);
                    hi = fmaxf(uf.x, uf.y);
                }
            } else {
                const __half* hv = reinterpret_cast<const __half*>(raw[i]);
#pragma unroll
                for (int c = 0; c < C; ++c) {
                    const float v = h2f(hv[c]);
                    nan |= (v != v);
                    if (MODE == Q_INT8 || MODE == Q_FP8SIM) m = fmaxf(m, fabsf(v));
                    else { lo = fminf(lo, v); hi = fmaxf(hi, v); }
                }
            }
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                if (MODE == Q_INT8 || MODE == Q_FP8SIM) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                else {
                    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
                    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
                }
                nan |= __shfl_xor_sync(0xffffffffu, (int)nan, o) != 0;
            }
            if (MODE == Q_INT8 || MODE == Q_FP8SIM) {
                const float div = (MODE == Q_INT8) ? 127.0f : 240.0f;
                sa[i] = nan ? __int_as_float(0x7fc00000) : rh(__fdiv_rn(m, div));
                sb[i] = 0.0f;
            } else {
                const float qmax = (MODE == Q_INT4) ? 15.0f : 3.0f;
                sa[i] = nan ? __int_as_float(0x7fc00000) : rh(__fdiv_rn(rh(__fsub_rn(hi, lo)), qmax));
                sb[i] = nan ? __int_as_float(0x7fc00000) : lo;
            }
            sr[i] = quot_recip(sa[i]);
        }
        uint32_t out[OW];
#pragma unroll
        for (int w = 0; w < OW; ++w) out[w] = 0u;
        bool fast = true;
#pragma unroll
        for (int i = 0; i < per; ++i) fast &= sr[i] != 0.0f;  // finite positive scales (no NaN row)
        if (fast) {
            // Column pairs in half2 lanes.  q = fl32(x / s) by the reciprocal and one FMA correction;
            // fp16(q) + 1536 rounds q to an integer (RNE at spacing 1) and puts its two's-complement
            // low byte in the half's low byte (|q| < 512 here), clamped in that offset domain.
            constexpr float kLo = (MODE == Q_INT8) ? -128.0f : (MODE == Q_FP8SIM ? -240.0f : 0.0f);
            constexpr float kHi = (MODE == Q_INT8) ? 127.0f : (MODE == Q_FP8SIM ? 240.0f : (MODE == Q_INT4 ? 15.0f : 3.0f));
            const __half2 off = __float2half2_rn(1536.0f);
            const __half2 clo = __float2half2_rn(1536.0f + kLo), chi = __float2half2_rn(1536.0f + kHi);
#pragma unroll
            for (int k = 0; k < C / 2; ++k) {
                uint32_t pairw = 0u;  // bytes 0 and 2: the two columns' output bytes
#pragma unroll
                for (int i = 0; i < per; ++i) {
                    __half2 h = reinterpret_cast<const __half2*>(raw[i])[k];
                    if (MODE == Q_INT4 || MODE == Q_INT2) h = __hsub2(h, __float2half2_rn(sb[i]));  // fp16(x - mn)
                    const float2 x2 = __half22float2(h);
                    const float2 r2 = make_float2(sr[i], sr[i]);
                    const float2 q0 = __fmul2_rn(x2, r2);
                    const float2 e = __ffma2_rn(make_float2(-sa[i], -sa[i]), q0, x2);
                    const float2 q = __ffma2_rn(e, r2, q0);
                    const __half2 m = __hmin2(__hmax2(__hadd2(__float22half2_rn(q), off), clo), chi);
                    const uint32_t cw = *reinterpret_cast<const uint32_t*>(&m);  // offset codes
                    if (MODE == Q_INT8 || MODE == Q_FP8SIM) pairw = cw & 0x00FF00FFu;
                    else if (MODE == Q_INT4) pairw |= (cw & 0x000F000Fu) << (4 * i);
                    else pairw |= (cw & 0x00030003u) << (2 * i);
                }
                // columns 2k, 2k+1 -> bytes (2k) & 3, (2k+1) & 3 of out[k / 2]
                if (k & 1) out[k >> 1] |= __byte_perm(pairw, 0u, 0x2044) & 0xFFFF0000u;
                else       out[k >> 1] |= __byte_perm(pairw, 0u, 0x4420) & 0x0000FFFFu;
            }
        } else {
#pragma unroll
            for (int c = 0; c < C; ++c) {
                uint32_t byte = 0;
#pragma unroll
                for (int i = 0; i < per; ++i) {
                    const float v = h2f(reinterpret_cast<const __half*>(raw[i])[c]);
                    if (MODE == Q_INT8 || MODE == Q_FP8SIM) {
                        const float lo = (MODE == Q_INT8) ? -128.0f : -240.0f;
                        const float hi = (MODE == Q_INT8) ? 127.0f : 240.0f;
                        byte = w8(clamp_nan(round_even(rh(quot(v, sa[i], sr[i]))), lo, hi));
                    } else {
                        const float qmax = (MODE == Q_INT4) ? 15.0f : 3.0f;
                        byte |= w8(clamp_nan(round_even(rh(quot(rh(__fsub_rn(v, sb[i])), sa[i], sr[i]))), 0.0f, qmax))
                                << ((MODE == Q_INT4 ? 4 : 2) * i);
                    }
                }
                out[c >> 2] |= (byte & 0xffu) << (8 * (c & 3));
            }
        }
        st_bytes<C>(dst.payload + g * dst.group_stride + (int64_t)((dst.row0 + prl * per) / per) * D + lane8 * C, out);
        if (lane8 < per) {
            // lane i writes row i's scale (and min)
            float a = sa[0], b = sb[0];
#pragma unroll
            for (int i = 1; i < per; ++i)
                if (lane8 == i) { a = sa[i]; b = sb[i]; }
            const int64_t si = g * dst.sgroup_stride + dst.row0 + prl * per + lane8;
            if (dst.scales) dst.scales[si] = f2h(a);
            if (MODE == Q_INT4 || MODE == Q_INT2) dst.mins[si] = f2h(b);
        }
    }
}

// 1-bit packing from fp16 without a block-wide tile: 8 lanes take one packed row (8 token rows),
// each lane D/8 consecutive columns of every row.  A row's mean |x| must follow ATen's cascade
// order (lane l sums columns 8c + l), so each row passes through a small per-group shared-memory
// buffer where the 8 lanes read it strided; the sign bits come from the lane's own registers.
template <int D>
__global__ void __launch_bounds__(256, D >= 256 ? 2 : (D >= 128 ? 3 : 4)) pack_sign_kernel(Rows src, Rows dst, int64_t n_groups, int group_rows) {
    constexpr int C = D / 8;
    constexpr int LW = (C * 2 + 3) / 4;
    constexpr int OW = (C + 3) / 4;
    constexpr int RS = D + 8;  // halves per buffered row: 16-byte pad staggers the groups' banks
    __shared__ __align__(16) __half rowbuf[256 / 8][RS];
    const int lane8 = threadIdx.x & 7;
    __half* buf = rowbuf[threadIdx.x >> 3];
    const int64_t prg = group_rows / 8;
    const int64_t total = n_groups * prg;
    const int64_t stride = ((int64_t)gridDim.x * blockDim.x) >> 3;
    // every lane runs the same number of iterations (the shuffles and warp barriers need the whole warp)
    const int64_t first = ((int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31)) >> 3;
    const __half2 zero2 = __float2half2_rn(0.0f);
    for (int64_t base = first; base < total; base += stride) {
        const int64_t pr = base + ((threadIdx.x & 31) >> 3);
        const bool live = pr < total;
        const int64_t g = (live && n_groups > 1) ? pr / prg : 0;  // one group (flat tensors): no division
        const int prl = live ? (int)(pr - g * prg) : 0;
        const unsigned char* rows = src.payload + g * src.group_stride + (int64_t)(src.row0 + prl * 8) * D * 2 + lane8 * C * 2;
        // the 8 token rows stream through: row i+1 loads while row i is summed and its sign bits taken
        uint32_t cur[LW], nxt[LW];
        if (live) ld_bytes<C * 2>(rows, cur);
        else
#pragma unroll
            for (int w = 0; w < LW; ++w) cur[w] = 0u;
        uint32_t pairw[C / 2];  // bit i of bytes 0 / 2: x >= 0 for row i, columns 2k / 2k+1 (NaN: 0, -0: 1)
#pragma unroll
        for (int k = 0; k < C / 2; ++k) pairw[k] = 0u;
        float sa[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (i < 7) {
                if (live) ld_bytes<C * 2>(rows + (int64_t)(i + 1) * D * 2, nxt);
                else
#pragma unroll
                    for (int w = 0; w < LW; ++w) nxt[w] = 0u;
            }
#pragma unroll
            for (int w = 0; w < LW; ++w) reinterpret_cast<uint32_t*>(buf + lane8 * C)[w] = cur[w];
            __syncwarp();
            const float lane_sum = cascade_lane_sum<true>(buf, D / 8, lane8);
            sa[i] = rh(__fdiv_rn(cascade_combine(lane_sum), (float)D));  // fp16(sum |x| / D)
            __syncwarp();
#pragma unroll
            for (int k = 0; k < C / 2; ++k)
                pairw[k] |= __hge2_mask(reinterpret_cast<const __half2*>(cur)[k], zero2) & (0x00010001u << i);
            if (i < 7)
#pragma unroll
                for (int w = 0; w < LW; ++w) cur[w] = nxt[w];
        }
        uint32_t out[OW];
#pragma unroll
        for (int w = 0; w < OW; ++w) out[w] = 0u;
#pragma unroll
        for (int k = 0; k < C / 2; ++k) {
            if (k & 1) out[k >> 1] |= __byte_perm(pairw[k], 0u, 0x2044) & 0xFFFF0000u;
            else       out[k >> 1] |= __byte_perm(pairw[k], 0u, 0x4420) & 0x0000FFFFu;
        }
        if (live) {
            st_bytes<C>(dst.payload + g * dst.group_stride + (int64_t)((dst.row0 + prl * 8) / 8) * D + lane8 * C, out);
            float a = sa[0];
#pragma unroll
            for (int i = 1; i < 8; ++i)
                if (lane8 == i) a = sa[i];
            if (dst.scales) dst.scales[g * dst.sgroup_stride + dst.row0 + prl * 8 + lane8] = f2h(a);
        }
    }
}

// Outlier isolation with sigma <= 0: cleanse NaN/Inf only, no outliers.
__global__ void cleanse_kernel(const __half* __restrict__ x, int64_t n, __half* __restrict__ normal,
                               __half* __restrict__ outv, uint8_t* __restrict__ mask) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        normal[i] = clean_nan_inf(x[i]);
        outv[i] = __ushort_as_half(0);
        mask[i] = 0;
    }
}

// ------------------------------------------------------------------------- dequantizers
// Register-only decode of SRC rows into fp16 rows: one packed row x 8 columns per thread.
template <int SRC>
__global__ void dequant_kernel(Rows src, Rows dst, int64_t n_groups, int group_rows, int D) {
    constexpr int per = mode_per(SRC);
    const int c8n = D / 8;
    const int prg = group_rows / per;
    const int64_t per_group = (int64_t)prg * c8n;
    const int64_t items = n_groups * per_group;
    // one group whose items fit 32 bits and a power-of-two column count (the usual flat tensors):
    // the item index splits with a shift and a mask instead of 64-bit divisions
    const bool flat32 = n_groups == 1 && per_group < ((int64_t)1 << 31) && (c8n & (c8n - 1)) == 0;
    const int sh = __ffs(c8n) - 1;
    for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < items; w += (int64_t)gridDim.x * blockDim.x) {
        int64_t g;
        int pr, c8;
        if (flat32) {
            g = 0;
            pr = (int)((uint32_t)w >> sh);
            c8 = (int)((uint32_t)w & (uint32_t)(c8n - 1));
        } else {
            g = w / per_group;
            const int64_t rem = w - g * per_group;
            pr = (int)(rem / c8n);
            c8 = (int)(rem - (int64_t)pr * c8n);
        }
        __half v[8][8];
        decode8<SRC>(src, g, pr, c8, D, v);
#pragma unroll
        for (int i = 0; i < per; ++i) {
            unsigned char* dp = dst.payload + g * dst.group_stride + (int64_t)(dst.row0 + pr * per + i) * D * 2;
            *reinterpret_cast<uint4*>(dp + c8 * 16) = *reinterpret_cast<uint4*>(v[i]);
        }
    }
}

// Packs 4-bit codes (uint8 0..15) two tokens per byte.
__global__ void pack_int4_codes_kernel(const uint8_t* __restrict__ codes, int64_t n_prows, int D,
                                       uint8_t* __restrict__ packed) {
    const int64_t items = n_prows * D;
    for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < items; w += (int64_t)gridDim.x * blockDim.x) {
        const int64_t pr = w / D;
        const int d = (int)(w - pr * D);
        packed[w] = (uint8_t)(codes[(2 * pr) * D + d] | (codes[(2 * pr + 1) * D + d] << 4));
    }
}

// ---------------------------------------------------------------------------- launchers
Rows flat_rows(const void* payload, const uint16_t* scales, const uint16_t* mins) {
    Rows r;
    r.payload = const_cast<unsigned char*>(static_cast<const unsigned char*>(payload));
    r.scales = const_cast<__half*>(reinterpret_cast<const __half*>(scales));
    r.mins = const_cast<__half*>(reinterpret_cast<const __half*>(mins));
    r.group_stride = 0;
    r.sgroup_stride = 0;
    r.row0 = 0;
    return r;
}

int tile_rows_for(int D, int group_rows) {
    int tr = 8192 / (2 * D);
    tr = (tr / 8) * 8;
    if (tr < 8) tr = 8;
    if (tr > 256) tr = 256;
    if (group_rows < tr) tr = ((group_rows + 7) / 8) * 8;
    return tr;
}

template <int MODE, int D>
int launch_pack_rows(const Rows& src, const Rows& dst, int64_t n_groups, int group_rows, cudaStream_t st) {
    const int64_t threads = n_groups * (group_rows / mode_per(MODE)) * 8;
    pack_rows_kernel<MODE, D><<<argus_grid_cap((threads + 255) / 256), 256, 0, st>>>(src, dst, n_groups, group_rows);
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

// Whether pack_rows_kernel / pack_sign_kernel take a launch: a tier packed from fp16, a head dim
// they are built for, whole packed rows per group and aligned rows (their vector loads and stores).
bool pack_rows_ok(int mode, int src_mode, const Rows& src, const Rows& dst, int group_rows, int D) {
    if (src_mode != Q_FP16 || !(mode == Q_INT8 || mode == Q_FP8SIM || mode == Q_INT4 || mode == Q_INT2 || mode == Q_SIGN1))
        return false;
    if (D != 16 && D != 32 && D != 64 && D != 128 && D != 256) return false;
    const int per = mode_per(mode);
    if (group_rows % per || src.row0 % per || dst.row0 % per) return false;
    const int lb = (D / 8) * 2;  // bytes one lane loads per row
    const int la = lb >= 16 ? 16 : lb;
    const int ob = D / 8;        // bytes one lane stores per packed row
    const int oa = ob >= 16 ? 16 : ob;
    return argus_aligned(src.payload, la) && src.group_stride % la == 0 && argus_aligned(dst.payload, oa) &&
           dst.group_stride % oa == 0;
}

template <int D>
int launch_pack_sign(const Rows& src, const Rows& dst, int64_t n_groups, int group_rows, cudaStream_t st) {
    const int64_t threads = n_groups * (group_rows / 8) * 8;
    pack_sign_kernel<D><<<argus_grid_cap((threads + 255) / 256), 256, 0, st>>>(src, dst, n_groups, group_rows);
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

template <int MODE>
int pack_rows_dispatch(const Rows& src, const Rows& dst, int64_t n_groups, int group_rows, int D, cudaStream_t st) {
    if constexpr (MODE == Q_SIGN1) {
        switch (D) {
            case 16: return launch_pack_sign<16>(src, dst, n_groups, group_rows, st);
            case 32: return launch_pack_sign<32>(src, dst, n_groups, group_rows, st);
            case 64: return launch_pack_sign<64>(src, dst, n_groups, group_rows, st);
            case 128: return launch_pack_sign<128>(src, dst, n_groups, group_rows, st);
            default: return launch_pack_sign<256>(src, dst, n_groups, group_rows, st);
        }
    } else {
        switch (D) {
            case 16: return launch_pack_rows<MODE, 16>(src, dst, n_groups, group_rows, st);
            case 32: return launch_pack_rows<MODE, 32>(src, dst, n_groups, group_rows, st);
            case 64: return launch_pack_rows<MODE, 64>(src, dst, n_groups, group_rows, st);
            case 128: return launch_pack_rows<MODE, 128>(src, dst, n_groups, group_rows, st);
            default: return launch_pack_rows<MODE, 256>(src, dst, n_groups, group_rows, st);
        }
    }
}

template <int MODE, int SRC>
int launch_quant(const Rows& src, const Rows& dst, int64_t n_groups, int group_rows, int D, float sigma,
                 uint16_t* outv, uint8_t* mask, cudaStream_t st) {
    if (n_groups == 0 || group_rows == 0) return ARGUS_OK;
    if constexpr (SRC == Q_FP16 && (MODE == Q_INT8 || MODE == Q_FP8SIM || MODE == Q_INT4 || MODE == Q_INT2 || MODE == Q_SIGN1)) {
        if (pack_rows_ok(MODE, SRC, src, dst, group_rows, D))
            return pack_rows_dispatch<MODE>(src, dst, n_groups, group_rows, D, st);
    }
    const int tile_rows = tile_rows_for(D, group_rows);
    const size_t smem = (size_t)tile_rows * (D + 8) * sizeof(__half) + 3 * tile_rows * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(quant_kernel<MODE, SRC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return argus_set_cuda_error(e);
    }
    const int64_t tiles = n_groups * ((group_rows + tile_rows - 1) / tile_rows);
    quant_kernel<MODE, SRC><<<argus_grid_cap(tiles), kQuantThreads, smem, st>>>(
        src, dst, n_groups, group_rows, D, tile_rows, sigma, reinterpret_cast<__half*>(outv), mask);
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

// Runtime dispatch over (destination mode, source mode).
int quant_dispatch(int mode, int src_mode, const Rows& src, const Rows& dst, int64_t n_groups, int group_rows, int D,
                   cudaStream_t st) {
#define ARGUS_Q(M)                                                                                            \
    switch (src_mode) {                                                                                       \
        case Q_FP16: return launch_quant<M, Q_FP16>(src, dst, n_groups, group_rows, D, 0.f, nullptr, nullptr, st); \
        case Q_FP8SIM: return launch_quant<M, Q_FP8SIM>(src, dst, n_groups, group_rows, D, 0.f, nullptr, nullptr, st); \
        case Q_INT8: return launch_quant<M, Q_INT8>(src, dst, n_groups, group_rows, D, 0.f, nullptr, nullptr, st); \
        case Q_INT4: return launch_quant<M, Q_INT4>(src, dst, n_groups, group_rows, D, 0.f, nullptr, nullptr, st); \
        case Q_INT2: return launch_quant<M, Q_INT2>(src, dst, n_groups, group_rows, D, 0.f, nullptr, nullptr, st); \
        case Q_SIGN1: return launch_quant<M, Q_SIGN1>(src, dst, n_groups, group_rows, D, 0.f, nullptr, nullptr, st); \
        case Q_E4M3: return launch_quant<M, Q_E4M3>(src, dst, n_groups, group_rows, D, 0.f, nullptr, nullptr, st); \
        default: return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad source tier");                       \
    }
    switch (mode) {
        case Q_INT8: ARGUS_Q(Q_INT8)
        case Q_FP8SIM: ARGUS_Q(Q_FP8SIM)
        case Q_INT4: ARGUS_Q(Q_INT4)
        case Q_INT2: ARGUS_Q(Q_INT2)
        case Q_SIGN1: ARGUS_Q(Q_SIGN1)
        case Q_FP16: ARGUS_Q(Q_FP16)
        case Q_E4M3: ARGUS_Q(Q_E4M3)
        default: return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad destination tier");
    }
#undef ARGUS_Q
}

int dq_blocks(int64_t items) { return argus_grid_cap((items + 255) / 256); }

int dequant_dispatch(int src_mode, const Rows& src, const Rows& dst, int64_t n_groups, int group_rows, int D,
                     cudaStream_t st) {
    if (n_groups == 0 || group_rows == 0) return ARGUS_OK;
    const int64_t items = n_groups * (group_rows / mode_per(src_mode)) * (D / 8);
    switch (src_mode) {
        case Q_FP16: dequant_kernel<Q_FP16><<<dq_blocks(items), 256, 0, st>>>(src, dst, n_groups, group_rows, D); break;
        case Q_FP8SIM: dequant_kernel<Q_FP8SIM><<<dq_blocks(items), 256, 0, st>>>(src, dst, n_groups, group_rows, D); break;
        case Q_INT8: dequant_kernel<Q_INT8><<<dq_blocks(items), 256, 0, st>>>(src, dst, n_groups, group_rows, D); break;
        case Q_INT4: dequant_kernel<Q_INT4><<<dq_blocks(items), 256, 0, st>>>(src, dst, n_groups, group_rows, D); break;
        case Q_INT2: dequant_kernel<Q_INT2><<<dq_blocks(items), 256, 0, st>>>(src, dst, n_groups, group_rows, D); break;
        case Q_SIGN1: dequant_kernel<Q_SIGN1><<<dq_blocks(items), 256, 0, st>>>(src, dst, n_groups, group_rows, D); break;
        case Q_E4M3: dequant_kernel<Q_E4M3><<<dq_blocks(items), 256, 0, st>>>(src, dst, n_groups, group_rows, D); break;
        default: return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad source tier");
    }
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

// Rows of the K (which = 0) or V (which = 1) half of page `slot` of a record arena, as B*H groups.
Rows page_rows(const argus_kv_arena* a, int slot, int which, int D) {
    const int P = a->page_tokens;
    const int bits = a->tier == ARGUS_TIER_FP16 ? 16 : a->tier == ARGUS_TIER_INT4 ? 4 : a->tier == ARGUS_TIER_INT2 ? 2 : a->tier == ARGUS_TIER_1BIT ? 1 : 8;
    const int64_t pb = (int64_t)P * D * bits / 8;
    unsigned char* rec = const_cast<unsigned char*>(static_cast<const unsigned char*>(a->k)) + (int64_t)slot * a->record_bytes;
    Rows r;
    r.payload = rec + (which ? pb : 0);
    r.scales = reinterpret_cast<__half*>(rec + 2 * pb + (which ? 2 * P : 0));
    r.mins = reinterpret_cast<__half*>(rec + 2 * pb + 4 * P + (which ? 2 * P : 0));
    r.group_stride = a->bh_stride;
    r.sgroup_stride = a->bh_stride / 2;
    r.row0 = 0;
    return r;
}

int check_arena(const argus_kv_arena* a, int D) {
    if (!a || !a->k) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null arena");
    if (a->layout != ARGUS_LAYOUT_RECORD) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "page codecs need a record arena");
    if (a->tier < ARGUS_TIER_FP16 || a->tier > ARGUS_TIER_E4M3) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad tier");
    if (D % 8 || D <= 0) return argus_set_error(ARGUS_ERR_UNSUPPORTED, "head dim must be a multiple of 8");
    if (a->page_tokens <= 0 || a->page_tokens % 8) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "page size must be a multiple of 8");
    if (!argus_aligned(a->k, 16) || a->bh_stride % 16 || a->record_bytes % 16)
        return argus_set_error(ARGUS_ERR_MISALIGNED, "record arena must be 16-byte aligned");
    return ARGUS_OK;
}

// Every pair of a finite fp16 value x and a positive finite fp16 value s (the divisors quot_recip
// admits): counts where quot_rn differs from the IEEE-rounded divide (for x = -0 it returns +0,
// which rounds, clamps and casts to the same code).  One CTA per divisor.
__global__ void quotient_selftest_kernel(unsigned long long* mismatches) {
    const unsigned short sb = (unsigned short)(blockIdx.x + 1);  // 0x0001 .. 0x7BFF
    const float sv = __half2float(__ushort_as_half(sb));
    const float r = __frcp_rn(sv);
    unsigned long long bad = 0;
    for (int xi = threadIdx.x; xi < 0x10000; xi += blockDim.x) {
        const __half xh = __ushort_as_half((unsigned short)xi);
        if ((xi & 0x7c00) == 0x7c00) continue;  // inf / NaN
        const float xv = __half2float(xh);
        const float a = quot_rn(xv, sv, r), b = __fdiv_rn(xv, sv);
        bad += a != b;  // +0 and -0 compare equal: the sign of a zero quotient reaches no code
    }
    if (bad) atomicAdd(mismatches, bad);
}

}  // namespace argus

using namespace argus;

// ------------------------------------------------------------------------------ C ABI
namespace {

int check_rows(const void* a, const void* b, int64_t n_rows, int D, int per) {
    if (!a || !b) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    if (n_rows < 0 || D <= 0) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "negative size");
    if (D % 8 != 0) return argus_set_error(ARGUS_ERR_UNSUPPORTED, "head dim must be a multiple of 8");
    if (D > 8192) return argus_set_error(ARGUS_ERR_UNSUPPORTED, "head dim above 8192");
    if (n_rows % per != 0)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "sequence length not a multiple of the packing factor");
    return ARGUS_OK;
}

// Flat tensors: one group, or groups of 2^24 rows when the row count exceeds the int range.
constexpr int64_t kFlatGroup = (int64_t)1 << 24;

int flat_quant(int mode, const uint16_t* x, int64_t n_rows, int D, void* payload, uint16_t* s, uint16_t* mn,
               cudaStream_t st) {
    if (!argus_aligned(x, 16)) return argus_set_error(ARGUS_ERR_MISALIGNED, "input must be 16-byte aligned");
    if (!argus_aligned(payload, 4)) return argus_set_error(ARGUS_ERR_MISALIGNED, "output must be 4-byte aligned");
    if (n_rows == 0) return ARGUS_OK;
    if (n_rows > ((int64_t)1 << 30)) {
        if (n_rows % kFlatGroup) return argus_set_error(ARGUS_ERR_UNSUPPORTED, "above 2^30 rows: use a multiple of 2^24");
        Rows src = flat_rows(x, nullptr, nullptr), dst = flat_rows(payload, s, mn);
        src.group_stride = kFlatGroup * D * 2;
        dst.group_stride = kFlatGroup / mode_per(mode) * D;
        dst.sgroup_stride = kFlatGroup;
        return quant_dispatch(mode, Q_FP16, src, dst, n_rows / kFlatGroup, (int)kFlatGroup, D, st);
    }
    return quant_dispatch(mode, Q_FP16, flat_rows(x, nullptr, nullptr), flat_rows(payload, s, mn), 1, (int)n_rows, D, st);
}

int flat_dequant(int mode, const void* payload, const uint16_t* s, const uint16_t* mn, int64_t n_rows, int D,
                 uint16_t* out, cudaStream_t st) {
    if (!argus_aligned(payload, 8) || !argus_aligned(out, 16))
        return argus_set_error(ARGUS_ERR_MISALIGNED, "payload must be 8-byte and output 16-byte aligned");
    if (n_rows == 0) return ARGUS_OK;
    if (n_rows > ((int64_t)1 << 30)) {
        if (n_rows % kFlatGroup) return argus_set_error(ARGUS_ERR_UNSUPPORTED, "above 2^30 rows: use a multiple of 2^24");
        Rows src = flat_rows(payload, s, mn), dst = flat_rows(out, nullptr, nullptr);
        src.group_stride = kFlatGroup / mode_per(mode) * D;
        src.sgroup_stride = kFlatGroup;
        dst.group_stride = kFlatGroup * D * 2;
        return dequant_dispatch(mode, src, dst, n_rows / kFlatGroup, (int)kFlatGroup, D, st);
    }
    return dequant_dispatch(mode, flat_rows(payload, s, mn), flat_rows(out, nullptr, nullptr), 1, (int)n_rows, D, st);
}

}  // namespace

extern "C" {

int argus_selftest_fp16_quotients(unsigned long long* mismatches, argus_stream_t stream) {
    if (!mismatches) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    unsigned long long* d = nullptr;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&d), sizeof(*d), st);
    if (e == cudaSuccess) e = cudaMemsetAsync(d, 0, sizeof(*d), st);
    if (e != cudaSuccess) return argus_set_cuda_error(e);
    argus::quotient_selftest_kernel<<<0x7BFF, 256, 0, st>>>(d);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(mismatches, d, sizeof(*d), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaFreeAsync(d, st);
    if (e != cudaSuccess) return argus_set_cuda_error(e);
    return ARGUS_OK;
}

int argus_quant_int8(const uint16_t* x, int64_t n_rows, int D, int8_t* q, uint16_t* scales, argus_stream_t stream) {
    int rc = check_rows(x, q, n_rows, D, 1);
    if (rc || !scales) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales");
    return flat_quant(Q_INT8, x, n_rows, D, q, scales, nullptr, (cudaStream_t)stream);
}

int argus_quant_fp8sim(const uint16_t* x, int64_t n_rows, int D, int8_t* q, uint16_t* scales, argus_stream_t stream) {
    int rc = check_rows(x, q, n_rows, D, 1);
    if (rc || !scales) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales");
    return flat_quant(Q_FP8SIM, x, n_rows, D, q, scales, nullptr, (cudaStream_t)stream);
}

int argus_quant_int4(const uint16_t* x, int64_t n_rows, int D, uint8_t* packed, uint16_t* scales, uint16_t* mins,
                     argus_stream_t stream) {
    int rc = check_rows(x, packed, n_rows, D, 2);
    if (rc || !scales || !mins) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales/mins");
    return flat_quant(Q_INT4, x, n_rows, D, packed, scales, mins, (cudaStream_t)stream);
}

int argus_quant_int2(const uint16_t* x, int64_t n_rows, int D, uint8_t* packed, uint16_t* scales, uint16_t* mins,
                     argus_stream_t stream) {
    int rc = check_rows(x, packed, n_rows, D, 4);
    if (rc || !scales || !mins) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales/mins");
    return flat_quant(Q_INT2, x, n_rows, D, packed, scales, mins, (cudaStream_t)stream);
}

int argus_quant_1bit(const uint16_t* x, int64_t n_rows, int D, uint8_t* packed, uint16_t* scales,
                     argus_stream_t stream) {
    int rc = check_rows(x, packed, n_rows, D, 8);
    if (rc || !scales) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales");
    return flat_quant(Q_SIGN1, x, n_rows, D, packed, scales, nullptr, (cudaStream_t)stream);
}

int argus_pack_1bit_signs(const uint16_t* x, int64_t n_rows, int D, uint8_t* packed, argus_stream_t stream) {
    // the 1-bit quantizer with its scale output switched off (null sink)
    int rc = check_rows(x, packed, n_rows, D, 8);
    if (rc) return rc;
    return flat_quant(Q_SIGN1, x, n_rows, D, packed, nullptr, nullptr, (cudaStream_t)stream);
}

int argus_isolate_outliers(const uint16_t* x, int64_t n_rows, int D, float sigma, uint16_t* normal, uint16_t* outv,
                           uint8_t* mask, argus_stream_t stream) {
    int rc = check_rows(x, normal, n_rows, D, 1);
    if (rc || !outv || !mask) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null output");
    if (n_rows == 0) return ARGUS_OK;
    if (!(sigma > 0.0f)) {
        const int64_t n = n_rows * D;
        cleanse_kernel<<<dq_blocks(n), 256, 0, (cudaStream_t)stream>>>(
            reinterpret_cast<const __half*>(x), n, reinterpret_cast<__half*>(normal), reinterpret_cast<__half*>(outv),
            mask);
        ARGUS_CHECK_LAUNCH();
        return ARGUS_OK;
    }
    if (!argus_aligned(x, 16) || !argus_aligned(outv, 8) || !argus_aligned(normal, 8) || !argus_aligned(mask, 4))
        return argus_set_error(ARGUS_ERR_MISALIGNED, "outputs must be 8-byte aligned");
    if (n_rows > ((int64_t)1 << 30)) return argus_set_error(ARGUS_ERR_UNSUPPORTED, "above 2^30 rows");
    return launch_quant<Q_OUTLIER, Q_FP16>(flat_rows(x, nullptr, nullptr), flat_rows(normal, nullptr, nullptr), 1,
                                           (int)n_rows, D, sigma, outv, mask, (cudaStream_t)stream);
}

int argus_dequant_int8(const int8_t* q, const uint16_t* scales, int64_t n_rows, int D, uint16_t* out,
                       argus_stream_t stream) {
    int rc = check_rows(q, out, n_rows, D, 1);
    if (rc || !scales) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales");
    return flat_dequant(Q_INT8, q, scales, nullptr, n_rows, D, out, (cudaStream_t)stream);
}

int argus_dequant_fp8sim(const int8_t* q, const uint16_t* scales, int64_t n_rows, int D, uint16_t* out,
                         argus_stream_t stream) {
    return argus_dequant_int8(q, scales, n_rows, D, out, stream);
}

int argus_quant_e4m3(const uint16_t* x, int64_t n_rows, int D, uint8_t* q, uint16_t* scales, argus_stream_t stream) {
    int rc = check_rows(x, q, n_rows, D, 1);
    if (rc || !scales) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales");
    return flat_quant(Q_E4M3, x, n_rows, D, q, scales, nullptr, (cudaStream_t)stream);
}

int argus_dequant_e4m3(const uint8_t* q, const uint16_t* scales, int64_t n_rows, int D, uint16_t* out,
                       argus_stream_t stream) {
    int rc = check_rows(q, out, n_rows, D, 1);
    if (rc || !scales) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales");
    return flat_dequant(Q_E4M3, q, scales, nullptr, n_rows, D, out, (cudaStream_t)stream);
}

int argus_dequant_int4(const uint8_t* packed, const uint16_t* scales, const uint16_t* mins, int64_t n_rows, int D,
                       uint16_t* out, argus_stream_t stream) {
    int rc = check_rows(packed, out, n_rows, D, 2);
    if (rc || !scales || !mins) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales/mins");
    return flat_dequant(Q_INT4, packed, scales, mins, n_rows, D, out, (cudaStream_t)stream);
}

int argus_dequant_int2(const uint8_t* packed, const uint16_t* scales, const uint16_t* mins, int64_t n_rows, int D,
                       uint16_t* out, argus_stream_t stream) {
    int rc = check_rows(packed, out, n_rows, D, 4);
    if (rc || !scales || !mins) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales/mins");
    return flat_dequant(Q_INT2, packed, scales, mins, n_rows, D, out, (cudaStream_t)stream);
}

int argus_dequant_1bit(const uint8_t* packed, const uint16_t* scales, int64_t n_rows, int D, uint16_t* out,
                       argus_stream_t stream) {
    int rc = check_rows(packed, out, n_rows, D, 8);
    if (rc || !scales) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales");
    return flat_dequant(Q_SIGN1, packed, scales, nullptr, n_rows, D, out, (cudaStream_t)stream);
}

int argus_pack_int4_codes(const uint8_t* codes, int64_t n_rows, int D, uint8_t* packed, argus_stream_t stream) {
    int rc = check_rows(codes, packed, n_rows, D, 2);
    if (rc) return rc;
    if (n_rows == 0) return ARGUS_OK;
    const int64_t pr = n_rows / 2;
    pack_int4_codes_kernel<<<dq_blocks(pr * D), 256, 0, (cudaStream_t)stream>>>(codes, pr, D, packed);
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

// ------------------------------------------------------------------------- page codecs
int argus_page_quantize(const uint16_t* k, const uint16_t* v, int32_t n_bh, int D, const argus_kv_arena* dst,
                        int32_t dst_slot, argus_stream_t stream) {
    int rc = check_arena(dst, D);
    if (rc) return rc;
    if (!k || !v || n_bh <= 0 || dst_slot < 0) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad page arguments");
    if (!argus_aligned(k, 16) || !argus_aligned(v, 16)) return argus_set_error(ARGUS_ERR_MISALIGNED, "k/v alignment");
    const int P = dst->page_tokens;
    for (int which = 0; which < 2; ++which) {
        Rows src = flat_rows(which ? v : k, nullptr, nullptr);
        src.group_stride = (int64_t)P * D * 2;
        rc = quant_dispatch(tier_mode(dst->tier), Q_FP16, src, page_rows(dst, dst_slot, which, D), n_bh, P, D,
                            (cudaStream_t)stream);
        if (rc) return rc;
    }
    return ARGUS_OK;
}

int argus_page_requant(const argus_kv_arena* src, int32_t src_slot, const argus_kv_arena* dst, int32_t dst_slot,
                       int32_t n_bh, int D, argus_stream_t stream) {
    int rc = check_arena(src, D);
    if (!rc) rc = check_arena(dst, D);
    if (rc) return rc;
    if (src->page_tokens != dst->page_tokens) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "page sizes differ");
    if (n_bh <= 0 || src_slot < 0 || dst_slot < 0) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad page arguments");
    for (int which = 0; which < 2; ++which) {
        rc = quant_dispatch(tier_mode(dst->tier), tier_mode(src->tier), page_rows(src, src_slot, which, D),
                            page_rows(dst, dst_slot, which, D), n_bh, src->page_tokens, D, (cudaStream_t)stream);
        if (rc) return rc;
    }
    return ARGUS_OK;
}

int argus_page_dequantize(const argus_kv_arena* src, int32_t src_slot, int32_t n_bh, int D, uint16_t* k_out,
                          uint16_t* v_out, int64_t out_bh_stride, int64_t out_tok0, argus_stream_t stream) {
    int rc = check_arena(src, D);
    if (rc) return rc;
    if (!k_out || !v_out || n_bh <= 0 || src_slot < 0 || out_tok0 < 0 || out_tok0 > (1 << 30))
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad page arguments");
    if (!argus_aligned(k_out, 16) || !argus_aligned(v_out, 16) || (out_bh_stride * 2) % 16)
        return argus_set_error(ARGUS_ERR_MISALIGNED, "outputs must be 16-byte aligned");
    for (int which = 0; which < 2; ++which) {
        Rows dst = flat_rows(which ? v_out : k_out, nullptr, nullptr);
        dst.group_stride = out_bh_stride * 2;
        dst.row0 = (int)out_tok0;
        rc = dequant_dispatch(tier_mode(src->tier), page_rows(src, src_slot, which, D), dst, n_bh, src->page_tokens, D,
                              (cudaStream_t)stream);
        if (rc) return rc;
    }
    return ARGUS_OK;
}

}  // extern "C"
