// Quantize/pack and unpack/dequantize kernels for ARGUS's storage tiers, bit-exact against the
// reference's CPU arithmetic (argus_cache 0.1.8, core/quantization.py, core/triton_kernels.py CPU
// path, core/memory_manager.py:89-113).
//
// Arithmetic model: every torch op on fp16 data is an fp32 op rounded to fp16 (rh); divisions use
// the IEEE-rounded fp32 divide so rh(x / s) equals the reference's fp16 quotient.  The
// per-token reductions (amax, min, max) are order-free; mean|x| (1-bit scale, outlier threshold)
// follows ATen's cascade_sum order: 8 fp32 lanes, 4 interleaved accumulators, 4 cascade levels,
// lanes combined 0..7 in order, then / D in fp32.
//
// HBM layout: [n_rows][D] fp16 rows (D contiguous), packed payload [n_rows/per][D] bytes, per-row
// fp16 scale/min.  The quantizers stage a tile of rows in shared memory (row stride padded by 16 B
// so 8-lane row groups hit distinct banks), reduce each row with 8 lanes, then emit 4 output bytes
// per thread; the dequantizers are register-only, 8 columns per thread, 16-byte stores.
#include "common.cuh"

namespace argus {

enum QuantMode { Q_INT8 = 0, Q_FP8SIM = 1, Q_INT4 = 2, Q_INT2 = 3, Q_SIGN1 = 4, Q_OUTLIER = 5 };

template <int MODE>
struct ModeTraits;
template <> struct ModeTraits<Q_INT8>    { static constexpr int per = 1; };
template <> struct ModeTraits<Q_FP8SIM>  { static constexpr int per = 1; };
template <> struct ModeTraits<Q_INT4>    { static constexpr int per = 2; };
template <> struct ModeTraits<Q_INT2>    { static constexpr int per = 4; };
template <> struct ModeTraits<Q_SIGN1>   { static constexpr int per = 8; };
template <> struct ModeTraits<Q_OUTLIER> { static constexpr int per = 1; };

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

// abs of fp16 bits with NaN/Inf cleaned to +0 (isolate_outliers' cleanse step).
__device__ __forceinline__ __half clean_nan_inf(__half h) {
    unsigned short b = __half_as_ushort(h);
    return ((b & 0x7c00u) == 0x7c00u) ? __ushort_as_half(0) : h;
}

template <int MODE>
__global__ void __launch_bounds__(kQuantThreads)
quant_kernel(const __half* __restrict__ x, int64_t n_rows, int D, int tile_rows, float sigma,
             uint8_t* __restrict__ payload, __half* __restrict__ s_out, __half* __restrict__ mn_out,
             __half* __restrict__ outv, uint8_t* __restrict__ mask) {
    constexpr int per = ModeTraits<MODE>::per;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int stride = D + 8;  // halfs; +16 B keeps 16 B alignment and staggers banks by row
    __half* tile = reinterpret_cast<__half*>(smem_raw);
    float* st_a = reinterpret_cast<float*>(smem_raw + (size_t)tile_rows * stride * sizeof(__half));
    float* st_b = st_a + tile_rows;

    const int vec_per_row = D / 8;
    const int64_t n_tiles = (n_rows + tile_rows - 1) / tile_rows;
    for (int64_t tix = blockIdx.x; tix < n_tiles; tix += gridDim.x) {
        const int64_t r0 = tix * tile_rows;
        const int rows = (int)((n_rows - r0) < tile_rows ? (n_rows - r0) : tile_rows);
        // 1. stage the tile (16-byte loads, coalesced: the tile is one contiguous block)
        const uint4* src = reinterpret_cast<const uint4*>(x + r0 * D);
        for (int v = threadIdx.x; v < rows * vec_per_row; v += kQuantThreads) {
            int r = v / vec_per_row, c = v - r * vec_per_row;
            uint4 val = __ldg(src + v);
            if (MODE == Q_OUTLIER) {
                __half* hv = reinterpret_cast<__half*>(&val);
#pragma unroll
                for (int e = 0; e < 8; ++e) hv[e] = clean_nan_inf(hv[e]);
            }
            *reinterpret_cast<uint4*>(tile + r * stride + c * 8) = val;
        }
        __syncthreads();
        // 2. per-row statistics, 8 lanes per row
        const int lane8 = threadIdx.x & 7;
        for (int rb = threadIdx.x >> 3; rb < ((rows + 3) & ~3); rb += kQuantThreads / kRowLanes) {
            const bool live = rb < rows;
            const __half* row = tile + (live ? rb : 0) * stride;
            float a = 0.0f, b = 0.0f;
            if (MODE == Q_INT8 || MODE == Q_FP8SIM) {
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
                const float div = (MODE == Q_INT8) ? 127.0f : 240.0f;
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
            } else {  // Q_SIGN1, Q_OUTLIER: mean|x| in ATen order (|x| of an fp16 value is exact)
                const float lane_sum = cascade_lane_sum<true>(row, D / 8, lane8);
                const float total = cascade_combine(lane_sum);
                const float mean = rh(__fdiv_rn(total, (float)D));  // fp16(sum / D)
                if (MODE == Q_SIGN1) {
                    a = mean;
                } else {
                    a = rh(__fmul_rn(mean, sigma));  // threshold fp16(mean * sigma)
                }
            }
            if (live && lane8 == 0) { st_a[rb] = a; st_b[rb] = b; }
        }
        __syncthreads();
        // 3. codes: 4 consecutive columns x `per` rows per thread -> 4 output bytes
        const int quads = D / 4;
        const int prows = rows / per;
        for (int w = threadIdx.x; w < prows * quads; w += kQuantThreads) {
            const int pr = w / quads, cq = w - pr * quads;
            uint32_t word = 0;
#pragma unroll
            for (int i = 0; i < per; ++i) {
                const int r = pr * per + i;
                const __half* hp = tile + r * stride + cq * 4;
                const float a = st_a[r], b = st_b[r];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float v = h2f(hp[e]);
                    uint32_t code;
                    if (MODE == Q_INT8 || MODE == Q_FP8SIM) {
                        const float lo = (MODE == Q_INT8) ? -128.0f : -240.0f;
                        const float hi = (MODE == Q_INT8) ? 127.0f : 240.0f;
                        code = w8(clamp_nan(round_even(rh(__fdiv_rn(v, a))), lo, hi));
                        word |= code << (8 * e);
                    } else if (MODE == Q_INT4 || MODE == Q_INT2) {
                        const float qmax = (MODE == Q_INT4) ? 15.0f : 3.0f;
                        code = w8(clamp_nan(round_even(rh(__fdiv_rn(rh(__fsub_rn(v, b)), a))), 0.0f, qmax));
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
            const int64_t prow = r0 / per + pr;
            if (MODE == Q_OUTLIER) {
                const int64_t base = (r0 + pr) * (int64_t)D + cq * 4;
                *reinterpret_cast<uint32_t*>(mask + base) = word;
                const __half* hp = tile + pr * stride + cq * 4;
                __half nv[4], ov[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const bool m = (word >> (8 * e)) & 1u;
                    nv[e] = m ? __ushort_as_half(0) : hp[e];
                    ov[e] = m ? hp[e] : __ushort_as_half(0);
                }
                *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(payload) + base) = *reinterpret_cast<uint2*>(nv);
                *reinterpret_cast<uint2*>(outv + base) = *reinterpret_cast<uint2*>(ov);
            } else {
                *reinterpret_cast<uint32_t*>(payload + prow * D + cq * 4) = word;
            }
        }
        // 4. per-row scales / mins
        if (MODE != Q_OUTLIER) {
            for (int r = threadIdx.x; r < rows; r += kQuantThreads) {
                if (s_out) s_out[r0 + r] = f2h(st_a[r]);
                if (MODE == Q_INT4 || MODE == Q_INT2) mn_out[r0 + r] = f2h(st_b[r]);
            }
        }
        __syncthreads();
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
// INT8 / FP8-sim: out = fp16(q * s); 8 columns per thread.
__global__ void dequant_sym8_kernel(const int8_t* __restrict__ q, const __half* __restrict__ s, int64_t n_rows,
                                    int D, __half* __restrict__ out) {
    const int cols8 = D / 8;
    const int64_t items = n_rows * cols8;
    for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < items; w += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = w / cols8;
        const int c = (int)(w - r * cols8);
        const uint2 raw = __ldg(reinterpret_cast<const uint2*>(q + r * D) + c);
        const __half2 s2 = __half2half2(s[r]);
        const int8_t* b = reinterpret_cast<const int8_t*>(&raw);
        __half2 o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
            o[e] = __hmul2_rn(__halves2half2(__short2half_rn(b[2 * e]), __short2half_rn(b[2 * e + 1])), s2);
        *reinterpret_cast<uint4*>(out + r * D + c * 8) = *reinterpret_cast<uint4*>(o);
    }
}

// INT4 / INT2: out = fp16(fp16(u * s) + min), `per` rows from each packed byte row.
template <int BITS>
__global__ void dequant_asym_kernel(const uint8_t* __restrict__ p, const __half* __restrict__ s,
                                    const __half* __restrict__ mn, int64_t n_prows, int D, __half* __restrict__ out) {
    constexpr int per = 8 / BITS;
    constexpr uint32_t m = (1u << BITS) - 1u;
    const int cols8 = D / 8;
    const int64_t items = n_prows * cols8;
    for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < items; w += (int64_t)gridDim.x * blockDim.x) {
        const int64_t pr = w / cols8;
        const int c = (int)(w - pr * cols8);
        const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p + pr * D) + c);
        const uint8_t* b = reinterpret_cast<const uint8_t*>(&raw);
#pragma unroll
        for (int i = 0; i < per; ++i) {
            const int64_t r = pr * per + i;
            const __half2 s2 = __half2half2(s[r]);
            const __half2 m2 = __half2half2(mn[r]);
            __half2 o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const __half2 u = __halves2half2(__uint2half_rn((b[2 * e] >> (BITS * i)) & m),
                                                 __uint2half_rn((b[2 * e + 1] >> (BITS * i)) & m));
                o[e] = __hadd2_rn(__hmul2_rn(u, s2), m2);
            }
            *reinterpret_cast<uint4*>(out + r * D + c * 8) = *reinterpret_cast<uint4*>(o);
        }
    }
}

// 1-bit: out = +s or -s (exactly (2b - 1) * s).
__global__ void dequant_sign1_kernel(const uint8_t* __restrict__ p, const __half* __restrict__ s, int64_t n_prows,
                                     int D, __half* __restrict__ out) {
    const int cols8 = D / 8;
    const int64_t items = n_prows * cols8;
    for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < items; w += (int64_t)gridDim.x * blockDim.x) {
        const int64_t pr = w / cols8;
        const int c = (int)(w - pr * cols8);
        const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p + pr * D) + c);
        const uint8_t* b = reinterpret_cast<const uint8_t*>(&raw);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t r = pr * 8 + i;
            const __half sv = s[r];
            const __half nv = __hneg(sv);
            __half o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = ((b[e] >> i) & 1u) ? sv : nv;
            *reinterpret_cast<uint4*>(out + r * D + c * 8) = *reinterpret_cast<uint4*>(o);
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

template <int MODE>
int launch_quant(const uint16_t* x, int64_t n_rows, int D, float sigma, void* payload, uint16_t* s, uint16_t* mn,
                 uint16_t* outv, uint8_t* mask, cudaStream_t st) {
    constexpr int per = ModeTraits<MODE>::per;
    if (!argus_aligned(x, 16)) return argus_set_error(ARGUS_ERR_MISALIGNED, "input must be 16-byte aligned");
    if (!argus_aligned(payload, 4)) return argus_set_error(ARGUS_ERR_MISALIGNED, "output must be 4-byte aligned");
    if (n_rows == 0) return ARGUS_OK;
    // ~8 KB of fp16 rows per tile, a multiple of 8 rows (and of `per`)
    int tile_rows = 8192 / (2 * D);
    tile_rows = (tile_rows / 8) * 8;
    if (tile_rows < 8) tile_rows = 8;
    if (tile_rows > 256) tile_rows = 256;
    const size_t smem = (size_t)tile_rows * (D + 8) * sizeof(__half) + 2 * tile_rows * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(quant_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return argus_set_cuda_error(e);
    }
    const int64_t tiles = (n_rows + tile_rows - 1) / tile_rows;
    quant_kernel<MODE><<<argus_grid_cap(tiles), kQuantThreads, smem, st>>>(
        reinterpret_cast<const __half*>(x), n_rows, D, tile_rows, sigma, reinterpret_cast<uint8_t*>(payload),
        reinterpret_cast<__half*>(s), reinterpret_cast<__half*>(mn), reinterpret_cast<__half*>(outv), mask);
    static_assert(per >= 1, "packing factor");
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

int dq_blocks(int64_t items) { return argus_grid_cap((items + 255) / 256); }

}  // namespace

extern "C" {

int argus_quant_int8(const uint16_t* x, int64_t n_rows, int D, int8_t* q, uint16_t* scales, argus_stream_t stream) {
    int rc = check_rows(x, q, n_rows, D, 1);
    if (rc || !scales) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales");
    return launch_quant<Q_INT8>(x, n_rows, D, 0.f, q, scales, nullptr, nullptr, nullptr, (cudaStream_t)stream);
}

int argus_quant_fp8sim(const uint16_t* x, int64_t n_rows, int D, int8_t* q, uint16_t* scales, argus_stream_t stream) {
    int rc = check_rows(x, q, n_rows, D, 1);
    if (rc || !scales) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales");
    return launch_quant<Q_FP8SIM>(x, n_rows, D, 0.f, q, scales, nullptr, nullptr, nullptr, (cudaStream_t)stream);
}

int argus_quant_int4(const uint16_t* x, int64_t n_rows, int D, uint8_t* packed, uint16_t* scales, uint16_t* mins,
                     argus_stream_t stream) {
    int rc = check_rows(x, packed, n_rows, D, 2);
    if (rc || !scales || !mins) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales/mins");
    return launch_quant<Q_INT4>(x, n_rows, D, 0.f, packed, scales, mins, nullptr, nullptr, (cudaStream_t)stream);
}

int argus_quant_int2(const uint16_t* x, int64_t n_rows, int D, uint8_t* packed, uint16_t* scales, uint16_t* mins,
                     argus_stream_t stream) {
    int rc = check_rows(x, packed, n_rows, D, 4);
    if (rc || !scales || !mins) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales/mins");
    return launch_quant<Q_INT2>(x, n_rows, D, 0.f, packed, scales, mins, nullptr, nullptr, (cudaStream_t)stream);
}

int argus_quant_1bit(const uint16_t* x, int64_t n_rows, int D, uint8_t* packed, uint16_t* scales,
                     argus_stream_t stream) {
    int rc = check_rows(x, packed, n_rows, D, 8);
    if (rc || !scales) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales");
    return launch_quant<Q_SIGN1>(x, n_rows, D, 0.f, packed, scales, nullptr, nullptr, nullptr, (cudaStream_t)stream);
}

int argus_isolate_outliers(const uint16_t* x, int64_t n_rows, int D, float sigma, uint16_t* normal, uint16_t* outv,
                           uint8_t* mask, argus_stream_t stream) {
    int rc = check_rows(x, normal, n_rows, D, 1);
    if (rc || !outv || !mask) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null output");
    if (!(sigma > 0.0f)) {
        if (n_rows == 0) return ARGUS_OK;
        const int64_t n = n_rows * D;
        cleanse_kernel<<<dq_blocks(n), 256, 0, (cudaStream_t)stream>>>(
            reinterpret_cast<const __half*>(x), n, reinterpret_cast<__half*>(normal), reinterpret_cast<__half*>(outv),
            mask);
        ARGUS_CHECK_LAUNCH();
        return ARGUS_OK;
    }
    if (!argus_aligned(outv, 8) || !argus_aligned(normal, 8) || !argus_aligned(mask, 4))
        return argus_set_error(ARGUS_ERR_MISALIGNED, "outputs must be 8-byte aligned");
    return launch_quant<Q_OUTLIER>(x, n_rows, D, sigma, normal, nullptr, nullptr, outv, mask, (cudaStream_t)stream);
}

static int dequant_check(const void* a, const void* s, const void* out, int64_t n_rows, int D, int per) {
    int rc = check_rows(a, out, n_rows, D, per);
    if (rc) return rc;
    if (!s) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null scales");
    if (!argus_aligned(a, 8) || !argus_aligned(out, 16))
        return argus_set_error(ARGUS_ERR_MISALIGNED, "payload must be 8-byte and output 16-byte aligned");
    return ARGUS_OK;
}

int argus_dequant_int8(const int8_t* q, const uint16_t* scales, int64_t n_rows, int D, uint16_t* out,
                       argus_stream_t stream) {
    int rc = dequant_check(q, scales, out, n_rows, D, 1);
    if (rc) return rc;
    if (n_rows == 0) return ARGUS_OK;
    dequant_sym8_kernel<<<dq_blocks(n_rows * (D / 8)), 256, 0, (cudaStream_t)stream>>>(
        q, reinterpret_cast<const __half*>(scales), n_rows, D, reinterpret_cast<__half*>(out));
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

int argus_dequant_fp8sim(const int8_t* q, const uint16_t* scales, int64_t n_rows, int D, uint16_t* out,
                         argus_stream_t stream) {
    return argus_dequant_int8(q, scales, n_rows, D, out, stream);
}

int argus_dequant_int4(const uint8_t* packed, const uint16_t* scales, const uint16_t* mins, int64_t n_rows, int D,
                       uint16_t* out, argus_stream_t stream) {
    int rc = dequant_check(packed, scales, out, n_rows, D, 2);
    if (rc || !mins) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null mins");
    if (n_rows == 0) return ARGUS_OK;
    const int64_t pr = n_rows / 2;
    dequant_asym_kernel<4><<<dq_blocks(pr * (D / 8)), 256, 0, (cudaStream_t)stream>>>(
        packed, reinterpret_cast<const __half*>(scales), reinterpret_cast<const __half*>(mins), pr, D,
        reinterpret_cast<__half*>(out));
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

int argus_dequant_int2(const uint8_t* packed, const uint16_t* scales, const uint16_t* mins, int64_t n_rows, int D,
                       uint16_t* out, argus_stream_t stream) {
    int rc = dequant_check(packed, scales, out, n_rows, D, 4);
    if (rc || !mins) return rc ? rc : argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null mins");
    if (n_rows == 0) return ARGUS_OK;
    const int64_t pr = n_rows / 4;
    dequant_asym_kernel<2><<<dq_blocks(pr * (D / 8)), 256, 0, (cudaStream_t)stream>>>(
        packed, reinterpret_cast<const __half*>(scales), reinterpret_cast<const __half*>(mins), pr, D,
        reinterpret_cast<__half*>(out));
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

int argus_dequant_1bit(const uint8_t* packed, const uint16_t* scales, int64_t n_rows, int D, uint16_t* out,
                       argus_stream_t stream) {
    int rc = dequant_check(packed, scales, out, n_rows, D, 8);
    if (rc) return rc;
    if (n_rows == 0) return ARGUS_OK;
    const int64_t pr = n_rows / 8;
    dequant_sign1_kernel<<<dq_blocks(pr * (D / 8)), 256, 0, (cudaStream_t)stream>>>(
        packed, reinterpret_cast<const __half*>(scales), pr, D, reinterpret_cast<__half*>(out));
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
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

int argus_pack_1bit_signs(const uint16_t* x, int64_t n_rows, int D, uint8_t* packed, argus_stream_t stream) {
    // The sign pack is the 1-bit quantizer with its scale output switched off (null sink).
    int rc = check_rows(x, packed, n_rows, D, 8);
    if (rc) return rc;
    return launch_quant<Q_SIGN1>(x, n_rows, D, 0.f, packed, nullptr, nullptr, nullptr, nullptr, (cudaStream_t)stream);
}

}  // extern "C"
