/*
 * CPU oracle for the ARGUS tiered-KV hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the arithmetic of the reference's CPU code path so
 * that the CUDA kernels can be checked bit for bit.  Only the tests, the smoke check and
 * bench.py's CPU-baseline leg load it; the product path never does.
 *
 * Arithmetic model (verified against the reference's golden vectors in tests/golden):
 *   - every elementwise torch op on fp16 tensors is an fp32 op followed by
 *     round-to-nearest-even to fp16:  rh(v);
 *   - float -> int8/uint8 casts truncate to int32 and keep the low byte, NaN -> 0
 *     (x86 cvttss2si semantics): w8(v);
 *   - torch.mean over the last dim of an fp16 tensor (ATen ReduceOps mean_out, torch
 *     2.11): the input is widened to fp32 and summed by ATen's cascade_sum
 *     (SumKernel.cpp: vectorized_inner_sum -> row_sum -> multi_row_sum) with 8 fp32
 *     vector lanes, 4 interleaved accumulators and 4 cascade levels; the scalar tail
 *     is added first, then lanes 0..7 in order; the sum is divided by D in fp32 and
 *     rounded to fp16.  Restated here as cascade_rowsum() / torch_mean_abs_row().
 *
 * Functions and the reference lines they follow (argus_cache 0.1.8):
 *   oracle_quant_sym8     quantization.py:3-22  (int8, bound 127) and :203-216 (fp8-sim, 240)
 *   oracle_dequant_sym8   quantization.py:24-28, :218-222
 *   oracle_quant_asym     quantization.py:30-59 (int4) and :69-124 (int2), pack fallback
 *                         triton_kernels.py:178-189
 *   oracle_dequant_asym   quantization.py:61-67, :126-171; unpack fallback triton_kernels.py:218-239
 *   oracle_quant_1bit     quantization.py:173-194; pack fallback triton_kernels.py:264-278
 *   oracle_dequant_1bit   quantization.py:196-201; unpack fallback triton_kernels.py:334-386
 *   oracle_isolate_outliers memory_manager.py:89-113
 *   oracle_quant_e4m3 / oracle_dequant_e4m3: the true-e4m3 storage mode, a separately named
 *                         non-parity tier (the reference's "FP8" is the int8-with-wrap simulation of
 *                         quantization.py:203-216); its arithmetic is defined in the comment below
 *
 * Layout convention: a tensor is [rows][T][D] with D contiguous; packing runs along T.
 */
#include <stdint.h>
#include <string.h>
#include <math.h>

/* ---------------------------------------------------------------- fp16 helpers */
static inline float h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do { e++; man <<= 1; } while ((man & 0x400u) == 0);
            man &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* fp32 -> fp16, round to nearest even, with subnormals, overflow to inf and NaN. */
static inline uint16_t f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) { /* inf or NaN */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477ff000u) { /* rounds to >= 65520: overflow */
        return (uint16_t)(sign | 0x7c00u);
    }
    if (ax < 0x38800000u) { /* below 2^-14: fp16 subnormal or zero */
        if (ax < 0x33000000u) return (uint16_t)sign; /* < 2^-25: rounds to 0 */
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7fffffu) | 0x800000u; /* value = m * 2^(e-150) */
        uint32_t sh = 126u - e;                       /* to units of 2^-24, the fp16 subnormal ulp */
        uint32_t q = m >> sh;
        uint32_t rem = m & ((1u << sh) - 1u);
        uint32_t half = 1u << (sh - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (ax >> 23) - 127 + 15;
    uint32_t m = ax & 0x7fffffu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++; /* may carry into exponent */
    return (uint16_t)(sign | q);
}

static inline float rh(float v) { return h2f(f2h(v)); }

/* float -> int8 as torch's CPU cast does it: truncate to int32, keep the low byte.
 * NaN and out-of-range give INT32_MIN (x86 cvttss2si), whose low byte is 0. */
static inline uint8_t w8(float v) {
    if (isnan(v) || v >= 2147483648.0f || v < -2147483648.0f) return 0;
    int32_t i = (int32_t)v; /* truncation toward zero */
    return (uint8_t)(i & 0xff);
}

/* round half to even on an fp16-valued float (torch.round on fp16 tensors). */
static inline float round_even(float v) { return rintf(v); }

static inline int is_nan_h(uint16_t h) { return ((h & 0x7c00u) == 0x7c00u) && (h & 0x3ffu); }

/* torch.clamp(x, lo, hi) on fp16: NaN propagates. */
static inline float clampf_nan(float v, float lo, float hi) {
    if (isnan(v)) return v;
    return v < lo ? lo : (v > hi ? hi : v);
}

/* torch.amax / torch.amin over a row: NaN propagates. */
static float row_amax_abs(const uint16_t* x, int D) {
    float m = 0.0f;
    for (int d = 0; d < D; ++d) {
        float a = fabsf(h2f(x[d]));
        if (isnan(a)) return a;
        if (a > m) m = a;
    }
    return m;
}

static void row_minmax(const uint16_t* x, int D, float* mn, float* mx) {
    float lo = h2f(x[0]), hi = lo;
    if (isnan(lo)) { *mn = *mx = lo; return; }
    for (int d = 1; d < D; ++d) {
        float v = h2f(x[d]);
        if (isnan(v)) { *mn = *mx = v; return; }
        if (v < lo) lo = v;
        if (v > hi) hi = v;
    }
    *mn = lo;
    *mx = hi;
}

/* ------------------------------------------------- ATen cascade_sum restatement */
static int ceil_log2_i64(int64_t x) {
    if (x <= 2) return 1;
    int b = 0;
    uint64_t v = (uint64_t)(x - 1);
    while (v) { b++; v >>= 1; }
    return b;
}

/* Sum of n fp32 values in the order ATen's cascade_sum uses for a contiguous inner
 * reduction with 8-lane fp32 vectors (vectorized_inner_sum), or its scalar path for
 * n < 8 (scalar_inner_sum).  Both go through row_sum: 4 interleaved accumulators fed
 * by multi_row_sum's 4-level cascade. */
static float cascade_rowsum(const float* x, int n) {
    enum { VL = 8, ILP = 4, LEVELS = 4 };
    int vector = n >= VL;
    int width = vector ? VL : 1;                 /* lanes per "element" of row_sum */
    int64_t count = vector ? n / VL : n;         /* elements row_sum iterates over */
    float acc[LEVELS][ILP][VL];
    memset(acc, 0, sizeof(acc));
    int64_t size_ilp = count / ILP;
    int level_power = ceil_log2_i64(size_ilp) / LEVELS;
    if (level_power < 4) level_power = 4;
    int64_t level_step = (int64_t)1 << level_power;
    int64_t level_mask = level_step - 1;
#define ELEM(idx, lane) (vector ? x[(idx) * VL + (lane)] : x[(idx)])
    int64_t i = 0;
    while (i + level_step <= size_ilp) {
        for (int64_t j = 0; j < level_step; ++j, ++i)
            for (int k = 0; k < ILP; ++k)
                for (int l = 0; l < width; ++l) acc[0][k][l] += ELEM(i * ILP + k, l);
        for (int j = 1; j < LEVELS; ++j) {
            for (int k = 0; k < ILP; ++k)
                for (int l = 0; l < width; ++l) { acc[j][k][l] += acc[j - 1][k][l]; acc[j - 1][k][l] = 0.0f; }
            int64_t mask = level_mask << (j * level_power);
            if ((i & mask) != 0) break;
        }
    }
    for (; i < size_ilp; ++i)
        for (int k = 0; k < ILP; ++k)
            for (int l = 0; l < width; ++l) acc[0][k][l] += ELEM(i * ILP + k, l);
    for (int j = 1; j < LEVELS; ++j)
        for (int k = 0; k < ILP; ++k)
            for (int l = 0; l < width; ++l) acc[0][k][l] += acc[j][k][l];
    float part[ILP][VL];
    memcpy(part, acc[0], sizeof(part));
    for (int64_t t = size_ilp * ILP; t < count; ++t)
        for (int l = 0; l < width; ++l) part[0][l] += ELEM(t, l);
    for (int k = 1; k < ILP; ++k)
        for (int l = 0; l < width; ++l) part[0][l] += part[k][l];
#undef ELEM
    if (!vector) return part[0][0];
    float fin = 0.0f;
    for (int t = (int)(count * VL); t < n; ++t) fin += x[t];
    for (int l = 0; l < VL; ++l) fin += part[0][l];
    return fin;
}

/* torch.mean(torch.abs(x), dim=-1) for one fp16 row, returned as fp16 bits. */
static uint16_t torch_mean_abs_row(const uint16_t* x, int D) {
    float buf[1024];
    float s;
    if (D <= 1024) {
        for (int d = 0; d < D; ++d) buf[d] = fabsf(h2f(x[d]));
        s = cascade_rowsum(buf, D);
    } else {
        s = 0.0f; /* head dims above 1024 are not supported by the oracle */
    }
    return f2h(s / (float)D);
}

/* ------------------------------------------------------------ exported oracle API */

/* Symmetric per-row quantization: s = rh(amax|x| / div), q = w8(clamp(round(rh(x / s)), lo, hi)).
 * INT8: div 127, lo -128, hi 127.  Simulated FP8: div 240, lo -240, hi 240 (the int8 cast then
 * wraps codes above 127).  clamp(min=1e-8) on the fp16 scale is a no-op: 1e-8 rounds to 0 in fp16.
 * x: [n_rows][D] fp16 bits -> q: [n_rows][D] int8, s: [n_rows] fp16 bits. */
void oracle_quant_sym8(const uint16_t* x, int64_t n_rows, int D, float div, float lo, float hi, int8_t* q,
                       uint16_t* s) {
    for (int64_t r = 0; r < n_rows; ++r) {
        const uint16_t* row = x + r * D;
        float sc = rh(row_amax_abs(row, D) / div);
        s[r] = f2h(sc);
        for (int d = 0; d < D; ++d) {
            float v = round_even(rh(h2f(row[d]) / sc));
            q[r * D + d] = (int8_t)w8(clampf_nan(v, lo, hi));
        }
    }
}

/* q * s (fp16 result). */
void oracle_dequant_sym8(const int8_t* q, const uint16_t* s, int64_t n_rows, int D, uint16_t* out) {
    for (int64_t r = 0; r < n_rows; ++r) {
        float sc = h2f(s[r]);
        for (int d = 0; d < D; ++d) out[r * D + d] = f2h((float)q[r * D + d] * sc);
    }
}

/* ------------------------------------------------------------ true e4m3 (non-parity) */
/* OCP FP8 E4M3 ("e4m3fn"): sign, 4 exponent bits (bias 7), 3 mantissa bits, no infinities, NaN =
 * S.1111.111, largest finite 448, smallest subnormal 2^-9.  Encoding: round to nearest even,
 * magnitudes from 448 up (and infinities) saturate to +-448; NaN stores code 0 (the tier's rule,
 * as the int8 tiers store 0 for NaN). */
static uint8_t e4m3_encode(float v) {
    if (isnan(v)) return 0;
    const uint8_t sign = signbit(v) ? 0x80u : 0u;
    const float a = fabsf(v);
    if (a >= 448.0f) return (uint8_t)(sign | 0x7eu);
    if (a < 0.015625f) { /* below 2^-6: subnormal grid of 2^-9 (a * 512 is exact) */
        const float q = rintf(a * 512.0f);   /* 8 is the smallest normal, code 0x08 */
        return (uint8_t)(sign | (uint8_t)q);
    }
    int e2;
    (void)frexpf(a, &e2);                    /* a = f * 2^e2, f in [0.5, 1) */
    int E = e2 - 1;                          /* a = 1.m * 2^E, E in [-6, 8] */
    float q = rintf(ldexpf(a, 3 - E));       /* 1.m * 8 rounded: [8, 16] */
    if (q >= 16.0f) { q = 8.0f; E += 1; }
    if (E > 8 || (E == 8 && q > 14.0f)) return (uint8_t)(sign | 0x7eu);
    return (uint8_t)(sign | (uint8_t)((E + 7) << 3) | (uint8_t)((int)q - 8));
}

static float e4m3_decode(uint8_t c) {
    const float sign = (c & 0x80u) ? -1.0f : 1.0f;
    const int E = (c >> 3) & 0xf, m = c & 7;
    if (E == 0xf && m == 7) return NAN;
    if (E == 0) return sign * ldexpf((float)m, -9);
    return sign * ldexpf((float)(8 + m), E - 10);
}

/* The e4m3 tier: s = rh(amax|x| / 448) per row, code = e4m3(x / s) from the fp32 quotient (one
 * rounding), value = rh(e4m3(code) * s).  A zero row has s = 0, its quotients are NaN and store 0.
 * x: [n_rows][D] fp16 bits -> q: [n_rows][D] codes, s: [n_rows] fp16 bits. */
void oracle_quant_e4m3(const uint16_t* x, int64_t n_rows, int D, uint8_t* q, uint16_t* s) {
    for (int64_t r = 0; r < n_rows; ++r) {
        const uint16_t* row = x + r * D;
        const float sc = rh(row_amax_abs(row, D) / 448.0f);
        s[r] = f2h(sc);
        for (int d = 0; d < D; ++d) q[r * D + d] = e4m3_encode(h2f(row[d]) / sc);
    }
}

void oracle_dequant_e4m3(const uint8_t* q, const uint16_t* s, int64_t n_rows, int D, uint16_t* out) {
    for (int64_t r = 0; r < n_rows; ++r) {
        const float sc = h2f(s[r]);
        for (int d = 0; d < D; ++d) out[r * D + d] = f2h(e4m3_decode(q[r * D + d]) * sc);
    }
}

/* e4m3 codes of n fp32 values (the encoder alone). */
void oracle_e4m3_encode(const float* v, int64_t n, uint8_t* q) {
    for (int64_t i = 0; i < n; ++i) q[i] = e4m3_encode(v[i]);
}

/* Asymmetric quantization with sequence packing.  bits = 4 (2 codes/byte) or 2 (4 codes/byte).
 * x: [n_groups][T][D] -> packed: [n_groups][T*bits/8][D], s, mn: [n_groups][T]. */
void oracle_quant_asym(const uint16_t* x, int64_t n_groups, int T, int D, int bits,
                       uint8_t* packed, uint16_t* s, uint16_t* mn) {
    int per = 8 / bits;
    float qmax = (float)((1 << bits) - 1);
    uint8_t codes[1024];
    for (int64_t g = 0; g < n_groups; ++g) {
        for (int t = 0; t < T; ++t) {
            const uint16_t* row = x + (g * T + t) * (int64_t)D;
            float lo, hi;
            row_minmax(row, D, &lo, &hi);
            float sc = rh(rh(hi - lo) / qmax);
            /* clamp(min=1e-8): 1e-8 is below the smallest fp16 subnormal, a no-op */
            s[g * T + t] = f2h(sc);
            mn[g * T + t] = f2h(lo);
            for (int d = 0; d < D; ++d) {
                float v = rh(rh(h2f(row[d]) - lo) / sc);
                v = round_even(v);
                v = clampf_nan(v, 0.0f, qmax);
                codes[d] = w8(v);
            }
            int pr = t / per, sh = (t % per) * bits;
            uint8_t* dst = packed + (g * (T / per) + pr) * (int64_t)D;
            for (int d = 0; d < D; ++d) {
                if (sh == 0) dst[d] = 0;
                dst[d] |= (uint8_t)(codes[d] << sh);
            }
        }
    }
}

/* rh(rh(u * s) + mn), unpacking along T. */
void oracle_dequant_asym(const uint8_t* packed, const uint16_t* s, const uint16_t* mn, int64_t n_groups,
                         int T, int D, int bits, uint16_t* out) {
    int per = 8 / bits;
    uint8_t mask = (uint8_t)((1 << bits) - 1);
    for (int64_t g = 0; g < n_groups; ++g)
        for (int t = 0; t < T; ++t) {
            float sc = h2f(s[g * T + t]), lo = h2f(mn[g * T + t]);
            const uint8_t* src = packed + (g * (T / per) + t / per) * (int64_t)D;
            int sh = (t % per) * bits;
            for (int d = 0; d < D; ++d) {
                float u = (float)((src[d] >> sh) & mask);
                out[(g * T + t) * (int64_t)D + d] = f2h(rh(u * sc) + lo);
            }
        }
}

/* Sign bits packed 8 tokens per byte along T; scale = mean|x| over D (ATen order). */
void oracle_quant_1bit(const uint16_t* x, int64_t n_groups, int T, int D, uint8_t* packed, uint16_t* s) {
    for (int64_t g = 0; g < n_groups; ++g)
        for (int t = 0; t < T; ++t) {
            const uint16_t* row = x + (g * T + t) * (int64_t)D;
            s[g * T + t] = torch_mean_abs_row(row, D);
            uint8_t* dst = packed + (g * (T / 8) + t / 8) * (int64_t)D;
            int sh = t % 8;
            for (int d = 0; d < D; ++d) {
                float v = h2f(row[d]);
                uint8_t bit = (!isnan(v) && v >= 0.0f) ? 1 : 0; /* -0 >= 0 holds */
                if (sh == 0) dst[d] = 0;
                dst[d] |= (uint8_t)(bit << sh);
            }
        }
}

/* (2b - 1) * s. */
void oracle_dequant_1bit(const uint8_t* packed, const uint16_t* s, int64_t n_groups, int T, int D,
                         uint16_t* out) {
    for (int64_t g = 0; g < n_groups; ++g)
        for (int t = 0; t < T; ++t) {
            float sc = h2f(s[g * T + t]);
            const uint8_t* src = packed + (g * (T / 8) + t / 8) * (int64_t)D;
            for (int d = 0; d < D; ++d) {
                float b = (float)((src[d] >> (t % 8)) & 1);
                out[(g * T + t) * (int64_t)D + d] = f2h(rh(rh(b * 2.0f) - 1.0f) * sc);
            }
        }
}

/* isolate_outliers on [n_rows][D]: NaN/Inf -> 0, threshold rh(mean|x| * sigma).
 * Writes normal (fp16), outlier values (fp16, zeros elsewhere) and a 0/1 mask. */
void oracle_isolate_outliers(const uint16_t* x, int64_t n_rows, int D, float sigma, uint16_t* normal,
                             uint16_t* outv, uint8_t* mask) {
    uint16_t clean[1024];
    for (int64_t r = 0; r < n_rows; ++r) {
        const uint16_t* row = x + r * D;
        for (int d = 0; d < D; ++d) {
            uint16_t h = row[d];
            clean[d] = ((h & 0x7c00u) == 0x7c00u) ? 0 : h; /* NaN or Inf -> +0 */
        }
        if (!(sigma > 0.0f)) {
            for (int d = 0; d < D; ++d) { normal[r * D + d] = clean[d]; outv[r * D + d] = 0; mask[r * D + d] = 0; }
            continue;
        }
        float thr = rh(h2f(torch_mean_abs_row(clean, D)) * sigma);
        for (int d = 0; d < D; ++d) {
            float a = fabsf(h2f(clean[d]));
            int m = a > thr;
            mask[r * D + d] = (uint8_t)m;
            outv[r * D + d] = m ? clean[d] : 0;
            normal[r * D + d] = m ? 0 : clean[d];
        }
    }
}

/* Exposed for tests of the rounding helpers themselves. */
void oracle_f32_to_f16(const float* x, int64_t n, uint16_t* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = f2h(x[i]);
}

float oracle_torch_mean_abs(const uint16_t* x, int D) { return h2f(torch_mean_abs_row(x, D)); }

int oracle_is_nan_h(uint16_t h) { return is_nan_h(h); }
