/*
 * argus_b200.h -- C ABI of the B200 (sm_100a) implementation of ARGUS's tiered-KV hot path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (cudaStream_t passed
 * as argus_stream_t; NULL is the legacy default stream), enqueues its work on that stream and
 * returns an argus status code (0 = success).  Nothing here allocates memory unless its comment
 * says so; outputs are caller-owned.  fp16 data is passed as uint16_t bit patterns.
 *
 * Tensor layout convention for the codecs: a tensor of n_rows = groups * T rows of D values,
 * row-major with D contiguous ([groups][T][D]).  Sequence packing (INT4 2 tokens/byte, INT2 4,
 * 1-bit 8) combines `per` consecutive rows, so T must be a multiple of `per` and n_rows too;
 * packed outputs are [n_rows / per][D] bytes, per-token scales/mins are [n_rows] fp16.
 *
 * Each declaration names the reference (argus_cache 0.1.8) interface it replaces, as
 * file:line within that project.
 */
#ifndef ARGUS_B200_H
#define ARGUS_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* argus_stream_t; /* a cudaStream_t */

enum argus_status {
    ARGUS_OK = 0,
    ARGUS_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size, divisibility */
    ARGUS_ERR_MISALIGNED = 2,       /* a pointer or stride breaks the kernel's alignment rule */
    ARGUS_ERR_CUDA = 3,             /* a CUDA runtime call or launch failed */
    ARGUS_ERR_UNSUPPORTED = 4,      /* shape outside what the kernels implement */
    ARGUS_ERR_TIMEOUT = 5,          /* a bounded device-side wait gave up */
    ARGUS_ERR_CAPACITY = 6          /* request larger than a fixed-size buffer */
};

/* Text for a status code; the last error's detail is in argus_last_error(). */
const char* argus_status_string(int status);
/* Detail of the most recent failure on this host thread ("" if none). */
const char* argus_last_error(void);
/* Library version as 10000*major + 100*minor + patch. */
int argus_version(void);

/* ------------------------------------------------------------------------------- codecs */

/* Symmetric per-token INT8: s = fp16(amax|x|/127), q = int8(clamp(round(fp16(x/s)), -128, 127)).
 * Replaces quantize_to_int8, core/quantization.py:3-22.  x:[n_rows][D] -> q:[n_rows][D], s:[n_rows]. */
int argus_quant_int8(const uint16_t* x, int64_t n_rows, int D, int8_t* q, uint16_t* scales,
                     argus_stream_t stream);
/* q * s in fp16.  Replaces dequantize_from_int8, core/quantization.py:24-28. */
int argus_dequant_int8(const int8_t* q, const uint16_t* scales, int64_t n_rows, int D, uint16_t* out,
                       argus_stream_t stream);
/* Simulated FP8: as INT8 with 240 and clamp(-240, 240), then the int8 cast wraps codes above 127.
 * Replaces quantize_to_fp8_simulated, core/quantization.py:203-216. */
int argus_quant_fp8sim(const uint16_t* x, int64_t n_rows, int D, int8_t* q, uint16_t* scales,
                       argus_stream_t stream);
/* Replaces dequantize_from_fp8_simulated, core/quantization.py:218-222. */
int argus_dequant_fp8sim(const int8_t* q, const uint16_t* scales, int64_t n_rows, int D, uint16_t* out,
                         argus_stream_t stream);

/* Asymmetric INT4, 2 tokens per byte along the sequence (low nibble = even token).
 * s = fp16(fp16(max-min)/15), u = uint8(clamp(round(fp16(fp16(x-min)/s)), 0, 15)).
 * Replaces quantize_to_int4_packed, core/quantization.py:30-59 with the pack of
 * triton_pack_int4, core/triton_kernels.py:173-189 (its CPU path).  n_rows % 2 == 0. */
int argus_quant_int4(const uint16_t* x, int64_t n_rows, int D, uint8_t* packed, uint16_t* scales,
                     uint16_t* mins, argus_stream_t stream);
/* fp16(fp16(u*s) + min).  Replaces dequantize_from_int4_packed / triton_unpack_int4,
 * core/quantization.py:61-67, core/triton_kernels.py:213-239.  n_rows = unpacked rows. */
int argus_dequant_int4(const uint8_t* packed, const uint16_t* scales, const uint16_t* mins, int64_t n_rows,
                       int D, uint16_t* out, argus_stream_t stream);
/* Asymmetric INT2, 4 tokens per byte (token 4j+i in bits 2i..2i+1), /3 and clamp(0, 3).
 * Replaces quantize_to_int2_packed, core/quantization.py:69-124.  n_rows % 4 == 0. */
int argus_quant_int2(const uint16_t* x, int64_t n_rows, int D, uint8_t* packed, uint16_t* scales,
                     uint16_t* mins, argus_stream_t stream);
/* Replaces dequantize_from_int2_packed, core/quantization.py:126-171. */
int argus_dequant_int2(const uint8_t* packed, const uint16_t* scales, const uint16_t* mins, int64_t n_rows,
                       int D, uint16_t* out, argus_stream_t stream);
/* 1-bit sign packing, 8 tokens per byte (token 8j+i in bit i, bit = x >= 0), scale = mean|x| over D
 * in torch's CPU summation order.  Replaces quantize_to_1bit_packed, core/quantization.py:173-194
 * with triton_pack_1bit, core/triton_kernels.py:260-308 (its CPU path).  n_rows % 8 == 0. */
int argus_quant_1bit(const uint16_t* x, int64_t n_rows, int D, uint8_t* packed, uint16_t* scales,
                     argus_stream_t stream);
/* (2b-1)*s.  Replaces dequantize_from_1bit_packed / triton_unpack_1bit,
 * core/quantization.py:196-201, core/triton_kernels.py:330-386. */
int argus_dequant_1bit(const uint8_t* packed, const uint16_t* scales, int64_t n_rows, int D, uint16_t* out,
                       argus_stream_t stream);

/* Packs already-quantized 4-bit codes (uint8 0..15) two tokens per byte along the sequence.
 * Replaces triton_pack_int4, core/triton_kernels.py:173-211.  n_rows % 2 == 0. */
int argus_pack_int4_codes(const uint8_t* codes, int64_t n_rows, int D, uint8_t* packed, argus_stream_t stream);
/* Packs the sign bits (x >= 0) of fp16 values 8 tokens per byte.
 * Replaces triton_pack_1bit, core/triton_kernels.py:260-328.  n_rows % 8 == 0. */
int argus_pack_1bit_signs(const uint16_t* x, int64_t n_rows, int D, uint8_t* packed, argus_stream_t stream);

/* Outlier isolation: NaN/Inf -> 0; mask = |x| > fp16(mean|x| * sigma) per row (torch's mean order);
 * normal = x with outliers zeroed, outv = outliers only.  sigma <= 0: no outliers.
 * Replaces isolate_outliers, core/memory_manager.py:89-113.  mask is one byte per element. */
int argus_isolate_outliers(const uint16_t* x, int64_t n_rows, int D, float sigma, uint16_t* normal,
                           uint16_t* outv, uint8_t* mask, argus_stream_t stream);

/* --------------------------------------------------------------------------- JL archive */

/* C[b] = A . X[b] for a shared fp16 operator A [M][K] and fp16 pages X[b] [K][N], fp32
 * accumulation, fp16 output [batch][M][N].  Used for the sequence projection W.X
 * (core/quantization.py:243, core/memory_manager.py:1139-1141) and the reconstruction R.Y
 * (core/quantization.py:255,290, core/memory_manager.py:1176-1178). */
int argus_jl_apply(const uint16_t* A, const uint16_t* X, int64_t batch, int M, int K, int N, uint16_t* C,
                   argus_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* ARGUS_B200_H */
