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

struct argus_kv_arena;

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

/* Asynchronous copy of `bytes` between any two of device memory and pinned host memory on `stream`
 * (one cudaMemcpyAsync).  The host-spill transport: replaces the synchronous pageable .to("cpu") /
 * .to(device) moves of swap_out_to_host / swap_in_to_device (core/memory_manager.py:1658-1713). */
int argus_memcpy_async(void* dst, const void* src, int64_t bytes, argus_stream_t stream);
/* Asynchronous 2-D copy (one cudaMemcpy2DAsync): `height` rows of `width` bytes, row starts
 * `src_pitch` / `dst_pitch` bytes apart, between pinned host and device memory on `stream`.  Moves a
 * run of slots of every (batch, kv_head) of a spilled record arena in one call, for streaming a
 * host-resident tier into a device staging arena (the swap_in_to_device of
 * core/memory_manager.py:1686-1713, in pieces that overlap the attention of the resident tiers). */
int argus_memcpy2d_async(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch, int64_t width,
                         int64_t height, argus_stream_t stream);

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
/* True e4m3 per token (ARGUS_TIER_E4M3; no reference counterpart: a separately named non-parity
 * mode beside the simulated FP8 above).  x:[n_rows][D] -> codes:[n_rows][D], s:[n_rows]. */
int argus_quant_e4m3(const uint16_t* x, int64_t n_rows, int D, uint8_t* q, uint16_t* scales,
                     argus_stream_t stream);
/* fp16(e4m3(code) * s). */
int argus_dequant_e4m3(const uint8_t* q, const uint16_t* scales, int64_t n_rows, int D, uint16_t* out,
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

/* ----------------------------------------------------------------------- page codecs (cascade) */
/* These address pages of record arenas (see argus_kv_arena below): page `slot` holds B*H_kv
 * (batch, kv_head) blocks `bh_stride` bytes apart, each [K payload][V payload][K scales][V scales]
 * [K mins][V mins].  n_bh = B*H_kv. */

/* Quantizes an fp16 page, k and v contiguous [n_bh][page_tokens][D], into slot dst_slot of a record
 * arena of any tier.  The K/V halves of _demote_active_to_fp8's quantize step
 * (core/memory_manager.py:944-949) and of building any tier directly from fp16. */
int argus_page_quantize(const uint16_t* k, const uint16_t* v, int32_t n_bh, int D, const struct argus_kv_arena* dst,
                        int32_t dst_slot, argus_stream_t stream);
/* Fused demotion of one page: dequantize slot src_slot of `src` exactly as the reference does and
 * re-quantize it into slot dst_slot of `dst` (any tier pair with equal page size), without leaving
 * the chip.  Replaces the dequantize + quantize pairs of _demote_fp8_to_int8, _demote_int8_to_int4,
 * _demote_int4_to_int2 and _demote_int2_to_one_bit (core/memory_manager.py:989-1123). */
int argus_page_requant(const struct argus_kv_arena* src, int32_t src_slot, const struct argus_kv_arena* dst,
                       int32_t dst_slot, int32_t n_bh, int D, argus_stream_t stream);
/* Dequantizes page src_slot of `src` to fp16 rows: K into k_out + bh*out_bh_stride + (out_tok0 + t)*D
 * (elements), V likewise into v_out.  The per-page dequantization of get_all_keys_values,
 * _resurrect_page and speculate_and_prefetch (core/memory_manager.py:832-866, 1157-1290, 1578-1621). */
int argus_page_dequantize(const struct argus_kv_arena* src, int32_t src_slot, int32_t n_bh, int D, uint16_t* k_out,
                          uint16_t* v_out, int64_t out_bh_stride, int64_t out_tok0, argus_stream_t stream);

/* Overwrites out[(b*H + h)*out_bh_stride + (out_tok0 + t)*D + d] with vals[i] for each COO entry
 * idx[i] = (b, h, t, d) (int16); entries outside [B, H, P, D] are skipped.  The sidecar scatter of
 * core/memory_manager.py:1190-1199 (and every other reader of key/value_out_indices). */
int argus_scatter_coo(uint16_t* out, int64_t out_bh_stride, int64_t out_tok0, int B, int H, int P, int D,
                      const int16_t* idx, const uint16_t* vals, int64_t n, argus_stream_t stream);
/* Compacts a [B,H,P,D] outlier mask (one byte per element) and its values into COO entries in
 * row-major order, as torch.nonzero(mask).to(int16) and outv[mask] (core/memory_manager.py:951-955).
 * Writes at most `capacity` entries; *count_out (device int64) receives the total count. */
int argus_outliers_to_coo(const uint8_t* mask, const uint16_t* outv, int B, int H, int P, int D, int16_t* idx_out,
                          uint16_t* vals_out, int64_t capacity, int64_t* count_out, argus_stream_t stream);

/* One outlier of a page as the fused attention applies it: the page's rebuilt value at (tok, dim)
 * (the sidecar's fp16 value, scattered over the dequantized page by core/memory_manager.py:1190-1199,
 * 1402-1409) minus the dequantized value there, in fp32. */
typedef struct argus_outlier {
    uint16_t tok;  /* token within the page */
    uint16_t dim;
    float delta;
} argus_outlier;

/* Bytes of the correction blocks of one page (argus_outlier_corrections) for bh = B*H (b, h)
 * pairs, nk key and nv value sidecar entries (the last 16 bytes are the builder's own scratch). */
int64_t argus_outlier_blocks_bytes(int32_t bh, int32_t page_tokens, int64_t nk, int64_t nv);
/* Correction blocks of one quantized page for the fused decode attention, so that the attention
 * reads the page compressed and still sees its sidecars (the reference scatters them over the
 * dequantized page before attending, core/memory_manager.py:1402-1409).  Inputs: the page's key and
 * value sidecars as COO (b, h, t, d) int16 indices in row-major order (torch.nonzero order, as
 * argus_outliers_to_coo writes them) with fp16 values; k_deq / v_deq: the page dequantized without
 * its sidecars, [B][H][P][D] fp16 (argus_page_dequantize).  Writes into `blocks` (16-byte aligned,
 * argus_outlier_blocks_bytes) one block per (b, h) with entries (NT = ceil(P / 16), NH = 8 NT + 1):
 *     uint32 k_off[NH]   first key entry of token pair j (tokens 2j, 2j+1); k_off[8 NT] = key count
 *     uint32 v_off[NH]   first value entry of tile i (tokens 16i ..) and dim group g (dims g D/8 ..
 *                        (g+1) D/8 - 1) at 8i + g; v_off[8 NT] = key count + value count
 *     argus_outlier entries[]   key entries in (token, dim) order, then value entries ordered by
 *                               tile, dim, token
 * (offsets index entries[]), and block_addr[b*H + h] = the block's device address, or 0 for a
 * (b, h) without entries.  A sidecar with an index outside [B, H, P, D] or out of row-major order
 * makes every address 0 and sets the status word argus_device_status reports
 * (ARGUS_ERR_INVALID_ARGUMENT). */
int argus_outlier_corrections(const int16_t* k_idx, const uint16_t* k_val, int64_t nk, const int16_t* v_idx,
                              const uint16_t* v_val, int64_t nv, const uint16_t* k_deq, const uint16_t* v_deq,
                              int32_t batch, int32_t heads, int32_t page_tokens, int32_t head_dim, void* blocks,
                              uint64_t* block_addr, argus_stream_t stream);

/* --------------------------------------------------------------------------- JL archive */

/* C[b] = A . X[b] for a shared fp16 operator A [M][K] and fp16 pages X[b] [K][N], fp32
 * accumulation, fp16 output [batch][M][N].  Used for the sequence projection W.X
 * (core/quantization.py:243, core/memory_manager.py:1139-1141) and the reconstruction R.Y
 * (core/quantization.py:255,290, core/memory_manager.py:1176-1178). */
int argus_jl_apply(const uint16_t* A, const uint16_t* X, int64_t batch, int M, int K, int N, uint16_t* C,
                   argus_stream_t stream);

/* ---------------------------------------------------------------- JL archive decode attention */

/* One decode step of attention over JL-archived blocks: each block of `block_tokens` tokens is
 * stored as Yk = W . K, Yv = W . V ([block_rows][head_dim] fp16), and the reference rebuilds it as
 * R . Yk, R . Yv before softmax attention (core/memory_manager.py:1176-1178, 1317-1447).  The kernel
 * computes the same attention without rebuilding K and V: s = R (Yk q^T), w = R^T p, o = Yv^T w.
 * Block j of (b, h) is at yk + (b*heads_kv + h)*bh_stride + j*block_stride (elements); supported:
 * head_dim 64 or 128, block_rows 64 or 128, block_tokens a multiple of 128, group*q_len <= 8. */
typedef struct argus_jl_attn_shape {
    int32_t batch;
    int32_t heads_kv;
    int32_t group;
    int32_t q_len;
    int32_t head_dim;
    int32_t block_rows;    /* rows of a projected block (N / ratio) */
    int32_t block_tokens;  /* tokens a block stands for (N) */
    int32_t n_blocks;
    int32_t n_splits;      /* split-K partitions of each (batch, kv_head)'s blocks (<= n_blocks) */
    int32_t n_ctas;        /* > 0: this many CTAs share the blocks of all (batch, kv_head) in equal
                              contiguous ranges (a range may span heads), instead of n_splits per
                              (batch, kv_head); at most the number of blocks */
    float scale;
    int32_t reserved;
    int64_t bh_stride;     /* elements */
    int64_t block_stride;  /* elements */
} argus_jl_attn_shape;

/* Writes R [n_tokens][n_rows] (fp16, the reconstruction operator of core/memory_manager.py:241-282)
 * into the operator pieces the JL attention copies: R for every 128 tokens and R^T for every 64
 * tokens, as K-major tensor-core operands in 128-byte swizzle (r_frag and rt_frag,
 * n_tokens*n_rows*2 bytes each, 16-byte aligned; n_tokens a multiple of 128, n_rows of 64).  Done
 * once per operator. */
int argus_jl_operator_fragments(const uint16_t* R, int n_tokens, int n_rows, void* r_frag, void* rt_frag,
                                argus_stream_t stream);
/* Workspace bytes of argus_jl_attention: one arrival counter per (batch, kv_head) at the front
 * (zero before the first use with a shape; every completed launch leaves them zero) and the split
 * partials. */
int64_t argus_jl_attention_workspace_size(const argus_jl_attn_shape* shape);
/* q [B, heads_kv*group, q_len, D] fp16 (D 64 or 128; blocks of 64 or 128 rows) -> out (same shape,
 * fp16) and optional lse (natural log,
 * [B, heads_kv*group, q_len] fp32) over the archived tokens only.  Optional block_lse
 * [B*heads_kv][n_blocks][8] fp32 receives each block's natural-log LSE per query (group*q_len
 * queries used): the per-page attention mass of the importance policy
 * (core/memory_manager.py:1453-1522) is exp(block_lse - lse). */
int argus_jl_attention(const argus_jl_attn_shape* shape, const uint16_t* yk, const uint16_t* yv, const void* r_frag,
                       const void* rt_frag, const uint16_t* q, uint16_t* out, float* lse, float* block_lse,
                       void* workspace, argus_stream_t stream);
/* Merges two attention results over disjoint token sets: rows of head_dim fp16 values with their
 * natural-log LSE -> out (and lse, if given).  Used to join the JL archive with the other tiers
 * (the concatenation of core/memory_manager.py:1373-1430). */
int argus_attention_merge(const uint16_t* out_a, const float* lse_a, const uint16_t* out_b, const float* lse_b,
                          int64_t rows, int head_dim, uint16_t* out, float* lse, argus_stream_t stream);
/* In-place fp32 form of argus_attention_merge for joining many partial results (runs of a streamed
 * host-resident tier): acc_o [rows][head_dim] fp32 and acc_lse (natural log; -inf and zeros before
 * the first join) <- join(acc, (out_b, lse_b)). */
int argus_attention_accumulate(float* acc_o, float* acc_lse, const uint16_t* out_b, const float* lse_b, int64_t rows,
                               int head_dim, argus_stream_t stream);

/* ------------------------------------------------------------------- mixed-tier decode attention */

/* Storage tiers of a KV arena. */
enum argus_tier {
    ARGUS_TIER_FP16 = 0,   /* fp16 values; no scales */
    ARGUS_TIER_FP8SIM = 1, /* int8 codes (simulated-FP8 wraparound), fp16 scale per token */
    ARGUS_TIER_INT8 = 2,   /* int8 codes, fp16 scale per token */
    ARGUS_TIER_INT4 = 3,   /* 2 tokens per byte, fp16 scale + min per token */
    ARGUS_TIER_INT2 = 4,   /* 4 tokens per byte, fp16 scale + min per token */
    ARGUS_TIER_1BIT = 5,   /* 8 tokens per byte (sign), fp16 scale per token */
    ARGUS_TIER_E4M3 = 6    /* true e4m3 codes (OCP FP8 E4M3), fp16 scale per token: a separately named
                              non-parity tier (the reference's FP8 tier is ARGUS_TIER_FP8SIM);
                              s = fp16(amax / 448), code = e4m3(x / s) from the fp32 quotient (nearest
                              even, saturating at 448, NaN -> 0), value = fp16(e4m3(code) * s) */
};

/* Arena layouts. */
enum argus_layout {
    /* One record per (batch*kv_head, slot): [K payload][V payload][K scales][V scales][K mins][V mins],
     * record r of (b, h) at  base + (b*H_kv + h)*bh_stride + slot*record_bytes.  Payload = page_tokens/per
     * packed rows of D bytes (fp16: page_tokens rows of 2D bytes); scales/mins = page_tokens fp16 each. */
    ARGUS_LAYOUT_RECORD = 0,
    /* Separate fp16 K and V tensors [B][H_kv][L][D] (sinks, anchors, the staging buffer); slot j is
     * tokens 16j .. 16j+15, at  k + (b*H_kv + h)*bh_stride + j*16*D*2. */
    ARGUS_LAYOUT_SPLIT_FP16 = 1
};

/* One storage arena.  All pointers and byte strides must be 16-byte aligned. */
typedef struct argus_kv_arena {
    int32_t tier;         /* argus_tier; ARGUS_TIER_FP16 for the split layout */
    int32_t layout;       /* argus_layout */
    const void* k;        /* record base, or the K tensor */
    const void* v;        /* the V tensor (split layout); unused for records */
    int64_t bh_stride;    /* bytes between consecutive (b, h) blocks */
    int32_t record_bytes; /* bytes per record (record layout) */
    int32_t page_tokens;  /* tokens per slot: page size for records, 16 for the split layout */
    /* Outlier sidecars of the arena's pages (quantized record arenas only; null = none):
     * outlier_dir[(b*H_kv + h)*dir_slots + slot] is the device address of that page's
     * correction block for (b, h), as argus_outlier_corrections writes it, or 0. */
    const uint64_t* outlier_dir;
    int32_t dir_slots;
    int32_t reserved;
    /* Occupancy of the arena's slots (null = every slot the chunk list names holds a page): a device
     * array of one byte per slot (per 16-token slot in the split layout), nonzero where the slot holds
     * live tokens.  Tiles of dead slots are skipped (their tile_lse entries read -inf); a chunk of a
     * record page longer than 16 tokens, or of the split layout, is live or dead as a whole (its first
     * slot's byte).  So a chunk list covering a whole pool
     * stays valid while pages come and go: the cache updates one byte per page move (demotion,
     * resurrection, a new page: core/memory_manager.py:383-489, 832-917, 944-1155) instead of rebuilding
     * its tables. */
    const uint8_t* slot_live;
} argus_kv_arena;

/* A run of up to 16 consecutive 16-token tiles of one arena, staged as one unit:
 *   page_tokens <= 16 (records): tiles are the slots slot0 .. slot0+ntiles-1, one page each;
 *   page_tokens  > 16 (records): tiles are tokens tok0 .. tok0+16*ntiles-1 of slot slot0;
 *   split layout: tiles are the 16-token slots slot0 .. slot0+ntiles-1.
 * The last tile holds ntok_last tokens (1..16; a multiple of 8 for quantized tiers). */
typedef struct argus_kv_chunk {
    int32_t slot0;
    uint16_t tok0;
    uint8_t arena;
    uint8_t ntiles;
    uint8_t ntok_last;
    uint8_t reserved[3];
} argus_kv_chunk;

#define ARGUS_MAX_ARENAS 8

/* Geometry of one decode-attention call. */
typedef struct argus_attn_shape {
    int32_t batch;      /* B */
    int32_t heads_kv;   /* H_kv */
    int32_t group;      /* query heads per KV head (H_q / H_kv) */
    int32_t q_len;      /* query tokens per sequence (all attend to every cached token) */
    int32_t head_dim;   /* D: 16, 32, 64, 128 or 256 */
    int32_t n_splits;   /* split-K partitions of the chunk list */
    int32_t n_arenas;
    int32_t n_chunks;
    float scale;        /* softmax scale (1/sqrt(D) by default in the reference) */
    int32_t flags;      /* ARGUS_ATTN_* bits */
} argus_attn_shape;

/* argus_attn_shape.flags: feed the softmax weights to the V contraction as an fp16 hi + lo pair
 * (two MMAs), keeping ~22 bits of each weight instead of fp16's 11; costs ~12% at head_dim 128. */
#define ARGUS_ATTN_PRECISE_PV 1

/* Bytes of scratch argus_decode_attention needs for split-K partials (0 when n_splits == 1).  The
 * workspace begins with one arrival counter per (batch, kv_head, query group): it must be
 * zero-filled before its first use with a given shape (or after a call that reported an error);
 * every completed launch leaves the counters at zero again. */
int64_t argus_decode_attention_workspace_size(const argus_attn_shape* shape);

/* Chunk capacity: the largest number of tiles of an arena that one staged chunk may hold for
 * head dim D (the chunk list passed to argus_decode_attention must respect it); page_tokens and
 * layout as in argus_kv_arena. */
int argus_decode_attention_chunk_tiles(int tier, int layout, int page_tokens, int head_dim);

/* Bytes of one record of the record layout for a tier, page size and head dim. */
int argus_record_bytes(int tier, int page_tokens, int head_dim);

/* Decode attention over a paged KV cache held in mixed tiers, fused with the dequantization:
 * out = softmax(q K^T * scale) V for every query token, K/V read straight from the compressed
 * pages.  q: [B][H_q][q_len][D] fp16 (H_q = H_kv * group), out: same shape fp16, lse: optional
 * [B][H_q][q_len] fp32 natural-log sum-exp.  The chunk list covers the cached tokens in any order;
 * split_chunk0[s] .. split_chunk0[s+1] are the chunks of split s (n_splits + 1 entries, device).
 * chunks and split_chunk0 are device arrays; arenas is a host array copied into the launch.
 * tile_lse: optional [B*H_kv*ceil(group*q_len/8)][n_chunks][16][8] fp32 receiving, per tile of
 * each chunk and per query of each 8-query group, log2 of the tile's sum of exp2-scaled scores
 * (natural scores times log2 e); with lse it gives each page's share of the attention mass, the
 * signal of the reference's importance and resurrection policy (core/memory_manager.py:1453-1522).
 * workspace: device scratch of argus_decode_attention_workspace_size bytes (may be null when
 * n_splits == 1).
 * Replaces PagedDynamicKVCache.inplace_paged_attention, core/memory_manager.py:1317-1447 (its
 * dequantize-concatenate-softmax part), and the reconstruct-then-SDPA path of
 * get_all_keys_values + transformers' attention (core/memory_manager.py:1157-1315,
 * models/attention_wrapper.py:87-88), which it matches within fp32-accumulation tolerance. */
int argus_decode_attention(const argus_attn_shape* shape, const argus_kv_arena* arenas, const argus_kv_chunk* chunks,
                           const int32_t* split_chunk0, const uint16_t* q, uint16_t* out, float* lse, float* tile_lse,
                           void* workspace, argus_stream_t stream);

/* Allocation-free variant of argus_decode_attention, for callers that cannot allocate device memory
 * (a host that must not call cudaMalloc during decode, such as an embedding runtime holding a fixed
 * memory budget or code running inside a region where allocation is forbidden): the split-K
 * partials go to a fixed scratch array that the library holds in its own device memory (8 MiB,
 * argus_decode_attention_noalloc_capacity(); every GPU that loads the library keeps it until the
 * process exits), so nothing is allocated.  Arguments as argus_decode_attention without workspace;
 * shapes whose partials need more than the capacity fail with ARGUS_ERR_CAPACITY.  The first call on
 * a device looks up the array's device address (cudaGetSymbolAddress) once, with that device current,
 * so make that first call before any stream capture.  All calls on a device share the one array; each
 * call clears its split-arrival counters (an asynchronous memset on `stream`) and writes every
 * partial it reads, so nothing else has to start at zero.  Calls that overlap on the GPU (concurrent
 * streams) race on the array and must be serialised by the caller.
 * This entry point has no counterpart in the reference. */
int argus_decode_attention_noalloc(const argus_attn_shape* shape, const argus_kv_arena* arenas,
                                   const argus_kv_chunk* chunks, const int32_t* split_chunk0, const uint16_t* q,
                                   uint16_t* out, float* lse, float* tile_lse, argus_stream_t stream);
/* Bytes of the built-in scratch of argus_decode_attention_noalloc. */
int64_t argus_decode_attention_noalloc_capacity(void);

/* ---- KV-head-sharded decode with the output all-gather fused into the attention kernel ----
 * Rank r of `world` GPUs (one process each) holds KV heads [r*Hl, (r+1)*Hl) of every page
 * (Hl = shape.heads_kv; the reference lays a page out as one [B, H_kv, P, D] block per tier,
 * core/memory_manager.py:333-379, so every rank keeps the same page table).  The kernel that
 * finishes a (batch, kv_head, query group) writes its output rows straight into every rank's output
 * buffer at their place in the full [B][H_q total][q_len][D] layout (plain 16-byte stores to peer
 * memory mapped with CUDA IPC); argus_gather_wait, queued after it on the same stream, then adds one
 * to every rank's arrival counter (after a system-scope fence, with release semantics) and holds the
 * stream until every rank has signalled the step.  This replaces the local attention + NCCL
 * all-gather + head-order copy of a head-sharded step; the reference has no multi-GPU path. */
#define ARGUS_MAX_PEERS 8
typedef struct argus_peer_gather {
    int32_t world;                   /* ranks, 1 .. ARGUS_MAX_PEERS */
    int32_t rank;                    /* this rank */
    int32_t heads_kv_total;          /* H_kv of the whole layer: shape.heads_kv * world */
    int32_t parity;                  /* half of every rank's output pair this step writes: 0 or 1 */
    void* out[ARGUS_MAX_PEERS];      /* per rank, mapped in this process: fp16 [2][B][H_q total][q_len][D] */
    void* arrivals[ARGUS_MAX_PEERS]; /* per rank, mapped in this process: one uint64 arrival counter */
} argus_peer_gather;

/* argus_decode_attention for rank g->rank of a head-sharded layer, the output going to every rank
 * (see above) instead of a local `out`.  q is the full query [B][H_q total][q_len][D] (the same on
 * every rank; this rank reads its own heads' rows); lse, tile_lse and workspace stay local (this
 * rank's heads).
 * Follow each call with argus_gather_wait on the same stream.  Consecutive steps alternate `parity`,
 * so a rank one step ahead never overwrites rows its peers may still be reading.  The caller keeps
 * every rank's calls in the same order. */
int argus_decode_attention_gather(const argus_attn_shape* shape, const argus_kv_arena* arenas,
                                  const argus_kv_chunk* chunks, const int32_t* split_chunk0, const uint16_t* q,
                                  const argus_peer_gather* g, float* lse, float* tile_lse, void* workspace,
                                  argus_stream_t stream);
/* Arrivals every rank's counter receives per step (one signal from each rank): world. */
int64_t argus_gather_arrivals_per_step(int world);
/* Queues a one-thread kernel on `stream` that signals every rank of g (the step's rows of this rank
 * are stored) and then waits until this rank's counter reaches `target` (steps so far times
 * argus_gather_arrivals_per_step), polling at most max_polls times about 0.25 us apart; on timeout
 * it records ARGUS_ERR_TIMEOUT in the status word read by argus_device_status and returns. */
int argus_gather_wait(const argus_peer_gather* g, uint64_t target, int64_t max_polls, argus_stream_t stream);
/* Device memory another process can map: `bytes` zero-filled bytes (cudaMalloc) and their 64-byte
 * CUDA IPC handle in ipc_handle. */
int argus_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle);
/* Maps a peer's argus_peer_alloc memory into this process (peer access enabled lazily). */
int argus_peer_open(const void* ipc_handle, void** ptr);
/* Unmaps memory mapped by argus_peer_open. */
int argus_peer_close(void* ptr);
/* Frees memory from argus_peer_alloc (after every peer has closed its mapping). */
int argus_peer_free(void* ptr);

/* Self-test of the quantizers' fast exact quotient: for every finite fp16 x and positive finite
 * fp16 s, the quotient computed from the correctly rounded reciprocal of s with one FMA correction
 * is compared with the IEEE-rounded fp32 divide (equal values; a zero quotient may differ in sign,
 * which reaches no code); *mismatches (host) receives the count (0 when the fast path may stand in
 * for the divide).  Synchronises `stream`.  No counterpart in the
 * reference. */
int argus_selftest_fp16_quotients(unsigned long long* mismatches, argus_stream_t stream);

/* Self-test of the bounded device waits: one CTA waits, with the wait the decode kernel's staging
 * rings use, on an mbarrier that nothing ever completes, gives up after `polls` polls (1 .. 2^20)
 * and sets the status word to ARGUS_ERR_TIMEOUT as a timed-out ring consumer does; *gave_up (host)
 * receives 1.  The status stays set for argus_device_status to read; the context stays usable.
 * Synchronises `stream`.  No counterpart in the reference. */
int argus_selftest_wait_timeout(int64_t polls, int* gave_up, argus_stream_t stream);

/* Reads (and clears) the device-side status words that bounded waits in the kernels set on a
 * timeout, and argus_outlier_corrections on a bad sidecar; writes ARGUS_OK, ARGUS_ERR_TIMEOUT or
 * ARGUS_ERR_INVALID_ARGUMENT to *status after synchronising `stream`. */
int argus_device_status(int* status, argus_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* ARGUS_B200_H */
