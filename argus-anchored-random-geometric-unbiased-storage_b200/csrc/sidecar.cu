// Outlier sidecars: COO (b, h, t, d) int16 indices + fp16 values, as _demote_active_to_fp8 builds
// them (core/memory_manager.py:951-955) and as every reader scatters them back over a dequantized
// page (core/memory_manager.py:1190-1199, 1402-1409).
#include "common.cuh"

namespace argus {

// out[(b*H + h)*bh_stride + (tok0 + t)*D + d] = val for every entry; entries outside [B,H,P,D] are
// skipped and counted in *bad (when given).
__global__ void scatter_coo_kernel(__half* __restrict__ out, int64_t bh_stride, int64_t tok0, int B, int H, int P, int D,
                                   const int16_t* __restrict__ idx, const __half* __restrict__ vals, int64_t n,
                                   unsigned long long* bad) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int b = idx[4 * i], h = idx[4 * i + 1], t = idx[4 * i + 2], d = idx[4 * i + 3];
        if (b < 0 || b >= B || h < 0 || h >= H || t < 0 || t >= P || d < 0 || d >= D) {
            if (bad) atomicAdd(bad, 1ull);
            continue;
        }
        out[((int64_t)b * H + h) * bh_stride + (tok0 + t) * (int64_t)D + d] = vals[i];
    }
}

constexpr int kCompactThreads = 1024;

// Row-major compaction of a [B,H,P,D] mask into COO entries (the order of torch.nonzero), one CTA:
// each thread owns a contiguous run of elements, a block scan gives each run its output offset.
__global__ void __launch_bounds__(kCompactThreads)
outliers_to_coo_kernel(const uint8_t* __restrict__ mask, const __half* __restrict__ outv, int B, int H, int P, int D,
                       int16_t* __restrict__ idx_out, __half* __restrict__ vals_out, int64_t capacity,
                       int64_t* __restrict__ count_out) {
    __shared__ int64_t warp_tot[kCompactThreads / 32];
    __shared__ int64_t warp_off[kCompactThreads / 32];
    const int64_t n = (int64_t)B * H * P * D;
    const int64_t per_thread = (n + kCompactThreads - 1) / kCompactThreads;
    const int64_t lo = min(n, (int64_t)threadIdx.x * per_thread), hi = min(n, lo + per_thread);
    int64_t mine = 0;
    for (int64_t i = lo; i < hi; ++i) mine += mask[i] != 0;
    // inclusive scan within the warp, then across warps
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int64_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int64_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (threadIdx.x == 0) {
        int64_t acc = 0;
        for (int w = 0; w < kCompactThreads / 32; ++w) { warp_off[w] = acc; acc += warp_tot[w]; }
        *count_out = acc;
    }
    __syncthreads();
    int64_t pos = warp_off[warp] + incl - mine;
    for (int64_t i = lo; i < hi; ++i) {
        if (!mask[i]) continue;
        if (pos < capacity) {
            const int64_t d = i % D, r = i / D, t = r % P, r2 = r / P, h = r2 % H, b = r2 / H;
            idx_out[4 * pos] = (int16_t)b;
            idx_out[4 * pos + 1] = (int16_t)h;
            idx_out[4 * pos + 2] = (int16_t)t;
            idx_out[4 * pos + 3] = (int16_t)d;
            vals_out[pos] = outv[i];
        }
        ++pos;
    }
}

// ------------------------------------------------------- correction blocks for the fused attention
// Layout of one (b, h) block (NT = ceil(P / 16) tiles, NH = 8 NT + 1):
//     uint32 k_off[NH]    first key entry of token pair j (tokens 2j, 2j+1); k_off[8 NT] = key count
//     uint32 v_off[NH]    first value entry of (tile i, dim group g) at 8i + g, dim group g being
//                         dims [g D/8, (g+1) D/8); v_off[8 NT] = key count + value count
//     argus_outlier entries[]   key entries in (token, dim) order, then value entries ordered by tile,
//                               then dim, then token
// at byte offset  bh * 8 NH + 8 (key entries of earlier (b, h) + value entries of earlier (b, h))  of
// the page's buffer.  The offsets give each lane of the attention kernel its own run: key entries by
// the token pair whose scores a lane holds, value entries by the dims of the output it holds.  A
// row-major sidecar is already grouped by (b, h) and sorted by (token, dim), so every offset is a
// binary search or a count over one tile.

__device__ int g_side_status = 0;

__device__ __forceinline__ int64_t coo_row(const int16_t* idx, int64_t i, int H, int P) {
    return ((int64_t)idx[4 * i] * H + idx[4 * i + 1]) * P + idx[4 * i + 2];
}

// flag |= 1 when an entry lies outside [B,H,P,D] or precedes its predecessor in row-major order.
__global__ void outlier_validate_kernel(const int16_t* __restrict__ idx, int64_t n, int B, int H, int P, int D,
                                        int* flag) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int b = idx[4 * i], h = idx[4 * i + 1], t = idx[4 * i + 2], d = idx[4 * i + 3];
        bool bad = b < 0 || b >= B || h < 0 || h >= H || t < 0 || t >= P || d < 0 || d >= D;
        if (!bad && i > 0) {
            const int64_t prev = coo_row(idx, i - 1, H, P) * D + idx[4 * (i - 1) + 3];
            bad = prev >= coo_row(idx, i, H, P) * D + d;
        }
        if (bad) atomicOr(flag, 1);
    }
}

// first i in [lo, hi) with row(i) >= key (row = (b*H + h)*P + t)
__device__ __forceinline__ int64_t lower_row(const int16_t* idx, int64_t lo, int64_t hi, int64_t key, int H, int P) {
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (coo_row(idx, mid, H, P) < key) lo = mid + 1; else hi = mid;
    }
    return lo;
}

// One CTA per (b, h).
__global__ void outlier_blocks_kernel(const int16_t* __restrict__ k_idx, const __half* __restrict__ k_val, int64_t nk,
                                      const int16_t* __restrict__ v_idx, const __half* __restrict__ v_val, int64_t nv,
                                      const __half* __restrict__ k_deq, const __half* __restrict__ v_deq, int H,
                                      int P, int D, unsigned char* __restrict__ blocks,
                                      unsigned long long* __restrict__ block_addr, const int* __restrict__ flag) {
    const int bh = blockIdx.x;
    if (*flag) {
        if (threadIdx.x == 0) {
            block_addr[bh] = 0ull;
            if (bh == 0) atomicExch(&g_side_status, (int)ARGUS_ERR_INVALID_ARGUMENT);
        }
        return;
    }
    const int NT = (P + 15) >> 4, NH = 8 * NT + 1, DG = D / 8;
    const int64_t r0 = (int64_t)bh * P, r1 = r0 + P;
    const int64_t kb = lower_row(k_idx, 0, nk, r0, H, P), ke = lower_row(k_idx, kb, nk, r1, H, P);
    const int64_t vb = lower_row(v_idx, 0, nv, r0, H, P), ve = lower_row(v_idx, vb, nv, r1, H, P);
    const int64_t nkb = ke - kb, nvb = ve - vb;
    unsigned char* blk = blocks + (int64_t)bh * 8 * NH + 8 * (kb + vb);
    if (threadIdx.x == 0) block_addr[bh] = (nkb + nvb) > 0 ? (unsigned long long)(uintptr_t)blk : 0ull;
    if (nkb + nvb == 0) return;
    uint32_t* koff = reinterpret_cast<uint32_t*>(blk);
    uint32_t* voff = koff + NH;
    argus_outlier* ent = reinterpret_cast<argus_outlier*>(voff + NH);
    for (int j = threadIdx.x; j < NH; j += blockDim.x) {
        koff[j] = (uint32_t)(lower_row(k_idx, kb, ke, r0 + min((int64_t)P, 2 * (int64_t)j), H, P) - kb);
        if (j == 8 * NT) {
            voff[j] = (uint32_t)(nkb + nvb);
        } else {
            const int tile = j >> 3, g = j & 7;
            const int64_t t0 = lower_row(v_idx, vb, ve, r0 + 16 * (int64_t)tile, H, P);
            const int64_t t1 = lower_row(v_idx, t0, ve, r0 + min((int64_t)P, 16 * (int64_t)(tile + 1)), H, P);
            int64_t below = 0;
            for (int64_t i = t0; i < t1; ++i) below += v_idx[4 * i + 3] < g * DG;
            voff[j] = (uint32_t)(nkb + (t0 - vb) + below);
        }
    }
    const int64_t deq_bh = (int64_t)bh * P * D;
    for (int64_t e = threadIdx.x; e < nkb; e += blockDim.x) {
        const int64_t i = kb + e;
        const int t = k_idx[4 * i + 2], d = k_idx[4 * i + 3];
        argus_outlier o;
        o.tok = (uint16_t)t;
        o.dim = (uint16_t)d;
        o.delta = __half2float(k_val[i]) - __half2float(k_deq[deq_bh + (int64_t)t * D + d]);
        ent[e] = o;
    }
    for (int64_t e = threadIdx.x; e < nvb; e += blockDim.x) {
        const int64_t i = vb + e;
        const int t = v_idx[4 * i + 2], d = v_idx[4 * i + 3];
        // position within the tile: entries of smaller dim, or of the same dim and an earlier token
        const int tile = t >> 4;
        const int64_t t0 = lower_row(v_idx, vb, ve, r0 + 16 * (int64_t)tile, H, P);
        const int64_t t1 = lower_row(v_idx, t0, ve, r0 + min((int64_t)P, 16 * (int64_t)(tile + 1)), H, P);
        int64_t rank = 0;
        for (int64_t j = t0; j < t1; ++j) {
            const int dj = v_idx[4 * j + 3];
            rank += (dj < d) || (dj == d && j < i);
        }
        argus_outlier o;
        o.tok = (uint16_t)t;
        o.dim = (uint16_t)d;
        o.delta = __half2float(v_val[i]) - __half2float(v_deq[deq_bh + (int64_t)t * D + d]);
        ent[nkb + (t0 - vb) + rank] = o;
    }
}

}  // namespace argus

int argus_side_take_status(int* status, cudaStream_t st) {
    int v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(&v, argus::g_side_status, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(argus::g_side_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return argus_set_cuda_error(e);
    *status = v;
    return ARGUS_OK;
}

extern "C" {

int64_t argus_outlier_blocks_bytes(int32_t bh, int32_t page_tokens, int64_t nk, int64_t nv) {
    if (bh <= 0 || page_tokens <= 0 || nk < 0 || nv < 0) return 0;
    return (int64_t)bh * 8 * (8 * ((page_tokens + 15) / 16) + 1) + 8 * (nk + nv) + 16;
}

int argus_outlier_corrections(const int16_t* k_idx, const uint16_t* k_val, int64_t nk, const int16_t* v_idx,
                              const uint16_t* v_val, int64_t nv, const uint16_t* k_deq, const uint16_t* v_deq,
                              int32_t batch, int32_t heads, int32_t page_tokens, int32_t head_dim, void* blocks,
                              uint64_t* block_addr, argus_stream_t stream) {
    if (batch <= 0 || heads <= 0 || page_tokens <= 0 || head_dim <= 0 || nk < 0 || nv < 0 || page_tokens > 32767 ||
        head_dim > 32767 || (int64_t)batch * heads > 65535)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad sizes");
    if (!block_addr || !k_deq || !v_deq || !blocks || (nk > 0 && (!k_idx || !k_val)) || (nv > 0 && (!v_idx || !v_val)))
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    if (!argus_aligned(blocks, 16) || !argus_aligned(block_addr, 8) || (nk > 0 && !argus_aligned(k_idx, 8)) ||
        (nv > 0 && !argus_aligned(v_idx, 8)) || !argus_aligned(k_val ? (const void*)k_val : blocks, 2) ||
        !argus_aligned(v_val ? (const void*)v_val : blocks, 2))
        return argus_set_error(ARGUS_ERR_MISALIGNED, "blocks must be 16-byte aligned, indices 8-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    // the validation flag: the 16 bytes past the last entry (counted by argus_outlier_blocks_bytes)
    int* flag = reinterpret_cast<int*>(static_cast<unsigned char*>(blocks) +
                                       argus_outlier_blocks_bytes(batch * heads, page_tokens, nk, nv) - 16);
    cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(int), st);
    if (e != cudaSuccess) return argus_set_cuda_error(e);
    if (nk > 0)
        argus::outlier_validate_kernel<<<argus_grid_cap((nk + 255) / 256), 256, 0, st>>>(k_idx, nk, batch, heads,
                                                                                         page_tokens, head_dim, flag);
    if (nv > 0)
        argus::outlier_validate_kernel<<<argus_grid_cap((nv + 255) / 256), 256, 0, st>>>(v_idx, nv, batch, heads,
                                                                                         page_tokens, head_dim, flag);
    argus::outlier_blocks_kernel<<<batch * heads, 256, 0, st>>>(
        k_idx, reinterpret_cast<const __half*>(k_val), nk, v_idx, reinterpret_cast<const __half*>(v_val), nv,
        reinterpret_cast<const __half*>(k_deq), reinterpret_cast<const __half*>(v_deq), heads, page_tokens, head_dim,
        static_cast<unsigned char*>(blocks), reinterpret_cast<unsigned long long*>(block_addr), flag);
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

int argus_scatter_coo(uint16_t* out, int64_t out_bh_stride, int64_t out_tok0, int B, int H, int P, int D,
                      const int16_t* idx, const uint16_t* vals, int64_t n, argus_stream_t stream) {
    if (n < 0 || B <= 0 || H <= 0 || P <= 0 || D <= 0 || out_tok0 < 0)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad sizes");
    if (n == 0) return ARGUS_OK;
    if (!out || !idx || !vals) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    if (!argus_aligned(idx, 8)) return argus_set_error(ARGUS_ERR_MISALIGNED, "indices must be 8-byte aligned");
    argus::scatter_coo_kernel<<<argus_grid_cap((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<__half*>(out), out_bh_stride, out_tok0, B, H, P, D, idx, reinterpret_cast<const __half*>(vals),
        n, nullptr);
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

int argus_outliers_to_coo(const uint8_t* mask, const uint16_t* outv, int B, int H, int P, int D, int16_t* idx_out,
                          uint16_t* vals_out, int64_t capacity, int64_t* count_out, argus_stream_t stream) {
    if (!mask || !outv || !count_out || (capacity > 0 && (!idx_out || !vals_out)))
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    if (B <= 0 || H <= 0 || P <= 0 || D <= 0 || B > 32767 || H > 32767 || P > 32767 || D > 32767)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "dims must fit int16 indices");
    argus::outliers_to_coo_kernel<<<1, argus::kCompactThreads, 0, (cudaStream_t)stream>>>(
        mask, reinterpret_cast<const __half*>(outv), B, H, P, D, idx_out, reinterpret_cast<__half*>(vals_out), capacity,
        count_out);
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}

}  // extern "C"
