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

}  // namespace argus

extern "C" {

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
