// JL archive contraction: C[b] = A . X[b] for a shared fp16 operator A [M][K] and a batch of fp16
// pages X[b] [K][N] (sequence-axis projection W.X and reconstruction R.Y of
// core/memory_manager.py:1139-1141,1176-1178 and core/quantization.py:243,255).
// fp32 accumulation, one fp16 rounding of each output.
#include "common.cuh"

namespace argus {

constexpr int kJlTile = 16;

// Tiled CUDA-core version: a 16x16 output tile per block, A and X tiles staged in shared memory.
__global__ void jl_apply_simple_kernel(const __half* __restrict__ A, const __half* __restrict__ X, int64_t batch,
                                       int M, int K, int N, __half* __restrict__ C) {
    __shared__ float As[kJlTile][kJlTile + 1];
    __shared__ float Xs[kJlTile][kJlTile + 1];
    const int tiles_m = (M + kJlTile - 1) / kJlTile, tiles_n = (N + kJlTile - 1) / kJlTile;
    const int64_t tiles = batch * tiles_m * tiles_n;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        const int64_t b = t / (tiles_m * tiles_n);
        const int rem = (int)(t - b * tiles_m * tiles_n);
        const int tm = rem / tiles_n, tn = rem - tm * tiles_n;
        const int row = tm * kJlTile + threadIdx.y, col = tn * kJlTile + threadIdx.x;
        const __half* Xb = X + b * (int64_t)K * N;
        float acc = 0.0f;
        for (int k0 = 0; k0 < K; k0 += kJlTile) {
            const int ka = k0 + threadIdx.x, kx = k0 + threadIdx.y;
            As[threadIdx.y][threadIdx.x] = (row < M && ka < K) ? __half2float(A[(int64_t)row * K + ka]) : 0.0f;
            Xs[threadIdx.y][threadIdx.x] = (kx < K && col < N) ? __half2float(Xb[(int64_t)kx * N + col]) : 0.0f;
            __syncthreads();
#pragma unroll
            for (int k = 0; k < kJlTile; ++k) acc = fmaf(As[threadIdx.y][k], Xs[k][threadIdx.x], acc);
            __syncthreads();
        }
        if (row < M && col < N) C[b * (int64_t)M * N + (int64_t)row * N + col] = __float2half_rn(acc);
    }
}

}  // namespace argus

extern "C" int argus_jl_apply(const uint16_t* A, const uint16_t* X, int64_t batch, int M, int K, int N, uint16_t* C,
                              argus_stream_t stream) {
    if (!A || !X || !C) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    if (batch < 0 || M <= 0 || K <= 0 || N <= 0) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad size");
    if (batch == 0) return ARGUS_OK;
    const int64_t tiles = batch * ((M + 15) / 16) * ((N + 15) / 16);
    argus::jl_apply_simple_kernel<<<argus_grid_cap(tiles), dim3(16, 16), 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const __half*>(A), reinterpret_cast<const __half*>(X), batch, M, K, N,
        reinterpret_cast<__half*>(C));
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}
