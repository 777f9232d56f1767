// JL archive contraction: C[b] = A . X[b] for a shared fp16 operator A [M][K] and a batch of fp16
// pages X[b] [K][N] (sequence-axis projection W.X and reconstruction R.Y of
// core/memory_manager.py:1139-1141,1176-1178 and core/quantization.py:243,255).
// fp32 accumulation, one fp16 rounding of each output.
//
// Shapes with M % 128 == 0, K % 64 == 0 and N % 16 == 0 (N <= 256) run on the 5th-generation
// tensor cores: one CTA per 128-row tile of one page, the fp32 accumulator in tensor memory
// (tcgen05.mma, kind::f16, A and B^T K-major in shared memory without swizzle), 64-deep K stages
// completed through tcgen05.commit on an mbarrier; other shapes (small pages) use a CUDA-core
// kernel.
#include "common.cuh"

namespace argus {

__device__ int g_jl_status = 0;  // ARGUS_ERR_TIMEOUT after a bounded wait ran out

// Two fp32 bit patterns -> one fp16x2 word (round to nearest even).
__device__ __forceinline__ uint32_t pack2(uint32_t lo, uint32_t hi) {
    __half2 h = __floats2half2_rn(__uint_as_float(lo), __uint_as_float(hi));
    return *reinterpret_cast<uint32_t*>(&h);
}

namespace tc {

constexpr int kM = 128;      // rows per CTA = tensor-memory lanes
constexpr int kKT = 64;      // K per shared-memory stage (4 MMAs of K = 16)
constexpr int kThreads = 128;
constexpr long long kSpinLimit = 1ll << 26;

__host__ __device__ constexpr int xrow_bytes(int N) { return 2 * N + 16; }  // staging rows, padded
__host__ __device__ constexpr size_t smem_bytes(int N) {
    return (size_t)kM * kKT * 2 + (size_t)N * kKT * 2 + (size_t)kKT * xrow_bytes(N) + 64;
}
__host__ __device__ constexpr int tmem_cols(int N) { return N <= 32 ? 32 : (N <= 64 ? 64 : (N <= 128 ? 128 : 256)); }

// Shared-memory matrix descriptor (tcgen05): start address, leading-dimension byte offset (next
// 8x16-byte core matrix along K), stride-dimension byte offset (next 8-row group), version 1,
// no swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor, kind::f16: fp32 accumulator, fp16 A and B, both K-major, N and M.
__host__ __device__ constexpr uint32_t instr_desc(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t phase) {
    for (long long i = 0; i < kSpinLimit; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(bar), "r"(phase)
            : "memory");
        if (ok) return true;
    }
    return false;
}

__global__ void __launch_bounds__(kThreads) jl_apply_tc_kernel(const __half* __restrict__ A, const __half* __restrict__ X,
                                                               int M, int K, int N, __half* __restrict__ C) {
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* a_tile = smem;                                   // [M 128 x K 64] canonical K-major
    unsigned char* b_tile = a_tile + kM * kKT * 2;                  // [N x K 64] canonical K-major (B^T)
    unsigned char* x_stage = b_tile + (size_t)N * kKT * 2;          // [K 64][N] row-major, padded rows
    uint64_t* mbar = reinterpret_cast<uint64_t*>(x_stage + (size_t)kKT * xrow_bytes(N));
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mbar + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tiles_m = M / kM;
    const int64_t b = blockIdx.x / tiles_m;
    const int m0 = (int)(blockIdx.x - b * tiles_m) * kM;
    const __half* Xb = X + b * (int64_t)K * N;
    const int ncols = tmem_cols(N);
    const uint32_t bar = smem_u32(mbar);

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(ncols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        mbar_init(bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem_d = *tmem_slot;

    const uint32_t a_base = smem_u32(a_tile), b_base = smem_u32(b_tile), x_base = smem_u32(x_stage);
    const uint32_t idesc = instr_desc(kM, N);
    const int nk = K / kKT;
    const int xchunks = N / 8;  // 16-byte chunks per staging row
    // Every wait's outcome is voted over the CTA (__syncthreads_and), so all threads leave the k-loop
    // on the same iteration and the barriers, the warp-collective tensor-memory loads and the
    // deallocation below are reached by whole warps.  `pending`: parity of the last committed MMA
    // group not yet seen complete (-1: none).
    bool ok = true;
    int pending = -1;
    for (int kt = 0; kt < nk; ++kt) {
        if (kt > 0) {
            // previous MMAs done with the tiles
            ok = __syncthreads_and(mbar_wait(bar, (uint32_t)((kt - 1) & 1)) ? 1 : 0) != 0;
            if (!ok) break;
            pending = -1;
        }
        // A tile: row m, 8-element group g -> core matrix (m / 8, g) row m % 8
        for (int idx = tid; idx < kM * (kKT / 8); idx += kThreads) {
            const int m = idx >> 3, g = idx & 7;
            cp_async16(a_base + (uint32_t)((m >> 3) * 1024 + g * 128 + (m & 7) * 16),
                       A + (int64_t)(m0 + m) * K + kt * kKT + g * 8);
        }
        // X tile rows k (N contiguous) into the padded staging rows
        for (int idx = tid; idx < kKT * xchunks; idx += kThreads) {
            const int r = idx / xchunks, c = idx - r * xchunks;
            cp_async16(x_base + (uint32_t)(r * xrow_bytes(N) + c * 16), Xb + (int64_t)(kt * kKT + r) * N + c * 8);
        }
        asm volatile("cp.async.commit_group;\n cp.async.wait_group 0;" ::: "memory");
        __syncthreads();
        // B^T core matrices (n-group, k-group) = transposed 8x8 blocks of the staged X, four per ldmatrix
        for (int op = warp; op < N / 4; op += kThreads / 32) {
            const int i = lane >> 3, r = lane & 7;
            const int core = op * 4 + i, ng = core >> 3, kg = core & 7;
            uint32_t d0, d1, d2, d3;
            asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                         : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
                         : "r"(x_base + (uint32_t)((kg * 8 + r) * xrow_bytes(N) + ng * 16)));
            const uint32_t d[4] = {d0, d1, d2, d3};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int cq = op * 4 + q;
                const uint32_t dst = b_base + (uint32_t)((cq >> 3) * 1024 + (cq & 7) * 128 + lane * 4);
                asm volatile("st.shared.b32 [%0], %1;" ::"r"(dst), "r"(d[q]) : "memory");
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
            for (int s = 0; s < kKT / 16; ++s) {
                const uint64_t ad = smem_desc(a_base + s * 256, 128, 1024);
                const uint64_t bd = smem_desc(b_base + s * 256, 128, 1024);
                const uint32_t acc = (kt > 0 || s > 0) ? 1u : 0u;
                asm volatile(
                    "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                    " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
                    "l"(ad), "l"(bd), "r"(idesc), "r"(acc));
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                         : "memory");
        }
        pending = kt & 1;
    }
    if (ok) {
        ok = __syncthreads_and(mbar_wait(bar, (uint32_t)((nk - 1) & 1)) ? 1 : 0) != 0;
        if (ok) pending = -1;
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok) {
        // epilogue: warp w reads tensor-memory lanes 32w .. 32w+31 (rows), 32 columns at a time
        const int m = m0 + warp * 32 + lane;
        __half* crow = C + (b * (int64_t)M + m) * N;
        for (int c0 = 0; c0 < N; c0 += 32) {
            uint32_t v[32];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                  "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                  "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
                  "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
                  "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                : "r"(tmem_d + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            const int nv = (N - c0) < 32 ? (N - c0) : 32;  // N % 16 == 0: 16 or 32
            for (int j = 0; j < nv; j += 8) {
                uint4 w;
                w.x = pack2(v[j], v[j + 1]); w.y = pack2(v[j + 2], v[j + 3]);
                w.z = pack2(v[j + 4], v[j + 5]); w.w = pack2(v[j + 6], v[j + 7]);
                *reinterpret_cast<uint4*>(crow + c0 + j) = w;
            }
        }
    } else {
        if (tid == 0) atomicExch(&g_jl_status, (int)ARGUS_ERR_TIMEOUT);
        // MMAs still in flight write tensor memory: give them one more bounded wait before it is freed
        if (pending >= 0) (void)__syncthreads_and(mbar_wait(bar, (uint32_t)pending) ? 1 : 0);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(ncols));
    }
}

}  // namespace tc

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

// Reads and clears the JL kernels' status word (ARGUS_OK or ARGUS_ERR_TIMEOUT) after synchronising.
int argus_jl_take_status(int* status, cudaStream_t st) {
    int v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(&v, argus::g_jl_status, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(argus::g_jl_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return argus_set_cuda_error(e);
    *status = v;
    return ARGUS_OK;
}

extern "C" int argus_jl_apply(const uint16_t* A, const uint16_t* X, int64_t batch, int M, int K, int N, uint16_t* C,
                              argus_stream_t stream) {
    if (!A || !X || !C) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    if (batch < 0 || M <= 0 || K <= 0 || N <= 0) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad size");
    if (batch == 0) return ARGUS_OK;
    const bool tc_shape = M % argus::tc::kM == 0 && K % argus::tc::kKT == 0 && N % 16 == 0 && N <= 256 &&
                          argus_aligned(A, 16) && argus_aligned(X, 16) && argus_aligned(C, 16) &&
                          batch * (M / argus::tc::kM) <= 0x7fffffffLL;
    if (tc_shape) {
        const size_t smem = argus::tc::smem_bytes(N);
        cudaError_t e = cudaFuncSetAttribute(argus::tc::jl_apply_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return argus_set_cuda_error(e);
        argus::tc::jl_apply_tc_kernel<<<(unsigned)(batch * (M / argus::tc::kM)), argus::tc::kThreads, smem,
                                        (cudaStream_t)stream>>>(reinterpret_cast<const __half*>(A),
                                                                reinterpret_cast<const __half*>(X), M, K, N,
                                                                reinterpret_cast<__half*>(C));
        ARGUS_CHECK_LAUNCH();
        return ARGUS_OK;
    }
    const int64_t tiles = batch * ((M + 15) / 16) * ((N + 15) / 16);
    argus::jl_apply_simple_kernel<<<argus_grid_cap(tiles), dim3(16, 16), 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const __half*>(A), reinterpret_cast<const __half*>(X), batch, M, K, N,
        reinterpret_cast<__half*>(C));
    ARGUS_CHECK_LAUNCH();
    return ARGUS_OK;
}
