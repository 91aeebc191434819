// SIMT GEMMs: the few-row GEMV used at batch 1 (the reference's gemv_nt role, 11_gemv.metal:45-128, M <= 8
// there) and a tiled FFMA GEMM for the fp32 engine at larger M. C = epilogue(A . W^T), W [N, K] row-major.
//
// The GEMV is bound by streaming W from HBM once (A is a few rows). One warp owns one output column; each lane
// issues all of its 16-byte weight loads for a block of U chunks at once, and the first block is issued before the
// grid-dependency wait, since W does not depend on the previous kernel, so the weight fetch overlaps the kernel
// before. A is staged once per CTA in shared memory.
#include "common.cuh"
#include "kernels.h"

namespace ud {
namespace {

__device__ __forceinline__ float apply_epi_scalar(const GemmEpilogue& epi, float acc, int m, int n) {
    float y = acc + (epi.bias ? epi.bias[n] : 0.f);
    if (epi.act == ACT_RELU) y = fmaxf(y, 0.f);
    else if (epi.act == ACT_SILU) y = epi.out_bf16 ? x_sigmoid_bf16out(y, y) : silu(y);
    y *= epi.out_scale;
    if (epi.residual) y += epi.res_scale * epi.residual[static_cast<size_t>(m) * epi.ldr + n];
    return y;
}

__device__ __forceinline__ void store_scalar(const GemmEpilogue& epi, int m, int n, float y) {
    if (epi.out_bf16)
        reinterpret_cast<bf16*>(epi.out)[static_cast<size_t>(m) * epi.ldo + n] = __float2bfloat16_rn(y);
    else
        reinterpret_cast<float*>(epi.out)[static_cast<size_t>(m) * epi.ldo + n] = y;
}

// One warp per output column; rows in chunks of MR held in registers. Weight rows stream once per chunk
// with 16-byte loads (4 in flight per lane).
template <typename T, int MR, bool VEC>
__global__ void __launch_bounds__(256) gemv_rows_kernel(const T* __restrict__ A, int lda, const T* __restrict__ W,
                                                        int M, int N, int K, const GemmEpilogue epi) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int VW = VEC ? Vec16<T>::N : 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x * 8 + warp;
    if (n >= N) return;
    const T* w = W + static_cast<size_t>(n) * K;
    for (int m0 = 0; m0 < M; m0 += MR) {
        const int mr = min(MR, M - m0);
        float acc[MR];
#pragma unroll
        for (int r = 0; r < MR; ++r) acc[r] = 0.f;
        for (int k = lane * VW; k < K; k += 32 * VW) {
            float wv[VW];
            if constexpr (VEC) load16<T>(w + k, wv);
            else wv[0] = to_f<T>(w[k]);
#pragma unroll
            for (int r = 0; r < MR; ++r) {
                if (r < mr) {
                    float av[VW];
                    if constexpr (VEC) load16<T>(A + static_cast<size_t>(m0 + r) * lda + k, av);
                    else av[0] = to_f<T>(A[static_cast<size_t>(m0 + r) * lda + k]);
#pragma unroll
                    for (int j = 0; j < VW; ++j) acc[r] = fmaf(wv[j], av[j], acc[r]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < MR; ++r) acc[r] = warp_sum(acc[r]);
        if (lane == 0) {
            for (int r = 0; r < mr; ++r) store_scalar(epi, m0 + r, n, apply_epi_scalar(epi, acc[r], m0 + r, n));
        }
    }
}

constexpr int kGemvWarps = 8;
constexpr int kGemvStageSmem = 64 * 1024;   // largest A staging (M x K x sizeof(T)) in shared memory

// Where the GEMV's A rows come from: global memory (read by every warp), or staged once per CTA into shared
// memory by 16-byte loads of all threads (one memory round trip instead of one per chunk).
enum GemvSrc { kSrcGlobal = 0, kSrcStaged = 1 };
// Few-row GEMV, M <= MR rows. K % VW == 0 and 16-byte aligned A, W and lda (checked by the host).
// U 16-byte weight chunks per lane are in flight at once (4 for K <= 1024 bf16, 16 above, where the extra
// registers are worth it).
template <typename T, int MR, int SRC, int U>
__global__ void __launch_bounds__(256) gemv_kernel(const T* __restrict__ A, int lda, const T* __restrict__ W, int M,
                                                   int N, int K, const GemmEpilogue epi) {
    constexpr int VW = Vec16<T>::N;
    extern __shared__ __align__(16) unsigned char gemv_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x * kGemvWarps + warp;
    const bool has_col = n < N;
    const T* w = W + static_cast<size_t>(has_col ? n : 0) * K;
    const int nchunks = K / VW;
    uint4 wr[U];
    auto load_w = [&](int base) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = base + u * 32 + lane;
            wr[u] = (has_col && c < nchunks) ? __ldcs(reinterpret_cast<const uint4*>(w) + c) : make_uint4(0, 0, 0, 0);
        }
    };
    pdl_launch_dependents();
    load_w(0);
    pdl_wait();
    const T* a_rows = A;
    int a_ld = lda;
    if constexpr (SRC == kSrcStaged) {
        T* as = reinterpret_cast<T*>(gemv_smem);
        const int total = M * nchunks;
        for (int i = threadIdx.x; i < total; i += 256) {
            const int r = i / nchunks, c = i - r * nchunks;
            reinterpret_cast<uint4*>(as)[i] =
                *reinterpret_cast<const uint4*>(A + static_cast<size_t>(r) * lda + static_cast<size_t>(c) * VW);
        }
        __syncthreads();
        a_rows = as;
        a_ld = K;
    }
    if (!has_col) return;
    float acc[MR];
#pragma unroll
    for (int r = 0; r < MR; ++r) acc[r] = 0.f;
    for (int base = 0; base < nchunks; base += U * 32) {
        if (base > 0) load_w(base);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = base + u * 32 + lane;
            if (c < nchunks) {
                float wf[VW];
                if constexpr (sizeof(T) == 4) {
                    wf[0] = __uint_as_float(wr[u].x); wf[1] = __uint_as_float(wr[u].y);
                    wf[2] = __uint_as_float(wr[u].z); wf[3] = __uint_as_float(wr[u].w);
                } else {
                    const bf16* h = reinterpret_cast<const bf16*>(&wr[u]);
#pragma unroll
                    for (int j = 0; j < VW; ++j) wf[j] = __bfloat162float(h[j]);
                }
#pragma unroll
                for (int r = 0; r < MR; ++r) {
                    if (r < M) {
                        float av[VW];
                        load16<T>(a_rows + static_cast<size_t>(r) * a_ld + static_cast<size_t>(c) * VW, av);
#pragma unroll
                        for (int j = 0; j < VW; ++j) acc[r] = fmaf(wf[j], av[j], acc[r]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < MR; ++r) {
        const float v = warp_sum(acc[r]);
        if (lane == r && r < M) store_scalar(epi, r, n, apply_epi_scalar(epi, v, r, n));
    }
}

// 64x64 output tile, 256 threads, 4x4 per thread, K step 16 through shared memory (fp32 engine, M > 16).
template <typename T>
__global__ void __launch_bounds__(256) gemm_tiled_kernel(const T* __restrict__ A, int lda, const T* __restrict__ W,
                                                         int M, int N, int K, const GemmEpilogue epi) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float As[16][64 + 4];
    __shared__ float Ws[16][64 + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int i = threadIdx.x; i < 64 * 16; i += 256) {
            const int r = i >> 4, kk = i & 15;
            const int m = m0 + r, n = n0 + r, k = k0 + kk;
            As[kk][r] = (m < M && k < K) ? to_f<T>(A[static_cast<size_t>(m) * lda + k]) : 0.f;
            Ws[kk][r] = (n < N && k < K) ? to_f<T>(W[static_cast<size_t>(n) * K + k]) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) { a[i] = As[kk][ty * 4 + i]; b[i] = Ws[kk][tx * 4 + i]; }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
            if (m < M && n < N) store_scalar(epi, m, n, apply_epi_scalar(epi, acc[i][j], m, n));
        }
}

template <typename T, int MR, int U>
void launch_gemv_u(const T* A, int lda, const T* W, int M, int N, int K, const GemmEpilogue& epi, cudaStream_t s) {
    static size_t attr[kMaxDevices] = {};
    ensure_dyn_smem(gemv_kernel<T, MR, kSrcStaged, U>, kGemvStageSmem, attr);
    const dim3 grid((N + kGemvWarps - 1) / kGemvWarps), block(256);
    const size_t smem = static_cast<size_t>(M) * K * sizeof(T);
    if (smem <= static_cast<size_t>(kGemvStageSmem))
        launch_pdl(gemv_kernel<T, MR, kSrcStaged, U>, grid, block, smem, s, A, lda, W, M, N, K, epi);
    else launch_pdl(gemv_kernel<T, MR, kSrcGlobal, U>, grid, block, 0, s, A, lda, W, M, N, K, epi);
}

template <typename T, int MR>
void launch_gemv(const T* A, int lda, const T* W, int M, int N, int K, const GemmEpilogue& epi, cudaStream_t s) {
    if (K / Vec16<T>::N <= 4 * 32) launch_gemv_u<T, MR, 4>(A, lda, W, M, N, K, epi, s);
    else launch_gemv_u<T, MR, 16>(A, lda, W, M, N, K, epi, s);
}

}  // namespace

template <typename TA, typename TW>
void gemm_simt(const TA* A, int lda, const TW* W, int M, int N, int K, const GemmEpilogue& epi, cudaStream_t s) {
    static_assert(std::is_same<TA, TW>::value, "A and W share a type");
    if (M <= 16) {
        constexpr int VW = Vec16<TA>::N;
        const bool vec = K % VW == 0 && lda % VW == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(W) & 15) == 0;
        if (vec) {
            if (M <= 2) launch_gemv<TA, 2>(A, lda, W, M, N, K, epi, s);
            else if (M <= 4) launch_gemv<TA, 4>(A, lda, W, M, N, K, epi, s);
            else if (M <= 8) launch_gemv<TA, 8>(A, lda, W, M, N, K, epi, s);
            else launch_gemv<TA, 16>(A, lda, W, M, N, K, epi, s);
        } else {
            launch_pdl(gemv_rows_kernel<TA, 8, false>, dim3((N + 7) / 8), dim3(256), 0, s, A, lda, W, M, N, K, epi);
        }
    } else {
        dim3 grid((N + 63) / 64, (M + 63) / 64);
        launch_pdl(gemm_tiled_kernel<TA>, dim3(grid), dim3(256), 0, s, A, lda, W, M, N, K, epi);
    }
}

template void gemm_simt<float, float>(const float*, int, const float*, int, int, int, const GemmEpilogue&, cudaStream_t);
template void gemm_simt<bf16, bf16>(const bf16*, int, const bf16*, int, int, int, const GemmEpilogue&, cudaStream_t);

}  // namespace ud
