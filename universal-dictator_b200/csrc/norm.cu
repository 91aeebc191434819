// LayerNorm over rows (eps 1e-5), one warp per row, fp32 statistics (two passes over registers).
// Replaces layer_norm_f32 (Sources/DictatorEngine/Metal/20_conformer.metal:26-49); `layer_norm2` fuses a
// layer's norm_out with the next layer's norm_feed_forward1 (FastConformer.swift:320 then :276).
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace ud {
namespace {

// D = 128 * NV: each lane holds NV float4 of its row (D <= 1024).
#define UD_LN_DISPATCH(KERNEL, ...)                                                              \
    switch (D / 128) {                                                                           \
        case 1: launch_pdl(KERNEL<TO, 1>, dim3((M + 7) / 8), dim3(256), 0, s, __VA_ARGS__); break;                   \
        case 2: launch_pdl(KERNEL<TO, 2>, dim3((M + 7) / 8), dim3(256), 0, s, __VA_ARGS__); break;                   \
        case 4: launch_pdl(KERNEL<TO, 4>, dim3((M + 7) / 8), dim3(256), 0, s, __VA_ARGS__); break;                   \
        case 6: launch_pdl(KERNEL<TO, 6>, dim3((M + 7) / 8), dim3(256), 0, s, __VA_ARGS__); break;                   \
        default: launch_pdl(KERNEL<TO, 8>, dim3((M + 7) / 8), dim3(256), 0, s, __VA_ARGS__); break;                  \
    }

template <typename TO>
__device__ __forceinline__ void store4(TO* p, const float* v) {
    if constexpr (std::is_same<TO, float>::value) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
        __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
        __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&a);
        u.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(p) = u;
    }
}

template <int NV>
__device__ __forceinline__ void row_stats(const float (&v)[NV][4], int D, float& mean, float& rstd) {
    constexpr int nv = NV;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < nv; ++i) s += v[i][0] + v[i][1] + v[i][2] + v[i][3];
    mean = warp_sum(s) / static_cast<float>(D);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < nv; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float d = v[i][j] - mean;
            q += d * d;
        }
    const float var = warp_sum(q) / static_cast<float>(D);
    rstd = rsqrtf(var + 1e-5f);
}

// Copies gamma and beta (D <= 1024 floats each) into shared memory: the CTA does it before it waits for the
// previous kernel (they are weights), so the affine step after the row statistics reads shared memory instead of
// making another round trip to L2.
__device__ __forceinline__ void stage_affine(const float* __restrict__ g, const float* __restrict__ b, float* sg,
                                             float* sb, int D) {
    for (int c = threadIdx.x * 4; c < D; c += blockDim.x * 4) {
        *reinterpret_cast<float4*>(sg + c) = *reinterpret_cast<const float4*>(g + c);
        *reinterpret_cast<float4*>(sb + c) = *reinterpret_cast<const float4*>(b + c);
    }
}

// gamma/beta for one float4 of this lane's columns.
__device__ __forceinline__ void load_affine4(const float* g, const float* b, int c, float (&gg)[4],
                                             float (&bb)[4]) {
    const float4 g4 = *reinterpret_cast<const float4*>(g + c), b4 = *reinterpret_cast<const float4*>(b + c);
    gg[0] = g4.x; gg[1] = g4.y; gg[2] = g4.z; gg[3] = g4.w;
    bb[0] = b4.x; bb[1] = b4.y; bb[2] = b4.z; bb[3] = b4.w;
}

template <int NV>
__device__ __forceinline__ void load_row(const float* xr, int lane, float (&v)[NV][4]) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const float4 t = *reinterpret_cast<const float4*>(xr + (i * 32 + lane) * 4);
        v[i][0] = t.x; v[i][1] = t.y; v[i][2] = t.z; v[i][3] = t.w;
    }
}

template <typename TO, int NV>
__global__ void __launch_bounds__(256) ln_kernel(const float* x, const float* __restrict__ g,
                                                 const float* __restrict__ b, TO* y, int M, int D,
                                                 unsigned long long* timer) {
    pdl_launch_dependents();
    __shared__ __align__(16) float sg[1024], sb[1024];
    stage_affine(g, b, sg, sb, D);
    __syncthreads();
    pdl_wait();
    if (threadIdx.x == 0) timer_start(timer);
    // x and y may alias (in-place): each warp reads its whole row before writing it.
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + warp;
    if (row >= M) return;
    float v[NV][4];
    load_row<NV>(x + static_cast<size_t>(row) * D, lane, v);
    float mean, rstd;
    row_stats<NV>(v, D, mean, rstd);
    TO* yr = y + static_cast<size_t>(row) * D;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        float gg[4], bb[4], o[4];
        load_affine4(sg, sb, (i * 32 + lane) * 4, gg, bb);
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = (v[i][j] - mean) * rstd * gg[j] + bb[j];
        store4<TO>(yr + (i * 32 + lane) * 4, o);
    }
    if (lane == 0) timer_end(timer);
}

template <typename TO, int NV>
__global__ void __launch_bounds__(256) ln2_kernel(float* __restrict__ x, const float* __restrict__ g1,
                                                  const float* __restrict__ b1, const float* __restrict__ g2,
                                                  const float* __restrict__ b2, TO* __restrict__ y, int M, int D,
                                                  unsigned long long* timer) {
    pdl_launch_dependents();
    __shared__ __align__(16) float sg1[1024], sb1[1024], sg2[1024], sb2[1024];
    stage_affine(g1, b1, sg1, sb1, D);
    stage_affine(g2, b2, sg2, sb2, D);
    __syncthreads();
    pdl_wait();
    if (threadIdx.x == 0) timer_start(timer);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + warp;
    if (row >= M) return;
    float* xr = x + static_cast<size_t>(row) * D;
    float v[NV][4];
    load_row<NV>(xr, lane, v);
    float mean, rstd;
    row_stats<NV>(v, D, mean, rstd);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        float gg[4], bb[4];
        load_affine4(sg1, sb1, (i * 32 + lane) * 4, gg, bb);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[i][j] = (v[i][j] - mean) * rstd * gg[j] + bb[j];
        *reinterpret_cast<float4*>(xr + (i * 32 + lane) * 4) = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
    }
    row_stats<NV>(v, D, mean, rstd);
    TO* yr = y + static_cast<size_t>(row) * D;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        float gg[4], bb[4], o[4];
        load_affine4(sg2, sb2, (i * 32 + lane) * 4, gg, bb);
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = (v[i][j] - mean) * rstd * gg[j] + bb[j];
        store4<TO>(yr + (i * 32 + lane) * 4, o);
    }
    if (lane == 0) timer_end(timer);
}

}  // namespace

template <typename TO>
void layer_norm(const float* x, const float* g, const float* b, TO* y, int M, int D, cudaStream_t s,
                unsigned long long* timer) {
    if (M <= 0) return;
    UD_LN_DISPATCH(ln_kernel, x, g, b, y, M, D, timer);
}

template <typename TO>
void layer_norm2(float* x, const float* g1, const float* b1, const float* g2, const float* b2, TO* y, int M, int D,
                 cudaStream_t s, unsigned long long* timer) {
    if (M <= 0) return;
    UD_LN_DISPATCH(ln2_kernel, x, g1, b1, g2, b2, y, M, D, timer);
}

template void layer_norm<float>(const float*, const float*, const float*, float*, int, int, cudaStream_t,
                                unsigned long long*);
template void layer_norm<bf16>(const float*, const float*, const float*, bf16*, int, int, cudaStream_t,
                               unsigned long long*);
template void layer_norm2<float>(float*, const float*, const float*, const float*, const float*, float*, int, int,
                                 cudaStream_t, unsigned long long*);
template void layer_norm2<bf16>(float*, const float*, const float*, const float*, const float*, bf16*, int, int,
                                cudaStream_t, unsigned long long*);

}  // namespace ud
