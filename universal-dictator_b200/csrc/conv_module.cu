// Conformer convolution-module core for one streaming step, one CTA per stream:
//   g_t = value_t * sigmoid(gate_t)   (GLU over the pointwise_conv1 output, first half value)   glu_f32
//   g_t = 0 for t >= validT            (pad mask, FastConformer.swift:300-302)
//   y_t = sum_k w[c, k] * [cache ; g]_{t+k}   (causal depthwise conv, k = 9, cache = last 8 inputs)   dwconv1d_f32
//   out_t = SiLU(LayerNorm(y_t))       (conv.batch_norm is a LayerNorm, FastConformer.swift:304-306)
// and the cache update (the reference's conv-cache roll, FastConformer.swift:472): the conv cache is a
// ring of 8 rows per (layer, stream) addressed by absolute frame % 8, so only the last min(T, 8) new rows
// are written and nothing is shifted. Reference kernels: Sources/DictatorEngine/Metal/20_conformer.metal:77-101.
#include "common.cuh"
#include "kernels.h"

namespace ud {
namespace {

template <typename T> struct Pair;
template <> struct Pair<float> {
    using V = float2;
    static __device__ __forceinline__ float2 ld(const float* p) { return *reinterpret_cast<const float2*>(p); }
    static __device__ __forceinline__ void st(float* p, float a, float b) { *reinterpret_cast<float2*>(p) = make_float2(a, b); }
};
template <> struct Pair<bf16> {
    static __device__ __forceinline__ float2 ld(const bf16* p) {
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    }
    static __device__ __forceinline__ void st(bf16* p, float a, float b) {
        *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
    }
};

// Each thread owns a channel pair; the time loop reads only the GLU input and this thread's ring rows, so
// loads of different frames are independent (restrict pointers) and stay in flight together. Taps are stored
// tap-major, w[k * D + c], so a warp reads each tap of its 64 channels with one coalesced 256-byte load. Two
// CTAs fit on an SM (64 registers), so the 256 streams of a C3 batch run in one wave.
template <typename T, int KW>
__global__ void __launch_bounds__(512, 2) conv_module_kernel(const T* __restrict__ pw, int ld_pw,
                                                          const float* __restrict__ dw, const float* __restrict__ g,
                                                          const float* __restrict__ beta,
                                                          const BatchEntry* __restrict__ meta, const CacheGeom cg,
                                                          int layer, T* __restrict__ out, int ldo) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int R = KW - 1;
    extern __shared__ float ys[];  // [T][D] pre-norm conv output
    const int b = blockIdx.x;
    const BatchEntry& me = meta[b];
    const int D = cg.D, T_ = me.T, vt = me.valid_t, head = me.head, row_off = me.row_off;
    T* __restrict__ ring = reinterpret_cast<T*>(cg.conv) + (static_cast<size_t>(layer) * cg.max_streams + me.slot) * R * D;

    for (int c = threadIdx.x * 2; c < D; c += blockDim.x * 2) {
        float w0[KW], w1[KW], a[KW], bq[KW];
#pragma unroll
        for (int k = 0; k < KW; ++k) {
            const float2 wk = *reinterpret_cast<const float2*>(dw + k * D + c);
            w0[k] = wk.x;
            w1[k] = wk.y;
        }
#pragma unroll
        for (int i = 0; i < R; ++i) {  // frame head - R + i, read before any ring row is rewritten
            const float2 v = Pair<T>::ld(ring + ((head + i) % R) * D + c);
            a[i] = v.x;
            bq[i] = v.y;
        }
        // Pass 1: GLU of every frame (independent loads, all in flight), into ys; the last R frames to the ring.
#pragma unroll 4
        for (int t = 0; t < T_; ++t) {
            float g0 = 0.f, g1 = 0.f;
            if (t < vt) {
                const T* pr = pw + static_cast<size_t>(row_off + t) * ld_pw + c;
                const float2 val = Pair<T>::ld(pr), gate = Pair<T>::ld(pr + D);
                g0 = __fdividef(val.x, 1.f + __expf(-gate.x));   // value * sigmoid(gate)
                g1 = __fdividef(val.y, 1.f + __expf(-gate.y));
            }
            *reinterpret_cast<float2*>(ys + t * D + c) = make_float2(g0, g1);
            if (t >= T_ - R) Pair<T>::st(ring + ((head + t) % R) * D + c, g0, g1);
        }
        // Pass 2: causal depthwise conv over [ring ; new], in place (ys[t] is read before it is overwritten).
        for (int t = 0; t < T_; ++t) {
            const float2 gv = *reinterpret_cast<const float2*>(ys + t * D + c);
            a[R] = gv.x;
            bq[R] = gv.y;
            float y0 = 0.f, y1 = 0.f;
#pragma unroll
            for (int k = 0; k < KW; ++k) {
                y0 = fmaf(w0[k], a[k], y0);
                y1 = fmaf(w1[k], bq[k], y1);
            }
            *reinterpret_cast<float2*>(ys + t * D + c) = make_float2(y0, y1);
#pragma unroll
            for (int k = 0; k < R; ++k) {
                a[k] = a[k + 1];
                bq[k] = bq[k + 1];
            }
        }
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    for (int t = warp; t < T_; t += nwarps) {
        const float* yr = ys + t * D;
        float s = 0.f;
        for (int c = lane * 4; c < D; c += 128) {
            const float4 v = *reinterpret_cast<const float4*>(yr + c);
            s += v.x + v.y + v.z + v.w;
        }
        const float mean = warp_sum(s) / static_cast<float>(D);
        float q = 0.f;
        for (int c = lane * 4; c < D; c += 128) {
            const float4 v = *reinterpret_cast<const float4*>(yr + c);
            q += (v.x - mean) * (v.x - mean) + (v.y - mean) * (v.y - mean) + (v.z - mean) * (v.z - mean) +
                 (v.w - mean) * (v.w - mean);
        }
        const float rstd = rsqrtf(warp_sum(q) / static_cast<float>(D) + 1e-5f);
        T* orow = out + static_cast<size_t>(row_off + t) * ldo;
        for (int c = lane * 2; c < D; c += 64) {
            const float2 v = *reinterpret_cast<const float2*>(yr + c);
            const float2 gg = *reinterpret_cast<const float2*>(g + c), bb = *reinterpret_cast<const float2*>(beta + c);
            const float z0 = (v.x - mean) * rstd * gg.x + bb.x;
            const float z1 = (v.y - mean) * rstd * gg.y + bb.y;
            Pair<T>::st(orow + c, silu(z0), silu(z1));
        }
    }
}

}  // namespace

template <typename T>
void conv_module(const T* pw, int ld_pw, const float* dw, const float* ln_g, const float* ln_b, const BatchEntry* meta,
                 int n, int tmax_batch, const CacheGeom& cg, int layer, int K, T* out, int ldo, cudaStream_t s) {
    if (n <= 0 || K != 9) return;
    const size_t smem = sizeof(float) * static_cast<size_t>(tmax_batch) * cg.D;
    static size_t attr_set[kMaxDevices] = {};
    if (smem > 48 * 1024) ensure_dyn_smem(conv_module_kernel<T, 9>, smem, attr_set);
    launch_pdl(conv_module_kernel<T, 9>, dim3(n), dim3(512), smem, s, pw, ld_pw, dw, ln_g, ln_b, meta, cg, layer, out, ldo);
}

template void conv_module<float>(const float*, int, const float*, const float*, const float*, const BatchEntry*, int,
                                 int, const CacheGeom&, int, int, float*, int, cudaStream_t);
template void conv_module<bf16>(const bf16*, int, const float*, const float*, const float*, const BatchEntry*, int, int,
                                const CacheGeom&, int, int, bf16*, int, cudaStream_t);

}  // namespace ud
