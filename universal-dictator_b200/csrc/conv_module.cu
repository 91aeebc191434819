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

template <typename T, int KW>
__global__ void __launch_bounds__(256) conv_module_kernel(const T* __restrict__ pw, int ld_pw,
                                                          const float* __restrict__ dw, const float* __restrict__ g,
                                                          const float* __restrict__ beta,
                                                          const BatchEntry* __restrict__ meta, const CacheGeom cg,
                                                          int layer, T* __restrict__ out, int ldo) {
    constexpr int R = KW - 1;
    extern __shared__ float ys[];  // [T][D] pre-norm conv output
    const int b = blockIdx.x;
    const BatchEntry& me = meta[b];
    const int D = cg.D, T_ = me.T, vt = me.valid_t, head = me.head, row_off = me.row_off;
    T* ring = reinterpret_cast<T*>(cg.conv) + (static_cast<size_t>(layer) * cg.max_streams + me.slot) * R * D;

    for (int c = threadIdx.x; c < D; c += blockDim.x) {
        float w[KW], win[KW];
#pragma unroll
        for (int k = 0; k < KW; ++k) w[k] = dw[c * KW + k];
#pragma unroll
        for (int i = 0; i < R; ++i) win[i] = to_f<T>(ring[((head + i) % R) * D + c]);  // frame head - R + i
        for (int t = 0; t < T_; ++t) {
            float gv = 0.f;
            if (t < vt) {
                const T* pr = pw + static_cast<size_t>(row_off + t) * ld_pw;
                const float a = to_f<T>(pr[c]), gate = to_f<T>(pr[D + c]);
                gv = a / (1.f + expf(-gate));
            }
            win[R] = gv;
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < KW; ++k) acc = fmaf(w[k], win[k], acc);
            ys[t * D + c] = acc;
            // Ring row (head + t) % R held frame head + t - R, already consumed above.
            if (t >= T_ - R) ring[((head + t) % R) * D + c] = from_f<T>(gv);
#pragma unroll
            for (int k = 0; k < R; ++k) win[k] = win[k + 1];
        }
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    for (int t = warp; t < T_; t += nwarps) {
        const float* yr = ys + t * D;
        float s = 0.f;
        for (int c = lane; c < D; c += 32) s += yr[c];
        const float mean = warp_sum(s) / static_cast<float>(D);
        float q = 0.f;
        for (int c = lane; c < D; c += 32) {
            const float d = yr[c] - mean;
            q += d * d;
        }
        const float rstd = rsqrtf(warp_sum(q) / static_cast<float>(D) + 1e-5f);
        T* orow = out + static_cast<size_t>(row_off + t) * ldo;
        for (int c = lane; c < D; c += 32) {
            const float v = (yr[c] - mean) * rstd * g[c] + beta[c];
            orow[c] = from_f<T>(v / (1.f + expf(-v)));
        }
    }
}

}  // namespace

template <typename T>
void conv_module(const T* pw, int ld_pw, const float* dw, const float* ln_g, const float* ln_b, const BatchEntry* meta,
                 int n, int tmax_batch, const CacheGeom& cg, int layer, int K, T* out, int ldo, cudaStream_t s) {
    if (n <= 0 || K != 9) return;
    const size_t smem = sizeof(float) * static_cast<size_t>(tmax_batch) * cg.D;
    static size_t attr_set = 0;
    if (smem > 48 * 1024 && smem > attr_set) {
        cudaFuncSetAttribute(conv_module_kernel<T, 9>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
        attr_set = smem;
    }
    conv_module_kernel<T, 9><<<n, 256, smem, s>>>(pw, ld_pw, dw, ln_g, ln_b, meta, cg, layer, out, ldo);
}

template void conv_module<float>(const float*, int, const float*, const float*, const float*, const BatchEntry*, int,
                                 int, const CacheGeom&, int, int, float*, int, cudaStream_t);
template void conv_module<bf16>(const bf16*, int, const float*, const float*, const float*, const BatchEntry*, int, int,
                                const CacheGeom&, int, int, bf16*, int, cudaStream_t);

}  // namespace ud
