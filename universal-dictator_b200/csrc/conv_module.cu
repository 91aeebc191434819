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
    using Raw = float2;  // a channel pair as loaded
    static __device__ __forceinline__ float2 ld(const float* p) { return *reinterpret_cast<const float2*>(p); }
    static __device__ __forceinline__ Raw ldr(const float* p) { return *reinterpret_cast<const float2*>(p); }
    static __device__ __forceinline__ float2 cvt(Raw r) { return r; }
    static __device__ __forceinline__ void st(float* p, float a, float b) { *reinterpret_cast<float2*>(p) = make_float2(a, b); }
};
template <> struct Pair<bf16> {
    using Raw = __nv_bfloat162;
    static __device__ __forceinline__ float2 ld(const bf16* p) {
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    }
    static __device__ __forceinline__ Raw ldr(const bf16* p) { return *reinterpret_cast<const __nv_bfloat162*>(p); }
    static __device__ __forceinline__ float2 cvt(Raw r) { return __bfloat1622float2(r); }
    static __device__ __forceinline__ void st(bf16* p, float a, float b) {
        *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
    }
};

// Each thread owns a channel pair (D <= 1024 = 2 x 512 threads). One CTA's work is a short dependent chain, so
// the kernel is built to make that chain short:
//   * before the grid-dependency wait (overlapping the pointwise GEMM's tail): the taps and the LayerNorm
//     parameters go to shared memory, and the thread's 8 ring rows to registers. None of them is written by
//     the preceding kernel: the ring of this layer only by this kernel in an earlier step, which finished
//     before the step's input copies; weights only at load;
//   * after it: the GLU inputs of up to 16 frames (8 for fp32) are loaded with one round of independent loads,
//     kept packed until all have been issued;
//   * the depthwise convolution runs from registers over [ring ; new] into ys, and the row LayerNorm reads ys
//     and the staged parameters from shared memory (a warp per frame).
// Taps are stored tap-major, w[k * D + c]. Two CTAs fit on an SM (64 registers, about 100 KB of shared memory
// at T = 14), so the 256 streams of a C3 batch run in one wave.
template <typename T, int KW>
__global__ void __launch_bounds__(512, 2) conv_module_kernel(const T* __restrict__ pw, int ld_pw,
                                                          const float* __restrict__ dw, const float* __restrict__ g,
                                                          const float* __restrict__ beta,
                                                          const BatchEntry* __restrict__ meta, const CacheGeom cg,
                                                          int layer, int tmax, T* __restrict__ out, int ldo) {
    pdl_launch_dependents();
    constexpr int R = KW - 1;
    constexpr int FB = sizeof(T) == 2 ? 16 : 8;  // frames whose GLU inputs a thread has in flight at once
    using Raw = typename Pair<T>::Raw;
    extern __shared__ float sm[];
    const int D = cg.D;
    float* __restrict__ ys = sm;                                    // [tmax][D] GLU output, then conv output
    float* __restrict__ taps = sm + static_cast<size_t>(tmax) * D;  // [KW][D]
    float* __restrict__ gs = taps + KW * D;                         // LayerNorm gain, then bias
    float* __restrict__ bs = gs + D;
    for (int i = threadIdx.x * 4; i < KW * D; i += blockDim.x * 4)
        *reinterpret_cast<float4*>(taps + i) = __ldg(reinterpret_cast<const float4*>(dw + i));
    for (int i = threadIdx.x * 4; i < D; i += blockDim.x * 4) {
        *reinterpret_cast<float4*>(gs + i) = __ldg(reinterpret_cast<const float4*>(g + i));
        *reinterpret_cast<float4*>(bs + i) = __ldg(reinterpret_cast<const float4*>(beta + i));
    }
    const BatchEntry& me = meta[blockIdx.x];
    const int T_ = me.T, vt = me.valid_t, head = me.head, row_off = me.row_off;
    T* __restrict__ ring = reinterpret_cast<T*>(cg.conv) + (static_cast<size_t>(layer) * cg.max_streams + me.slot) * R * D;
    const int c = threadIdx.x * 2;
    const bool own = c < D;
    Raw rr[R];  // frames head - R + i, read before any ring row is rewritten
    if (own) {
#pragma unroll
        for (int i = 0; i < R; ++i) rr[i] = Pair<T>::ldr(ring + ((head + i) % R) * D + c);
    }
    pdl_wait();
    if (own) {
        for (int t0 = 0; t0 < T_; t0 += FB) {
            Raw val[FB], gate[FB];
#pragma unroll
            for (int u = 0; u < FB; ++u) {
                if (t0 + u < vt) {
                    const T* pr = pw + static_cast<size_t>(row_off + t0 + u) * ld_pw + c;
                    val[u] = Pair<T>::ldr(pr);
                    gate[u] = Pair<T>::ldr(pr + D);
                }
            }
#pragma unroll
            for (int u = 0; u < FB; ++u) {
                const int t = t0 + u;
                if (t < T_) {
                    float g0 = 0.f, g1 = 0.f;  // pad mask: frames from validT on enter as zero
                    if (t < vt) {
                        const float2 v = Pair<T>::cvt(val[u]), q = Pair<T>::cvt(gate[u]);
                        g0 = __fdividef(v.x, 1.f + __expf(-q.x));  // value * sigmoid(gate)
                        g1 = __fdividef(v.y, 1.f + __expf(-q.y));
                    }
                    *reinterpret_cast<float2*>(ys + t * D + c) = make_float2(g0, g1);
                    if (t >= T_ - R) Pair<T>::st(ring + ((head + t) % R) * D + c, g0, g1);
                }
            }
        }
        float w0[KW], w1[KW], a[KW], bq[KW];
#pragma unroll
        for (int k = 0; k < KW; ++k) {
            const float2 wk = *reinterpret_cast<const float2*>(taps + k * D + c);
            w0[k] = wk.x;
            w1[k] = wk.y;
        }
#pragma unroll
        for (int i = 0; i < R; ++i) {
            const float2 v = Pair<T>::cvt(rr[i]);
            a[i] = v.x;
            bq[i] = v.y;
        }
        // Causal depthwise conv over [ring ; new], in place (ys[t] is read before it is overwritten; each
        // thread reads and writes only its own columns, so no barrier is needed before this loop).
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
        for (int c4 = lane * 4; c4 < D; c4 += 128) {
            const float4 v = *reinterpret_cast<const float4*>(yr + c4);
            s += v.x + v.y + v.z + v.w;
        }
        const float mean = warp_sum(s) / static_cast<float>(D);
        float q = 0.f;
        for (int c4 = lane * 4; c4 < D; c4 += 128) {
            const float4 v = *reinterpret_cast<const float4*>(yr + c4);
            q += (v.x - mean) * (v.x - mean) + (v.y - mean) * (v.y - mean) + (v.z - mean) * (v.z - mean) +
                 (v.w - mean) * (v.w - mean);
        }
        const float rstd = rsqrtf(warp_sum(q) / static_cast<float>(D) + 1e-5f);
        T* orow = out + static_cast<size_t>(row_off + t) * ldo;
        for (int c2 = lane * 2; c2 < D; c2 += 64) {
            const float2 v = *reinterpret_cast<const float2*>(yr + c2);
            const float2 gg = *reinterpret_cast<const float2*>(gs + c2), bb = *reinterpret_cast<const float2*>(bs + c2);
            const float z0 = (v.x - mean) * rstd * gg.x + bb.x;
            const float z1 = (v.y - mean) * rstd * gg.y + bb.y;
            Pair<T>::st(orow + c2, silu(z0), silu(z1));
        }
    }
}

}  // namespace

template <typename T>
void conv_module(const T* pw, int ld_pw, const float* dw, const float* ln_g, const float* ln_b, const BatchEntry* meta,
                 int n, int tmax_batch, const CacheGeom& cg, int layer, int K, T* out, int ldo, cudaStream_t s) {
    if (n <= 0 || K != 9) return;
    const size_t smem = sizeof(float) * (static_cast<size_t>(tmax_batch) + 9 + 2) * cg.D;
    static size_t attr_set[kMaxDevices] = {};
    if (smem > 48 * 1024) ensure_dyn_smem(conv_module_kernel<T, 9>, smem, attr_set);
    launch_pdl(conv_module_kernel<T, 9>, dim3(n), dim3(512), smem, s, pw, ld_pw, dw, ln_g, ln_b, meta, cg, layer,
               tmax_batch, out, ldo);
}

template void conv_module<float>(const float*, int, const float*, const float*, const float*, const BatchEntry*, int,
                                 int, const CacheGeom&, int, int, float*, int, cudaStream_t);
template void conv_module<bf16>(const bf16*, int, const float*, const float*, const float*, const BatchEntry*, int, int,
                                const CacheGeom&, int, int, bf16*, int, cudaStream_t);

}  // namespace ud
