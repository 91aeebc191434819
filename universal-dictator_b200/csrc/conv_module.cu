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

// x * sigmoid(q). fp32 engine: x / (1 + e^-q) with the fast exponential and division (two special-function
// operations). bf16 engine, whose outputs are rounded to bf16 (relative 2^-9): x * (0.5 + 0.5 tanh(q / 2)) with the
// one-instruction tanh.approx.f32 (relative error about 2^-11). The special-function unit (16 results per clock
// per SM) is what the GLU and SiLU of a C3 launch queue on, so one operation instead of two halves that work.
template <typename T> __device__ __forceinline__ float x_sigmoid(float x, float q);
template <> __device__ __forceinline__ float x_sigmoid<float>(float x, float q) { return __fdividef(x, 1.f + __expf(-q)); }
template <> __device__ __forceinline__ float x_sigmoid<bf16>(float x, float q) { return x_sigmoid_bf16out(x, q); }

template <typename T> __device__ __forceinline__ void st4(T* p, float a, float b, float c, float d);
template <> __device__ __forceinline__ void st4<float>(float* p, float a, float b, float c, float d) {
    *reinterpret_cast<float4*>(p) = make_float4(a, b, c, d);
}
template <> __device__ __forceinline__ void st4<bf16>(bf16* p, float a, float b, float c, float d) {
    const __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&lo);
    u.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(p) = u;
}

// Each thread owns a channel pair (D <= 1024 = 2 x 512 threads). One CTA's work is a short dependent chain, so
// the kernel is built to keep that chain short and its per-thread work small:
//   * before the grid-dependency wait (overlapping the pointwise GEMM's tail), one thread starts three bulk
//     copies into shared memory on an mbarrier: the stream's 8 ring rows (contiguous in the ring pool) and the
//     LayerNorm gain and bias; each warp prefetches its taps into L2. None of these is written by the preceding
//     kernel: the ring of this layer only by this kernel in an earlier step, which finished before the step's
//     input copies; weights only at load;
//   * after it: the GLU inputs of up to 16 frames (8 for fp32) are loaded with one round of independent loads,
//     kept packed until all have been issued, and their GLU goes to ys;
//   * the depthwise convolution runs from registers over [ring ; new] into ys, and puts the new frames' GLU
//     values into the shared copy of the ring as it passes them; one bulk store writes the 8 rows back (rows of
//     frames older than the last 8 hold their old values again);
//   * the row LayerNorm (a warp per frame) holds its row in registers: one pass over shared memory, 8- or
//     16-byte stores.
// Taps are stored tap-major, w[k * D + c]. Two CTAs fit on an SM (64 registers, 80 KB of shared memory at
// T = 14), so the 256 streams of a C3 batch run in one wave.
template <typename T, int KW>
__global__ void __launch_bounds__(512, 2) conv_module_kernel(const T* __restrict__ pw, int ld_pw,
                                                          const float* __restrict__ dw, const float* __restrict__ g,
                                                          const float* __restrict__ beta,
                                                          const BatchEntry* __restrict__ meta, const CacheGeom cg,
                                                          int layer, int tmax, T* __restrict__ out, int ldo, int* err,
                                                          unsigned long long* timer) {
    pdl_launch_dependents();
    constexpr int R = KW - 1;
    constexpr int FB = sizeof(T) == 2 ? 16 : 8;  // frames whose GLU inputs a thread has in flight at once
    using Raw = typename Pair<T>::Raw;
    extern __shared__ __align__(16) float sm[];
    __shared__ uint64_t bar;
    __shared__ int fail;
    const int D = cg.D;
    float* __restrict__ ys = sm;                                    // [tmax][D] GLU output, then conv output
    float* __restrict__ gs = sm + static_cast<size_t>(tmax) * D;    // LayerNorm gain [D], bias [D]
    float* __restrict__ bs = gs + D;
    T* __restrict__ rs = reinterpret_cast<T*>(bs + D);              // [R][D] ring rows, in ring order
    const BatchEntry& me = meta[blockIdx.x];
    const int slot = me.slot;
    T* __restrict__ ring = reinterpret_cast<T*>(cg.conv) + (static_cast<size_t>(layer) * cg.max_streams + slot) * R * D;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    const uint32_t ring_bytes = static_cast<uint32_t>(R * D * sizeof(T));
    if (threadIdx.x == 0) {
        fail = 0;
        mbar_init(&bar, 1);
        fence_mbarrier_init();
        const uint32_t par_bytes = static_cast<uint32_t>(D * 4);
        mbar_arrive_expect_tx(&bar, ring_bytes + 2 * par_bytes);
        bulk_load(rs, ring, ring_bytes, &bar);
        bulk_load(gs, g, par_bytes, &bar);
        bulk_load(bs, beta, par_bytes, &bar);
    }
    if (warp * 64 < D && lane < 2 * KW) {  // this warp's 64 channels of tap lane / 2: two 128-byte lines
        const float* line = dw + (lane >> 1) * D + warp * 64 + (lane & 1) * 32;
        asm volatile("prefetch.global.L2 [%0];" ::"l"(line));
    }
    __syncthreads();  // the barrier is initialised before anyone waits on it
    const int T_ = me.T, vt = me.valid_t, head = me.head, row_off = me.row_off;
    const int c = threadIdx.x * 2;
    const bool own = c < D;
    pdl_wait();
    if (threadIdx.x == 0) timer_start(timer);
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
                        g0 = x_sigmoid<T>(v.x, q.x);  // value * sigmoid(gate)
                        g1 = x_sigmoid<T>(v.y, q.y);
                    }
                    *reinterpret_cast<float2*>(ys + t * D + c) = make_float2(g0, g1);
                }
            }
        }
    }
    if (!mbar_wait_bounded(&bar, 0, err, DEV_TIMEOUT_CONV, &fail)) fail = 1;
    __syncthreads();
    if (fail) {   // the wait expired (error recorded): give copies already issued into this CTA time to land
        __nanosleep(100000);
        return;
    }
    if (own) {
        float w0[KW], w1[KW], xa[KW], xb[KW];
#pragma unroll
        for (int k = 0; k < KW; ++k) {
            const float2 wk = __ldg(reinterpret_cast<const float2*>(dw + k * D + c));
            w0[k] = wk.x;
            w1[k] = wk.y;
        }
        // Input j (frames -R .. T-1, negative ones from the ring) lives in register (j + KW) % KW of xa / xb, so
        // with the frame loop unrolled KW-fold every index is a compile-time constant: nothing is shifted.
#pragma unroll
        for (int i = 0; i < R; ++i) {  // frame i - R sits in ring row (head + i) % R
            const float2 v = Pair<T>::ld(rs + ((head + i) % R) * D + c);
            xa[i + 1] = v.x;
            xb[i + 1] = v.y;
        }
        // Causal depthwise conv over [ring ; new], in place (ys[t] is read before it is overwritten; each
        // thread reads and writes only its own columns). The last R new frames' GLU values replace, in the
        // shared copy, the ring rows of the frames R older, which this thread has already read.
        for (int t0 = 0; t0 < T_; t0 += KW) {
#pragma unroll
            for (int u = 0; u < KW; ++u) {
                const int t = t0 + u;
                if (t < T_) {
                    const float2 gv = *reinterpret_cast<const float2*>(ys + t * D + c);
                    xa[u] = gv.x;
                    xb[u] = gv.y;
                    if (t >= T_ - R) Pair<T>::st(rs + ((head + t) % R) * D + c, gv.x, gv.y);
                    float y0 = 0.f, y1 = 0.f;
#pragma unroll
                    for (int k = 0; k < KW; ++k) {  // input t - R + k
                        y0 = fmaf(w0[k], xa[(u + 1 + k) % KW], y0);
                        y1 = fmaf(w1[k], xb[(u + 1 + k) % KW], y1);
                    }
                    *reinterpret_cast<float2*>(ys + t * D + c) = make_float2(y0, y1);
                }
            }
        }
    }
    fence_proxy_async_smem();  // the ring rows written above, before the bulk store reads them
    __syncthreads();
    if (threadIdx.x == 0) {
        bulk_store(ring, rs, ring_bytes);
        tma_store_commit();
    }
    constexpr int kV = 8;  // float4 per lane: D <= 1024
    for (int t = warp; t < T_; t += nwarps) {
        const float* yr = ys + t * D;
        float4 v[kV];
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < kV; ++j) {
            const int c4 = lane * 4 + 128 * j;
            v[j] = c4 < D ? *reinterpret_cast<const float4*>(yr + c4) : make_float4(0.f, 0.f, 0.f, 0.f);
            s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
        }
        const float mean = warp_sum(s) / static_cast<float>(D);
        float q = 0.f;
#pragma unroll
        for (int j = 0; j < kV; ++j) {
            if (lane * 4 + 128 * j < D) {
                const float a0 = v[j].x - mean, a1 = v[j].y - mean, a2 = v[j].z - mean, a3 = v[j].w - mean;
                q = fmaf(a0, a0, fmaf(a1, a1, fmaf(a2, a2, fmaf(a3, a3, q))));
            }
        }
        const float rstd = rsqrtf(warp_sum(q) / static_cast<float>(D) + 1e-5f);
        T* orow = out + static_cast<size_t>(row_off + t) * ldo;
#pragma unroll
        for (int j = 0; j < kV; ++j) {
            const int c4 = lane * 4 + 128 * j;
            if (c4 < D) {
                const float4 gg = *reinterpret_cast<const float4*>(gs + c4), bb = *reinterpret_cast<const float4*>(bs + c4);
                const float z0 = (v[j].x - mean) * rstd * gg.x + bb.x, z1 = (v[j].y - mean) * rstd * gg.y + bb.y;
                const float z2 = (v[j].z - mean) * rstd * gg.z + bb.z, z3 = (v[j].w - mean) * rstd * gg.w + bb.w;
                st4<T>(orow + c4, x_sigmoid<T>(z0, z0), x_sigmoid<T>(z1, z1), x_sigmoid<T>(z2, z2),
                       x_sigmoid<T>(z3, z3));
            }
        }
    }
    if (threadIdx.x == 0) tma_store_wait_all();  // the ring rows are in global memory before the CTA exits
    if (lane == 0) timer_end(timer);
}

}  // namespace

template <typename T>
void conv_module(const T* pw, int ld_pw, const float* dw, const float* ln_g, const float* ln_b, const BatchEntry* meta,
                 int n, int tmax_batch, const CacheGeom& cg, int layer, int K, T* out, int ldo, int* dev_err,
                 cudaStream_t s, unsigned long long* timer) {
    if (n <= 0 || K != 9) return;
    const size_t smem = (sizeof(float) * (static_cast<size_t>(tmax_batch) + 2) + sizeof(T) * 8) * cg.D;
    static size_t attr_set[kMaxDevices] = {};
    ensure_dyn_smem(conv_module_kernel<T, 9>, smem, attr_set);  // also below 48 KB: the kernel has static shared memory too
    launch_pdl(conv_module_kernel<T, 9>, dim3(n), dim3(512), smem, s, pw, ld_pw, dw, ln_g, ln_b, meta, cg, layer,
               tmax_batch, out, ldo, dev_err, timer);
}

template void conv_module<float>(const float*, int, const float*, const float*, const float*, const BatchEntry*, int,
                                 int, const CacheGeom&, int, int, float*, int, int*, cudaStream_t,
                                 unsigned long long*);
template void conv_module<bf16>(const bf16*, int, const float*, const float*, const float*, const BatchEntry*, int, int,
                                const CacheGeom&, int, int, bf16*, int, int*, cudaStream_t, unsigned long long*);

}  // namespace ud
