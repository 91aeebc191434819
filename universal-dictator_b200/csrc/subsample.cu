// Causal dw-striding x8 subsampling (NeMo pre_encode as restated in tools/nemotron_ane.py:73-83 and
// FastConformer.swift:219-250), batched over streams that share one padded mel length. Activations are
// channel-last [stream][time][freq][channel] so the 1x1 convs are plain GEMMs (run by the GEMM kernels)
// and the final flatten is a reshape (the engine permutes pre_encode.out's columns to f*C + c at load,
// as FastConformer.swift:78-94 does).
//
// Time masks: rows at or beyond each stage's valid length are zero (MaskedConvSequential; lengths
// v1 = v0/2+1, v2 = v1/2+1, v3 = v2/2+1). conv0 masks its output; the depthwise stages mask their input
// on read (the input of stage 2 is relu(pw3(...)) whose rows >= v2 must read as zero); sub_select applies
// the last mask by substituting pre_encode.out's bias for masked rows (a zero row times W plus b).
#include "common.cuh"
#include "kernels.h"

namespace ud {
namespace {

__device__ __forceinline__ int nxt(int t) { return t / 2 + 1; }

// Taps are stored tap-major, w[k * C + c] (transposed from the checkpoint's [C][1][3][3] at load).
// One CTA per (stream, output row). Each thread owns one 8-channel group (its 72 taps in registers) and steps
// over output frequencies; the three input mel rows sit in shared memory and are read as broadcasts.
template <typename T>
__global__ void __launch_bounds__(256) conv0_kernel(const float* __restrict__ mel, int rows_stride, int mel_bins,
                                                    const BatchEntry* __restrict__ meta, int Tin,
                                                    const float* __restrict__ w, const float* __restrict__ bias,
                                                    T* __restrict__ out, int T1, int F1, int C) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int VW = Vec16<T>::N;
    extern __shared__ float xs[];           // [3][mel_bins + 3], frequency index shifted by the left pad of 2
    const int W = mel_bins + 3;
    const int b = blockIdx.x, t = blockIdx.y;
    const int vm = meta[b].valid_mel;
    const int v1 = nxt(vm);
    for (int i = threadIdx.x; i < 3 * W; i += blockDim.x) {
        const int r = i / W, q = i % W - 2;
        const int row = 2 * t - 2 + r;
        const bool ok = row >= 0 && row < vm && row < Tin && q >= 0 && q < mel_bins;
        xs[i] = ok ? mel[(static_cast<size_t>(b) * rows_stride + row) * mel_bins + q] : 0.f;
    }
    __syncthreads();
    const int groups = C / VW;
    const int lanes_f = blockDim.x / groups;  // threads sharing a channel group, each taking every lanes_f-th f
    const int g = threadIdx.x % groups, f0 = threadIdx.x / groups;
    if (f0 >= lanes_f) return;
    const int c = g * VW;
    float wr[9][VW], br[VW];
#pragma unroll
    for (int e = 0; e < VW; e += 4) {
        const float4 bb = *reinterpret_cast<const float4*>(bias + c + e);
        br[e] = bb.x; br[e + 1] = bb.y; br[e + 2] = bb.z; br[e + 3] = bb.w;
    }
#pragma unroll
    for (int k = 0; k < 9; ++k)   // taps stored tap-major [9][C]: this thread's channels are contiguous
#pragma unroll
        for (int e = 0; e < VW; e += 4) {
            const float4 ww = *reinterpret_cast<const float4*>(w + k * C + c + e);
            wr[k][e] = ww.x; wr[k][e + 1] = ww.y; wr[k][e + 2] = ww.z; wr[k][e + 3] = ww.w;
        }
    T* orow = out + (static_cast<size_t>(b) * T1 + t) * F1 * C;
    const bool live = t < v1;
    for (int f = f0; f < F1; f += lanes_f) {
        float acc[VW];
#pragma unroll
        for (int e = 0; e < VW; ++e) acc[e] = br[e];
#pragma unroll
        for (int kh = 0; kh < 3; ++kh)
#pragma unroll
            for (int kw = 0; kw < 3; ++kw) {
                const float xv = xs[kh * W + 2 * f + kw];
#pragma unroll
                for (int e = 0; e < VW; ++e) acc[e] = fmaf(wr[kh * 3 + kw][e], xv, acc[e]);
            }
#pragma unroll
        for (int e = 0; e < VW; ++e) acc[e] = live ? fmaxf(acc[e], 0.f) : 0.f;
        store16<T>(orow + static_cast<size_t>(f) * C + c, acc);
    }
}

// One CTA per (stream, output row); each thread owns one 8-channel group (taps in registers), steps over output
// frequencies, and reads its inputs with 16-byte loads.
template <typename T>
__global__ void __launch_bounds__(256) dwconv_kernel(const T* __restrict__ in, int Tin, int Fin, int stage,
                                                     const BatchEntry* __restrict__ meta, const float* __restrict__ w,
                                                     const float* __restrict__ bias, T* __restrict__ out, int Tout,
                                                     int Fout, int C) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int VW = Vec16<T>::N;
    const int b = blockIdx.x, t = blockIdx.y;
    const int v1 = nxt(meta[b].valid_mel);
    const int vin = stage == 1 ? v1 : nxt(v1);
    const int groups = C / VW;
    const int lanes_f = blockDim.x / groups;
    const int g = threadIdx.x % groups, f0 = threadIdx.x / groups;
    if (f0 >= lanes_f) return;
    const int c = g * VW;
    float wr[9][VW], br[VW];
#pragma unroll
    for (int e = 0; e < VW; e += 4) {
        const float4 bb = *reinterpret_cast<const float4*>(bias + c + e);
        br[e] = bb.x; br[e + 1] = bb.y; br[e + 2] = bb.z; br[e + 3] = bb.w;
    }
#pragma unroll
    for (int k = 0; k < 9; ++k)   // taps stored tap-major [9][C]: this thread's channels are contiguous
#pragma unroll
        for (int e = 0; e < VW; e += 4) {
            const float4 ww = *reinterpret_cast<const float4*>(w + k * C + c + e);
            wr[k][e] = ww.x; wr[k][e + 1] = ww.y; wr[k][e + 2] = ww.z; wr[k][e + 3] = ww.w;
        }
    for (int f = f0; f < Fout; f += lanes_f) {
        float acc[VW];
#pragma unroll
        for (int e = 0; e < VW; ++e) acc[e] = br[e];
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) {
            const int r = 2 * t + kh - 2;
            if (r < 0 || r >= Tin || r >= vin) continue;
#pragma unroll
            for (int kw = 0; kw < 3; ++kw) {
                const int q = 2 * f + kw - 2;
                if (q < 0 || q >= Fin) continue;
                float x[VW];
                load16<T>(in + ((static_cast<size_t>(b) * Tin + r) * Fin + q) * C + c, x);
#pragma unroll
                for (int e = 0; e < VW; ++e) acc[e] = fmaf(wr[kh * 3 + kw][e], x[e], acc[e]);
            }
        }
        store16<T>(out + ((static_cast<size_t>(b) * Tout + t) * Fout + f) * C + c, acc);
    }
}

__global__ void select_kernel(const float* __restrict__ sub_out, int T3, const float* __restrict__ out_bias,
                              const BatchEntry* __restrict__ meta, float* __restrict__ x, int D) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x, t = blockIdx.y;
    const BatchEntry& me = meta[b];
    if (t >= me.T) return;
    const int v3 = nxt(nxt(nxt(me.valid_mel)));
    const int st = me.drop + t;
    const float* src = st < v3 ? sub_out + (static_cast<size_t>(b) * T3 + st) * D : out_bias;
    float* dst = x + static_cast<size_t>(me.row_off + t) * D;
    for (int c = threadIdx.x * 4; c < D; c += blockDim.x * 4)
        *reinterpret_cast<float4*>(dst + c) = *reinterpret_cast<const float4*>(src + c);
}

__global__ void pack_frames_kernel(const float* __restrict__ frames, int rows_stride,
                                   const BatchEntry* __restrict__ meta, float* __restrict__ x, int D) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x, t = blockIdx.y;
    const BatchEntry& me = meta[b];
    if (t >= me.T) return;
    const float* src = frames + (static_cast<size_t>(b) * rows_stride + t) * D;
    float* dst = x + static_cast<size_t>(me.row_off + t) * D;
    for (int c = threadIdx.x * 4; c < D; c += blockDim.x * 4)
        *reinterpret_cast<float4*>(dst + c) = *reinterpret_cast<const float4*>(src + c);
}

__global__ void scatter_rows_kernel(const float* __restrict__ src, const BatchEntry* __restrict__ meta,
                                    float* __restrict__ dst, int tmax, int W) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x, t = blockIdx.y;
    const BatchEntry& me = meta[b];
    if (t >= me.keep) return;
    const float* s = src + static_cast<size_t>(me.row_off + t) * W;
    float* d = dst + (static_cast<size_t>(b) * tmax + t) * W;
    for (int c = threadIdx.x * 4; c < W; c += blockDim.x * 4)
        *reinterpret_cast<float4*>(d + c) = *reinterpret_cast<const float4*>(s + c);
}

}  // namespace

template <typename T>
void sub_conv0(const float* mel, int rows_stride, int mel_bins, const BatchEntry* meta, int n, int Tin, const float* w,
               const float* b, T* out, int T1, int F1, int C, cudaStream_t s) {
    dim3 grid(n, T1);
    const size_t smem = sizeof(float) * (3 * (mel_bins + 3));
    launch_pdl(conv0_kernel<T>, dim3(grid), dim3(256), smem, s, mel, rows_stride, mel_bins, meta, Tin, w, b, out, T1, F1, C);
}

template <typename T>
void sub_dwconv(const T* in, int Tin, int Fin, const int*, int stage, const BatchEntry* meta, int n, const float* w,
                const float* b, T* out, int Tout, int Fout, int C, cudaStream_t s) {
    dim3 grid(n, Tout);
    launch_pdl(dwconv_kernel<T>, dim3(grid), dim3(256), 0, s, in, Tin, Fin, stage, meta, w, b, out, Tout, Fout, C);
}

template <typename T>
void sub_select(const float* sub_out, int T3, const float* out_bias, const BatchEntry* meta, int n, float* x, int D,
                cudaStream_t s) {
    dim3 grid(n, T3);
    launch_pdl(select_kernel, dim3(grid), dim3(256), 0, s, sub_out, T3, out_bias, meta, x, D);
}

void pack_frames(const float* frames, int rows_stride, const BatchEntry* meta, int n, int tmax, float* x, int D,
                 cudaStream_t s) {
    dim3 grid(n, tmax);
    launch_pdl(pack_frames_kernel, dim3(grid), dim3(256), 0, s, frames, rows_stride, meta, x, D);
}

void scatter_rows(const float* src, const BatchEntry* meta, int n, float* dst, int tmax, int W, cudaStream_t s) {
    dim3 grid(n, tmax);
    launch_pdl(scatter_rows_kernel, dim3(grid), dim3(128), 0, s, src, meta, dst, tmax, W);
}

template void sub_conv0<float>(const float*, int, int, const BatchEntry*, int, int, const float*, const float*, float*,
                               int, int, int, cudaStream_t);
template void sub_conv0<bf16>(const float*, int, int, const BatchEntry*, int, int, const float*, const float*, bf16*, int,
                              int, int, cudaStream_t);
template void sub_dwconv<float>(const float*, int, int, const int*, int, const BatchEntry*, int, const float*,
                                const float*, float*, int, int, int, cudaStream_t);
template void sub_dwconv<bf16>(const bf16*, int, int, const int*, int, const BatchEntry*, int, const float*, const float*,
                               bf16*, int, int, int, cudaStream_t);
template void sub_select<float>(const float*, int, const float*, const BatchEntry*, int, float*, int, cudaStream_t);

}  // namespace ud
