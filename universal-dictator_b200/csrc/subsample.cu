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
//
// conv0 (1 -> C channels, 3x3 stride 2, ReLU, rows >= v1 zero) fused with the stage-1 depthwise conv (3x3
// stride 2 over conv0's output, input rows >= v1 zero): conv0's output is never stored. Persistent: each CTA
// walks stage-1 output rows (stream b, row t2) with a stride of the grid; a row needs conv0 rows 2 t2 - 2 .. 2 t2,
// i.e. mel rows 4 t2 - 6 .. 4 t2 (7 rows), staged in shared memory by zero-filling cp.async, the next row's
// while the current one is computed. Each thread owns four channels (conv0 taps in registers, loaded once)
// and a contiguous run of output columns, carrying the conv0 column shared by neighbouring outputs
// (f1 = 2 f2); 64 channel groups x 4 column lanes (9, 9, 9, 6 of the 33 columns), two CTAs per SM. Sums keep
// the order of the two separate convolutions (bias, then taps kh-major, kw-minor), in fp32 throughout.

// Four consecutive channels: 16 bytes (fp32) or 8 bytes (bf16).
template <typename T>
__device__ __forceinline__ void store4v(T* p, const float* v) {
    if constexpr (sizeof(T) == 4) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
        __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]), hi = __floats2bfloat162_rn(v[2], v[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&lo);
        u.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(p) = u;
    }
}

__device__ __forceinline__ void cp_async4_zfill(float* smem, const float* gmem, bool ok) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(ok ? 4 : 0)
                 : "memory");
}

// 16 bytes global -> shared, or 16 zero bytes when !ok (the source is then not read).
__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, bool ok) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(ok ? 16 : 0)
                 : "memory");
}

template <typename T>
__global__ void __launch_bounds__(256, 2) conv01_kernel(const float* __restrict__ mel, int rows_stride, int mel_bins,
                                                        const BatchEntry* __restrict__ meta, int Tin,
                                                        const float* __restrict__ w0, const float* __restrict__ b0,
                                                        int T1, int F1, const float* __restrict__ w1,
                                                        const float* __restrict__ b1, T* __restrict__ out, int T2,
                                                        int F2, int C, int rows_total) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int VW = 4;   // channels per thread: 64 channel groups x 4 column lanes, two CTAs per SM
    extern __shared__ __align__(16) float sm[];
    const int W = mel_bins + 3;                           // mel columns shifted by the left pad of 2
    float* w1s = sm;                                      // [9][C]
    float* b1s = w1s + 9 * C;                             // [C]
    float* xs = b1s + C;                                  // [2][7][W]
    // mel rows 4 t2 - 6 .. 4 t2 of row r into dst (zeros outside the stream's valid rows and the frequency pad)
    auto prefetch = [&](int r, float* dst) {
        const int b = r / T2, t2 = r % T2;
        const int vm = meta[b].valid_mel;
        const int mel0 = 4 * t2 - 6;
        for (int i = threadIdx.x; i < 7 * W; i += blockDim.x) {
            const int rr = i / W, q = i % W - 2;
            const int row = mel0 + rr;
            const bool ok = row >= 0 && row < vm && row < Tin && q >= 0 && q < mel_bins;
            cp_async4_zfill(dst + i, ok ? mel + (static_cast<size_t>(b) * rows_stride + row) * mel_bins + q : mel, ok);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (blockIdx.x < rows_total) prefetch(blockIdx.x, xs);
    for (int i = threadIdx.x; i < 9 * C; i += blockDim.x) w1s[i] = w1[i];
    for (int i = threadIdx.x; i < C; i += blockDim.x) b1s[i] = b1[i];

    const int groups = C / VW;
    const int lanes_f = blockDim.x / groups;
    const int g = threadIdx.x % groups, fl = threadIdx.x / groups;
    const int per = (F2 + lanes_f - 1) / lanes_f;
    const int fa = fl * per, fb = fl < lanes_f ? min(F2, fa + per) : fa;
    const int c = fl < lanes_f ? g * VW : 0;
    float wr[9][VW], br[VW];
#pragma unroll
    for (int e = 0; e < VW; e += 4) {
        const float4 bb = *reinterpret_cast<const float4*>(b0 + c + e);
        br[e] = bb.x; br[e + 1] = bb.y; br[e + 2] = bb.z; br[e + 3] = bb.w;
    }
#pragma unroll
    for (int k = 0; k < 9; ++k)
#pragma unroll
        for (int e = 0; e < VW; e += 4) {
            const float4 ww = *reinterpret_cast<const float4*>(w0 + k * C + c + e);
            wr[k][e] = ww.x; wr[k][e + 1] = ww.y; wr[k][e + 2] = ww.z; wr[k][e + 3] = ww.w;
        }

    int buf = 0;
    for (int r = blockIdx.x; r < rows_total; r += gridDim.x) {
        const int rn = r + gridDim.x;
        if (rn < rows_total) prefetch(rn, xs + (buf ^ 1) * 7 * W);
        else asm volatile("cp.async.commit_group;" ::: "memory");    // keeps one group per iteration
        asm volatile("cp.async.wait_group 1;" ::: "memory");           // row r's group has landed
        __syncthreads();
        const float* x = xs + buf * 7 * W;
        const int b = r / T2, t2 = r % T2;
        const int v1 = nxt(meta[b].valid_mel);
        bool row_ok[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const int t1 = 2 * t2 - 2 + k;
            row_ok[k] = t1 >= 0 && t1 < T1 && t1 < v1;
        }
        // conv0 output at (row 2 t2 - 2 + k, column f1) for this thread's channels; zero where masked or padded.
        auto conv0 = [&](int k, int f1, float (&dst)[VW]) {
            if (!row_ok[k] || f1 < 0 || f1 >= F1) {
#pragma unroll
                for (int e = 0; e < VW; ++e) dst[e] = 0.f;
                return;
            }
#pragma unroll
            for (int e = 0; e < VW; ++e) dst[e] = br[e];
#pragma unroll
            for (int kh = 0; kh < 3; ++kh)
#pragma unroll
                for (int kw = 0; kw < 3; ++kw) {
                    const float xv = x[(2 * k + kh) * W + 2 * f1 + kw];
#pragma unroll
                    for (int e = 0; e < VW; ++e) dst[e] = fmaf(wr[kh * 3 + kw][e], xv, dst[e]);
                }
#pragma unroll
            for (int e = 0; e < VW; ++e) dst[e] = fmaxf(dst[e], 0.f);
        };
        if (fa < fb) {
            float left[3][VW];   // conv0 column 2 f2 - 2, carried from the previous output
#pragma unroll
            for (int k = 0; k < 3; ++k) conv0(k, 2 * fa - 2, left[k]);
            for (int f2 = fa; f2 < fb; ++f2) {
                float acc[VW];
#pragma unroll
                for (int e = 0; e < VW; e += 4) {
                    const float4 bb = *reinterpret_cast<const float4*>(b1s + c + e);
                    acc[e] = bb.x; acc[e + 1] = bb.y; acc[e + 2] = bb.z; acc[e + 3] = bb.w;
                }
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    float mid[VW], right[VW];
                    conv0(k, 2 * f2 - 1, mid);
                    conv0(k, 2 * f2, right);
#pragma unroll
                    for (int e = 0; e < VW; e += 4) {
                        const float4 wa = *reinterpret_cast<const float4*>(w1s + (k * 3 + 0) * C + c + e);
                        const float4 wb = *reinterpret_cast<const float4*>(w1s + (k * 3 + 1) * C + c + e);
                        const float4 wc = *reinterpret_cast<const float4*>(w1s + (k * 3 + 2) * C + c + e);
                        const float a4[4] = {wa.x, wa.y, wa.z, wa.w}, b4[4] = {wb.x, wb.y, wb.z, wb.w};
                        const float c4[4] = {wc.x, wc.y, wc.z, wc.w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            acc[e + i] = fmaf(a4[i], left[k][e + i], acc[e + i]);
                            acc[e + i] = fmaf(b4[i], mid[e + i], acc[e + i]);
                            acc[e + i] = fmaf(c4[i], right[e + i], acc[e + i]);
                        }
                    }
#pragma unroll
                    for (int e = 0; e < VW; ++e) left[k][e] = right[e];
                }
                store4v<T>(out + ((static_cast<size_t>(b) * T2 + t2) * F2 + f2) * C + c, acc);
            }
        }
        __syncthreads();   // xs[buf] is refilled by the next iteration's prefetch
        buf ^= 1;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// Stage-2 depthwise conv (3x3 stride 2; input rows >= v2 = nxt(nxt(valid_mel)) read as zero). One CTA per
// (stream, output row t): the three input rows 2t-2 .. 2t are staged in shared memory by 16-byte cp.async, all in
// flight at once (masked rows zero-filled); each thread owns one channel group (taps in registers, loaded before
// the grid-dependency wait) and a run of output columns.
template <typename T>
__global__ void __launch_bounds__(256, 3) dwconv2_kernel(const T* __restrict__ in, int Tin, int Fin,
                                                      const BatchEntry* __restrict__ meta, const float* __restrict__ w,
                                                      const float* __restrict__ bias, T* __restrict__ out, int Tout,
                                                      int Fout, int C) {
    pdl_launch_dependents();
    constexpr int VW = Vec16<T>::N;
    extern __shared__ __align__(16) unsigned char smraw[];
    T* xs = reinterpret_cast<T*>(smraw);   // [3][Fin][C]
    float* ws = reinterpret_cast<float*>(smraw + sizeof(T) * 3 * static_cast<size_t>(Fin) * C);   // [9][C] taps, [C] bias
    const int b = blockIdx.x, t = blockIdx.y;
    const int groups = C / VW;
    const int lanes_f = blockDim.x / groups;
    const int g = threadIdx.x % groups, fl = threadIdx.x / groups;
    const int per = (Fout + lanes_f - 1) / lanes_f;
    const int fa = fl * per, fb = fl < lanes_f ? min(Fout, fa + per) : fa;
    const int c = g * VW;
    // Taps and bias (weights, never written by the previous kernel) to shared memory before the grid-dependency
    // wait; kept out of registers so that three CTAs fit on an SM.
    for (int i = threadIdx.x * 4; i < 9 * C; i += blockDim.x * 4)
        *reinterpret_cast<float4*>(ws + i) = *reinterpret_cast<const float4*>(w + i);
    for (int i = threadIdx.x * 4; i < C; i += blockDim.x * 4)
        *reinterpret_cast<float4*>(ws + 9 * C + i) = *reinterpret_cast<const float4*>(bias + i);
    pdl_wait();
    // The three input rows 2 t - 2 .. 2 t (zero where masked), every 16-byte chunk in flight at once.
    const int vin = nxt(nxt(meta[b].valid_mel));
    const int row_chunks = Fin * C / VW;
    for (int i = threadIdx.x; i < 3 * row_chunks; i += blockDim.x) {
        const int k = i / row_chunks, j = i - k * row_chunks;
        const int r = 2 * t - 2 + k;
        const bool ok = r >= 0 && r < Tin && r < vin;
        const T* src = in + (static_cast<size_t>(b) * Tin + (ok ? r : 0)) * Fin * C + static_cast<size_t>(j) * VW;
        cp_async16_zfill(xs + static_cast<size_t>(i) * VW, src, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    for (int f = fa; f < fb; ++f) {
        float acc[VW];
#pragma unroll
        for (int e = 0; e < VW; e += 4) {
            const float4 bb = *reinterpret_cast<const float4*>(ws + 9 * C + c + e);
            acc[e] = bb.x; acc[e + 1] = bb.y; acc[e + 2] = bb.z; acc[e + 3] = bb.w;
        }
#pragma unroll
        for (int kh = 0; kh < 3; ++kh)
#pragma unroll
            for (int kw = 0; kw < 3; ++kw) {
                const int q = 2 * f + kw - 2;
                if (q < 0 || q >= Fin) continue;
                float x[VW];
                load16<T>(xs + (kh * Fin + q) * C + c, x);
#pragma unroll
                for (int e = 0; e < VW; e += 4) {
                    const float4 ww = *reinterpret_cast<const float4*>(ws + (kh * 3 + kw) * C + c + e);
                    acc[e] = fmaf(ww.x, x[e], acc[e]);
                    acc[e + 1] = fmaf(ww.y, x[e + 1], acc[e + 1]);
                    acc[e + 2] = fmaf(ww.z, x[e + 2], acc[e + 2]);
                    acc[e + 3] = fmaf(ww.w, x[e + 3], acc[e + 3]);
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
void sub_conv01(const float* mel, int rows_stride, int mel_bins, const BatchEntry* meta, int n, int Tin, const float* w0,
                const float* b0, int T1, int F1, const float* w1, const float* b1, T* out, int T2, int F2, int C,
                int num_sms, cudaStream_t s) {
    const int rows = n * T2;
    if (rows <= 0) return;
    const size_t smem = sizeof(float) * (9 * C + C + 2 * 7 * (mel_bins + 3));
    const int grid = rows < 2 * num_sms ? rows : 2 * num_sms;
    launch_pdl(conv01_kernel<T>, dim3(grid), dim3(256), smem, s, mel, rows_stride, mel_bins, meta, Tin, w0, b0, T1, F1,
               w1, b1, out, T2, F2, C, rows);
}

template <typename T>
void sub_dwconv2(const T* in, int Tin, int Fin, const BatchEntry* meta, int n, const float* w, const float* b, T* out,
                 int Tout, int Fout, int C, cudaStream_t s) {
    const size_t smem = sizeof(T) * 3 * static_cast<size_t>(Fin) * C + sizeof(float) * 10 * C;
    static size_t attr_set[kMaxDevices] = {};   // per instantiation (T) and device
    ensure_dyn_smem(dwconv2_kernel<T>, smem, attr_set);
    launch_pdl(dwconv2_kernel<T>, dim3(n, Tout), dim3(256), smem, s, in, Tin, Fin, meta, w, b, out, Tout, Fout, C);
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

template void sub_conv01<float>(const float*, int, int, const BatchEntry*, int, int, const float*, const float*, int, int,
                                const float*, const float*, float*, int, int, int, int, cudaStream_t);
template void sub_conv01<bf16>(const float*, int, int, const BatchEntry*, int, int, const float*, const float*, int, int,
                               const float*, const float*, bf16*, int, int, int, int, cudaStream_t);
template void sub_dwconv2<float>(const float*, int, int, const BatchEntry*, int, const float*, const float*, float*, int,
                                 int, int, cudaStream_t);
template void sub_dwconv2<bf16>(const bf16*, int, int, const BatchEntry*, int, const float*, const float*, bf16*, int,
                                int, int, cudaStream_t);
template void sub_select<float>(const float*, int, const float*, const BatchEntry*, int, float*, int, cudaStream_t);

}  // namespace ud
