// Fused RNN-T greedy decoding, one CTA per stream, fp32 throughout.
//
// Reference: Sources/DictatorCore/Decoding/RNNT.swift
//   predict  :73-114  x = embed[token] (blank -> zeros); per layer gates = W_ih x + W_hh h + (b_ih + b_hh),
//                     order i, f, g, o; c' = s(f) c + s(i) tanh(g); h' = s(o) tanh(c'); g = joint.pred(h_top)
//   joint    :117-123 logits = W_out relu(f_t + g) + b_out
//   greedy   :127-151 per frame at most max_symbols emissions; blank advances; the prediction for the last
//                     token is computed lazily and committed (h, c, lastToken) only when a token is emitted
// The decoder state (committed h/c, last token, pending prediction) lives per stream slot in device memory and
// carries across calls. argmax keeps the first maximum (RNNT.swift:138-140).
#include "common.cuh"
#include "kernels.h"

namespace ud {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;

// out[r] = bias[r] + W1[r] . x1 (+ W2[r] . x2), rows split across warps, float4 loads along K.
__device__ void matvec(const float* __restrict__ W1, const float* __restrict__ x1, const float* __restrict__ W2,
                       const float* __restrict__ x2, const float* __restrict__ bias, float* __restrict__ out,
                       int rows, int K) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k4 = K / 4;
    for (int r = warp; r < rows; r += kWarps) {
        const float4* w1 = reinterpret_cast<const float4*>(W1 + static_cast<size_t>(r) * K);
        const float4* xa = reinterpret_cast<const float4*>(x1);
        float acc = 0.f;
        for (int i = lane; i < k4; i += 32) {
            const float4 w = w1[i], x = xa[i];
            acc = fmaf(w.x, x.x, fmaf(w.y, x.y, fmaf(w.z, x.z, fmaf(w.w, x.w, acc))));
        }
        if (W2) {
            const float4* w2 = reinterpret_cast<const float4*>(W2 + static_cast<size_t>(r) * K);
            const float4* xb = reinterpret_cast<const float4*>(x2);
            for (int i = lane; i < k4; i += 32) {
                const float4 w = w2[i], x = xb[i];
                acc = fmaf(w.x, x.x, fmaf(w.y, x.y, fmaf(w.z, x.z, fmaf(w.w, x.w, acc))));
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) out[r] = acc + (bias ? bias[r] : 0.f);
    }
}

__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + expf(-x)); }

__global__ void __launch_bounds__(kThreads) rnnt_kernel(const RnntWeights w, const RnntState st,
                                                        const float* __restrict__ proj, int ld_proj,
                                                        const BatchEntry* __restrict__ meta,
                                                        int32_t* __restrict__ tokens, int tok_stride,
                                                        int* __restrict__ n_tokens) {
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ __align__(16) float sm[];
    const int Hp = w.Hp, J = w.J, V = w.V, NLp = w.layers;
    float* f = sm;                  // [J]
    float* g = f + J;               // [J]  pending prediction output
    float* hs = g + J;              // [J]  relu(f + g)
    float* x = hs + J;              // [Hp] layer input
    float* hc = x + Hp;             // [NLp][Hp] committed h
    float* cc = hc + NLp * Hp;      // [NLp][Hp] committed c
    float* ph = cc + NLp * Hp;      // [NLp][Hp] pending h
    float* pc = ph + NLp * Hp;      // [NLp][Hp] pending c
    float* gates = pc + NLp * Hp;   // [4 Hp]
    __shared__ float red_v[kWarps];
    __shared__ int red_i[kWarps];
    __shared__ int s_best, s_pend, s_last;

    const int b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const BatchEntry& me = meta[b];
    const int slot = me.slot;
    const int blank = V - 1;
    for (int i = tid; i < NLp * Hp; i += kThreads) {
        hc[i] = st.h[static_cast<size_t>(slot) * NLp * Hp + i];
        cc[i] = st.c[static_cast<size_t>(slot) * NLp * Hp + i];
        ph[i] = st.pend_h[static_cast<size_t>(slot) * NLp * Hp + i];
        pc[i] = st.pend_c[static_cast<size_t>(slot) * NLp * Hp + i];
    }
    for (int i = tid; i < J; i += kThreads) g[i] = st.pend_g[static_cast<size_t>(slot) * J + i];
    if (tid == 0) {
        s_pend = st.pend_valid[slot];
        s_last = st.last_tok[slot];
    }
    __syncthreads();

    int ntok = 0;
    for (int t = 0; t < me.keep; ++t) {
        for (int i = tid; i < J; i += kThreads) f[i] = proj[static_cast<size_t>(me.row_off + t) * ld_proj + i];
        __syncthreads();
        for (int emitted = 0; emitted < w.max_symbols;) {
            if (!s_pend) {
                const int tok = s_last;
                for (int i = tid; i < Hp; i += kThreads)
                    x[i] = tok != blank ? w.embed[static_cast<size_t>(tok) * Hp + i] : 0.f;
                __syncthreads();
                for (int l = 0; l < NLp; ++l) {
                    const float* in = l == 0 ? x : ph + (l - 1) * Hp;
                    matvec(w.w_ih[l], in, w.w_hh[l], hc + l * Hp, w.bias[l], gates, 4 * Hp, Hp);
                    __syncthreads();
                    for (int k = tid; k < Hp; k += kThreads) {
                        const float ig = sigm(gates[k]), fg = sigm(gates[Hp + k]);
                        const float gg = tanhf(gates[2 * Hp + k]), og = sigm(gates[3 * Hp + k]);
                        const float cn = fg * cc[l * Hp + k] + ig * gg;
                        pc[l * Hp + k] = cn;
                        ph[l * Hp + k] = og * tanhf(cn);
                    }
                    __syncthreads();
                }
                matvec(w.pred_w, ph + (NLp - 1) * Hp, nullptr, nullptr, w.pred_b, g, J, Hp);
                if (tid == 0) s_pend = 1;
                __syncthreads();
            }
            for (int i = tid; i < J; i += kThreads) hs[i] = fmaxf(f[i] + g[i], 0.f);
            __syncthreads();
            // Joint logits and first-maximum argmax.
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int r = warp; r < V; r += kWarps) {
                const float4* wr = reinterpret_cast<const float4*>(w.out_w + static_cast<size_t>(r) * J);
                const float4* hv = reinterpret_cast<const float4*>(hs);
                float acc = 0.f;
                for (int i = lane; i < J / 4; i += 32) {
                    const float4 a = wr[i], h4 = hv[i];
                    acc = fmaf(a.x, h4.x, fmaf(a.y, h4.y, fmaf(a.z, h4.z, fmaf(a.w, h4.w, acc))));
                }
                acc = warp_sum(acc) + w.out_b[r];
                if (acc > bv || (acc == bv && r < bi)) { bv = acc; bi = r; }
            }
            if (lane == 0) { red_v[warp] = bv; red_i[warp] = bi; }
            __syncthreads();
            if (tid == 0) {
                float v0 = red_v[0];
                int i0 = red_i[0];
                for (int k = 1; k < kWarps; ++k)
                    if (red_v[k] > v0 || (red_v[k] == v0 && red_i[k] < i0)) { v0 = red_v[k]; i0 = red_i[k]; }
                s_best = i0;
            }
            __syncthreads();
            const int best = s_best;
            if (best == blank) break;
            if (tid == 0) {
                tokens[static_cast<size_t>(b) * tok_stride + ntok] = best;
                s_last = best;
                s_pend = 0;
            }
            for (int i = tid; i < NLp * Hp; i += kThreads) { hc[i] = ph[i]; cc[i] = pc[i]; }
            ++ntok;
            ++emitted;
            __syncthreads();
        }
    }
    for (int i = tid; i < NLp * Hp; i += kThreads) {
        st.h[static_cast<size_t>(slot) * NLp * Hp + i] = hc[i];
        st.c[static_cast<size_t>(slot) * NLp * Hp + i] = cc[i];
        st.pend_h[static_cast<size_t>(slot) * NLp * Hp + i] = ph[i];
        st.pend_c[static_cast<size_t>(slot) * NLp * Hp + i] = pc[i];
    }
    for (int i = tid; i < J; i += kThreads) st.pend_g[static_cast<size_t>(slot) * J + i] = g[i];
    if (tid == 0) {
        st.pend_valid[slot] = s_pend;
        st.last_tok[slot] = s_last;
        n_tokens[b] = ntok;
    }
}

__global__ void rnnt_reset_kernel(const RnntState st, const int* __restrict__ slots, int layers, int Hp, int J,
                                  int blank) {
    const int slot = slots[blockIdx.x];
    for (int i = threadIdx.x; i < layers * Hp; i += blockDim.x) {
        st.h[static_cast<size_t>(slot) * layers * Hp + i] = 0.f;
        st.c[static_cast<size_t>(slot) * layers * Hp + i] = 0.f;
        st.pend_h[static_cast<size_t>(slot) * layers * Hp + i] = 0.f;
        st.pend_c[static_cast<size_t>(slot) * layers * Hp + i] = 0.f;
    }
    for (int i = threadIdx.x; i < J; i += blockDim.x) st.pend_g[static_cast<size_t>(slot) * J + i] = 0.f;
    if (threadIdx.x == 0) {
        st.pend_valid[slot] = 0;
        st.last_tok[slot] = blank;
    }
}

}  // namespace

size_t rnnt_smem_bytes(const RnntWeights& w) {
    return sizeof(float) * (3 * w.J + w.Hp + 4 * w.layers * w.Hp + 4 * w.Hp);
}

void rnnt_greedy(const RnntWeights& w, const RnntState& st, const float* proj, int ld_proj, const BatchEntry* meta,
                 int n, int32_t* tokens, int tok_stride, int* n_tokens, cudaStream_t s) {
    if (n <= 0) return;
    const size_t smem = rnnt_smem_bytes(w);
    static size_t attr_set = 0;
    if (smem > 48 * 1024 && smem > attr_set) {
        cudaFuncSetAttribute(rnnt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        attr_set = smem;
    }
    launch_pdl(rnnt_kernel, dim3(n), dim3(kThreads), smem, s, w, st, proj, ld_proj, meta, tokens, tok_stride, n_tokens);
}

void rnnt_reset(const RnntState& st, const int* slots, int n, const RnntWeights& w, cudaStream_t s) {
    if (n <= 0) return;
    rnnt_reset_kernel<<<n, 256, 0, s>>>(st, slots, w.layers, w.Hp, w.J, w.V - 1);
}

}  // namespace ud
