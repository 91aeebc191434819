// Pieces shared by the two lock-step RNN-T decoders (rnnt.cu: fp32 SIMT dot products; rnnt_tc.cu: tcgen05 with a
// three-term fp16 split): the bounded grid barrier, the per-frame lists of streams still in the frame and the
// greedy decision.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace ud {
namespace {

constexpr int kLsThreads = 512;
constexpr int kLsWarps = kLsThreads / 32;

__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + expf(-x)); }

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier: all CTAs of the launch are resident (cooperative launch, one CTA per SM). Returns false (and
// records DEV_TIMEOUT_GRID) when the wait exceeds kWaitLimitNs; the caller then leaves the kernel.
__device__ bool grid_sync(unsigned long long* ctr, unsigned long long& target, int* err, volatile int* s_fail) {
    __syncthreads();
    if (threadIdx.x == 0) {
        target += gridDim.x;
        __threadfence();
        atomicAdd(ctr, 1ull);
        const uint64_t t0 = global_timer_ns();
        while (ld_acquire_u64(ctr) < target) {
            if (global_timer_ns() - t0 > kWaitLimitNs) {
                report_error(err, DEV_TIMEOUT_GRID);
                *s_fail = 1;
                break;
            }
            __nanosleep(32);
        }
        __threadfence();
    }
    __syncthreads();
    return *s_fail == 0;
}

// Appends the streams b (in order) that are still in frame t, and those of them without a pending prediction.
// Every CTA computes the same lists from the state published before the last grid barrier.
__device__ void ls_lists(const BatchEntry* meta, int n, int t, const RnntState& st, const RnntScratch& scr, int* act,
                         int* need, int* s_cnt, int* s_wa, int* s_wn) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int na = 0, nn = 0;
    for (int b0 = 0; b0 < n; b0 += kLsThreads) {
        const int b = b0 + tid;
        bool fa = false, fn = false;
        if (b < n && t < meta[b].keep && __ldcg(scr.done_frame + b) <= t) {
            fa = true;
            fn = __ldcg(st.pend_valid + meta[b].slot) == 0;
        }
        const unsigned ba = __ballot_sync(0xffffffffu, fa), bn = __ballot_sync(0xffffffffu, fn);
        if (lane == 0) { s_wa[warp] = __popc(ba); s_wn[warp] = __popc(bn); }
        __syncthreads();
        int pa = na, pn = nn, ta = 0, tn = 0;
        for (int w = 0; w < kLsWarps; ++w) {
            if (w < warp) { pa += s_wa[w]; pn += s_wn[w]; }
            ta += s_wa[w];
            tn += s_wn[w];
        }
        const unsigned lt = (1u << lane) - 1u;
        if (fa) act[pa + __popc(ba & lt)] = b;
        if (fn) need[pn + __popc(bn & lt)] = b;
        na += ta;
        nn += tn;
        __syncthreads();
    }
    if (threadIdx.x == 0) { s_cnt[0] = na; s_cnt[1] = nn; }
    __syncthreads();
}

// The greedy decision of stream b from its per-slice joint maxima part_val/part_idx[b * nparts + k], k < nparts
// (slices in vocabulary order; the first maximum wins, RNNT.swift:138-140), taken by one warp: blank ends the
// frame (the prediction stays pending); a symbol is emitted, the pending LSTM state committed and the frame ends
// after max_symbols emissions. Returns the emitted symbol, or -1 for blank.
__device__ int ls_decide(int b, int t, int nparts, const BatchEntry* meta, const RnntState& st,
                          const RnntScratch& scr, int NLp, int Hp, int blank, int max_symbols, int32_t* tokens,
                          int tok_stride, int* n_tokens) {
    const int lane = threadIdx.x & 31;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int kk = lane; kk < nparts; kk += 32) {
        const float v = __ldcg(scr.part_val + static_cast<size_t>(b) * nparts + kk);
        const int ix = __ldcg(scr.part_idx + static_cast<size_t>(b) * nparts + kk);
        if (v > bv || (v == bv && ix < bi)) { bv = v; bi = ix; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    const int slot = meta[b].slot;
    if (bi > blank) bi = blank;   // no maximum at all (every logit NaN): end the frame, the state stays as it is
    if (bi == blank) {
        if (lane == 0) {
            st.pend_valid[slot] = 1;
            scr.done_frame[b] = t + 1;
            scr.emitted[b] = 0;
        }
        return -1;
    }
    {   // commit: h, c <- the pending state (Hp a multiple of 4), four float4 pairs in flight per lane
        const size_t o = static_cast<size_t>(slot) * NLp * Hp;
        const float4* ph = reinterpret_cast<const float4*>(st.pend_h + o);
        const float4* pc = reinterpret_cast<const float4*>(st.pend_c + o);
        float4* h = reinterpret_cast<float4*>(st.h + o);
        float4* c = reinterpret_cast<float4*>(st.c + o);
        const int n4 = NLp * Hp / 4;
        for (int x0 = lane; x0 < n4; x0 += 128) {
            float4 a[4], d[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (x0 + 32 * u < n4) {
                    a[u] = __ldcg(ph + x0 + 32 * u);
                    d[u] = __ldcg(pc + x0 + 32 * u);
                }
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (x0 + 32 * u < n4) {
                    h[x0 + 32 * u] = a[u];
                    c[x0 + 32 * u] = d[u];
                }
        }
    }
    if (lane == 0) {
        const int nt = __ldcg(n_tokens + b);
        tokens[static_cast<size_t>(b) * tok_stride + nt] = bi;
        n_tokens[b] = nt + 1;
        st.last_tok[slot] = bi;
        st.pend_valid[slot] = 0;
        const int em = __ldcg(scr.emitted + b) + 1;
        if (em >= max_symbols) {
            scr.done_frame[b] = t + 1;
            scr.emitted[b] = 0;
        } else {
            scr.emitted[b] = em;
        }
    }
    return bi;
}

}  // namespace
}  // namespace ud
