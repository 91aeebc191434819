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
#include <algorithm>

#include "rnnt_common.cuh"

namespace ud {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kSpec = 16;   // frames whose joints one pass of the per-stream kernel evaluates together

// out[r] = bias[r] + W1[r] . x1 (+ W2[r] . x2), rows split across warps, float4 loads along K. Each warp takes
// four rows at a time (four independent accumulators), so four rows' weight loads are in flight together.
__device__ void matvec(const float* __restrict__ W1, const float* __restrict__ x1, const float* __restrict__ W2,
                       const float* __restrict__ x2, const float* __restrict__ bias, float* __restrict__ out,
                       int rows, int K) {
    constexpr int RB = 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k4 = K / 4;
    const float4* xa = reinterpret_cast<const float4*>(x1);
    const float4* xb = reinterpret_cast<const float4*>(x2);
    for (int r0 = warp * RB; r0 < rows; r0 += kWarps * RB) {
        float acc[RB];
#pragma unroll
        for (int u = 0; u < RB; ++u) acc[u] = 0.f;
        for (int i = lane; i < k4; i += 32) {
            const float4 x = xa[i];
            const float4 y = W2 ? xb[i] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int u = 0; u < RB; ++u) {
                if (r0 + u < rows) {
                    const float4 w = reinterpret_cast<const float4*>(W1 + static_cast<size_t>(r0 + u) * K)[i];
                    acc[u] = fmaf(w.x, x.x, fmaf(w.y, x.y, fmaf(w.z, x.z, fmaf(w.w, x.w, acc[u]))));
                    if (W2) {
                        const float4 v = reinterpret_cast<const float4*>(W2 + static_cast<size_t>(r0 + u) * K)[i];
                        acc[u] = fmaf(v.x, y.x, fmaf(v.y, y.y, fmaf(v.z, y.z, fmaf(v.w, y.w, acc[u]))));
                    }
                }
            }
        }
#pragma unroll
        for (int u = 0; u < RB; ++u) {
            const float v = warp_sum(acc[u]);
            if (lane == 0 && r0 + u < rows) out[r0 + u] = v + (bias ? bias[r0 + u] : 0.f);
        }
    }
}

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
    float* x = g + J;               // [Hp] layer input
    float* hc = x + Hp;             // [NLp][Hp] committed h
    float* cc = hc + NLp * Hp;      // [NLp][Hp] committed c
    float* ph = cc + NLp * Hp;      // [NLp][Hp] pending h
    float* pc = ph + NLp * Hp;      // [NLp][Hp] pending c
    float* gates = pc + NLp * Hp;   // [4 Hp]
    float* hsm = gates + 4 * Hp;    // [kSpec][J] relu(f_t + g) of the frames of one joint pass
    __shared__ float red_v[kWarps][kSpec];
    __shared__ int red_i[kWarps][kSpec];
    __shared__ int s_bestf[kSpec];
    __shared__ int s_pend, s_last;

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

    // The prediction for the last token (LSTM + joint.pred) into g, when it is not pending.
    auto predict = [&]() {
        const int tok = s_last;
        for (int i = tid; i < Hp; i += kThreads) x[i] = tok != blank ? w.embed[static_cast<size_t>(tok) * Hp + i] : 0.f;
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
    };
    // Joint logits of F frames (rows of hsm) and each frame's first-maximum argmax into s_bestf[0, F).
    auto joint = [&](int F) {
        float bv[kSpec];
        int bi[kSpec];
#pragma unroll
        for (int ff = 0; ff < kSpec; ++ff) { bv[ff] = -INFINITY; bi[ff] = 0x7fffffff; }
        for (int r = warp; r < V; r += kWarps) {
            const float4* wr = reinterpret_cast<const float4*>(w.out_w + static_cast<size_t>(r) * J);
            float acc[kSpec];
#pragma unroll
            for (int ff = 0; ff < kSpec; ++ff) acc[ff] = 0.f;
            for (int i = lane; i < J / 4; i += 32) {
                const float4 a = wr[i];
#pragma unroll
                for (int ff = 0; ff < kSpec; ++ff) {
                    if (ff < F) {
                        const float4 h4 = reinterpret_cast<const float4*>(hsm + ff * J)[i];
                        acc[ff] = fmaf(a.x, h4.x, fmaf(a.y, h4.y, fmaf(a.z, h4.z, fmaf(a.w, h4.w, acc[ff]))));
                    }
                }
            }
            const float ob = w.out_b[r];
#pragma unroll
            for (int ff = 0; ff < kSpec; ++ff) {
                if (ff < F) {
                    const float v = warp_sum(acc[ff]) + ob;
                    if (v > bv[ff] || (v == bv[ff] && r < bi[ff])) { bv[ff] = v; bi[ff] = r; }
                }
            }
        }
        if (lane == 0)
#pragma unroll
            for (int ff = 0; ff < kSpec; ++ff)
                if (ff < F) { red_v[warp][ff] = bv[ff]; red_i[warp][ff] = bi[ff]; }
        __syncthreads();
        if (tid < F) {
            float v0 = red_v[0][tid];
            int i0 = red_i[0][tid];
            for (int k = 1; k < kWarps; ++k)
                if (red_v[k][tid] > v0 || (red_v[k][tid] == v0 && red_i[k][tid] < i0)) { v0 = red_v[k][tid]; i0 = red_i[k][tid]; }
            s_bestf[tid] = i0;
        }
        __syncthreads();
    };

    // While no symbol is emitted the prediction g does not change, so the joints of the next frames are
    // computed in one pass over the joint weights (the weight rows are read once for up to kSpec frames; the
    // pass length adapts to the gaps between emissions, so frames evaluated past an emission stay few). The
    // first frame whose maximum is not blank continues the reference's loop exactly: it emits that symbol,
    // then alternates prediction and joint until blank or max_symbols; later frames of the pass are discarded.
    int ntok = 0;
    int t = 0;
    int spec = kSpec;   // frames per pass: doubled after a pass of blanks, the last gap to an emission after one
    while (t < me.keep) {
        if (!s_pend) predict();
        const int F = min(spec, me.keep - t);
        for (int i = tid; i < F * J; i += kThreads) {
            const int ff = i / J, j = i - ff * J;
            hsm[ff * J + j] = fmaxf(proj[static_cast<size_t>(me.row_off + t + ff) * ld_proj + j] + g[j], 0.f);
        }
        __syncthreads();
        joint(F);
        int first = F;
        for (int ff = 0; ff < F; ++ff)
            if (s_bestf[ff] != blank) { first = ff; break; }
        t += first;   // frames before it end with blank
        if (first == F) {
            spec = min(kSpec, 2 * spec);
            continue;
        }
        spec = max(2, first + 1);
        int best = s_bestf[first];
        __syncthreads();   // every thread has read s_bestf
        for (int i = tid; i < J; i += kThreads) f[i] = proj[static_cast<size_t>(me.row_off + t) * ld_proj + i];
        for (int emitted = 0;;) {
            if (tid == 0) {
                tokens[static_cast<size_t>(b) * tok_stride + ntok] = best;
                s_last = best;
                s_pend = 0;
            }
            for (int i = tid; i < NLp * Hp; i += kThreads) { hc[i] = ph[i]; cc[i] = pc[i]; }
            ++ntok;
            ++emitted;
            __syncthreads();
            if (emitted >= w.max_symbols) break;
            predict();
            for (int i = tid; i < J; i += kThreads) hsm[i] = fmaxf(f[i] + g[i], 0.f);
            __syncthreads();
            joint(1);
            best = s_bestf[0];
            __syncthreads();   // every thread has read s_bestf before the next joint rewrites it
            if (best == blank) break;
        }
        ++t;
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

// ---------------------------------------------------------------- lock-step decoder
// The same greedy semantics with the streams of a batch advanced together: per frame t, every stream that has
// not finished the frame takes one symbol iteration at a time,
//   [LSTM layers + prediction for the streams without a pending prediction]  ->  joint + argmax  ->  decide,
// and the frame ends when every stream has emitted blank or the symbol limit. Each CTA owns a slice of the
// hidden units (all four gates of each, so it can apply the cell update itself), of the prediction rows and of
// the vocabulary rows; those weight slices stay in shared memory for the whole launch, so each iteration reads
// only the streams' vectors (from L2). A grid barrier (bounded wait) separates the stages; the owner CTA of a
// stream (b mod grid) combines the per-CTA maxima in vocabulary order (first maximum, RNNT.swift:138-140),
// emits, commits the LSTM state and marks the stream's progress. Data written by other CTAs during the launch is
// read through L2 (ld.global.cg).

// Dot product of one weight row [a ; b] (len each) with [x ; y], lanes over float4 chunks; full sum in every lane.
__device__ __forceinline__ float dot2(const float* a, const float* x, const float* b, const float* y, int len,
                                      int lane) {
    float acc = 0.f;
    for (int i = lane * 4; i < len; i += 128) {
        const float4 w = *reinterpret_cast<const float4*>(a + i), v = *reinterpret_cast<const float4*>(x + i);
        acc = fmaf(w.x, v.x, fmaf(w.y, v.y, fmaf(w.z, v.z, fmaf(w.w, v.w, acc))));
    }
    if (b) {
        for (int i = lane * 4; i < len; i += 128) {
            const float4 w = *reinterpret_cast<const float4*>(b + i), v = *reinterpret_cast<const float4*>(y + i);
            acc = fmaf(w.x, v.x, fmaf(w.y, v.y, fmaf(w.z, v.z, fmaf(w.w, v.w, acc))));
        }
    }
    return warp_sum(acc);
}

// Y[s * ldy + r] = W[r] . X[s] for r < rows, s < ns: weight rows (row stride ldw) and vectors (stride ldx) in
// shared memory, K a multiple of 4. A warp takes a tile of 4 rows x 8 vectors: its lanes split K in 16-byte
// chunks, so each weight chunk loaded feeds 8 vectors and each vector chunk 4 rows (32 products per 12 loads);
// the 32 partial sums are then reduced across the lanes by halving exchanges (31 shuffles), after which lane L
// holds tile element L (row L / 8, vector L % 8).
__device__ void tile_dots(const float* __restrict__ W, int ldw, int rows, const float* __restrict__ X, int ldx, int ns,
                          int K, float* __restrict__ Y, int ldy) {
    constexpr int TR = 4, TS = 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nrt = (rows + TR - 1) / TR, nst = (ns + TS - 1) / TS;
    const int k4 = K / 4;
    for (int tile = warp; tile < nrt * nst; tile += kLsWarps) {
        const int r0 = (tile / nst) * TR, s0 = (tile % nst) * TS;
        float v[TR * TS];
#pragma unroll
        for (int i = 0; i < TR * TS; ++i) v[i] = 0.f;
        for (int c = lane; c < k4; c += 32) {
            float4 wv[TR], xv[TS];
#pragma unroll
            for (int r = 0; r < TR; ++r)
                wv[r] = r0 + r < rows ? reinterpret_cast<const float4*>(W + static_cast<size_t>(r0 + r) * ldw)[c]
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int q = 0; q < TS; ++q)
                xv[q] = s0 + q < ns ? reinterpret_cast<const float4*>(X + static_cast<size_t>(s0 + q) * ldx)[c]
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int r = 0; r < TR; ++r)
#pragma unroll
                for (int q = 0; q < TS; ++q)
                    v[r * TS + q] = fmaf(wv[r].x, xv[q].x, fmaf(wv[r].y, xv[q].y,
                                    fmaf(wv[r].z, xv[q].z, fmaf(wv[r].w, xv[q].w, v[r * TS + q]))));
        }
        // halving exchanges: at distance o the lanes with bit o set keep the upper half of their values
#pragma unroll
        for (int o = 16, h = 16; o >= 1; o >>= 1, h >>= 1) {
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < h; ++i) {
                const float send = up ? v[i] : v[i + h];
                const float keep = up ? v[i + h] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        }
        const int r = r0 + lane / TS, q = s0 + lane % TS;
        if (r < rows && q < ns) Y[static_cast<size_t>(q) * ldy + r] = v[0];
    }
}

struct LsGeom {
    int nu, nj, nv;     // hidden units, prediction rows and vocabulary rows per CTA
    int sb;             // streams per staged tile
    int wl_smem;        // LSTM slices in shared memory (else read from global)
};

__global__ void __launch_bounds__(kLsThreads, 1) rnnt_lockstep_kernel(
    const RnntWeights w, const RnntState st, const float* __restrict__ proj, int ld_proj,
    const BatchEntry* __restrict__ meta, int n, int32_t* __restrict__ tokens, int tok_stride, int* __restrict__ n_tokens,
    const RnntScratch scr, const LsGeom gm, int* err) {
    pdl_wait();
    extern __shared__ __align__(16) float lsm[];
    const int Hp = w.Hp, J = w.J, V = w.V, NLp = w.layers, G = gridDim.x, k = blockIdx.x;
    const int H2 = 2 * Hp, XW = max(H2, J), YW = max(4 * gm.nu, gm.nv), SB = gm.sb;
    float* Wl = lsm;                                                            // [NLp][4][nu][2Hp] (if wl_smem)
    float* Wp = Wl + (gm.wl_smem ? static_cast<size_t>(NLp) * 4 * gm.nu * H2 : 0);  // [nj][Hp]
    float* Wo = Wp + static_cast<size_t>(gm.nj) * Hp;                           // [nv][J]
    float* X = Wo + static_cast<size_t>(gm.nv) * J;                             // [SB][XW]
    float* Y = X + static_cast<size_t>(SB) * XW;                                // [SB][YW]
    int* act = reinterpret_cast<int*>(Y + static_cast<size_t>(SB) * YW);        // [n]
    int* need = act + n;                                                        // [n]
    __shared__ int s_fail, s_cnt[2], s_wa[kLsWarps], s_wn[kLsWarps];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int u0 = k * gm.nu, nuk = max(0, min(Hp, u0 + gm.nu) - u0);
    const int j0 = k * gm.nj, njk = max(0, min(J, j0 + gm.nj) - j0);
    const int v0 = k * gm.nv, nvk = max(0, min(V, v0 + gm.nv) - v0);
    const int blank = V - 1;
    if (tid == 0) s_fail = 0;

    // This CTA's weight slices into shared memory (float4 rows; Hp and J are multiples of 4).
    if (gm.wl_smem) {
        const int h4 = Hp / 4;
        const int total = NLp * 4 * nuk * 2 * h4;
        for (int i = tid; i < total; i += kLsThreads) {
            int r = i;
            const int c = r % h4; r /= h4;
            const int half = r % 2; r /= 2;
            const int uu = r % nuk; r /= nuk;
            const int q = r % 4, l = r / 4;
            const float* src = (half ? w.w_hh[l] : w.w_ih[l]) + static_cast<size_t>(q * Hp + u0 + uu) * Hp;
            reinterpret_cast<float4*>(Wl + (static_cast<size_t>(l * 4 + q) * gm.nu + uu) * H2 + half * Hp)[c] =
                reinterpret_cast<const float4*>(src)[c];
        }
    }
    for (int i = tid; i < njk * (Hp / 4); i += kLsThreads) {
        const int jj = i / (Hp / 4), c = i % (Hp / 4);
        reinterpret_cast<float4*>(Wp + static_cast<size_t>(jj) * Hp)[c] =
            reinterpret_cast<const float4*>(w.pred_w + static_cast<size_t>(j0 + jj) * Hp)[c];
    }
    for (int i = tid; i < nvk * (J / 4); i += kLsThreads) {
        const int vv = i / (J / 4), c = i % (J / 4);
        reinterpret_cast<float4*>(Wo + static_cast<size_t>(vv) * J)[c] =
            reinterpret_cast<const float4*>(w.out_w + static_cast<size_t>(v0 + vv) * J)[c];
    }
    if (tid == 0)
        for (int b = k; b < n; b += G) {
            scr.done_frame[b] = 0;
            scr.emitted[b] = 0;
            n_tokens[b] = 0;
        }
    int tmax = 0;
    for (int b = 0; b < n; ++b) tmax = max(tmax, meta[b].keep);
    unsigned long long target = 0;
    if (!grid_sync(scr.barrier, target, err, &s_fail)) return;

    for (int t = 0; t < tmax; ++t) {
        for (;;) {
            ls_lists(meta, n, t, st, scr, act, need, s_cnt, s_wa, s_wn);
            const int na = s_cnt[0], nn = s_cnt[1];
            if (na == 0) break;
            if (nn > 0) {
                // ---- LSTM layers for the streams that need a new prediction: gates for this CTA's units
                for (int l = 0; l < NLp; ++l) {
                    for (int s0 = 0; s0 < nn; s0 += SB) {
                        const int sb = min(SB, nn - s0);
                        for (int s = warp; s < sb; s += kLsWarps) {   // one warp per stream: [x ; h]
                            const int slot = meta[need[s0 + s]].slot;
                            const float4* xs = nullptr;
                            if (l == 0) {
                                const int tok = __ldcg(st.last_tok + slot);
                                if (tok != blank) xs = reinterpret_cast<const float4*>(w.embed + static_cast<size_t>(tok) * Hp);
                            } else {
                                xs = reinterpret_cast<const float4*>(st.pend_h + (static_cast<size_t>(slot) * NLp + l - 1) * Hp);
                            }
                            const float4* hs4 = reinterpret_cast<const float4*>(st.h + (static_cast<size_t>(slot) * NLp + l) * Hp);
                            float4* xr = reinterpret_cast<float4*>(X + s * XW);
#pragma unroll 4
                            for (int c = lane; c < Hp / 4; c += 32) {
                                xr[c] = xs ? (l == 0 ? xs[c] : __ldcg(xs + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
                                xr[Hp / 4 + c] = __ldcg(hs4 + c);
                            }
                        }
                        __syncthreads();
                        const int rows = 4 * nuk;
                        if (gm.wl_smem) {
                            // gate rows (q, uu) sit at Wl[l][q][uu] with stride nu rows per gate: one tiled pass per
                            // gate over [w_ih ; w_hh] . [x ; h]
                            for (int q = 0; q < 4; ++q)
                                tile_dots(Wl + static_cast<size_t>(l * 4 + q) * gm.nu * H2, H2, nuk, X, XW, sb, H2,
                                          Y + q * nuk, YW);
                            __syncthreads();
                            for (int i = tid; i < sb * rows; i += kLsThreads) {
                                const int s = i / rows, lr = i - s * rows;
                                const int q = lr / nuk, uu = lr - q * nuk;
                                Y[s * YW + lr] += w.bias[l][q * Hp + u0 + uu];
                            }
                        } else {
                            for (int it = warp; it < rows * sb; it += kLsWarps) {
                                const int lr = it / sb, s = it - lr * sb;
                                const int q = lr / nuk, uu = lr - q * nuk;
                                const float* ra = w.w_ih[l] + static_cast<size_t>(q * Hp + u0 + uu) * Hp;
                                const float* rb = w.w_hh[l] + static_cast<size_t>(q * Hp + u0 + uu) * Hp;
                                const float v = dot2(ra, X + s * XW, rb, X + s * XW + Hp, Hp, lane);
                                if (lane == 0) Y[s * YW + lr] = v + w.bias[l][q * Hp + u0 + uu];
                            }
                        }
                        __syncthreads();
                        for (int i = tid; i < sb * nuk; i += kLsThreads) {
                            const int s = i / nuk, uu = i - s * nuk;
                            const int slot = meta[need[s0 + s]].slot;
                            const float* gy = Y + s * YW;
                            const float ig = sigm(gy[uu]), fg = sigm(gy[nuk + uu]);
                            const float gg = tanhf(gy[2 * nuk + uu]), og = sigm(gy[3 * nuk + uu]);
                            const size_t o = (static_cast<size_t>(slot) * NLp + l) * Hp + u0 + uu;
                            const float cn = fg * __ldcg(st.c + o) + ig * gg;
                            st.pend_c[o] = cn;
                            st.pend_h[o] = og * tanhf(cn);
                        }
                        __syncthreads();
                    }
                    if (!grid_sync(scr.barrier, target, err, &s_fail)) return;
                }
                // ---- prediction output g = joint.pred(h_top) for this CTA's rows
                for (int s0 = 0; s0 < nn; s0 += SB) {
                    const int sb = min(SB, nn - s0);
                    for (int s = warp; s < sb; s += kLsWarps) {
                        const int slot = meta[need[s0 + s]].slot;
                        const float4* src = reinterpret_cast<const float4*>(st.pend_h + (static_cast<size_t>(slot) * NLp + NLp - 1) * Hp);
                        float4* xr = reinterpret_cast<float4*>(X + s * XW);
#pragma unroll 4
                        for (int c = lane; c < Hp / 4; c += 32) xr[c] = __ldcg(src + c);
                    }
                    __syncthreads();
                    tile_dots(Wp, Hp, njk, X, XW, sb, Hp, Y, YW);
                    __syncthreads();
                    for (int i = tid; i < sb * njk; i += kLsThreads) {
                        const int s = i / njk, jj = i - s * njk;
                        st.pend_g[static_cast<size_t>(meta[need[s0 + s]].slot) * J + j0 + jj] = Y[s * YW + jj] + w.pred_b[j0 + jj];
                    }
                    __syncthreads();
                }
                if (!grid_sync(scr.barrier, target, err, &s_fail)) return;
            }
            // ---- joint logits for this CTA's vocabulary rows and their first maximum, per active stream
            for (int s0 = 0; s0 < na; s0 += SB) {
                const int sb = min(SB, na - s0);
                for (int s = warp; s < sb; s += kLsWarps) {   // one warp per stream: relu(f_t + g)
                    const BatchEntry& me = meta[act[s0 + s]];
                    const float4* fp = reinterpret_cast<const float4*>(proj + static_cast<size_t>(me.row_off + t) * ld_proj);
                    const float4* gp = reinterpret_cast<const float4*>(st.pend_g + static_cast<size_t>(me.slot) * J);
                    float4* xr = reinterpret_cast<float4*>(X + s * XW);
#pragma unroll 4
                    for (int c = lane; c < J / 4; c += 32) {
                        const float4 a = fp[c], g = __ldcg(gp + c);
                        xr[c] = make_float4(fmaxf(a.x + g.x, 0.f), fmaxf(a.y + g.y, 0.f), fmaxf(a.z + g.z, 0.f),
                                            fmaxf(a.w + g.w, 0.f));
                    }
                }
                __syncthreads();
                tile_dots(Wo, J, nvk, X, XW, sb, J, Y, YW);
                __syncthreads();
                for (int i = tid; i < sb * nvk; i += kLsThreads) {
                    const int s = i / nvk, vv = i - s * nvk;
                    Y[s * YW + vv] += w.out_b[v0 + vv];
                }
                __syncthreads();
                for (int s = warp; s < sb; s += kLsWarps) {
                    float bv = -INFINITY;
                    int bi = 0x7fffffff;
                    for (int vv = lane; vv < nvk; vv += 32) {
                        const float v = Y[s * YW + vv];
                        if (v > bv) { bv = v; bi = v0 + vv; }
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
                    }
                    if (lane == 0) {
                        const size_t pi = static_cast<size_t>(act[s0 + s]) * G + k;
                        scr.part_val[pi] = bv;
                        scr.part_idx[pi] = bi;
                    }
                }
                __syncthreads();
            }
            if (!grid_sync(scr.barrier, target, err, &s_fail)) return;
            // ---- decide, by the owner CTA of each active stream
            for (int i = warp; i < na; i += kLsWarps) {
                const int b = act[i];
                if (b % G == k) ls_decide(b, t, G, meta, st, scr, NLp, Hp, blank, w.max_symbols, tokens, tok_stride, n_tokens);
            }
            if (!grid_sync(scr.barrier, target, err, &s_fail)) return;
        }
    }
}

}  // namespace

size_t rnnt_smem_bytes(const RnntWeights& w) {
    return sizeof(float) * (2 * w.J + w.Hp + 4 * w.layers * w.Hp + 4 * w.Hp + kSpec * w.J);
}

void rnnt_greedy(const RnntWeights& w, const RnntState& st, const float* proj, int ld_proj, const BatchEntry* meta,
                 int n, int32_t* tokens, int tok_stride, int* n_tokens, const RnntScratch* scr, int num_sms,
                 int* dev_err, cudaStream_t s) {
    if (n <= 0) return;
    if (scr && scr->tc_min_n > 0 && n >= scr->tc_min_n &&
        rnnt_greedy_tc(w, st, proj, ld_proj, meta, n, tokens, tok_stride, n_tokens, *scr, num_sms, dev_err, s))
        return;
    if (scr && scr->barrier && n <= scr->max_n && n <= scr->lockstep_max_n && w.Hp % 4 == 0 && w.J % 4 == 0 &&
        ld_proj % 4 == 0 && (reinterpret_cast<uintptr_t>(proj) & 15) == 0 && w.max_symbols > 0) {
        const int G = std::min(num_sms, scr->max_grid);
        LsGeom gm;
        gm.nu = (w.Hp + G - 1) / G;
        gm.nj = (w.J + G - 1) / G;
        gm.nv = (w.V + G - 1) / G;
        const size_t XW = std::max(2 * w.Hp, w.J), YW = std::max(4 * gm.nu, gm.nv);
        const size_t wl = sizeof(float) * static_cast<size_t>(w.layers) * 4 * gm.nu * 2 * w.Hp;
        const size_t fixed = sizeof(float) * (static_cast<size_t>(gm.nj) * w.Hp + static_cast<size_t>(gm.nv) * w.J) +
                             sizeof(int) * 2 * static_cast<size_t>(n);
        const size_t per_stream = sizeof(float) * (XW + YW);
        constexpr size_t kSmemMax = 227 * 1024 - 1024;   // static shared memory of the kernel stays below 1 KB
        gm.wl_smem = wl + fixed + 4 * per_stream <= kSmemMax ? 1 : 0;
        const size_t base = fixed + (gm.wl_smem ? wl : 0);
        if (base + per_stream <= kSmemMax) {
            gm.sb = static_cast<int>(std::min<size_t>(16, (kSmemMax - base) / per_stream));
            const size_t smem = base + per_stream * gm.sb;
            static size_t attr_set[kMaxDevices] = {};
            ensure_dyn_smem(rnnt_lockstep_kernel, kSmemMax, attr_set);
            cudaMemsetAsync(scr->barrier, 0, sizeof(unsigned long long), s);
            // A cooperative launch: the runtime refuses it unless all G CTAs can be resident at once, so the grid
            // barriers never wait on a CTA that has not been scheduled (the bounded waits stay as a second guard).
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(G);
            cfg.blockDim = dim3(kLsThreads);
            cfg.dynamicSmemBytes = smem;
            cfg.stream = s;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeCooperative;
            attr[0].val.cooperative = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            cudaLaunchKernelEx(&cfg, rnnt_lockstep_kernel, w, st, proj, ld_proj, meta, n, tokens, tok_stride, n_tokens,
                               *scr, gm, dev_err);
            return;
        }
    }
    const size_t smem = rnnt_smem_bytes(w);
    static size_t attr_set[kMaxDevices] = {};
    ensure_dyn_smem(rnnt_kernel, smem, attr_set);  // also below 48 KB: the kernel has static shared memory too
    launch_pdl(rnnt_kernel, dim3(n), dim3(kThreads), smem, s, w, st, proj, ld_proj, meta, tokens, tok_stride, n_tokens);
}

void rnnt_reset(const RnntState& st, const int* slots, int n, const RnntWeights& w, cudaStream_t s) {
    if (n <= 0) return;
    rnnt_reset_kernel<<<n, 256, 0, s>>>(st, slots, w.layers, w.Hp, w.J, w.V - 1);
}

}  // namespace ud
