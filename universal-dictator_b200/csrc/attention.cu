// Transformer-XL relative-position attention over the paged per-stream K/V window plus the new chunk,
// with the append of the chunk's projected K/V rows into the ring pages fused in.
//
// Semantics (Sources/DictatorEngine/Metal/20_conformer.metal:140-219 and FastConformer.swift:455-462):
//   keys are [L cached ; T new], query i sits at key position L + i, rel(i, j) = L + i - j;
//   score(i, j) = ((q_i + u) . k_j + (q_i + v) . P[rel(i, j)]) / sqrt(dk)
//   visible keys j in [L - cacheLen, L + validT) for every query row; other keys get probability 0;
//   an empty visible range gives a zero output.
// P is the per-layer table of projected sinusoids for rel in [-(tmax-1), L+tmax-1] (row = rel + tmax - 1).
//
// One CTA per (stream, head). Cached rows live in pages: frame f of a stream is row f % page_frames of
// page pages[(f / page_frames) % kPageSlots] (absolute frame addressing, so the cache roll moves no data).
#include "common.cuh"
#include "kernels.h"

namespace ud {
namespace {

constexpr int DK = 128;
constexpr int RS = 130;  // shared-memory row stride in elements: conflict-free 4/8-byte reads per lane

__device__ __forceinline__ float2 load_pair(const float* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ float2 load_pair(const bf16* p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
__device__ __forceinline__ void store_pair(float* p, float a, float b) {
    *reinterpret_cast<float2*>(p) = make_float2(a, b);
}
__device__ __forceinline__ void store_pair(bf16* p, float a, float b) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
}

// Copies one 16-byte chunk from global into a padded shared row as 4-byte words.
template <typename T>
__device__ __forceinline__ void chunk_to_smem(T* dst, const T* src) {
    uint4 u = *reinterpret_cast<const uint4*>(src);
    uint32_t* d = reinterpret_cast<uint32_t*>(dst);
    d[0] = u.x; d[1] = u.y; d[2] = u.z; d[3] = u.w;
}
template <typename T>
__device__ __forceinline__ void zero_chunk_smem(T* dst) {
    uint32_t* d = reinterpret_cast<uint32_t*>(dst);
    d[0] = 0u; d[1] = 0u; d[2] = 0u; d[3] = 0u;
}

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

template <typename T>
struct AttnSmem {
    size_t qu, qv, S, K, V, P, total;
    __host__ __device__ AttnSmem(int tb, int L) {
        size_t o = 0;
        qu = o; o = align16(o + sizeof(float) * tb * DK);
        qv = o; o = align16(o + sizeof(float) * tb * DK);
        S = o;  o = align16(o + sizeof(float) * tb * (L + tb));
        K = o;  o = align16(o + sizeof(T) * (L + tb) * RS);
        V = o;  o = align16(o + sizeof(T) * (L + tb) * RS);
        P = o;  o = align16(o + sizeof(T) * (L + 2 * tb - 1) * RS);
        total = o;
    }
};

template <typename T>
__global__ void __launch_bounds__(256) relpos_attn_kernel(const T* __restrict__ qkv, int ld_qkv,
                                                          const T* __restrict__ ptab, int tmax,
                                                          const float* __restrict__ bias_u,
                                                          const float* __restrict__ bias_v,
                                                          const BatchEntry* __restrict__ meta, const CacheGeom cg,
                                                          int layer, T* __restrict__ out, int ldo, int tb, int* err) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int CH = 16 / sizeof(T);  // elements per 16-byte chunk
    constexpr int CPR = DK / CH;        // chunks per head row
    const int b = blockIdx.x, h = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    const BatchEntry& me = meta[b];
    const int T_ = me.T, L = cg.L, D = cg.D, PF = cg.page_frames;
    const int row_off = me.row_off, head = me.head;
    const int lo = L - me.cache_len, hi = L + me.valid_t;
    const int nk = hi > lo ? hi - lo : 0;
    const int rel_min = L - hi + 1;           // smallest rel(i, j) over visible keys
    const int np = nk > 0 ? T_ + nk - 1 : 0;  // P rows needed
    const int hoff = h * DK;

    extern __shared__ __align__(16) uint8_t sm[];
    const AttnSmem<T> lay(tb, L);
    float* qu = reinterpret_cast<float*>(sm + lay.qu);
    float* qv = reinterpret_cast<float*>(sm + lay.qv);
    float* S = reinterpret_cast<float*>(sm + lay.S);
    T* Ks = reinterpret_cast<T*>(sm + lay.K);
    T* Vs = reinterpret_cast<T*>(sm + lay.V);
    T* Ps = reinterpret_cast<T*>(sm + lay.P);
    const int SW = L + tb;

    // Queries with the two position biases.
    for (int idx = tid; idx < T_ * (DK / 2); idx += blockDim.x) {
        const int i = idx / (DK / 2), d = (idx % (DK / 2)) * 2;
        const float2 q = load_pair(qkv + static_cast<size_t>(row_off + i) * ld_qkv + hoff + d);
        qu[i * DK + d] = q.x + bias_u[hoff + d];
        qu[i * DK + d + 1] = q.y + bias_u[hoff + d + 1];
        qv[i * DK + d] = q.x + bias_v[hoff + d];
        qv[i * DK + d + 1] = q.y + bias_v[hoff + d + 1];
    }
    // Visible keys and values: cached frames from the pages, new frames from the QKV rows.
    const T* kpool = reinterpret_cast<const T*>(cg.kpool);
    const T* vpool = reinterpret_cast<const T*>(cg.vpool);
    for (int idx = tid; idx < nk * CPR; idx += blockDim.x) {
        const int r = idx / CPR, c = (idx % CPR) * CH;
        const int j = lo + r;
        T* kd = Ks + r * RS + c;
        T* vd = Vs + r * RS + c;
        if (j < L) {
            const int f = head - L + j;
            const int page = me.pages[(f / PF) % kPageSlots];
            if (page < 0 || page >= cg.n_pages) {
                report_error(err, DEV_BAD_PAGE);
                zero_chunk_smem(kd);
                zero_chunk_smem(vd);
                continue;
            }
            const size_t off = ((static_cast<size_t>(layer) * cg.n_pages + page) * PF + (f % PF)) * D + hoff + c;
            chunk_to_smem(kd, kpool + off);
            chunk_to_smem(vd, vpool + off);
        } else {
            const T* src = qkv + static_cast<size_t>(row_off + (j - L)) * ld_qkv + hoff + c;
            chunk_to_smem(kd, src + D);
            chunk_to_smem(vd, src + 2 * D);
        }
    }
    // Position rows rel_min .. rel_min + np - 1.
    for (int idx = tid; idx < np * CPR; idx += blockDim.x) {
        const int r = idx / CPR, c = (idx % CPR) * CH;
        const int trow = rel_min + r + tmax - 1;
        chunk_to_smem(Ps + r * RS + c, ptab + static_cast<size_t>(trow) * D + hoff + c);
    }
    __syncthreads();

    // Scores: warp per query row, lanes over keys.
    const float scale = rsqrtf(static_cast<float>(DK));
    for (int i = warp; i < T_; i += nwarps) {
        const float* qa = qu + i * DK;
        const float* qb = qv + i * DK;
        for (int jj = lane; jj < nk; jj += 32) {
            const int j = lo + jj;
            const T* kr = Ks + jj * RS;
            const T* pr = Ps + ((L + i - j) - rel_min) * RS;
            float s0 = 0.f, s1 = 0.f;
#pragma unroll 8
            for (int d = 0; d < DK; d += 2) {
                const float2 k2 = load_pair(kr + d), p2 = load_pair(pr + d);
                const float2 a2 = *reinterpret_cast<const float2*>(qa + d);
                const float2 b2 = *reinterpret_cast<const float2*>(qb + d);
                s0 = fmaf(a2.x, k2.x, s0);
                s0 = fmaf(a2.y, k2.y, s0);
                s1 = fmaf(b2.x, p2.x, s1);
                s1 = fmaf(b2.y, p2.y, s1);
            }
            S[i * SW + jj] = (s0 + s1) * scale;
        }
    }
    __syncthreads();
    // Softmax over the visible keys of each row.
    for (int i = warp; i < T_; i += nwarps) {
        float* sr = S + i * SW;
        float m = -INFINITY;
        for (int jj = lane; jj < nk; jj += 32) m = fmaxf(m, sr[jj]);
        m = warp_max(m);
        float sum = 0.f;
        for (int jj = lane; jj < nk; jj += 32) {
            const float e = expf(sr[jj] - m);
            sr[jj] = e;
            sum += e;
        }
        sum = warp_sum(sum);
        const float inv = sum > 0.f ? 1.f / sum : 0.f;
        for (int jj = lane; jj < nk; jj += 32) sr[jj] *= inv;
    }
    __syncthreads();
    // Weighted values.
    for (int idx = tid; idx < T_ * (DK / 2); idx += blockDim.x) {
        const int i = idx / (DK / 2), d = (idx % (DK / 2)) * 2;
        const float* sr = S + i * SW;
        float o0 = 0.f, o1 = 0.f;
        for (int jj = 0; jj < nk; ++jj) {
            const float p = sr[jj];
            const float2 v2 = load_pair(Vs + jj * RS + d);
            o0 = fmaf(p, v2.x, o0);
            o1 = fmaf(p, v2.y, o1);
        }
        store_pair(out + static_cast<size_t>(row_off + i) * ldo + hoff + d, o0, o1);
    }
    // Append this chunk's K/V rows (all T of them, as the reference's roll keeps them) at frames head + t.
    T* kw = reinterpret_cast<T*>(cg.kpool);
    T* vw = reinterpret_cast<T*>(cg.vpool);
    for (int idx = tid; idx < T_ * CPR; idx += blockDim.x) {
        const int t = idx / CPR, c = (idx % CPR) * CH;
        const int f = head + t;
        const int page = me.pages[(f / PF) % kPageSlots];
        if (page < 0 || page >= cg.n_pages) {
            report_error(err, DEV_BAD_PAGE);
            continue;
        }
        const size_t off = ((static_cast<size_t>(layer) * cg.n_pages + page) * PF + (f % PF)) * D + hoff + c;
        const T* src = qkv + static_cast<size_t>(row_off + t) * ld_qkv + hoff + c;
        *reinterpret_cast<uint4*>(kw + off) = *reinterpret_cast<const uint4*>(src + D);
        *reinterpret_cast<uint4*>(vw + off) = *reinterpret_cast<const uint4*>(src + 2 * D);
    }
}

// ---------------------------------------------------------------- tensor-core variant (bf16, T <= 16)
// The same attention with mma.sync m16n8k16 (bf16 in, fp32 accumulate):
//   AC    = (Q + u) [16 x dk] . K^T [dk x nk]           score content term
//   BDraw = (Q + v) [16 x dk] . P^T [dk x np]           position term for every rel in the window
//   S[i, j] = (AC[i, j] + BDraw[i, (L + i - j) - rel_min]) / sqrt(dk), softmax over visible keys (fp32)
//   O     = softmax [16 x nk] (bf16) . V [nk x dk]
// One CTA (16 warps, two CTAs per SM) per (stream, head). A first pass writes each key's source row (cache
// page or this chunk's QKV row) to a small table, so the copies of K, V, the needed P rows and the raw queries
// into shared memory (cp.async) need no per-chunk page arithmetic; the chunk's K/V rows are appended to their
// pages from the staged copies, so no synchronous global load sits in the CTA's chain. Fragments come from
// ldmatrix (row stride 136 elements: conflict-free, 16-byte aligned rows). The 13 AC/BD jobs of 16 columns run
// in one round over the warps, each warp then normalises one query row, and each warp computes 8 output
// columns of O.
namespace tc {

constexpr int TM = 16;
constexpr int RSB = 136;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t* r, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t* r, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

struct Lay {
    int nkp, npp, psw, acw, bdw;  // padded key rows (x16), padded position rows (x16), row strides
    size_t qu, qv, k, v, p, ac, bd, pb, kp, vp, total;
    __host__ __device__ Lay(int L) {
        nkp = (L + TM + 15) / 16 * 16;
        npp = (TM + L + TM - 1 + 15) / 16 * 16;
        psw = nkp + 8;
        acw = nkp + 8;   // == 8 (mod 32) for 16-multiples of 32k+... : float2 stores of the mma D fragment are
        bdw = npp + 8;   // conflict-free per half-warp when the row stride is 8 or 24 (mod 32)
        size_t o = 0;
        qu = o; o += sizeof(bf16) * TM * RSB;
        qv = o; o += sizeof(bf16) * TM * RSB;
        k = o;  o += sizeof(bf16) * nkp * RSB;
        v = o;  o += sizeof(bf16) * nkp * RSB;
        p = o;  o += sizeof(bf16) * npp * RSB;
        ac = o; o += sizeof(float) * TM * acw;
        bd = o; o += sizeof(float) * TM * bdw;
        pb = o; o += sizeof(bf16) * TM * psw;
        o = (o + 15) / 16 * 16;
        kp = o; o += sizeof(void*) * nkp;   // per-key source rows of K and V
        vp = o; o += sizeof(void*) * nkp;
        total = (o + 127) / 128 * 128;
    }
};

constexpr int kAttnThreads = 512;
constexpr int kAttnWarps = kAttnThreads / 32;

__global__ void __launch_bounds__(kAttnThreads, 2) attn_tc_kernel(const bf16* __restrict__ qkv, int ld_qkv,
                                                         const bf16* __restrict__ ptab, int tmax,
                                                         const float* __restrict__ bias_u,
                                                         const float* __restrict__ bias_v,
                                                         const BatchEntry* __restrict__ meta, const CacheGeom cg,
                                                         int layer, bf16* __restrict__ out, int ldo, int* err) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int DKk = 128;
    const int b = blockIdx.x, h = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const BatchEntry& me = meta[b];
    const int T_ = me.T, L = cg.L, D = cg.D, PF = cg.page_frames;
    const int row_off = me.row_off, head = me.head;
    const int lo = L - me.cache_len, hi = L + me.valid_t;
    const int nk = hi > lo ? hi - lo : 0;
    const int rel_min = L - hi + 1;
    const int np = nk > 0 ? T_ + nk - 1 : 0;
    const int hoff = h * DKk;
    const int na = L + T_ - lo;   // staged key rows: the visible ones and the chunk's invalid frames (appended too)
    const Lay lay(L);

    extern __shared__ __align__(128) uint8_t sm[];
    bf16* QU = reinterpret_cast<bf16*>(sm + lay.qu);
    bf16* QV = reinterpret_cast<bf16*>(sm + lay.qv);
    bf16* Ks = reinterpret_cast<bf16*>(sm + lay.k);
    bf16* Vs = reinterpret_cast<bf16*>(sm + lay.v);
    bf16* Ps = reinterpret_cast<bf16*>(sm + lay.p);
    float* AC = reinterpret_cast<float*>(sm + lay.ac);
    float* BD = reinterpret_cast<float*>(sm + lay.bd);
    bf16* Pb = reinterpret_cast<bf16*>(sm + lay.pb);
    const bf16** KP = reinterpret_cast<const bf16**>(sm + lay.kp);
    const bf16** VP = reinterpret_cast<const bf16**>(sm + lay.vp);

    // ---- per-key source rows: cached frame f = head - L + j in its page, or this chunk's row j - L (null when
    //      the page is not mapped, which is reported and read as zeros). Rows past the visible ones (this chunk's
    //      invalid frames) are staged for the append; the softmax gives them probability 0.
    const bf16* kpool = reinterpret_cast<const bf16*>(cg.kpool);
    const bf16* vpool = reinterpret_cast<const bf16*>(cg.vpool);
    for (int r = tid; r < na; r += kAttnThreads) {
        const int j = lo + r;
        const bf16 *ks = nullptr, *vs = nullptr;
        if (j < L) {
            const int f = head - L + j;
            const int page = me.pages[(f / PF) % kPageSlots];
            if (page >= 0 && page < cg.n_pages) {
                const size_t off = ((static_cast<size_t>(layer) * cg.n_pages + page) * PF + (f % PF)) * D + hoff;
                ks = kpool + off;
                vs = vpool + off;
            } else {
                report_error(err, DEV_BAD_PAGE);
            }
        } else {
            const bf16* src = qkv + static_cast<size_t>(row_off + (j - L)) * ld_qkv + hoff;
            ks = src + D;
            vs = src + 2 * D;
        }
        KP[r] = ks;
        VP[r] = vs;
    }
    __syncthreads();
    // ---- stage K, P and the raw queries (group 0) and V (group 1) with cp.async; zero the padding rows.
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    for (int idx = tid; idx < na * 16; idx += kAttnThreads) {
        const int r = idx >> 4, c = (idx & 15) * 8;
        const bf16* ks = KP[r];
        if (ks) cp_async16(Ks + r * RSB + c, ks + c);
        else *reinterpret_cast<uint4*>(Ks + r * RSB + c) = z;
    }
    for (int idx = tid; idx < np * 16; idx += kAttnThreads) {
        const int r = idx >> 4, c = (idx & 15) * 8;
        cp_async16(Ps + r * RSB + c, ptab + static_cast<size_t>(rel_min + r + tmax - 1) * D + hoff + c);
    }
    for (int idx = tid; idx < TM * 16; idx += kAttnThreads) {   // raw queries into QU (biased in place below)
        const int i = idx >> 4, c = (idx & 15) * 8;
        if (i < T_) cp_async16(QU + i * RSB + c, qkv + static_cast<size_t>(row_off + i) * ld_qkv + hoff + c);
        else *reinterpret_cast<uint4*>(QU + i * RSB + c) = z;
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int idx = tid; idx < na * 16; idx += kAttnThreads) {
        const int r = idx >> 4, c = (idx & 15) * 8;
        const bf16* vs = VP[r];
        if (vs) cp_async16(Vs + r * RSB + c, vs + c);
        else *reinterpret_cast<uint4*>(Vs + r * RSB + c) = z;
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int idx = tid; idx < (lay.nkp - na) * 16; idx += kAttnThreads) {
        const int r = na + (idx >> 4), c = (idx & 15) * 8;
        *reinterpret_cast<uint4*>(Ks + r * RSB + c) = z;
        *reinterpret_cast<uint4*>(Vs + r * RSB + c) = z;
    }
    for (int idx = tid; idx < (lay.npp - np) * 16; idx += kAttnThreads) {
        const int r = np + (idx >> 4), c = (idx & 15) * 8;
        *reinterpret_cast<uint4*>(Ps + r * RSB + c) = z;
    }
    asm volatile("cp.async.wait_group 1;" ::: "memory");   // K, P and the queries have landed; V may be in flight
    __syncthreads();
    // queries with the position biases, rounded to bf16 (rows >= T are zero), from the raw queries in QU
    for (int idx = tid; idx < TM * 16; idx += kAttnThreads) {
        const int i = idx >> 4, c = (idx & 15) * 8;
        float q[8], a[8], bb[8];
        load16<bf16>(QU + i * RSB + c, q);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            a[e] = i < T_ ? q[e] + bias_u[hoff + c + e] : 0.f;
            bb[e] = i < T_ ? q[e] + bias_v[hoff + c + e] : 0.f;
        }
        store16<bf16>(QU + i * RSB + c, a);
        store16<bf16>(QV + i * RSB + c, bb);
    }
    bf16* kw = reinterpret_cast<bf16*>(cg.kpool);
    bf16* vw = reinterpret_cast<bf16*>(cg.vpool);
    __syncthreads();

    // ---- AC and BDraw: jobs of two n-tiles (16 columns), one round over the warps.
    {
        const int arow = (lane & 7) + ((lane >> 3) & 1) * 8, acol = (lane >> 4) * 8;
        const int n_ac = (nk + 15) / 16, n_bd = (np + 15) / 16;
        const int g = lane >> 2, t4 = lane & 3;
        const int brow = (lane & 7) + ((lane >> 4) << 3), bcol = ((lane >> 3) & 1) * 8;
        for (int job = warp; job < n_ac + n_bd; job += kAttnWarps) {
            const bool is_ac = job < n_ac;
            const int n0 = (is_ac ? job : job - n_ac) * 16;
            const bf16* Bs = is_ac ? Ks : Ps;
            const bf16* As = is_ac ? QU : QV;
            float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                uint32_t a[4], bfr[4];
                ldsm_x4(a, As + arow * RSB + ks * 16 + acol);
                ldsm_x4(bfr, Bs + (n0 + brow) * RSB + ks * 16 + bcol);
                mma16816(c0, a, bfr[0], bfr[1]);
                mma16816(c1, a, bfr[2], bfr[3]);
            }
            float* dst = is_ac ? AC : BD;
            const int w = is_ac ? lay.acw : lay.bdw;
            *reinterpret_cast<float2*>(dst + g * w + n0 + 2 * t4) = make_float2(c0[0], c0[1]);
            *reinterpret_cast<float2*>(dst + (g + 8) * w + n0 + 2 * t4) = make_float2(c0[2], c0[3]);
            *reinterpret_cast<float2*>(dst + g * w + n0 + 8 + 2 * t4) = make_float2(c1[0], c1[1]);
            *reinterpret_cast<float2*>(dst + (g + 8) * w + n0 + 8 + 2 * t4) = make_float2(c1[2], c1[3]);
        }
    }
    __syncthreads();

    // ---- softmax rows (fp32), probabilities to bf16: one query row per warp
    const float scale = rsqrtf(static_cast<float>(DKk));
    for (int i = warp; i < TM; i += kAttnWarps) {
        bf16* prow = Pb + i * lay.psw;
        if (i >= T_ || nk == 0) {
            for (int jj = lane; jj < lay.nkp; jj += 32) prow[jj] = __float2bfloat16_rn(0.f);
            continue;
        }
        const float* acr = AC + i * lay.acw;
        const float* bdr = BD + i * lay.bdw + i + nk - 1;   // BDraw column for key jj is (i + nk - 1 - jj)
        constexpr int kPer = 4;                              // nkp <= 128 keys: at most 4 per lane
        float sv[kPer];
        float m = -INFINITY;
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int jj = lane + 32 * u;
            sv[u] = jj < nk ? (acr[jj] + bdr[-jj]) * scale : -INFINITY;
            m = fmaxf(m, sv[u]);
        }
        m = warp_max(m);
        float sum = 0.f;
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int jj = lane + 32 * u;
            sv[u] = jj < nk ? __expf(sv[u] - m) : 0.f;
            sum += sv[u];
        }
        sum = warp_sum(sum);
        const float inv = 1.f / sum;
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int jj = lane + 32 * u;
            if (jj < lay.nkp) prow[jj] = __float2bfloat16_rn(sv[u] * inv);
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");   // V
    __syncthreads();
    // ---- append this chunk's K/V rows (staged rows L - lo + t) at frames head + t, off the path to the AC/BD
    //      phase. Those pool rows are not read by this launch (the window is frames head - cacheLen .. head - 1,
    //      and the 8 page slots hold 128 frames).
    for (int idx = tid; idx < T_ * 16; idx += kAttnThreads) {
        const int t = idx >> 4, c = (idx & 15) * 8;
        const int f = head + t;
        const int page = me.pages[(f / PF) % kPageSlots];
        if (page < 0 || page >= cg.n_pages) {
            report_error(err, DEV_BAD_PAGE);
            continue;
        }
        const size_t off = ((static_cast<size_t>(layer) * cg.n_pages + page) * PF + (f % PF)) * D + hoff + c;
        *reinterpret_cast<uint4*>(kw + off) = *reinterpret_cast<const uint4*>(Ks + (L - lo + t) * RSB + c);
        *reinterpret_cast<uint4*>(vw + off) = *reinterpret_cast<const uint4*>(Vs + (L - lo + t) * RSB + c);
    }

    // ---- O = P . V: warp w owns output columns [8w, 8w + 8)
    {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const int arow = (lane & 7) + ((lane >> 3) & 1) * 8, acol = (lane >> 4) * 8;
        const int n0 = warp * 8;
        const int ksteps = (nk + 15) / 16;
        for (int ks = 0; ks < ksteps; ++ks) {
            uint32_t a[4], bfr[2];
            ldsm_x4(a, Pb + arow * lay.psw + ks * 16 + acol);
            ldsm_x2_t(bfr, Vs + (ks * 16 + (lane & 15)) * RSB + n0);
            mma16816(acc, a, bfr[0], bfr[1]);
        }
        const int g = lane >> 2, t4 = lane & 3;
        const int col = hoff + n0 + 2 * t4;
        if (g < T_)
            *reinterpret_cast<__nv_bfloat162*>(out + static_cast<size_t>(row_off + g) * ldo + col) =
                __floats2bfloat162_rn(acc[0], acc[1]);
        if (g + 8 < T_)
            *reinterpret_cast<__nv_bfloat162*>(out + static_cast<size_t>(row_off + g + 8) * ldo + col) =
                __floats2bfloat162_rn(acc[2], acc[3]);
    }

}

}  // namespace tc

// ---------------------------------------------------------------- persistent TMA-fed variant (bf16, T <= 16)
// The same attention and append as attn_tc_kernel, restructured so that a CTA's copies cost a few instructions
// and overlap its compute:
//   * one CTA per SM walks a contiguous range of (head, stream) items, head-major, so consecutive items share one
//     head; that head's slice of the projected position table (128 rows x 128 columns) is staged once per head and
//     stays resident (the items of one CTA span at most two heads);
//   * a producer warp stages item k + 1 while 16 compute warps work on item k (two stage buffers on mbarriers).
//     An item is staged by about 30 TMA tensor loads: one box of 16 frames x 64 columns per cache page touched by
//     the window and column half (the window's first and last page boxes start at the window's ends, so frames
//     outside it arrive as zeros without being read: the first box from the window's first frame, the last one
//     from a negative frame coordinate), one box for this chunk's new K, V and Q rows from the QKV projection;
//   * the compute warps address staged K and V rows through a per-item key -> row table (ldmatrix takes one row
//     address per lane), so the page boxes need not be contiguous; the staged rows keep TMA's 128-byte swizzle
//     (16-byte chunk c of row r at position c ^ (r % 8)), which makes the ldmatrix reads conflict-free.
// Math per item is attn_tc_kernel's: AC = (Q + u) K^T and BDraw = (Q + v) P^T with mma.sync m16n8k16, the band
// shift and softmax in fp32, O = softmax . V, and the chunk's K and V rows appended to their pages.
namespace tma_attn {

constexpr int kTM = 16;          // query rows per item (T <= 16)
constexpr int kKVRows = 112;     // staged K (and V) rows: 6 page boxes of 16 frames, then the chunk's rows
constexpr int kNewRow = 96;      // first staged row of this chunk's K / V
constexpr int kPRows = 128;      // staged position-table rows per head
constexpr int kNKP = 96;         // padded key count (at most L + T = 86 visible keys)
constexpr int kNPP = 112;        // padded position-row count (at most T + 86 - 1 = 101)
constexpr int kComputeWarps = 16;
constexpr int kThreads = (kComputeWarps + 1) * 32;
constexpr int RSB = 136;         // padded row of the biased queries (elements): conflict-free ldmatrix
constexpr int ACW = kNKP + 8, BDW = kNPP + 8, PSW = kNKP + 8;

struct Window {
    int T, valid_t, cl, head, row_off, lo, hi, nk, rel_min, np;
    int f0, p_first, p_last, npg, y0, ylast;
    int pages[kPageSlots];
};

struct Lay {
    static constexpr uint32_t HALF_KV = kKVRows * 128;                 // one 64-column half of the staged K rows
    static constexpr uint32_t STAGE = 4 * HALF_KV + 2 * kTM * 128;     // K0 K1 V0 V1 Q0 Q1
    static constexpr uint32_t PBUF = 2 * kPRows * 128;                 // one head's position rows: two column halves
    static constexpr uint32_t P = 0;                                   // a CTA's (at most two) heads' position rows
    static constexpr uint32_t S0 = 2 * PBUF;
    static constexpr uint32_t AC = S0 + 2 * STAGE;
    static constexpr uint32_t BD = AC + kTM * ACW * 4;
    static constexpr uint32_t PB = BD + kTM * BDW * 4;
    static constexpr uint32_t KROW = PB + kTM * PSW * 2;               // staged row of each key, per stage
    static constexpr uint32_t BIAS = KROW + 2 * kNKP * 4;              // this head's pos_bias_u, pos_bias_v (fp32)
    static constexpr uint32_t WIN = BIAS + 2 * 128 * 4;                // the item window of each stage
    static constexpr uint32_t ZERO = (WIN + 2 * sizeof(Window) + 127) / 128 * 128;   // one zero row (256 bytes)
    static constexpr uint32_t BAR = ZERO + 256;
    static constexpr uint32_t TOTAL = BAR + 64;
    static constexpr uint32_t SMEM = TOTAL + 1024;                     // room to align the base to 1024 bytes
};
static_assert(Lay::STAGE % 1024 == 0 && Lay::S0 % 1024 == 0 && Lay::HALF_KV % 1024 == 0, "swizzle alignment");
static_assert(Lay::SMEM <= 232448, "shared memory of the TMA attention kernel");

// Address of the 16-byte chunk c (0..15) of staged row r in a region of two 64-column halves of `rows` rows each,
// 128-byte swizzled; r < 0 is the zero row.
__device__ __forceinline__ const uint8_t* chunk_addr(const uint8_t* region, int rows, int r, int c, const uint8_t* zero) {
    if (r < 0) return zero + ((c & 7) << 4);
    return region + (c >> 3) * rows * 128 + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}

// Two bf16 values (a packed pair) plus two fp32 biases, rounded back to a bf16 pair.
__device__ __forceinline__ uint32_t add_bias2(uint32_t x, float2 bv) {
    __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&x);
    const float2 f = __bfloat1622float2(v);
    const __nv_bfloat162 r = __floats2bfloat162_rn(f.x + bv.x, f.y + bv.y);
    return *reinterpret_cast<const uint32_t*>(&r);
}

__device__ __forceinline__ void compute_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kComputeWarps * 32) : "memory"); }

__device__ __forceinline__ Window window_of(const BatchEntry& me, int L) {
    Window w;
    w.T = me.T;
    w.valid_t = me.valid_t;
    w.cl = me.cache_len;
    w.head = me.head;
    w.row_off = me.row_off;
    w.lo = L - w.cl;
    w.hi = L + w.valid_t;
    w.nk = w.hi > w.lo ? w.hi - w.lo : 0;
    w.rel_min = L - w.hi + 1;
    w.np = w.nk > 0 ? w.T + w.nk - 1 : 0;
    w.f0 = w.head - w.cl;
    if (w.cl > 0) {
        w.p_first = w.f0 >> 4;
        w.p_last = (w.head - 1) >> 4;
        w.npg = w.p_last - w.p_first + 1;
        w.y0 = w.f0 & 15;
        w.ylast = ((w.head - 1) & 15) + 1 - 16;
    } else {
        w.p_first = w.p_last = w.npg = w.y0 = w.ylast = 0;
    }
    for (int i = 0; i < kPageSlots; ++i) w.pages[i] = me.pages[i];
    return w;
}

// Staged row of key j (window index; keys [0, nk) visible), -1 for the padding keys.
__device__ __forceinline__ int key_row(const Window& w, int L, int j) {
    if (j >= w.nk) return -1;
    const int jj = w.lo + j;
    if (jj >= L) return kNewRow + (jj - L);
    const int f = w.f0 + j;
    const int pg = f >> 4, bx = pg - w.p_first;
    const int y = bx == 0 ? w.y0 : (pg == w.p_last ? w.ylast : 0);
    return 16 * bx + (f & 15) - y;
}

__global__ void __launch_bounds__(kThreads, 1) attn_tma_kernel(
    const __grid_constant__ CUtensorMap mqkv, const __grid_constant__ CUtensorMap mk,
    const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mp, int D, int L, int ptab_row0,
    const float* __restrict__ bias_u, const float* __restrict__ bias_v, const BatchEntry* __restrict__ meta, int n,
    int n_heads, int ipc, int layer, int n_pages, bf16* __restrict__ kw, bf16* __restrict__ vw, bf16* __restrict__ out,
    int ldo, int* err, unsigned long long* timer) {
    constexpr int DKk = 128;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + Lay::BAR);
    uint64_t* empty = full + 2;
    uint64_t* pfull = full + 4;   // per head of the CTA: its position rows have landed
    int* abort_flag = reinterpret_cast<int*>(full + 6);
    volatile int* abort_v = abort_flag;
    const uint8_t* zero = sm + Lay::ZERO;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int total = n * n_heads;
    const int first = blockIdx.x * ipc, last = min(total, first + ipc);

    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kComputeWarps);   // every compute warp releases the stage when done with it
        }
        mbar_init(&pfull[0], 1);
        mbar_init(&pfull[1], 1);
        *abort_flag = 0;
        fence_mbarrier_init();
        prefetch_tensormap(&mqkv);
        prefetch_tensormap(&mk);
        prefetch_tensormap(&mv);
        prefetch_tensormap(&mp);
    }
    if (tid < 64) reinterpret_cast<uint32_t*>(sm + Lay::ZERO)[tid] = 0u;
    __syncthreads();

    if (warp == kComputeWarps) {
        // ---------------------------------------------------------------- producer warp
        // Lane 0 issues the copies; the whole warp reads the next item's window (before waiting for its stage, so
        // the metadata load overlaps the wait) and writes the stage's key -> staged-row table. The first item's
        // position rows and cached page boxes are issued before the grid-dependency wait: none of them comes from
        // the previous kernel (the pages of this layer were written by this kernel in an earlier step, the
        // position table is a weight, the metadata is copied in before the step), so they overlap its tail; the
        // chunk's new K, V and Q rows, from the QKV projection, only after it.
        // The position rows of the CTA's heads (at most two: a CTA holds at most n items), each in its own buffer.
        if (lane == 0 && first < last) {
            const int h0 = first / n, h1 = (last - 1) / n;
            for (int hh = h0; hh <= h1 && hh <= h0 + 1; ++hh) {
                uint8_t* pbuf = sm + Lay::P + (hh - h0) * Lay::PBUF;
                mbar_arrive_expect_tx(&pfull[hh - h0], Lay::PBUF);
                tma_load_2d(pbuf, &mp, &pfull[hh - h0], hh * DKk, ptab_row0);
                tma_load_2d(pbuf + kPRows * 128, &mp, &pfull[hh - h0], hh * DKk + 64, ptab_row0);
            }
        }
        for (int k = 0; first + k < last; ++k) {
            const int item = first + k, h = item / n, b = item - h * n, s = k & 1;
            const Window wv = window_of(meta[b], L);
            int ok = 1;
            if (lane == 0 && k >= 2 && !mbar_wait_bounded(&empty[s], ((k - 2) >> 1) & 1, err, DEV_TIMEOUT_ATTN, abort_v))
                ok = 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            int* kr = reinterpret_cast<int*>(sm + Lay::KROW) + s * kNKP;
            for (int j = lane; j < kNKP; j += 32) kr[j] = key_row(wv, L, j);
            // The window and the table are published to the compute warps by the stage's full barrier: lane 0's
            // arrive (which also sets the expected bytes) follows them and precedes every copy.
            if (lane == 0) {
                reinterpret_cast<Window*>(sm + Lay::WIN)[s] = wv;
                mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>((wv.npg + 1) * 4 * 2048 + 2 * 2048));
            }
            __syncwarp();
            // The copies, spread over the warp's lanes: copy q < 4 npg is page box q / 4 (K or V, column half),
            // then the chunk's K, V and Q rows.
            uint8_t* st = sm + Lay::S0 + s * Lay::STAGE;
            const int n_copies = 4 * wv.npg + 6;
            for (int q = lane; q < n_copies; q += 32) {
                if (k == 0 && q >= 4 * wv.npg) continue;   // the first item's new rows: after the wait below
                if (q < 4 * wv.npg) {
                    const int bx = q >> 2, half = q & 1, isv = (q >> 1) & 1;
                    const int pg = wv.p_first + bx;
                    const int page = wv.pages[pg % kPageSlots];
                    int z = layer * n_pages + page;
                    if (page < 0 || page >= n_pages) {
                        report_error(err, DEV_BAD_PAGE);
                        z = -1;   // a page coordinate outside the pool: the box arrives as zeros
                    }
                    const int y = bx == 0 ? wv.y0 : (pg == wv.p_last ? wv.ylast : 0);
                    tma_load_3d(st + (2 * isv + half) * Lay::HALF_KV + bx * 16 * 128, isv ? &mv : &mk, &full[s],
                                h * DKk + half * 64, y, z);
                } else {
                    const int r = q - 4 * wv.npg, half = r & 1, which = r >> 1;   // which: 0 K, 1 V, 2 Q
                    uint8_t* dst = which < 2 ? st + (2 * which + half) * Lay::HALF_KV + kNewRow * 128
                                             : st + 4 * Lay::HALF_KV + half * kTM * 128;
                    const int xcol = (which == 0 ? D : which == 1 ? 2 * D : 0) + h * DKk + half * 64;
                    tma_load_2d(dst, &mqkv, &full[s], xcol, wv.row_off);
                }
            }
            if (k == 0) {
                pdl_wait();   // the QKV projection's outputs are read only from here on
                for (int r = lane; r < 6; r += 32) {
                    const int half = r & 1, which = r >> 1;   // which: 0 K, 1 V, 2 Q
                    uint8_t* dst = which < 2 ? st + (2 * which + half) * Lay::HALF_KV + kNewRow * 128
                                             : st + 4 * Lay::HALF_KV + half * kTM * 128;
                    const int xcol = (which == 0 ? D : which == 1 ? 2 * D : 0) + h * DKk + half * 64;
                    tma_load_2d(dst, &mqkv, &full[s], xcol, wv.row_off);
                }
            }
        }
        if (lane == 0) pdl_launch_dependents();
        return;
    }
    pdl_wait();   // compute warps: the previous kernel's grid has completed (its outputs reach them by the copies)
    if (tid == 0) timer_start(timer);

    // -------------------------------------------------------------------- compute warps
    float* AC = reinterpret_cast<float*>(sm + Lay::AC);
    float* BD = reinterpret_cast<float*>(sm + Lay::BD);
    bf16* Pb = reinterpret_cast<bf16*>(sm + Lay::PB);
    const int* krow_all = reinterpret_cast<const int*>(sm + Lay::KROW);
    float* bias = reinterpret_cast<float*>(sm + Lay::BIAS);   // [0, 128): pos_bias_u, [128, 256): pos_bias_v
    const float scale = rsqrtf(static_cast<float>(DKk));
    const int g = lane >> 2, t4 = lane & 3;
    volatile int* go = abort_flag + 1;
    const int h_first = first / n;
    int cur_h = -1;
    for (int k = 0; first + k < last; ++k) {
        const int item = first + k, h = item / n, s = k & 1;
        const int hoff = h * DKk, pb = (h - h_first) & 1;
        const uint8_t* Ps = sm + Lay::P + pb * Lay::PBUF;
        const bool new_head = h != cur_h;
        // One thread makes the bounded waits and the whole group follows its verdict, so that no warp leaves while
        // the others wait at a group barrier; then every thread observes the completed phases (at once).
        if (tid == 0) {
            bool ok = !new_head || mbar_wait_bounded(&pfull[pb], 0, err, DEV_TIMEOUT_ATTN, abort_v);
            ok = ok && mbar_wait_bounded(&full[s], (k >> 1) & 1, err, DEV_TIMEOUT_ATTN, abort_v);
            *go = ok ? 1 : 0;
        }
        if (new_head && tid < 2 * DKk) bias[tid] = (tid < DKk ? bias_u : bias_v)[hoff + (tid & (DKk - 1))];
        compute_sync();
        if (!*go) break;
        if (new_head) {
            mbar_wait_bounded(&pfull[pb], 0, err, DEV_TIMEOUT_ATTN, abort_v);
            cur_h = h;
        }
        mbar_wait_bounded(&full[s], (k >> 1) & 1, err, DEV_TIMEOUT_ATTN, abort_v);
        const Window& ws = reinterpret_cast<const Window*>(sm + Lay::WIN)[s];
        const uint8_t* st = sm + Lay::S0 + s * Lay::STAGE;
        const uint8_t* Ks = st;
        const uint8_t* Vs = st + 2 * Lay::HALF_KV;
        const uint8_t* Qs = st + 4 * Lay::HALF_KV;

        const int* krow = krow_all + s * kNKP;   // key -> staged row, written by the producer warp
        const int T_ = ws.T;
        const int nk = ws.nk, np = ws.np, rel_min = ws.rel_min, row_off = ws.row_off, head = ws.head;

        // ---- AC = (Q + u) K^T and BDraw = (Q + v) P^T: jobs of two n-tiles (16 columns), one round over the warps
        {
            // A: the staged query rows with the position bias added in the fragments, rounded to bf16 (rows >= T
            // zero): a[0] / a[1] hold columns 2 t4, 2 t4 + 1 of rows g / g + 8, a[2] / a[3] columns 8 + 2 t4,
            // 9 + 2 t4 of the same rows
            const int arow = (lane & 7) + ((lane >> 3) & 1) * 8, ahalf = lane >> 4;
            const bool z0 = g >= T_, z1 = g + 8 >= T_;
            const int n_ac = (nk + 15) / 16, n_bd = (np + 15) / 16;
            const int brow = (lane & 7) + ((lane >> 4) << 3), bsel = (lane >> 3) & 1;
            for (int job = warp; job < n_ac + n_bd; job += kComputeWarps) {
                const bool is_ac = job < n_ac;
                const int n0 = (is_ac ? job : job - n_ac) * 16;
                const float* bq = is_ac ? bias : bias + DKk;
                // this lane's B row: a key's staged K row, or a position-table row (rel_min + r -> row rel + 15)
                const int r = n0 + brow;
                const int brow_s = is_ac ? krow[r] : (rel_min + r + 15);
                const uint8_t* breg = is_ac ? Ks : Ps;
                const int brows = is_ac ? kKVRows : kPRows;
                float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    uint32_t a[4], bfr[4];
                    tc::ldsm_x4(a, chunk_addr(Qs, kTM, arow, 2 * ks + ahalf, zero));
                    {
                        const float2 b0 = *reinterpret_cast<const float2*>(bq + ks * 16 + 2 * t4);
                        const float2 b1 = *reinterpret_cast<const float2*>(bq + ks * 16 + 8 + 2 * t4);
                        a[0] = z0 ? 0u : add_bias2(a[0], b0);
                        a[1] = z1 ? 0u : add_bias2(a[1], b0);
                        a[2] = z0 ? 0u : add_bias2(a[2], b1);
                        a[3] = z1 ? 0u : add_bias2(a[3], b1);
                    }
                    tc::ldsm_x4(bfr, chunk_addr(breg, brows, brow_s, 2 * ks + bsel, zero));
                    tc::mma16816(c0, a, bfr[0], bfr[1]);
                    tc::mma16816(c1, a, bfr[2], bfr[3]);
                }
                float* dst = is_ac ? AC : BD;
                const int wd = is_ac ? ACW : BDW;
                *reinterpret_cast<float2*>(dst + g * wd + n0 + 2 * t4) = make_float2(c0[0], c0[1]);
                *reinterpret_cast<float2*>(dst + (g + 8) * wd + n0 + 2 * t4) = make_float2(c0[2], c0[3]);
                *reinterpret_cast<float2*>(dst + g * wd + n0 + 8 + 2 * t4) = make_float2(c1[0], c1[1]);
                *reinterpret_cast<float2*>(dst + (g + 8) * wd + n0 + 8 + 2 * t4) = make_float2(c1[2], c1[3]);
            }
        }
        compute_sync();

        // ---- softmax rows (fp32), probabilities to bf16: one query row per warp
        for (int i = warp; i < kTM; i += kComputeWarps) {
            bf16* prow = Pb + i * PSW;
            if (i >= T_ || nk == 0) {
                for (int jj = lane; jj < kNKP; jj += 32) prow[jj] = __float2bfloat16_rn(0.f);
                continue;
            }
            const float* acr = AC + i * ACW;
            const float* bdr = BD + i * BDW + i + nk - 1;   // BDraw column for key jj is (i + nk - 1 - jj)
            constexpr int kPer = kNKP / 32;
            float sv[kPer];
            float m = -INFINITY;
#pragma unroll
            for (int u = 0; u < kPer; ++u) {
                const int jj = lane + 32 * u;
                sv[u] = jj < nk ? (acr[jj] + bdr[-jj]) * scale : -INFINITY;
                m = fmaxf(m, sv[u]);
            }
            m = warp_max(m);
            float sum = 0.f;
#pragma unroll
            for (int u = 0; u < kPer; ++u) {
                const int jj = lane + 32 * u;
                sv[u] = jj < nk ? __expf(sv[u] - m) : 0.f;
                sum += sv[u];
            }
            sum = warp_sum(sum);
            const float inv = 1.f / sum;
#pragma unroll
            for (int u = 0; u < kPer; ++u) prow[lane + 32 * u] = __float2bfloat16_rn(sv[u] * inv);
        }
        compute_sync();

        // ---- append this chunk's K/V rows (staged rows kNewRow + t) at frames head + t
        for (int idx = tid; idx < T_ * 32; idx += kComputeWarps * 32) {
            const int t = idx >> 5, isv = (idx >> 4) & 1, c = idx & 15;
            const int f = head + t;
            const int page = ws.pages[(f >> 4) % kPageSlots];
            if (page < 0 || page >= n_pages) {
                report_error(err, DEV_BAD_PAGE);
                continue;
            }
            const size_t off = ((static_cast<size_t>(layer) * n_pages + page) * 16 + (f & 15)) * D + hoff + c * 8;
            const uint4 v = *reinterpret_cast<const uint4*>(chunk_addr(isv ? Vs : Ks, kKVRows, kNewRow + t, c, zero));
            *reinterpret_cast<uint4*>((isv ? vw : kw) + off) = v;
        }

        // ---- O = P . V: warp w owns output columns [8 w, 8 w + 8)
        {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            const int arow = (lane & 7) + ((lane >> 3) & 1) * 8, acol = (lane >> 4) * 8;
            const int ksteps = (nk + 15) / 16;
            for (int ks = 0; ks < ksteps; ++ks) {
                uint32_t a[4], bfr[2];
                tc::ldsm_x4(a, Pb + arow * PSW + ks * 16 + acol);
                tc::ldsm_x2_t(bfr, chunk_addr(Vs, kKVRows, krow[ks * 16 + (lane & 15)], warp, zero));
                tc::mma16816(acc, a, bfr[0], bfr[1]);
            }
            const int col = hoff + warp * 8 + 2 * t4;
            if (g < T_)
                *reinterpret_cast<__nv_bfloat162*>(out + static_cast<size_t>(row_off + g) * ldo + col) =
                    __floats2bfloat162_rn(acc[0], acc[1]);
            if (g + 8 < T_)
                *reinterpret_cast<__nv_bfloat162*>(out + static_cast<size_t>(row_off + g + 8) * ldo + col) =
                    __floats2bfloat162_rn(acc[2], acc[3]);
        }
        // This warp's reads of the stage and the window are done: it releases them (the scores are rewritten only
        // after the next item's group barrier, which every warp reaches after this point).
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    compute_sync();   // every compute warp has finished its last item
    if (tid == 0) timer_end(timer);   // after the last item's group barrier: every compute warp is done
    if (*abort_v) __nanosleep(100000);   // after a failed wait: let copies already issued into this CTA land
}

}  // namespace tma_attn

}  // namespace

template <typename T>
void relpos_attention(const T* qkv, int ld_qkv, const T* ptab, int tmax, const float* bias_u, const float* bias_v,
                      const BatchEntry* meta, int n, int tmax_batch, const CacheGeom& cg, int layer, T* out, int ldo,
                      int n_heads, int* dev_err, cudaStream_t s) {
    if (n <= 0) return;
    if constexpr (std::is_same<T, bf16>::value) {
        if (tmax_batch <= tc::TM && cg.L + tc::TM <= 128) {
            const tc::Lay lay(cg.L);
            static size_t tc_attr[kMaxDevices] = {};
            ensure_dyn_smem(tc::attn_tc_kernel, lay.total, tc_attr);
            dim3 grid(n, n_heads);
            launch_pdl(tc::attn_tc_kernel, dim3(grid), dim3(tc::kAttnThreads), lay.total, s, qkv, ld_qkv, ptab, tmax, bias_u, bias_v, meta, cg, layer,
                                                            out, ldo, dev_err);
            return;
        }
    }
    const AttnSmem<T> lay(tmax_batch, cg.L);
    static size_t attr_set[kMaxDevices] = {};
    if (lay.total > 48 * 1024) ensure_dyn_smem(relpos_attn_kernel<T>, lay.total, attr_set);
    dim3 grid(n, n_heads);
    launch_pdl(relpos_attn_kernel<T>, dim3(grid), dim3(256), lay.total, s, qkv, ld_qkv, ptab, tmax, bias_u, bias_v, meta, cg, layer, out,
                                                       ldo, tmax_batch, dev_err);
}

bool relpos_attention_tma(const TmaMatrix& qkv, const TmaMatrix& kpool, const TmaMatrix& vpool, const TmaMatrix& ptab,
                          int ptab_row0, const float* bias_u, const float* bias_v, const BatchEntry* meta, int n,
                          int tmax_batch, const CacheGeom& cg, int layer, bf16* out, int ldo, int n_heads, int num_sms,
                          int* dev_err, cudaStream_t s, unsigned long long* timer) {
    using namespace tma_attn;
    if (n <= 0) return true;
    if (tmax_batch > kTM || cg.page_frames != 16 || cg.L + kTM - 1 + 15 >= kPRows || cg.L + kTM > kNKP) return false;
    const int total = n * n_heads;
    int ipc = (total + num_sms - 1) / num_sms;
    if (ipc > n) ipc = n;   // a CTA's items then span at most two heads
    const int grid = (total + ipc - 1) / ipc;
    static size_t attr[kMaxDevices] = {};
    ensure_dyn_smem(attn_tma_kernel, Lay::SMEM, attr);
    launch_pdl(attn_tma_kernel, dim3(grid), dim3(kThreads), Lay::SMEM, s, qkv.map, kpool.map, vpool.map, ptab.map, cg.D,
               cg.L, ptab_row0, bias_u, bias_v, meta, n, n_heads, ipc, layer, cg.n_pages,
               reinterpret_cast<bf16*>(cg.kpool), reinterpret_cast<bf16*>(cg.vpool), out, ldo, dev_err, timer);
    return true;
}

size_t relpos_attention_smem_bytes(int tmax_batch, int L, int elem_bytes) {
    return elem_bytes == 2 ? AttnSmem<bf16>(tmax_batch, L).total : AttnSmem<float>(tmax_batch, L).total;
}

template void relpos_attention<float>(const float*, int, const float*, int, const float*, const float*,
                                      const BatchEntry*, int, int, const CacheGeom&, int, float*, int, int, int*,
                                      cudaStream_t);
template void relpos_attention<bf16>(const bf16*, int, const bf16*, int, const float*, const float*, const BatchEntry*,
                                     int, int, const CacheGeom&, int, bf16*, int, int, int*, cudaStream_t);

}  // namespace ud
