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

}  // namespace

template <typename T>
void relpos_attention(const T* qkv, int ld_qkv, const T* ptab, int tmax, const float* bias_u, const float* bias_v,
                      const BatchEntry* meta, int n, int tmax_batch, const CacheGeom& cg, int layer, T* out, int ldo,
                      int n_heads, int* dev_err, cudaStream_t s) {
    if (n <= 0) return;
    const AttnSmem<T> lay(tmax_batch, cg.L);
    static size_t attr_set = 0;
    if (lay.total > 48 * 1024 && lay.total > attr_set) {
        cudaFuncSetAttribute(relpos_attn_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(lay.total));
        attr_set = lay.total;
    }
    dim3 grid(n, n_heads);
    relpos_attn_kernel<T><<<grid, 256, lay.total, s>>>(qkv, ld_qkv, ptab, tmax, bias_u, bias_v, meta, cg, layer, out,
                                                       ldo, tmax_batch, dev_err);
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
