// Paged per-stream ring caches: append, gather and slot reset (the data movement of the reference's
// cache roll, FastConformer.swift:464-477, and its zero-initialised StreamState, :416-428).
//
// K/V: frame f of a stream lives at row f % PF of page pages[(f / PF) % kPageSlots] in the layer's pool;
// the roll only advances `head`, so it moves no data. Conv: ring of conv_ring rows per (layer, slot),
// frame f at row f % conv_ring. All copies are 16-byte vectors, one row per warp, coalesced.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace ud {
namespace {

// Rows are moved one warp per row: each lane copies up to kPer 16-byte chunks of the row (a bf16 row of 1024 is
// 128 chunks, 4 per lane), all its loads issued before its stores, so a warp keeps a whole 2 KB row in flight and no
// per-element index division is needed.
constexpr int kPer = 8;   // chunks per lane: rows of up to 256 chunks (d_model 1024 in fp32)

template <typename T>
__device__ __forceinline__ void copy_row(T* __restrict__ dst, const T* __restrict__ src, int cpr, int lane) {
    constexpr int CH = 16 / sizeof(T);
    uint4 v[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int c = lane + 32 * i;
        v[i] = (src && c < cpr) ? *reinterpret_cast<const uint4*>(src + c * CH) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int c = lane + 32 * i;
        if (c < cpr) *reinterpret_cast<uint4*>(dst + c * CH) = v[i];
    }
}

// Row f of a layer's K or V pool (nullptr, with the error recorded, when its page slot is unmapped).
template <typename T>
__device__ __forceinline__ T* pool_row(const CacheGeom& cg, int kind, int layer, const BatchEntry& me, int f, int* err) {
    const int PF = cg.page_frames;
    const int page = me.pages[(f / PF) % kPageSlots];
    if (page < 0 || page >= cg.n_pages) {
        report_error(err, DEV_BAD_PAGE);
        return nullptr;
    }
    T* pool = reinterpret_cast<T*>(kind == 0 ? cg.kpool : cg.vpool);
    return pool + ((static_cast<size_t>(layer) * cg.n_pages + page) * PF + (f % PF)) * cg.D;
}

// One warp per appended row over the whole call (appends are a few rows per stream and layer, so a CTA per
// (stream, layer) would leave most of its warps idle): row w of the call is (stream b, layer, r) with r in
// [0, 2k) a K (r < k) or V row and r in [2k, 2k + kc) one of the last kc = min(k, R) conv rows.
// kv_rows [n][NL][2][k][D], conv_rows [n][NL][k][D] (either may be null).
template <typename T>
__global__ void append_kernel(const T* __restrict__ kv_rows, const T* __restrict__ conv_rows, int k, int n,
                              const BatchEntry* __restrict__ meta, const CacheGeom cg, int* err) {
    constexpr int CH = 16 / sizeof(T);
    const int lane = threadIdx.x & 31;
    const int D = cg.D, NL = cg.n_layers, R = cg.conv_ring;
    const int cpr = D / CH;
    const int kc = conv_rows ? (k < R ? k : R) : 0;
    const int kv = kv_rows ? 2 * k : 0;
    const int per = kv + kc;   // rows per (stream, layer)
    const long long total = static_cast<long long>(n) * NL * per;
    for (long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < total;
         w += (static_cast<long long>(gridDim.x) * blockDim.x) >> 5) {
        const int r = static_cast<int>(w % per);
        const long long bl = w / per;
        const int layer = static_cast<int>(bl % NL), b = static_cast<int>(bl / NL);
        const BatchEntry& me = meta[b];
        if (r < kv) {
            const int kind = r >= k ? 1 : 0, t = r - kind * k;
            T* dst = pool_row<T>(cg, kind, layer, me, me.head + t, err);
            if (dst) copy_row<T>(dst, kv_rows + ((static_cast<size_t>(b) * NL + layer) * 2 * k + r) * D, cpr, lane);
        } else {
            const int t = k - kc + (r - kv);   // only the last R new frames survive in the ring
            T* ring = reinterpret_cast<T*>(cg.conv) + (static_cast<size_t>(layer) * cg.max_streams + me.slot) * R * D;
            copy_row<T>(ring + static_cast<size_t>((me.head + t) % R) * D,
                        conv_rows + ((static_cast<size_t>(b) * NL + layer) * k + t) * D, cpr, lane);
        }
    }
}

// grid (n, n_layers), 256 threads. kv_out [n][NL][2][L][D] (window, unfilled rows zero), conv_out [n][NL][R][D].
template <typename T>
__global__ void gather_kernel(T* __restrict__ kv_out, T* __restrict__ conv_out, const BatchEntry* __restrict__ meta,
                              const CacheGeom cg, int* err) {
    constexpr int CH = 16 / sizeof(T);
    const int b = blockIdx.x, layer = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const BatchEntry& me = meta[b];
    const int D = cg.D, NL = cg.n_layers, L = cg.L, R = cg.conv_ring;
    const int cpr = D / CH;
    if (kv_out) {
        T* dst = kv_out + (static_cast<size_t>(b) * NL + layer) * 2 * L * D;
        const int lo = L - me.cache_len;
        for (int row = warp; row < 2 * L; row += nw) {   // row = kind * L + j; window row j is frame head - L + j
            const int kind = row >= L ? 1 : 0, j = row - kind * L;
            const T* src = j >= lo ? pool_row<T>(cg, kind, layer, me, me.head - L + j, err) : nullptr;
            copy_row<T>(dst + static_cast<size_t>(row) * D, src, cpr, lane);
        }
    }
    if (conv_out) {
        const T* ring =
            reinterpret_cast<const T*>(cg.conv) + (static_cast<size_t>(layer) * cg.max_streams + me.slot) * R * D;
        T* dst = conv_out + (static_cast<size_t>(b) * NL + layer) * R * D;
        for (int i = warp; i < R; i += nw)   // frame head - R + i
            copy_row<T>(dst + static_cast<size_t>(i) * D, ring + static_cast<size_t>((me.head + i) % R) * D, cpr, lane);
    }
}

// The same gather by bulk copies (TMA engine, no multicast): a window's rows are contiguous within each page, and
// the conv ring's within each of its two wrapped parts, so one thread splits the CTA's output into runs of up to
// kGatherBytes and moves each run global -> shared (cp.async.bulk on an mbarrier, bounded wait) -> global (bulk
// store), two runs in flight. The window's unfilled rows are zeroed by all threads with plain stores first.
// grid (n, n_layers), 128 threads, 2 * kGatherBytes of dynamic shared memory.
constexpr int kGatherBytes = 32 * 1024;
constexpr int kMaxRuns = 40;

template <typename T>
__global__ void __launch_bounds__(128) gather_bulk_kernel(T* __restrict__ kv_out, T* __restrict__ conv_out,
                                                          const BatchEntry* __restrict__ meta, const CacheGeom cg,
                                                          int* err) {
    constexpr int CH = 16 / sizeof(T);
    extern __shared__ __align__(128) unsigned char gsm[];
    __shared__ uint64_t bar[2];
    __shared__ int fail;
    const int b = blockIdx.x, layer = blockIdx.y;
    const BatchEntry& me = meta[b];
    const int D = cg.D, NL = cg.n_layers, L = cg.L, R = cg.conv_ring, PF = cg.page_frames;
    const uint32_t row_bytes = static_cast<uint32_t>(D * sizeof(T));
    const int run_max = kGatherBytes / static_cast<int>(row_bytes);
    const int lo = L - me.cache_len;   // window rows j < lo hold no frame yet: zero
    T* kvd = kv_out ? kv_out + (static_cast<size_t>(b) * NL + layer) * 2 * L * D : nullptr;
    if (kvd && lo > 0) {
        const int n16 = lo * D / CH;
        for (int kind = 0; kind < 2; ++kind)
            for (int i = threadIdx.x; i < n16; i += blockDim.x)
                reinterpret_cast<uint4*>(kvd + static_cast<size_t>(kind) * L * D)[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    if (threadIdx.x == 0) {
        fail = 0;
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbarrier_init();
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    // The runs: (source, destination, rows).
    const T* rsrc[kMaxRuns];
    T* rdst[kMaxRuns];
    int rrows[kMaxRuns];
    int nr = 0;
    if (kvd) {
        T* pools[2] = {reinterpret_cast<T*>(cg.kpool), reinterpret_cast<T*>(cg.vpool)};
        for (int kind = 0; kind < 2; ++kind) {
            for (int j = lo > 0 ? lo : 0; j < L;) {
                const int f = me.head - L + j;
                const int page = me.pages[(f / PF) % kPageSlots];
                int rows = PF - f % PF;
                rows = min(rows, L - j);
                rows = min(rows, run_max);
                T* dst = kvd + (static_cast<size_t>(kind) * L + j) * D;
                if (page < 0 || page >= cg.n_pages) {   // unmapped: recorded, the rows read as zero
                    report_error(err, DEV_BAD_PAGE);
                    for (int i = 0; i < rows * D / CH; ++i) reinterpret_cast<uint4*>(dst)[i] = make_uint4(0u, 0u, 0u, 0u);
                } else if (nr < kMaxRuns) {
                    rsrc[nr] = pools[kind] + ((static_cast<size_t>(layer) * cg.n_pages + page) * PF + f % PF) * D;
                    rdst[nr] = dst;
                    rrows[nr++] = rows;
                }
                j += rows;
            }
        }
    }
    if (conv_out) {
        const T* ring = reinterpret_cast<const T*>(cg.conv) + (static_cast<size_t>(layer) * cg.max_streams + me.slot) * R * D;
        T* dst = conv_out + (static_cast<size_t>(b) * NL + layer) * R * D;
        for (int i = 0; i < R;) {   // output row i is frame head - R + i, ring row (head + i) % R
            const int rr = (me.head + i) % R;
            const int rows = min(min(R - rr, R - i), run_max);
            if (nr < kMaxRuns) {
                rsrc[nr] = ring + static_cast<size_t>(rr) * D;
                rdst[nr] = dst + static_cast<size_t>(i) * D;
                rrows[nr++] = rows;
            }
            i += rows;
        }
    }
    T* buf[2] = {reinterpret_cast<T*>(gsm), reinterpret_cast<T*>(gsm + kGatherBytes)};
    uint32_t phase[2] = {0u, 0u};
    auto issue = [&](int r) {
        const int s = r & 1;
        const uint32_t bytes = static_cast<uint32_t>(rrows[r]) * row_bytes;
        mbar_arrive_expect_tx(&bar[s], bytes);
        bulk_load(buf[s], rsrc[r], bytes, &bar[s]);
    };
    if (nr > 0) issue(0);
    for (int r = 0; r < nr; ++r) {
        const int s = r & 1;
        if (r + 1 < nr) {
            if (r >= 1) tma_store_wait_read<0>();   // run r - 1's store has read the buffer run r + 1 reuses
            issue(r + 1);
        }
        if (!mbar_wait_bounded(&bar[s], phase[s], err, DEV_TIMEOUT_COPY, &fail)) break;
        phase[s] ^= 1u;
        bulk_store(rdst[r], buf[s], static_cast<uint32_t>(rrows[r]) * row_bytes);
        tma_store_commit();
    }
    tma_store_wait_all();
    if (fail) __nanosleep(100000);   // an expired wait: give loads already issued into this CTA time to land
}

// grid (n, n_layers): zero the conv ring of each listed slot.
template <typename T>
__global__ void conv_zero_kernel(const int* __restrict__ slots, const CacheGeom cg) {
    constexpr int CH = 16 / sizeof(T);
    const int layer = blockIdx.y;
    T* ring = reinterpret_cast<T*>(cg.conv) + (static_cast<size_t>(layer) * cg.max_streams + slots[blockIdx.x]) *
                                                  cg.conv_ring * cg.D;
    const int n16 = cg.conv_ring * cg.D / CH;
    for (int i = threadIdx.x; i < n16; i += blockDim.x)
        reinterpret_cast<uint4*>(ring)[i] = make_uint4(0u, 0u, 0u, 0u);
}

}  // namespace

template <typename T>
void cache_append(const T* kv_rows, const T* conv_rows, int k, const BatchEntry* meta, int n, const CacheGeom& cg,
                  int* dev_err, cudaStream_t s) {
    if (n <= 0 || k <= 0 || cg.n_layers <= 0 || (!kv_rows && !conv_rows)) return;
    const long long rows = static_cast<long long>(n) * cg.n_layers *
                           ((kv_rows ? 2 * k : 0) + (conv_rows ? (k < cg.conv_ring ? k : cg.conv_ring) : 0));
    const long long blocks = (rows + 7) / 8;   // 8 warps per block, one row each; the kernel strides beyond
    const int grid = static_cast<int>(blocks < 65535LL * 16 ? blocks : 65535LL * 16);
    append_kernel<T><<<grid, 256, 0, s>>>(kv_rows, conv_rows, k, n, meta, cg, dev_err);
}

template <typename T>
void cache_gather(T* kv_out, T* conv_out, const BatchEntry* meta, int n, const CacheGeom& cg, int* dev_err,
                  cudaStream_t s) {
    if (n <= 0 || cg.n_layers <= 0) return;
    dim3 grid(n, cg.n_layers);
    static int bulk = -1;
    if (bulk < 0) {
        const char* v = std::getenv("UD_GATHER_BULK");
        bulk = v ? std::atoi(v) : 1;
    }
    const bool aligned = (cg.D * sizeof(T)) % 16 == 0 && static_cast<int>(cg.D * sizeof(T)) <= kGatherBytes;
    // runs: per kind at most one per page boundary or kGatherBytes of rows crossed, plus the ring's two parts
    const int rm = aligned ? std::min(kGatherBytes / static_cast<int>(cg.D * sizeof(T)), cg.page_frames) : 1;
    const bool fits = 2 * ((cg.L + rm - 1) / rm + 1) + 2 <= kMaxRuns;
    if (bulk && aligned && fits) {
        static size_t attr[kMaxDevices] = {};
        ensure_dyn_smem(gather_bulk_kernel<T>, 2 * kGatherBytes, attr);
        gather_bulk_kernel<T><<<grid, 128, 2 * kGatherBytes, s>>>(kv_out, conv_out, meta, cg, dev_err);
        return;
    }
    gather_kernel<T><<<grid, 256, 0, s>>>(kv_out, conv_out, meta, cg, dev_err);
}

template <typename T>
void conv_slot_zero(const int* slots, int n, const CacheGeom& cg, cudaStream_t s) {
    if (n <= 0 || cg.n_layers <= 0) return;
    dim3 grid(n, cg.n_layers);
    conv_zero_kernel<T><<<grid, 256, 0, s>>>(slots, cg);
}

template void cache_append<float>(const float*, const float*, int, const BatchEntry*, int, const CacheGeom&, int*,
                                  cudaStream_t);
template void cache_append<bf16>(const bf16*, const bf16*, int, const BatchEntry*, int, const CacheGeom&, int*,
                                 cudaStream_t);
template void cache_gather<float>(float*, float*, const BatchEntry*, int, const CacheGeom&, int*, cudaStream_t);
template void cache_gather<bf16>(bf16*, bf16*, const BatchEntry*, int, const CacheGeom&, int*, cudaStream_t);
template void conv_slot_zero<float>(const int*, int, const CacheGeom&, cudaStream_t);
template void conv_slot_zero<bf16>(const int*, int, const CacheGeom&, cudaStream_t);

}  // namespace ud
