// Paged per-stream ring caches: append, gather and slot reset (the data movement of the reference's
// cache roll, FastConformer.swift:464-477, and its zero-initialised StreamState, :416-428).
//
// K/V: frame f of a stream lives at row f % PF of page pages[(f / PF) % kPageSlots] in the layer's pool;
// the roll only advances `head`, so it moves no data. Conv: ring of conv_ring rows per (layer, slot),
// frame f at row f % conv_ring. All copies are 16-byte vectors, one row per warp group, coalesced.
#include "common.cuh"
#include "kernels.h"

namespace ud {
namespace {

// grid (n, n_layers), 256 threads. kv_rows [n][NL][2][k][D], conv_rows [n][NL][k][D].
template <typename T>
__global__ void append_kernel(const T* __restrict__ kv_rows, const T* __restrict__ conv_rows, int k,
                              const BatchEntry* __restrict__ meta, const CacheGeom cg, int* err) {
    constexpr int CH = 16 / sizeof(T);
    const int b = blockIdx.x, layer = blockIdx.y;
    const BatchEntry& me = meta[b];
    const int D = cg.D, PF = cg.page_frames, NL = cg.n_layers, R = cg.conv_ring;
    const int cpr = D / CH;
    if (kv_rows) {
        const T* src = kv_rows + (static_cast<size_t>(b) * NL + layer) * 2 * k * D;
        for (int idx = threadIdx.x; idx < 2 * k * cpr; idx += blockDim.x) {
            const int kind = idx / (k * cpr);
            const int rem = idx % (k * cpr);
            const int t = rem / cpr, c = (rem % cpr) * CH;
            const int f = me.head + t;
            const int page = me.pages[(f / PF) % kPageSlots];
            if (page < 0 || page >= cg.n_pages) {
                report_error(err, DEV_BAD_PAGE);
                continue;
            }
            T* pool = reinterpret_cast<T*>(kind == 0 ? cg.kpool : cg.vpool);
            const size_t off = ((static_cast<size_t>(layer) * cg.n_pages + page) * PF + (f % PF)) * D + c;
            *reinterpret_cast<uint4*>(pool + off) =
                *reinterpret_cast<const uint4*>(src + (static_cast<size_t>(kind) * k + t) * D + c);
        }
    }
    if (conv_rows) {
        const T* src = conv_rows + (static_cast<size_t>(b) * NL + layer) * k * D;
        T* ring = reinterpret_cast<T*>(cg.conv) + (static_cast<size_t>(layer) * cg.max_streams + me.slot) * R * D;
        const int t0 = k > R ? k - R : 0;  // only the last R new frames survive
        for (int idx = threadIdx.x; idx < (k - t0) * cpr; idx += blockDim.x) {
            const int t = t0 + idx / cpr, c = (idx % cpr) * CH;
            *reinterpret_cast<uint4*>(ring + static_cast<size_t>((me.head + t) % R) * D + c) =
                *reinterpret_cast<const uint4*>(src + static_cast<size_t>(t) * D + c);
        }
    }
}

// grid (n, n_layers), 256 threads. kv_out [n][NL][2][L][D] (window, unfilled rows zero), conv_out [n][NL][R][D].
template <typename T>
__global__ void gather_kernel(T* __restrict__ kv_out, T* __restrict__ conv_out, const BatchEntry* __restrict__ meta,
                              const CacheGeom cg, int* err) {
    constexpr int CH = 16 / sizeof(T);
    const int b = blockIdx.x, layer = blockIdx.y;
    const BatchEntry& me = meta[b];
    const int D = cg.D, PF = cg.page_frames, NL = cg.n_layers, L = cg.L, R = cg.conv_ring;
    const int cpr = D / CH;
    if (kv_out) {
        T* dst = kv_out + (static_cast<size_t>(b) * NL + layer) * 2 * L * D;
        for (int idx = threadIdx.x; idx < 2 * L * cpr; idx += blockDim.x) {
            const int kind = idx / (L * cpr);
            const int rem = idx % (L * cpr);
            const int j = rem / cpr, c = (rem % cpr) * CH;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (j >= L - me.cache_len) {
                const int f = me.head - L + j;
                const int page = me.pages[(f / PF) % kPageSlots];
                if (page < 0 || page >= cg.n_pages) {
                    report_error(err, DEV_BAD_PAGE);
                } else {
                    const T* pool = reinterpret_cast<const T*>(kind == 0 ? cg.kpool : cg.vpool);
                    v = *reinterpret_cast<const uint4*>(
                        pool + ((static_cast<size_t>(layer) * cg.n_pages + page) * PF + (f % PF)) * D + c);
                }
            }
            *reinterpret_cast<uint4*>(dst + (static_cast<size_t>(kind) * L + j) * D + c) = v;
        }
    }
    if (conv_out) {
        const T* ring =
            reinterpret_cast<const T*>(cg.conv) + (static_cast<size_t>(layer) * cg.max_streams + me.slot) * R * D;
        T* dst = conv_out + (static_cast<size_t>(b) * NL + layer) * R * D;
        for (int idx = threadIdx.x; idx < R * cpr; idx += blockDim.x) {
            const int i = idx / cpr, c = (idx % cpr) * CH;  // frame head - R + i
            *reinterpret_cast<uint4*>(dst + static_cast<size_t>(i) * D + c) =
                *reinterpret_cast<const uint4*>(ring + static_cast<size_t>((me.head + i) % R) * D + c);
        }
    }
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
    if (n <= 0 || k <= 0 || cg.n_layers <= 0) return;
    dim3 grid(n, cg.n_layers);
    append_kernel<T><<<grid, 256, 0, s>>>(kv_rows, conv_rows, k, meta, cg, dev_err);
}

template <typename T>
void cache_gather(T* kv_out, T* conv_out, const BatchEntry* meta, int n, const CacheGeom& cg, int* dev_err,
                  cudaStream_t s) {
    if (n <= 0 || cg.n_layers <= 0) return;
    dim3 grid(n, cg.n_layers);
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
