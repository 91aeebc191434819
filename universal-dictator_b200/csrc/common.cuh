// Shared device helpers for the B200 (sm_100a) kernels of libud.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <type_traits>

namespace ud {

using bf16 = __nv_bfloat16;

// Error codes a kernel writes into the engine's device error word (first writer wins).
enum DeviceError : int {
    DEV_OK = 0,
    DEV_TIMEOUT_FULL = 1,       // GEMM: waiting for a TMA stage
    DEV_TIMEOUT_EMPTY = 2,      // GEMM: waiting for a free stage
    DEV_TIMEOUT_ACC_FULL = 3,   // GEMM: waiting for the accumulator
    DEV_TIMEOUT_ACC_EMPTY = 4,  // GEMM: waiting for the epilogue to drain TMEM
    DEV_BAD_PAGE = 5,           // cache: a page slot needed by a kernel is unmapped
    DEV_TIMEOUT_TEST = 6,       // the failure-detection test wait
    DEV_TIMEOUT_GRID = 7,       // RNN-T: waiting at a grid barrier of the lock-step decoder
    DEV_TIMEOUT_ATTN = 8,       // attention: waiting for a staged item or a free stage
    DEV_RANGE_F16 = 9,          // RNN-T tensor-core decoder: an operand value beyond the fp16 range
    DEV_TIMEOUT_CONV = 10,      // conv module: waiting for its ring rows and LayerNorm parameters
    DEV_TIMEOUT_COPY = 11,      // cache gather: waiting for a staged run of rows
};

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<bf16>(bf16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ bf16 from_f<bf16>(float v) { return __float2bfloat16_rn(v); }

// 16-byte vector of T: 4 floats or 8 bf16.
template <typename T> struct Vec16;
template <> struct Vec16<float> { static constexpr int N = 4; };
template <> struct Vec16<bf16> { static constexpr int N = 8; };

template <typename T>
__device__ __forceinline__ void load16(const T* p, float* out) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    if constexpr (sizeof(T) == 4) {
        out[0] = __uint_as_float(u.x); out[1] = __uint_as_float(u.y);
        out[2] = __uint_as_float(u.z); out[3] = __uint_as_float(u.w);
    } else {
        const bf16* h = reinterpret_cast<const bf16*>(&u);
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] = __bfloat162float(h[i]);
    }
}

template <typename T>
__device__ __forceinline__ void store16(T* p, const float* v) {
    uint4 u;
    if constexpr (sizeof(T) == 4) {
        u.x = __float_as_uint(v[0]); u.y = __float_as_uint(v[1]);
        u.z = __float_as_uint(v[2]); u.w = __float_as_uint(v[3]);
    } else {
        bf16* h = reinterpret_cast<bf16*>(&u);
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = __float2bfloat16_rn(v[i]);
    }
    *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// The PTX tanh.approx.f32 instruction: one special-function operation, relative error about 2^-11.
__device__ __forceinline__ float tanh_approx(float x) {
    float t;
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(x));
    return t;
}
// x * sigmoid(q) for results that are rounded to bf16 (relative 2^-9): x * (0.5 + 0.5 tanh(q / 2)), one
// special-function operation where x / (1 + e^-q) takes two (exponential and reciprocal). The special-function
// unit delivers 16 results per clock per SM, and the GLU / SiLU epilogues of a C3 step queue on it.
__device__ __forceinline__ float x_sigmoid_bf16out(float x, float q) { return x * fmaf(0.5f, tanh_approx(0.5f * q), 0.5f); }
__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + __expf(-x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Graph-mode kernel timers (off unless the engine hands a kernel a slot): slot p receives in p[0] the earliest
// global-timer time (ns) at which a CTA passed the grid-dependency wait, in p[kTimerSlots] the latest at which a
// CTA's work ended. Slots start at (max, 0) before each timed step.
constexpr int kTimerSlots = 2048;
__device__ __forceinline__ void timer_start(unsigned long long* p) {
    if (p) atomicMin(p, static_cast<unsigned long long>(global_timer_ns()));
}
__device__ __forceinline__ void timer_end(unsigned long long* p) {
    if (p) atomicMax(p + kTimerSlots, static_cast<unsigned long long>(global_timer_ns()));
}

// Upper bound of any single wait inside a kernel. A healthy kernel never waits this long on one
// barrier; reaching it means a protocol bug, and the kernel reports instead of hanging.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ void report_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// ------------------------------------------------------------------ programmatic dependent launch
// A kernel of the step lets the next kernel start launching at once (its CTAs then run their prologue while
// this grid finishes) and waits for the previous grid to complete before touching its results. Both are
// no-ops when the launch did not ask for programmatic serialization.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------------ per-device launch setup
// A kernel's dynamic shared-memory limit is set on the current device; each device keeps its own record of the
// largest size set so far (one process may drive engines on several GPUs).
constexpr int kMaxDevices = 64;
inline int current_device_index() {
    int d = 0;
    cudaGetDevice(&d);
    return (d >= 0 && d < kMaxDevices) ? d : 0;
}
template <typename F>
inline void ensure_dyn_smem(F* kernel, size_t bytes, size_t (&done)[kMaxDevices]) {
    const int d = current_device_index();
    if (bytes > done[d]) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
        done[d] = bytes;
    }
}

// ------------------------------------------------------------------ mbarrier (shared::cta)
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// Raises the transaction count of the current phase without an arrival.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: returns false (after recording `code` in *err and raising *abort) if the phase with
// the given parity does not complete within kWaitLimitNs, or if another role already aborted.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err, int code,
                                                  volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (*abort) return false;
            if (global_timer_ns() - t0 > kWaitLimitNs) {
                report_error(err, code);
                *abort = 1;
                return false;
            }
        }
    }
}

// Untiled bulk copy global -> this CTA's shared memory, completing `bytes` transactions on `bar` (no multicast).
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(smem_dst)),
                 "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Untiled bulk copy this CTA's shared memory -> global, in the current bulk group (commit with tma_store_commit).
__device__ __forceinline__ void bulk_store(void* gdst, const void* smem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(smem_src)),
                 "r"(bytes)
                 : "memory");
}

// ------------------------------------------------------------------ TMA stores (shared -> global, bulk groups)
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(smem_src)), "r"(x), "r"(y)
                 : "memory");
}
// Element-wise global += shared tile (fp32 add performed at L2; the tensor map clips out-of-range rows).
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(smem_src)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed store groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void tma_store_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Orders this thread's generic shared-memory writes before later async-proxy (TMA) reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------ TMA (no cluster forms used)
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------------ tcgen05 (cta_group::1)
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] . B[smem desc]^T, bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives on the mbarrier once all previously issued tcgen05.mma of this thread have completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 bit, 32 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor for a K-major bf16 tile written by TMA with 128-byte swizzle:
// rows of 64 elements (128 B), 8-row groups 1024 B apart. The tile base must be 1024-byte aligned;
// `addr` may be advanced by 32 B steps along K inside the 128-byte row.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);          // start address
    d |= static_cast<uint64_t>(1u) << 16;                        // leading byte offset (unused for SW128 K-major)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;                // stride byte offset: 8 rows x 128 B
    d |= static_cast<uint64_t>(1u) << 46;                        // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2u) << 61;                        // swizzle mode: 128 B
    return d;
}

// Instruction descriptor, kind::f16: bf16 A and B (K-major), fp32 D, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
    return (1u << 4)                                  // D format fp32
           | (1u << 7)                                // A format bf16
           | (1u << 10)                               // B format bf16
           | (static_cast<uint32_t>(N >> 3) << 17)    // N / 8
           | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

}  // namespace ud
