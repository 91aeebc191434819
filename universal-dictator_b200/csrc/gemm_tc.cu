// Persistent tcgen05 GEMM for sm_100a: C = epilogue(A . W^T), bf16 operands, fp32 accumulation in TMEM.
//
// Replaces the reference's gemm2_nt (Sources/DictatorEngine/Metal/12_gemm2.metal:47-123, 32x64 tiles on
// Apple simdgroup 8x8 MMA) and gemv_nt (11_gemv.metal:45-128) for batched streams, where M = streams x T.
//
// Structure (one CTA per SM, 320 threads):
//   warp 0      TMA producer: A tile 128x64 and W tile BNx64 per stage, 128-byte swizzle, one mbarrier per stage
//   warp 1      TMEM allocator and single-thread MMA issuer: 4 x tcgen05.mma (M=128, N=BN, K=16) per stage,
//               tcgen05.commit frees the stage; a second commit publishes the finished accumulator
//   warps 2..9  epilogue: two warps per TMEM lane quadrant (32 rows), each taking half of the tile's columns;
//               tcgen05.ld 32 lanes x 32 columns, bias / activation / scale / residual (prefetched one chunk
//               ahead), 16-byte stores
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns) so the epilogue of tile i overlaps the
// main loop of tile i+1. Every mbarrier wait is bounded; on expiry the kernel records an error code in
// the engine's device error word, all roles leave their loops, and TMEM is freed before the CTA exits.
#include <cstdio>

#include "common.cuh"
#include "gemm_epi.cuh"
#include "kernels.h"

namespace ud {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 320;
constexpr int kEpiWarps = 8;

template <int BN>
struct TcCfg {
    static constexpr int STAGES = BN == 256 ? 4 : 6;
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int EPI_OFF = STAGES * STAGE_BYTES + 256;   // epilogue staging after the barriers
    static constexpr int SMEM = EPI_OFF + 8 * kEpiStageBytes + 1024;
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapW, int M, int N,
                   int K, const GemmEpilogue epi, int* err) {
    using C = TcCfg<BN>;
    pdl_launch_dependents();
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint8_t* sA = smem;
    uint8_t* sB = smem + C::STAGES * C::A_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
    uint64_t* empty = full + C::STAGES;
    uint64_t* acc_full = empty + C::STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
    volatile int* abort_v = abort_flag;
    float* epi_stage = reinterpret_cast<float*>(smem + C::EPI_OFF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_m = (M + BM - 1) / BM;
    const int num_tiles = num_m * (N / BN);
    const int num_kb = K / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], kEpiWarps);
        }
        *abort_flag = 0;
        fence_mbarrier_init();
        prefetch_tensormap(&mapA);
        prefetch_tensormap(&mapW);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();  // the prologue above overlaps the previous kernel; its outputs are read only from here on

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
                const int mb = tile % num_m, nb = tile / num_m;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, err, DEV_TIMEOUT_EMPTY, abort_v)) goto producer_done;
                    mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                    tma_load_2d(sA + stage * C::A_BYTES, &mapA, &full[stage], kb * BK, mb * BM);
                    tma_load_2d(sB + stage * C::B_BYTES, &mapW, &full[stage], kb * BK, nb * BN);
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                }
            }
        producer_done:;
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(BM, BN);
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
                if (!mbar_wait_bounded(&acc_empty[acc], acc_phase ^ 1u, err, DEV_TIMEOUT_ACC_EMPTY, abort_v)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait_bounded(&full[stage], phase, err, DEV_TIMEOUT_FULL, abort_v)) goto mma_done;
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + stage * C::A_BYTES);
                    const uint32_t b_addr = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        tc_mma_bf16(d_tmem, sw128_desc(a_addr + k * 32), sw128_desc(b_addr + k * 32), idesc,
                                    (kb | k) != 0 ? 1u : 0u);
                    }
                    tc_commit(&empty[stage]);
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                }
                tc_commit(&acc_full[acc]);
                if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
            }
        mma_done:;
        }
    } else {
        const int q = warp & 3;                       // TMEM lane quadrant accessible to this warp
        const int half = (warp - 2) >> 2;             // which half of the tile's columns
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            const int mb = tile % num_m, nb = tile / num_m;
            int ok = 1;
            if (lane == 0) ok = mbar_wait_bounded(&acc_full[acc], acc_phase, err, DEV_TIMEOUT_ACC_FULL, abort_v) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            const uint32_t t_row = tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(q * 32) << 16);
            // the two warps of a lane quadrant take the two halves of the tile's 16-column blocks
            epi_drain(epi, epi_stage + (warp - 2) * kEpiStageFloats, t_row, mb * BM + q * 32, M, nb * BN,
                      half * (BN / 32), (half + 1) * (BN / 32), lane);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
            if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        }
    }

    __syncthreads();
    if (*abort_v) __nanosleep(100000);  // let in-flight bulk copies / MMAs land before the CTA retires
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

template <int BN>
void launch(const TmaMatrix& A, const TmaMatrix& W, int M, int N, int K, const GemmEpilogue& epi, int* err,
            int num_sms, cudaStream_t s) {
    using C = TcCfg<BN>;
    static size_t attr[kMaxDevices] = {};
    ensure_dyn_smem(gemm_tc_kernel<BN>, C::SMEM, attr);
    const int tiles = ((M + BM - 1) / BM) * (N / BN);
    const int grid = tiles < num_sms ? tiles : num_sms;
    launch_pdl(gemm_tc_kernel<BN>, dim3(grid), dim3(kThreads), C::SMEM, s, A.map, W.map, M, N, K, epi, err);
}

}  // namespace

bool make_tma_bf16(TmaMatrix& t, const void* base, int rows, int cols, int ld, int box_rows) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (ld * 2) % 16 != 0 || cols % 64 != 0) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
    cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1u, 1u};
    CUresult r = enc(&t.map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
    t.base = base;
    t.rows = rows;
    t.cols = cols;
    t.ld = ld;
    t.box_rows = box_rows;
    return true;
}

bool make_tma_epi(TmaMatrix& t, const void* base, int rows, int cols, int ld, bool bf16) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    const int esz = bf16 ? 2 : 4;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (static_cast<long long>(ld) * esz) % 16 != 0 ||
        (cols * esz) % 128 != 0)
        return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * esz};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / esz), 32u};
    cuuint32_t estr[2] = {1u, 1u};
    CUresult r = enc(&t.map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                     const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
    t.base = base;
    t.rows = rows;
    t.cols = cols;
    t.ld = ld;
    t.box_rows = 32;
    return true;
}

bool make_tma_pages(TmaMatrix& t, const void* base, int pages_total, int page_frames, int cols) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || cols % 64 != 0 || page_frames < 1 || page_frames > 256)
        return false;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(page_frames),
                          static_cast<cuuint64_t>(pages_total)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols) * 2, static_cast<cuuint64_t>(page_frames) * cols * 2};
    cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(page_frames), 1u};
    cuuint32_t estr[3] = {1u, 1u, 1u};
    CUresult r = enc(&t.map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
    t.base = base;
    t.rows = pages_total * page_frames;
    t.cols = cols;
    t.ld = cols;
    t.box_rows = page_frames;
    return true;
}

int gemm_tc_pick_bn(int M, int N, int num_sms) {
    const int num_m = (M + BM - 1) / BM;
    if (N % 256 == 0 && num_m * (N / 256) >= num_sms) return 256;
    return 128;
}

void gemm_tc(const TmaMatrix& A, const TmaMatrix& W, int M, int N, int K, int bn, const GemmEpilogue& epi,
             int* dev_err, int num_sms, cudaStream_t s) {
    if (bn == 256)
        launch<256>(A, W, M, N, K, epi, dev_err, num_sms, s);
    else
        launch<128>(A, W, M, N, K, epi, dev_err, num_sms, s);
}

}  // namespace ud
