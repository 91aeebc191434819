// Persistent 2-CTA tcgen05 GEMM (cta_group::2) for sm_100a: the same C = epilogue(A . W^T) contract as
// gemm_tc.cu, with each CTA pair of a cluster computing a 256 x BN tile.
//
// Per pair and stage (64 along K): CTA r stages rows [128 r, 128 r + 128) of the A tile and rows
// [BN/2 r, BN/2 (r+1)) of the W tile in its own shared memory (TMA, 128-byte swizzle). Both CTAs' loads complete
// on the leader's (rank 0) stage barrier; the leader's single MMA thread issues tcgen05.mma.cta_group::2
// (M = 256, N = BN, K = 16), which reads A and W halves from both CTAs and accumulates each CTA's 128 rows in
// its own TMEM. Commits signal both CTAs' stage-free and accumulator-ready barriers; each CTA's 8 epilogue warps
// drain their TMEM rows and report back to the leader. Per CTA and stage that is 32 KB of shared memory for
// 128 x BN x 64 multiply-adds: half the operand bytes per FLOP of the one-CTA kernel, so six stages cover the
// TMA round trip. Every wait is bounded, as in gemm_tc.cu.
//
// Tile width: each launch uses one tile width tn, the fewest tiles per output row of at most BN columns with
// their width balanced and rounded up to a multiple of 16 (N = 1024 -> 256; N = 1040 -> 5 tiles of 208; the
// last tile of a row may be narrower). The MMA's N, the W rows each CTA loads (tile width / 2) and the epilogue
// width are read from the tile. Narrower tiles that would fill a partial last round of pairs measured slower
// than the wide tiles on the encoder's shapes, so the host does not trade width for rounds (256 x 128 tiles, two
// per pair, doubled the time from the first stage to the last MMA on every shape).
//
// TMA epilogues (every tile 256 wide, host-supplied tensor map of the output): bf16 outputs without a residual,
// and fp32 outputs whose residual is the output itself with unit scale (the encoder's x += s * f(x)). Each
// epilogue warp owns two 4 KB shared-memory blocks of 32 rows x 128 bytes (64 bf16 or 32 fp32 columns) in the
// 128-byte swizzled layout. Per block it reads its TMEM rows, applies bias / activation / scale, writes the block
// (conflict-free: lane = row, 16-byte chunk k at position k ^ (row % 8)) and one lane issues a TMA bulk store
// (bf16) or a TMA bulk reduce-add (fp32: the L2 adds the block to the output, so the residual never travels to
// the SM); out-of-range rows are clipped by the copy. A buffer is rewritten only after the copy issued from it
// two blocks earlier has read it (cp.async.bulk.wait_group.read). Five pipeline stages leave room for the 64 KB
// of blocks. The register epilogue (staged through shared memory, residual read by the SM) serves every other
// output form.
#include <cstdlib>

#include "common.cuh"
#include "gemm_epi.cuh"
#include "kernels.h"
#include "tc2_common.cuh"

namespace ud {
namespace {

using namespace tc2;

constexpr int BM2 = 256;  // rows per CTA pair
constexpr int BK = 64;
constexpr int kThreads = 320;
constexpr int kEpiWarps = 8;

// Epilogue modes: register epilogue (any output), TMA store of bf16 blocks, TMA reduce-add of fp32 blocks.
enum Tc2Epi { kEpiReg = 0, kEpiStoreBf16 = 1, kEpiAddF32 = 2 };

template <int BN, int EP>
struct Tc2Cfg {
    static constexpr int STAGES = EP != kEpiReg ? 5 : 6;
    static constexpr int A_BYTES = 128 * BK * 2;        // this CTA's half of the A tile
    static constexpr int B_BYTES = (BN / 2) * BK * 2;   // this CTA's half of the W tile (a full 128-row box)
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int BAR_BYTES = 256;                // pipeline and accumulator barriers
    static constexpr int EPI_OFF = (STAGES * STAGE_BYTES + BAR_BYTES + 1023) / 1024 * 1024;   // 1 KB aligned
    static constexpr int EPI_BYTES = EP != kEpiReg ? kEpiWarps * 2 * 4096 : kEpiWarps * kEpiStageBytes;
    static constexpr int SMEM = EPI_OFF + EPI_BYTES + 1024;
};

template <int BN, int EP>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapW,
                    const __grid_constant__ CUtensorMap mapO, int M, int N,
                    int K, int tn, const GemmEpilogue epi, int* err) {
    using C = Tc2Cfg<BN, EP>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint8_t* sA = smem;
    uint8_t* sB = smem + C::STAGES * C::A_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);  // used in the leader
    uint64_t* empty = full + C::STAGES;
    uint64_t* acc_full = empty + C::STAGES;
    uint64_t* acc_empty = acc_full + 2;                                                  // used in the leader
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
    volatile int* abort_v = abort_flag;
    float* epi_stage = reinterpret_cast<float*>(smem + C::EPI_OFF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
    const int num_m = (M + BM2 - 1) / BM2;
    const int tiles_per_row = (N + tn - 1) / tn;
    const int num_tiles = num_m * tiles_per_row;
    const int num_kb = K / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], 2 * kEpiWarps);
        }
        *abort_flag = 0;
        fence_mbarrier_init();
        prefetch_tensormap(&mapA);
        prefetch_tensormap(&mapW);
        if (EP != kEpiReg) prefetch_tensormap(&mapO);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(C::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // The weights do not depend on the previous kernel: the producer stages the W halves of the first tile's
    // first stages (all free at this point) before the dependency wait, so only the A loads follow it. Those
    // stages' barriers get the W bytes now (no arrival) and the A bytes with the producer's arrival below.
    int w_early = 0;
    if (warp == 0 && lane == 0 && pair < num_tiles) {
        const int nb = pair / num_m;
        const int c0 = nb * tn, w = min(tn, N - c0);
        w_early = min(C::STAGES, num_kb);
        for (int kb = 0; kb < w_early; ++kb) {
            if (rank == 0) mbar_expect_tx(&full[kb], 2 * C::B_BYTES);
            tma_load_2d_pair(sB + kb * C::B_BYTES, &mapW, peer_addr(smem_u32(&full[kb]), 0), kb * BK,
                             c0 + static_cast<int>(rank) * (w / 2));
        }
    }
    pdl_wait();  // the prologue above overlaps the previous kernel; its outputs are read only from here on
    if (threadIdx.x == 0) timer_start(epi.prof);

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            for (int tile = pair; tile < num_tiles; tile += num_pairs) {
                const int mb = tile % num_m, nb = tile / num_m;
                const int c0 = nb * tn, w = min(tn, N - c0);
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, err, DEV_TIMEOUT_EMPTY, abort_v)) goto producer_done;
                    const uint32_t leader_full = peer_addr(smem_u32(&full[stage]), 0);
                    const bool w_loaded = tile == pair && kb < w_early;
                    if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (w_loaded ? C::A_BYTES : C::STAGE_BYTES));
                    tma_load_2d_pair(sA + stage * C::A_BYTES, &mapA, leader_full, kb * BK, mb * BM2 + rank * 128);
                    if (!w_loaded)
                        tma_load_2d_pair(sB + stage * C::B_BYTES, &mapW, leader_full, kb * BK,
                                         c0 + static_cast<int>(rank) * (w / 2));
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                }
            }
        producer_done:;
            // This CTA has no more tiles to load: the next kernel may launch now. Its CTAs then take the SMs as this
            // grid's last tiles drain, instead of sharing them with this grid's epilogues from the start.
            pdl_launch_dependents();
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            for (int tile = pair; tile < num_tiles; tile += num_pairs) {
                const int nb = tile / num_m;
                const uint32_t idesc = idesc_bf16_f32(BM2, min(tn, N - nb * tn));
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
                        tc2_mma_bf16(d_tmem, sw128_desc(a_addr + k * 32), sw128_desc(b_addr + k * 32), idesc,
                                     (kb | k) != 0 ? 1u : 0u);
                    }
                    tc2_commit_both(&empty[stage]);
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                }
                tc2_commit_both(&acc_full[acc]);
                if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
            }
        mma_done:;
        }
    } else if constexpr (EP != kEpiReg) {
        // Blocks of 32 rows x 128 bytes: 64 bf16 columns (store) or 32 fp32 columns (reduce-add).
        constexpr int BC = EP == kEpiStoreBf16 ? 64 : 32;
        const int q = warp & 3;
        const int half = (warp - 2) >> 2;   // the two warps of a lane quadrant take column halves of the tile
        const int hw = tn / 2;              // columns per warp: 128 or 64 (a multiple of BC)
        uint8_t* eb = smem + C::EPI_OFF + (warp - 2) * 8192;   // this warp's two blocks
        const int swz = lane & 7;
        int acc = 0, g = 0;
        uint32_t acc_phase = 0;
        for (int tile = pair; tile < num_tiles; tile += num_pairs) {
            int ok = 1;
            if (lane == 0) ok = mbar_wait_bounded(&acc_full[acc], acc_phase, err, DEV_TIMEOUT_ACC_FULL, abort_v) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            const uint32_t t_base =
                tmem_base + static_cast<uint32_t>(acc * BN + half * hw) + (static_cast<uint32_t>(q * 32) << 16);
            const int y = (tile % num_m) * BM2 + static_cast<int>(rank) * 128 + q * 32;
            for (int ch = 0; ch < hw / BC; ++ch, ++g) {
                uint8_t* buf = eb + (g & 1) * 4096;
                const int x = (tile / num_m) * tn + half * hw + ch * BC;
                if (lane == 0) tma_store_wait_read<1>();   // the copy issued from buf two blocks ago has read it
                __syncwarp();
                float v[BC];
                tmem_ld32(t_base + static_cast<uint32_t>(ch * BC), v);
                if constexpr (BC == 64) tmem_ld32(t_base + static_cast<uint32_t>(ch * BC + 32), v + 32);
                uint8_t* row = buf + lane * 128;
                constexpr int PER = BC / 8;   // values per 16-byte chunk
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    float e[PER];
#pragma unroll
                    for (int j = 0; j < PER; ++j) e[j] = v[PER * k + j];
                    if (epi.bias) {
#pragma unroll
                        for (int j = 0; j < PER; j += 4) {
                            const float4 b = *reinterpret_cast<const float4*>(epi.bias + x + PER * k + j);
                            e[j] += b.x; e[j + 1] += b.y; e[j + 2] += b.z; e[j + 3] += b.w;
                        }
                    }
                    uint4 u;
                    if constexpr (EP == kEpiStoreBf16) {
                        uint32_t w[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            __nv_bfloat162 h = __floats2bfloat162_rn(epi_act_bf16(epi.act, e[2 * j]) * epi.out_scale,
                                                                     epi_act_bf16(epi.act, e[2 * j + 1]) * epi.out_scale);
                            w[j] = *reinterpret_cast<uint32_t*>(&h);
                        }
                        u = make_uint4(w[0], w[1], w[2], w[3]);
                    } else {
                        u = make_uint4(__float_as_uint(epi_act(epi.act, e[0]) * epi.out_scale),
                                       __float_as_uint(epi_act(epi.act, e[1]) * epi.out_scale),
                                       __float_as_uint(epi_act(epi.act, e[2]) * epi.out_scale),
                                       __float_as_uint(epi_act(epi.act, e[3]) * epi.out_scale));
                    }
                    *reinterpret_cast<uint4*>(row + ((k ^ swz) << 4)) = u;
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (EP == kEpiStoreBf16) tma_store_2d(&mapO, buf, x, y);
                    else tma_reduce_add_2d(&mapO, buf, x, y);
                    tma_store_commit();
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(peer_addr(smem_u32(&acc_empty[acc]), 0));
            if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        }
        if (lane == 0) tma_store_wait_all();
    } else {
        const int q = warp & 3;
        const int half = (warp - 2) >> 2;   // the two warps of a lane quadrant split the tile's columns
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = pair; tile < num_tiles; tile += num_pairs) {
            const int mb = tile % num_m, nb = tile / num_m;
            const int c0 = nb * tn, nblk = min(tn, N - c0) / 16;   // 16-column blocks in this tile
            const int hb = (nblk + 1) >> 1;
            const int b0 = half ? hb : 0, b1 = half ? nblk : hb;    // this warp's blocks [b0, b1)
            int ok = 1;
            if (lane == 0) ok = mbar_wait_bounded(&acc_full[acc], acc_phase, err, DEV_TIMEOUT_ACC_FULL, abort_v) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            const int row0 = mb * BM2 + static_cast<int>(rank) * 128 + q * 32;
            const uint32_t t_row = tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(q * 32) << 16);
            epi_drain(epi, epi_stage + (warp - 2) * kEpiStageFloats, t_row, row0, M, c0, b0, b1, lane);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(peer_addr(smem_u32(&acc_empty[acc]), 0));
            if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        }
    }

    tc_fence_before();
    cluster_sync();  // no CTA frees TMEM while its peer's MMAs or epilogue may still touch the pair's state
    if (threadIdx.x == 0) timer_end(epi.prof);
    if (*abort_v) __nanosleep(100000);
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(C::TMEM_COLS)
                     : "memory");
    }
}

template <int BN>
void launch2(const TmaMatrix& A, const TmaMatrix& W, int M, int N, int K, const GemmEpilogue& epi, int* err,
             int num_sms, const TmaMatrix* out_map, cudaStream_t s) {
    using C = Tc2Cfg<BN, kEpiReg>;
    using CT = Tc2Cfg<BN, kEpiStoreBf16>;
    static size_t attr0[kMaxDevices] = {}, attr1[kMaxDevices] = {}, attr2[kMaxDevices] = {};
    ensure_dyn_smem(gemm_tc2_kernel<BN, kEpiReg>, C::SMEM, attr0);
    ensure_dyn_smem(gemm_tc2_kernel<BN, kEpiStoreBf16>, CT::SMEM, attr1);
    ensure_dyn_smem(gemm_tc2_kernel<BN, kEpiAddF32>, CT::SMEM, attr2);
    // Persistent grid: no more pairs than can be resident at once (clusters are placed within GPCs).
    static int max_pairs_dev[kMaxDevices] = {};
    int& max_pairs = max_pairs_dev[current_device_index()];
    if (max_pairs <= 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(num_sms, 1, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = C::SMEM;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_tc2_kernel<BN, kEpiReg>, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = num_sms / 2;
        }
        max_pairs = n < num_sms / 2 ? n : num_sms / 2;
    }
    // Tile width: the fewest tiles per row, widths balanced and rounded up to a multiple of 16.
    const int num_m = (M + BM2 - 1) / BM2;
    const int per_row = (N + BN - 1) / BN;
    const int tn = ((N + per_row - 1) / per_row + 15) / 16 * 16;
    const int tiles = num_m * ((N + tn - 1) / tn);
    const int pairs = tiles < max_pairs ? tiles : max_pairs;
    // UD_TMA_EPI: unset = both TMA epilogues, 1 = bf16 stores only, 0 = the register epilogue everywhere.
    static int te_env = -1;
    if (te_env < 0) {
        const char* v = std::getenv("UD_TMA_EPI");
        te_env = v ? std::atoi(v) : 2;
    }
    const bool full_tiles = BN == 256 && out_map && tn == 256 && N % 256 == 0;
    int ep = kEpiReg;
    if (full_tiles && te_env >= 1 && epi.out_bf16 && epi.residual == nullptr) ep = kEpiStoreBf16;
    // out += out_scale * act(acc + bias): the residual is the output itself, added once per element at L2.
    if (full_tiles && te_env >= 2 && !epi.out_bf16 && epi.residual == epi.out && epi.ldr == epi.ldo &&
        epi.res_scale == 1.f)
        ep = kEpiAddF32;
    const dim3 grid(2 * pairs), block(kThreads);
    if (ep == kEpiStoreBf16)
        launch_pdl(gemm_tc2_kernel<BN, kEpiStoreBf16>, grid, block, CT::SMEM, s, A.map, W.map, out_map->map, M, N, K,
                   tn, epi, err);
    else if (ep == kEpiAddF32)
        launch_pdl(gemm_tc2_kernel<BN, kEpiAddF32>, grid, block, CT::SMEM, s, A.map, W.map, out_map->map, M, N, K,
                   tn, epi, err);
    else
        launch_pdl(gemm_tc2_kernel<BN, kEpiReg>, grid, block, C::SMEM, s, A.map, W.map, A.map, M, N, K, tn, epi, err);
}

}  // namespace

void gemm_tc2(const TmaMatrix& A, const TmaMatrix& W_half, int M, int N, int K, int bn, const GemmEpilogue& epi,
              int* dev_err, int num_sms, const TmaMatrix* out_map, cudaStream_t s) {
    if (bn == 256)
        launch2<256>(A, W_half, M, N, K, epi, dev_err, num_sms, out_map, s);
    else
        launch2<128>(A, W_half, M, N, K, epi, dev_err, num_sms, nullptr, s);
}

}  // namespace ud
