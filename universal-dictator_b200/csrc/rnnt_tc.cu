// Lock-step RNN-T greedy decoding on the tensor cores (tcgen05), with fp32-level accuracy from a three-term fp16
// split. Same semantics as the other decoders (RNNT.swift:73-151; see rnnt.cu): per frame, every stream still in
// the frame takes one symbol iteration at a time, and an iteration is a chain of batched products over the streams
//   LSTM layer l : gates[b, 4Hp] = [x_l ; h_l][b, 2Hp] . [W_ih ; W_hh]^T  -> cell update (epilogue)
//   prediction   : g[b, J]       = h_top[b, Hp] . W_pred^T + b             (streams without a pending prediction)
//   joint        : logits[b, V]  = relu(f_t + g)[b, J] . W_out^T + b -> per-slice first maximum (epilogue)
//   decision     : owner CTA of each stream combines the slice maxima, emits, commits the LSTM state,
// with bounded grid barriers between them.
//
// Numbers. Every operand value x is carried as two fp16 values, hi = fp16(x) and lo = fp16((x - hi) * 2^11), so
// x = hi + lo * 2^-11 to within 2^-22 |x|. A product is D0 + (D1 + D2) * 2^-11 with D0 = A_hi . B_hi,
// D1 = A_hi . B_lo, D2 = A_lo . B_hi (kind::f16, fp32 accumulation in TMEM); the dropped A_lo . B_lo and the
// rounding of the lo parts stay below 2^-21 of |a||b|, the size of fp32 accumulation error over these K. The
// weights are split once, at load (unit-major LSTM rows: row 4u + q is gate q of hidden unit u, so a slice of rows
// holds whole units and the cell update runs in the epilogue). The per-stream operand rows live in batch order in
// global memory and are written, already split, by whoever produces them: the decision (token embedding and
// committed h), the LSTM epilogue (the next layer's input, the prediction input), the prediction epilogue (the joint
// input relu(f_t + g)) and, once per frame, a pack of the joint input of the streams whose prediction was pending.
//
// Work. A product is cut into items of 128 streams (M) x BN output rows (N, chosen on the host so the items fill
// the grid once); an item runs K in chunks of 64. Warp 0 loads each chunk's four tiles with TMA (128-byte swizzle);
// warps 1-3 each issue one of the three product terms into its own accumulator (four MMAs per chunk: the issue
// rate of one thread, not the tensor core, bounds small-N MMAs, so three issuers run them three times faster);
// warps 4-11 drain the accumulators (TMEM lane = stream row) and run the epilogue, two warps per lane quadrant
// splitting the columns. All twelve warps take the per-stream passes (decision, packs). 384 threads leave each
// thread 168 registers: the epilogue's prefetched rows and accumulator columns stay out of local memory, which with
// nearly all of the SM's shared memory in use would be read from L2.
#include <algorithm>
#include <cstring>
#include <vector>

#include <cuda_fp16.h>

#include "rnnt_common.cuh"

namespace ud {
namespace {

constexpr int kTcWarps = 12, kTcThreads = 32 * kTcWarps;   // warp 0 TMA, 1-3 MMA, 4-11 epilogue
constexpr int kTcEpiWarps = kTcWarps - 4, kTcEpiSets = kTcEpiWarps / 4;
constexpr int kTM = 128;                        // streams per item (MMA M)
constexpr int kTK = 64;                         // fp16 elements per K chunk: one 128-byte swizzled row
constexpr int kTMaxBN = 128;                    // widest item slice (MMA N)
constexpr int kTMaxStages = 6;                  // shared-memory stages: as many as fit (plan.stages)
constexpr uint32_t kTileA = kTM * 128;          // bytes of one A tile (hi or lo)
constexpr uint32_t kTmemCols = 512;             // D0, D1, D2 at columns 0, 128, 256
constexpr float kLoScale = 2048.f, kLoUnscale = 1.f / 2048.f;
constexpr float kHalfMax = 65504.f;
enum { kPhLstm = 0, kPhPred = 1, kPhJoint = 2 };
enum : uint8_t { kFlagAct = 1, kFlagNeed = 2 };

struct TcMaps {
    CUtensorMap xl_hi[4], xl_lo[4], wl_hi[4], wl_lo[4];
    CUtensorMap xp_hi, xp_lo, wp_hi, wp_lo, xj_hi, xj_lo, wo_hi, wo_lo;
};
struct TcBufs {
    __half* xl_hi[4];
    __half* xl_lo[4];
    __half *xp_hi, *xp_lo, *xj_hi, *xj_lo;
};
struct TcPlan {
    int bn[3], ns[3], nk[3];   // per product (LSTM, prediction, joint): slice width, slices, K chunks
    int stages;                // stages of [A hi | A lo | B hi | B lo], B tiles sized for the widest slice
    uint32_t stage_bytes, b_lo;   // bytes of a stage; offset of its B lo tile (B hi is at 2 A tiles)
};

// Instruction descriptor, kind::f16 with fp16 A and B (K-major), fp32 D, shape M x N.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
    return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
    return static_cast<uint32_t>(__half_as_ushort(a)) | (static_cast<uint32_t>(__half_as_ushort(b)) << 16);
}
// Splits 4 values into their hi and lo fp16 parts (4 halves each); `bad` records a value beyond the fp16 range.
__device__ __forceinline__ void split4(float4 x, uint2& hi, uint2& lo, bool& bad) {
    const float v[4] = {x.x, x.y, x.z, x.w};
    __half h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        bad |= !(fabsf(v[i]) < kHalfMax);
        h[i] = __float2half_rn(v[i]);
        l[i] = __float2half_rn((v[i] - __half2float(h[i])) * kLoScale);
    }
    hi = make_uint2(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]));
    lo = make_uint2(pack_h2(l[0], l[1]), pack_h2(l[2], l[3]));
}
__device__ __forceinline__ void store_split4(__half* hi, __half* lo, size_t off, float4 x, bool& bad) {
    uint2 h, l;
    split4(x, h, l, bad);
    *reinterpret_cast<uint2*>(hi + off) = h;
    *reinterpret_cast<uint2*>(lo + off) = l;
}

// The LSTM cell's nonlinearities from the fast exponential and division intrinsics (about 1e-7 absolute error, the
// size of the product's own rounding); tanh(x) = 2 sigmoid(2x) - 1 saturates to +-1 as the exponential overflows.
__device__ __forceinline__ float sigm_fast(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }
__device__ __forceinline__ float tanh_fast(float x) { return 2.f * sigm_fast(2.f * x) - 1.f; }

// v = D0 + (D1 + D2) * 2^-11 for 16 consecutive columns of this warp's TMEM lanes: the three loads are issued
// before one wait.
__device__ __forceinline__ void tmem_sum3(uint32_t taddr, float* v) {
    uint32_t r[3][16];
#pragma unroll
    for (int m = 0; m < 3; ++m)
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(r[m][0]), "=r"(r[m][1]), "=r"(r[m][2]), "=r"(r[m][3]), "=r"(r[m][4]), "=r"(r[m][5]), "=r"(r[m][6]),
              "=r"(r[m][7]), "=r"(r[m][8]), "=r"(r[m][9]), "=r"(r[m][10]), "=r"(r[m][11]), "=r"(r[m][12]),
              "=r"(r[m][13]), "=r"(r[m][14]), "=r"(r[m][15])
            : "r"(taddr + m * 128));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int e = 0; e < 16; ++e)
        v[e] = __uint_as_float(r[0][e]) + (__uint_as_float(r[1][e]) + __uint_as_float(r[2][e])) * kLoUnscale;
}

// Generic-proxy global writes made visible to later TMA (async-proxy) reads, then the bounded grid barrier.
__device__ __forceinline__ bool tc_grid_sync(unsigned long long* ctr, unsigned long long& target, int* err,
                                             volatile int* fail) {
    asm volatile("fence.proxy.async.global;" ::: "memory");
    return grid_sync(ctr, target, err, fail);
}

struct TcShared {
    uint8_t* stages;
    uint64_t *full, *empty, *acc_full, *acc_empty;
    uint8_t* flag;       // [n] kFlagAct | kFlagNeed of the current iteration
    int* tiles_act;      // tiles (of 128 streams) holding an active stream
    int* tiles_need;     // tiles holding a stream without a pending prediction
    int* tile_bits;      // OR of the flags of each tile
    int* cnt;            // [4] active streams, streams needing the LSTM, active tiles, needing tiles
    float* bias;         // [kTcEpiWarps][kTMaxBN] per epilogue warp: the per-column bias of its current item
    volatile int* fail;
    uint32_t tmem;
};

struct TcPipe {            // pipeline positions of this thread's role, carried across products
    uint32_t stage = 0, phase = 0, acc_phase = 0;
};

struct TcCtx {
    RnntWeights w;
    RnntState st;
    TcBufs xb;
    const float* proj;
    int ld_proj;
    const BatchEntry* meta;
    int n;
    RnntScratch scr;
    int* err;
};

// One product over the current tile list; every thread of the CTA calls it and takes its warp's role.
__device__ __forceinline__ bool tc_product(const TcCtx& c, TcShared& sh, TcPipe& pp, int kind, int l, int t, const TcPlan& plan,
                           const CUtensorMap* ma_hi, const CUtensorMap* ma_lo, const CUtensorMap* mb_hi,
                           const CUtensorMap* mb_lo) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, G = gridDim.x;
    const int BN = plan.bn[kind], ns = plan.ns[kind], nk = plan.nk[kind];
    const int* tiles = kind == kPhJoint ? sh.tiles_act : sh.tiles_need;
    const int ntiles = kind == kPhJoint ? sh.cnt[2] : sh.cnt[3];
    const int items = ntiles * ns;
    const uint8_t mask = kind == kPhJoint ? kFlagAct : kFlagNeed;
    const RnntWeights& w = c.w;
    const int Hp = w.Hp, NLp = w.layers, J = w.J, V = w.V;

    if (warp == 0) {
        // ---- TMA producer
        if (lane == 0) {
            const uint32_t bytes = 2 * kTileA + 2 * static_cast<uint32_t>(BN) * 128;
            for (int it = blockIdx.x; it < items; it += G) {
                const int tile = tiles[it % ntiles], si = it / ntiles;
                for (int kc = 0; kc < nk; ++kc) {
                    if (!mbar_wait_bounded(&sh.empty[pp.stage], pp.phase ^ 1u, c.err, DEV_TIMEOUT_EMPTY, sh.fail))
                        return false;
                    uint8_t* s = sh.stages + pp.stage * plan.stage_bytes;
                    mbar_arrive_expect_tx(&sh.full[pp.stage], bytes);
                    tma_load_2d(s, ma_hi, &sh.full[pp.stage], kc * kTK, tile * kTM);
                    tma_load_2d(s + kTileA, ma_lo, &sh.full[pp.stage], kc * kTK, tile * kTM);
                    tma_load_2d(s + 2 * kTileA, mb_hi, &sh.full[pp.stage], kc * kTK, si * BN);
                    tma_load_2d(s + plan.b_lo, mb_lo, &sh.full[pp.stage], kc * kTK, si * BN);
                    if (++pp.stage == static_cast<uint32_t>(plan.stages)) { pp.stage = 0; pp.phase ^= 1u; }
                }
            }
        }
    } else if (warp <= 3) {
        // ---- MMA issuers: warp 1 A_hi.B_hi, warp 2 A_hi.B_lo, warp 3 A_lo.B_hi, each into its own accumulator
        if (lane == 0) {
            const int m = warp - 1;
            const uint32_t idesc = idesc_f16_f32(kTM, BN), d = sh.tmem + m * 128;
            for (int it = blockIdx.x; it < items; it += G) {
                if (!mbar_wait_bounded(sh.acc_empty, pp.acc_phase ^ 1u, c.err, DEV_TIMEOUT_ACC_EMPTY, sh.fail))
                    return false;
                tc_fence_after();
                for (int kc = 0; kc < nk; ++kc) {
                    if (!mbar_wait_bounded(&sh.full[pp.stage], pp.phase, c.err, DEV_TIMEOUT_FULL, sh.fail)) return false;
                    tc_fence_after();
                    const uint32_t s = smem_u32(sh.stages + pp.stage * plan.stage_bytes);
                    const uint32_t a = s + (m == 2 ? kTileA : 0u), b = s + (m == 1 ? plan.b_lo : 2 * kTileA);
#pragma unroll
                    for (int k = 0; k < kTK / 16; ++k)
                        tc_mma_bf16(d, sw128_desc(a + k * 32), sw128_desc(b + k * 32), idesc, (kc | k) != 0 ? 1u : 0u);
                    tc_commit(&sh.empty[pp.stage]);
                    if (kc == nk - 1) tc_commit(sh.acc_full);
                    if (++pp.stage == static_cast<uint32_t>(plan.stages)) { pp.stage = 0; pp.phase ^= 1u; }
                }
                pp.acc_phase ^= 1u;
            }
        }
    } else {
        // ---- epilogue: warps 4-11; warp w reads TMEM lane quadrant w % 4 (one stream row per thread) and, for the
        // LSTM and the prediction, the 16-column groups g with g % 2 == (w - 4) / 4 (the joint's running maximum
        // stays in warps 4-7; the others only wait for the accumulators and release them). While the MMAs run a
        // warp stages the slice's per-column bias in shared memory and loads its row's data for its first group;
        // in the column loop the next group's row data is in flight while the current group is computed.
        const int q = warp & 3, row = q * 32 + lane, set = (warp - 4) >> 2;
        const int g_first = kind == kPhJoint ? 0 : 16 * set, g_step = kind == kPhJoint ? 16 : 16 * kTcEpiSets;
        const bool drains = kind != kPhJoint || set == 0;
        const uint32_t trow = sh.tmem + (static_cast<uint32_t>(q * 32) << 16);
        bool bad = false;
        float* bias = sh.bias + (warp - 4) * kTMaxBN;   // this warp's copy (no barrier between the epilogue warps)
        for (int it = blockIdx.x; it < items; it += G) {
            const int tile = tiles[it % ntiles], si = it / ntiles;
            __syncwarp();   // the previous item's reads of `bias` are done
            for (int col = lane; drains && col < BN; col += 32) {
                float bv = 0.f;
                if (kind == kPhLstm) {
                    const int u = si * (BN / 4) + col / 4;
                    if (u < Hp) bv = __ldg(w.bias[l] + (col % 4) * Hp + u);
                } else if (kind == kPhPred) {
                    if (si * BN + col < J) bv = __ldg(w.pred_b + si * BN + col);
                } else if (si * BN + col < V) {
                    bv = __ldg(w.out_b + si * BN + col);
                }
                bias[col] = bv;
            }
            __syncwarp();
            const int b = tile * kTM + row;
            const bool valid = drains && b < c.n && (sh.flag[b] & mask);
            int slot = 0, row_off = 0;
            if (valid) {
                slot = c.meta[b].slot;
                row_off = c.meta[b].row_off;
            }
            // row data of a 16-column group: the LSTM's old cell state (4 units), the prediction's f_t (16 values)
            const size_t c_row = (static_cast<size_t>(slot) * NLp + l) * Hp;
            const float* f_row = c.proj + static_cast<size_t>(row_off + t) * c.ld_proj;
            auto load_group = [&](int g0, float4* r) {
                if (!valid) return;
                if (kind == kPhLstm) {
                    const int u0 = si * (BN / 4) + g0 / 4;
                    if (u0 < Hp) r[0] = __ldcg(reinterpret_cast<const float4*>(c.st.c + c_row + u0));
                } else if (kind == kPhPred) {
                    const int j0 = si * BN + g0;
                    if (j0 < J)
#pragma unroll
                        for (int e = 0; e < 4; ++e) r[e] = __ldg(reinterpret_cast<const float4*>(f_row + j0) + e);
                }
            };
            float4 pre[4];
            load_group(g_first, pre);
            int ok = 1;
            if (lane == 0) ok = mbar_wait_bounded(sh.acc_full, pp.acc_phase, c.err, DEV_TIMEOUT_ACC_FULL, sh.fail) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) return false;
            tc_fence_after();
            float best = -INFINITY;
            int besti = 0x7fffffff;
            for (int g0 = g_first; drains && g0 < BN; g0 += g_step) {
                float4 cur[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) cur[e] = pre[e];
                if (g0 + g_step < BN) load_group(g0 + g_step, pre);
                float v[16];
                tmem_sum3(trow + g0, v);
                if (!valid) continue;
                if (kind == kPhLstm) {
                    const int u0 = si * (BN / 4) + g0 / 4;   // 4 hidden units, a multiple of 4
                    if (u0 >= Hp) continue;
                    const float co[4] = {cur[0].x, cur[0].y, cur[0].z, cur[0].w};
                    float cn[4], hn[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float* bb = bias + g0 + 4 * e;
                        const float ig = sigm_fast(v[4 * e] + bb[0]), fg = sigm_fast(v[4 * e + 1] + bb[1]);
                        const float gg = tanh_fast(v[4 * e + 2] + bb[2]), og = sigm_fast(v[4 * e + 3] + bb[3]);
                        cn[e] = fg * co[e] + ig * gg;
                        hn[e] = og * tanh_fast(cn[e]);
                    }
                    const float4 h4 = make_float4(hn[0], hn[1], hn[2], hn[3]);
                    const size_t o = c_row + u0;
                    *reinterpret_cast<float4*>(c.st.pend_c + o) = make_float4(cn[0], cn[1], cn[2], cn[3]);
                    *reinterpret_cast<float4*>(c.st.pend_h + o) = h4;
                    if (l + 1 < NLp)   // the next layer's input x_{l+1}
                        store_split4(c.xb.xl_hi[l + 1], c.xb.xl_lo[l + 1], static_cast<size_t>(b) * 2 * Hp + u0, h4, bad);
                    else               // the prediction input
                        store_split4(c.xb.xp_hi, c.xb.xp_lo, static_cast<size_t>(b) * Hp + u0, h4, bad);
                } else if (kind == kPhPred) {
                    const int j0 = si * BN + g0;   // J is a multiple of 64: all 16 columns or none
                    if (j0 >= J) continue;
                    float* gd = c.st.pend_g + static_cast<size_t>(slot) * J + j0;
#pragma unroll
                    for (int e = 0; e < 16; e += 4) {
                        const float* bb = bias + g0 + e;
                        const float4 g4 = make_float4(v[e] + bb[0], v[e + 1] + bb[1], v[e + 2] + bb[2], v[e + 3] + bb[3]);
                        *reinterpret_cast<float4*>(gd + e) = g4;
                        const float4 f4 = cur[e / 4];
                        const float4 x = make_float4(fmaxf(f4.x + g4.x, 0.f), fmaxf(f4.y + g4.y, 0.f),
                                                     fmaxf(f4.z + g4.z, 0.f), fmaxf(f4.w + g4.w, 0.f));
                        store_split4(c.xb.xj_hi, c.xb.xj_lo, static_cast<size_t>(b) * J + j0 + e, x, bad);
                    }
                } else {
                    const int v0 = si * BN + g0;
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        if (v0 + e < V) {
                            const float x = v[e] + bias[g0 + e];
                            if (x > best) { best = x; besti = v0 + e; }   // increasing column order: first maximum
                        }
                    }
                }
            }
            if (valid && kind == kPhJoint) {   // set 0 only (valid is false elsewhere)
                const size_t pi = static_cast<size_t>(b) * ns + si;
                c.scr.part_val[pi] = best;
                c.scr.part_idx[pi] = besti;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(sh.acc_empty);
            pp.acc_phase ^= 1u;
        }
        if (bad) report_error(c.err, DEV_RANGE_F16);
    }
    return true;
}

// The flags of the streams in frame t and the tiles holding them; every CTA computes the same lists.
__device__ void tc_flags(const TcCtx& c, int t, TcShared& sh) {
    const int tid = threadIdx.x, n = c.n;
    if (tid < 4) sh.cnt[tid] = 0;
    __syncthreads();
    int na = 0, nn = 0;
    for (int b = tid; b < n; b += kTcThreads) {
        uint8_t f = 0;
        if (t < c.meta[b].keep && __ldcg(c.scr.done_frame + b) <= t) {
            f = kFlagAct;
            if (__ldcg(c.st.pend_valid + c.meta[b].slot) == 0) f |= kFlagNeed;
        }
        sh.flag[b] = f;
        na += f ? 1 : 0;
        nn += (f & kFlagNeed) ? 1 : 0;
    }
    na = __reduce_add_sync(0xffffffffu, na);
    nn = __reduce_add_sync(0xffffffffu, nn);
    if ((tid & 31) == 0 && (na | nn)) {
        atomicAdd(&sh.cnt[0], na);
        atomicAdd(&sh.cnt[1], nn);
    }
    __syncthreads();
    const int ntile = (n + kTM - 1) / kTM, warp = tid >> 5, lane = tid & 31;
    for (int tile = warp; tile < ntile; tile += kTcWarps) {   // a warp ORs a tile's 128 flags
        unsigned any = 0;
        for (int r = lane; r < kTM && tile * kTM + r < n; r += 32) any |= sh.flag[tile * kTM + r];
        any = __reduce_or_sync(0xffffffffu, any);
        if (lane == 0) sh.tile_bits[tile] = static_cast<int>(any);
    }
    __syncthreads();
    if (tid == 0) {
        int ta = 0, tn = 0;
        for (int tile = 0; tile < ntile; ++tile) {
            if (sh.tile_bits[tile] & kFlagAct) sh.tiles_act[ta++] = tile;
            if (sh.tile_bits[tile] & kFlagNeed) sh.tiles_need[tn++] = tile;
        }
        sh.cnt[2] = ta;
        sh.cnt[3] = tn;
    }
    __syncthreads();
}

// Per-stream passes: stream b = blockIdx.x + i * gridDim.x goes to warp i % 12 of its owner CTA.
// The LSTM operand rows of stream b: [embed(tok) ; h_0] for layer 0 (zeros for the blank token) and h_l of the
// deeper layers, h read from `h` ([layers][Hp] of the stream's slot).
__device__ void tc_pack_lstm_rows(const TcCtx& c, int b, int tok, const float* h, int lane, bool& bad) {
    const RnntWeights& w = c.w;
    const int Hp = w.Hp, NLp = w.layers;
    const float4* x0 = tok >= 0 && tok < w.V - 1 ? reinterpret_cast<const float4*>(w.embed + static_cast<size_t>(tok) * Hp)
                                                 : nullptr;
    for (int i = lane; i < Hp / 4; i += 32) {
        const float4 x = x0 ? __ldg(x0 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        store_split4(c.xb.xl_hi[0], c.xb.xl_lo[0], static_cast<size_t>(b) * 2 * Hp + 4 * i, x, bad);
    }
    for (int l = 0; l < NLp; ++l) {
        const float4* h4 = reinterpret_cast<const float4*>(h + static_cast<size_t>(l) * Hp);
        for (int i = lane; i < Hp / 4; i += 32)
            store_split4(c.xb.xl_hi[l], c.xb.xl_lo[l], static_cast<size_t>(b) * 2 * Hp + Hp + 4 * i, __ldcg(h4 + i), bad);
    }
}

// The joint input relu(f_t + g) of stream b from its pending prediction.
__device__ void tc_pack_joint_row(const TcCtx& c, int b, int t, int lane, bool& bad) {
    const int J = c.w.J;
    const BatchEntry& me = c.meta[b];
    const float4* f = reinterpret_cast<const float4*>(c.proj + static_cast<size_t>(me.row_off + t) * c.ld_proj);
    const float4* g = reinterpret_cast<const float4*>(c.st.pend_g + static_cast<size_t>(me.slot) * J);
    for (int i = lane; i < J / 4; i += 32) {
        const float4 a = __ldg(f + i), d = __ldcg(g + i);
        const float4 x = make_float4(fmaxf(a.x + d.x, 0.f), fmaxf(a.y + d.y, 0.f), fmaxf(a.z + d.z, 0.f),
                                     fmaxf(a.w + d.w, 0.f));
        store_split4(c.xb.xj_hi, c.xb.xj_lo, static_cast<size_t>(b) * J + 4 * i, x, bad);
    }
}

// The greedy decision of stream b (the semantics of ls_decide: first maximum over the slice maxima in vocabulary
// order; blank ends the frame; a symbol is emitted, the pending state committed, the frame ends after max_symbols),
// taken by one warp, and after an emission the stream's next LSTM operand rows (the symbol's embedding and the
// committed h). The pending state and the stream's counters are loaded together with the slice maxima, so the commit
// and the rows need no second round trip for them.
__device__ void tc_decide(const TcCtx& c, int b, int t, int nparts, int32_t* tokens, int tok_stride, int* n_tokens,
                          bool& bad) {
    constexpr int kPre = 5;   // float4 of the pending h and c a lane holds from the start (1 layer of 640 units)
    const RnntWeights& w = c.w;
    const RnntState& st = c.st;
    const RnntScratch& scr = c.scr;
    const int lane = threadIdx.x & 31, Hp = w.Hp, NLp = w.layers, blank = w.V - 1, h4n = Hp / 4;
    const int slot = c.meta[b].slot;
    const size_t so = static_cast<size_t>(slot) * NLp * Hp;
    const float4* ph = reinterpret_cast<const float4*>(st.pend_h + so);
    const float4* pc = reinterpret_cast<const float4*>(st.pend_c + so);
    const int n4 = NLp * h4n;
    float4 hp[kPre], cp[kPre];
#pragma unroll
    for (int u = 0; u < kPre; ++u)
        if (lane + 32 * u < n4) {
            hp[u] = __ldcg(ph + lane + 32 * u);
            cp[u] = __ldcg(pc + lane + 32 * u);
        }
    const int nt = lane == 0 ? __ldcg(n_tokens + b) : 0, em = lane == 0 ? __ldcg(scr.emitted + b) : 0;
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
    if (bi > blank) bi = blank;   // no maximum at all (every logit NaN): end the frame, the state stays as it is
    if (bi == blank) {
        if (lane == 0) {
            st.pend_valid[slot] = 1;
            scr.done_frame[b] = t + 1;
            scr.emitted[b] = 0;
        }
        return;
    }
    // commit h, c <- the pending state, and the next rows: [embed(bi) ; h_0] and h_l of the deeper layers
    float4* h = reinterpret_cast<float4*>(st.h + so);
    float4* cc = reinterpret_cast<float4*>(st.c + so);
    const float4* e4 = reinterpret_cast<const float4*>(w.embed + static_cast<size_t>(bi) * Hp);
    for (int i = lane; i < h4n; i += 32)
        store_split4(c.xb.xl_hi[0], c.xb.xl_lo[0], static_cast<size_t>(b) * 2 * Hp + 4 * i, __ldg(e4 + i), bad);
    auto put = [&](int x, float4 hv, float4 cv) {
        h[x] = hv;
        cc[x] = cv;
        const int l = x / h4n, i = x - l * h4n;
        store_split4(c.xb.xl_hi[l], c.xb.xl_lo[l], static_cast<size_t>(b) * 2 * Hp + Hp + 4 * i, hv, bad);
    };
#pragma unroll
    for (int u = 0; u < kPre; ++u)
        if (lane + 32 * u < n4) put(lane + 32 * u, hp[u], cp[u]);
    for (int x = lane + 32 * kPre; x < n4; x += 32) put(x, __ldcg(ph + x), __ldcg(pc + x));
    if (lane == 0) {
        tokens[static_cast<size_t>(b) * tok_stride + nt] = bi;
        n_tokens[b] = nt + 1;
        st.last_tok[slot] = bi;
        st.pend_valid[slot] = 0;
        if (em + 1 >= w.max_symbols) {
            scr.done_frame[b] = t + 1;
            scr.emitted[b] = 0;
        } else {
            scr.emitted[b] = em + 1;
        }
    }
}

__global__ void __launch_bounds__(kTcThreads, 1) rnnt_tc_kernel(
    const __grid_constant__ TcMaps maps, const RnntWeights w, const RnntState st, const TcBufs xb, const TcPlan plan,
    const float* __restrict__ proj, int ld_proj, const BatchEntry* __restrict__ meta, int n, int32_t* __restrict__ tokens,
    int tok_stride, int* __restrict__ n_tokens, const RnntScratch scr, int* err) {
    extern __shared__ uint8_t tc_raw[];
    __shared__ uint64_t s_full[kTMaxStages], s_empty[kTMaxStages], s_acc_full, s_acc_empty;
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail, s_cnt[4];
    __shared__ float s_bias[kTcEpiWarps * kTMaxBN];
    const uint32_t raw = smem_u32(tc_raw);
    uint8_t* base = tc_raw + ((1024u - (raw & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, G = gridDim.x, k = blockIdx.x;
    const int ntile_max = (n + kTM - 1) / kTM;

    // The launch's context, plan and shared-memory layout live in shared memory: with nearly all of it taken by the
    // stages, L1 has little room left for a stack copy of them (local memory would then be read from L2).
    __shared__ TcShared s_sh;
    __shared__ TcPlan s_plan;
    __shared__ __align__(16) unsigned char s_ctx[sizeof(TcCtx)];
    TcShared& sh = s_sh;
    const TcPlan& pl = s_plan;
    const TcCtx& c = *reinterpret_cast<const TcCtx*>(s_ctx);
    if (tid == 0) {
        sh.stages = base;
        sh.tiles_act = reinterpret_cast<int*>(base + static_cast<size_t>(plan.stages) * plan.stage_bytes);
        sh.tiles_need = sh.tiles_act + ntile_max;
        sh.tile_bits = sh.tiles_need + ntile_max;
        sh.flag = reinterpret_cast<uint8_t*>(sh.tile_bits + ntile_max);
        sh.full = s_full;
        sh.empty = s_empty;
        sh.acc_full = &s_acc_full;
        sh.acc_empty = &s_acc_empty;
        sh.cnt = s_cnt;
        sh.bias = s_bias;
        sh.fail = &s_fail;
        s_plan = plan;
        *reinterpret_cast<TcCtx*>(s_ctx) = TcCtx{w, st, xb, proj, ld_proj, meta, n, scr, err};
    }
    if (tid == 0) {
        for (int s = 0; s < plan.stages; ++s) {
            mbar_init(&s_full[s], 1);
            mbar_init(&s_empty[s], 3);
        }
        mbar_init(&s_acc_full, 3);
        mbar_init(&s_acc_empty, kTcEpiWarps);
        s_fail = 0;
        fence_mbarrier_init();
    }
    if (warp == 0) {
        if (lane == 0) {
            for (int l = 0; l < w.layers; ++l) {
                prefetch_tensormap(&maps.xl_hi[l]);
                prefetch_tensormap(&maps.xl_lo[l]);
                prefetch_tensormap(&maps.wl_hi[l]);
                prefetch_tensormap(&maps.wl_lo[l]);
            }
            const CUtensorMap* rest[8] = {&maps.xp_hi, &maps.xp_lo, &maps.wp_hi, &maps.wp_lo,
                                          &maps.xj_hi, &maps.xj_lo, &maps.wo_hi, &maps.wo_lo};
            for (int i = 0; i < 8; ++i) prefetch_tensormap(rest[i]);
        }
        tmem_alloc(&s_tmem, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) sh.tmem = s_tmem;
    __syncthreads();
    pdl_wait();

    TcPipe pp;
    bool bad = false;
    unsigned long long target = 0;
    const int Hp = w.Hp, NLp = w.layers;
    int tmax = 0;
    for (int b = 0; b < n; ++b) tmax = max(tmax, meta[b].keep);

    // Launch setup: progress counters, and the LSTM operand rows of every stream from its carried state.
    if (tid == 0)
        for (int b = k; b < n; b += G) {
            scr.done_frame[b] = 0;
            scr.emitted[b] = 0;
            n_tokens[b] = 0;
        }
    for (int b = k + warp * G; b < n; b += kTcWarps * G) {
        const int slot = meta[b].slot;
        tc_pack_lstm_rows(c, b, __ldcg(st.last_tok + slot), st.h + static_cast<size_t>(slot) * w.layers * w.Hp, lane, bad);
    }
    if (!tc_grid_sync(scr.barrier, target, err, sh.fail)) goto done;

    for (int t = 0; t < tmax; ++t) {
        for (int pass = 0;; ++pass) {
            tc_flags(c, t, sh);
            const int na = sh.cnt[0], nn = sh.cnt[1];
            if (na == 0) break;
            if (pass == 0) {
                // the joint inputs of the streams entering the frame with a pending prediction
                for (int b = k + warp * G; b < n; b += kTcWarps * G)
                    if (sh.flag[b] == kFlagAct) tc_pack_joint_row(c, b, t, lane, bad);
                if (nn == 0 && !tc_grid_sync(scr.barrier, target, err, sh.fail)) goto done;
            }
            if (nn > 0) {
                for (int l = 0; l < NLp; ++l) {
                    if (!tc_product(c, sh, pp, kPhLstm, l, t, pl, &maps.xl_hi[l], &maps.xl_lo[l], &maps.wl_hi[l],
                                    &maps.wl_lo[l]))
                        goto done;
                    if (!tc_grid_sync(scr.barrier, target, err, sh.fail)) goto done;
                }
                if (!tc_product(c, sh, pp, kPhPred, 0, t, pl, &maps.xp_hi, &maps.xp_lo, &maps.wp_hi, &maps.wp_lo))
                    goto done;
                if (!tc_grid_sync(scr.barrier, target, err, sh.fail)) goto done;
            }
            if (!tc_product(c, sh, pp, kPhJoint, 0, t, pl, &maps.xj_hi, &maps.xj_lo, &maps.wo_hi, &maps.wo_lo))
                goto done;
            if (!tc_grid_sync(scr.barrier, target, err, sh.fail)) goto done;
            for (int b = k + warp * G; b < n; b += kTcWarps * G)
                if (sh.flag[b] & kFlagAct) tc_decide(c, b, t, pl.ns[kPhJoint], tokens, tok_stride, n_tokens, bad);
            if (!tc_grid_sync(scr.barrier, target, err, sh.fail)) goto done;
        }
    }
done:
    if (bad) report_error(err, DEV_RANGE_F16);
    __syncthreads();
    if (*sh.fail) __nanosleep(100000);   // let in-flight copies and MMAs land before the accumulators are released
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(sh.tmem, kTmemCols);
    }
    (void)Hp;
}

// Host split of one value into its fp16 pair; false beyond the fp16 range.
inline bool split_host(float x, uint16_t& hi, uint16_t& lo) {
    if (!(std::fabs(x) < kHalfMax)) return false;
    const __half h = __float2half_rn(x);
    const __half l = __float2half_rn((x - __half2float(h)) * kLoScale);
    std::memcpy(&hi, &h, 2);
    std::memcpy(&lo, &l, 2);
    return true;
}

// Slice width of a product of N output rows and nk chunks over mt stream tiles: the multiple of 16 with the least
// estimated time, waves of items over the grid x a chunk's cost (issue of four MMAs per warp, tensor time of the
// twelve, and its bytes from L2).
int pick_bn(int N, int nk, int mt, int G) {
    int best_bn = 16;
    double best = 1e30;
    for (int bn = 16; bn <= kTMaxBN; bn += 16) {
        const int items = mt * ((N + bn - 1) / bn);
        const int waves = (items + G - 1) / G;
        const double chunk_ns = std::max({200.0, 12.0 * bn / 128.0 * 41.0, (32768.0 + 256.0 * bn) / 190.0});
        const double cost = waves * nk * chunk_ns;
        if (cost < best - 1e-9) { best = cost; best_bn = bn; }
    }
    return best_bn;
}

}  // namespace

bool rnnt_tc_split(const float* w, size_t count, uint16_t* hi, uint16_t* lo) {
    for (size_t i = 0; i < count; ++i)
        if (!split_host(w[i], hi[i], lo[i])) return false;
    return true;
}

bool rnnt_tc_split_lstm(const float* w_ih, const float* w_hh, int Hp, uint16_t* hi, uint16_t* lo) {
    for (int u = 0; u < Hp; ++u)
        for (int q = 0; q < 4; ++q) {
            const size_t dst = (static_cast<size_t>(u) * 4 + q) * 2 * Hp, src = static_cast<size_t>(q * Hp + u) * Hp;
            for (int x = 0; x < Hp; ++x) {
                if (!split_host(w_ih[src + x], hi[dst + x], lo[dst + x])) return false;
                if (!split_host(w_hh[src + x], hi[dst + Hp + x], lo[dst + Hp + x])) return false;
            }
        }
    return true;
}

bool rnnt_tc_build_row_maps(RnntTc& tc, int layers, int Hp, int J) {
    bool ok = true;
    for (int l = 0; l < layers; ++l) {
        ok = ok && make_tma_bf16(tc.m_xl_hi[l], tc.xl_hi[l], tc.n_pad, 2 * Hp, 2 * Hp, kTM);
        ok = ok && make_tma_bf16(tc.m_xl_lo[l], tc.xl_lo[l], tc.n_pad, 2 * Hp, 2 * Hp, kTM);
    }
    ok = ok && make_tma_bf16(tc.m_xp_hi, tc.xp_hi, tc.n_pad, Hp, Hp, kTM) &&
         make_tma_bf16(tc.m_xp_lo, tc.xp_lo, tc.n_pad, Hp, Hp, kTM) &&
         make_tma_bf16(tc.m_xj_hi, tc.xj_hi, tc.n_pad, J, J, kTM) && make_tma_bf16(tc.m_xj_lo, tc.xj_lo, tc.n_pad, J, J, kTM);
    tc.maps_ok = ok;
    return ok;
}

bool rnnt_greedy_tc(const RnntWeights& w, const RnntState& st, const float* proj, int ld_proj, const BatchEntry* meta,
                    int n, int32_t* tokens, int tok_stride, int* n_tokens, const RnntScratch& scr, int num_sms,
                    int* dev_err, cudaStream_t s) {
    RnntTc* tc = scr.tc;
    const int G = std::min(num_sms, scr.max_grid);
    const int ntile = (n + kTM - 1) / kTM;
    constexpr size_t kSmemMax = 227 * 1024 - 7168;   // static shared memory of the kernel stays below 7 KB
    const size_t lists = sizeof(int) * 3 * ntile + static_cast<size_t>(n);
    if (!tc || !tc->weights_ok || !tc->maps_ok || !scr.barrier || n <= 0 || n > scr.max_n || n > tc->n_pad ||
        w.max_symbols <= 0 || w.layers < 1 || w.layers > 4 || w.Hp % kTK || w.J % kTK || ld_proj % 4 ||
        (reinterpret_cast<uintptr_t>(proj) & 15) || (w.V + 15) / 16 > G)
        return false;
    TcPlan plan;
    const int N[3] = {4 * w.Hp, w.J, w.V}, K[3] = {2 * w.Hp, w.Hp, w.J};
    int bn_max = 16;
    for (int p = 0; p < 3; ++p) {
        plan.nk[p] = K[p] / kTK;
        plan.bn[p] = pick_bn(N[p], plan.nk[p], ntile, G);
        plan.ns[p] = (N[p] + plan.bn[p] - 1) / plan.bn[p];
        bn_max = std::max(bn_max, plan.bn[p]);
    }
    plan.b_lo = 2 * kTileA + static_cast<uint32_t>(bn_max) * 128;   // bn_max is a multiple of 8: 1024-byte aligned
    plan.stage_bytes = plan.b_lo + static_cast<uint32_t>(bn_max) * 128;
    plan.stages = static_cast<int>(std::min<size_t>(kTMaxStages, (kSmemMax - 1024 - lists) / plan.stage_bytes));
    const size_t smem = 1024 + static_cast<size_t>(plan.stages) * plan.stage_bytes + lists;
    if (plan.stages < 2) return false;
    if (plan.bn[0] != tc->bn_lstm || plan.bn[1] != tc->bn_pred || plan.bn[2] != tc->bn_joint) {
        bool ok = true;
        for (int l = 0; l < w.layers; ++l) {
            ok = ok && make_tma_bf16(tc->m_wl_hi[l], tc->wl_hi[l], 4 * w.Hp, 2 * w.Hp, 2 * w.Hp, plan.bn[0]);
            ok = ok && make_tma_bf16(tc->m_wl_lo[l], tc->wl_lo[l], 4 * w.Hp, 2 * w.Hp, 2 * w.Hp, plan.bn[0]);
        }
        ok = ok && make_tma_bf16(tc->m_wp_hi, tc->wp_hi, w.J, w.Hp, w.Hp, plan.bn[1]) &&
             make_tma_bf16(tc->m_wp_lo, tc->wp_lo, w.J, w.Hp, w.Hp, plan.bn[1]) &&
             make_tma_bf16(tc->m_wo_hi, tc->wo_hi, w.V, w.J, w.J, plan.bn[2]) &&
             make_tma_bf16(tc->m_wo_lo, tc->wo_lo, w.V, w.J, w.J, plan.bn[2]);
        if (!ok) {
            tc->bn_lstm = tc->bn_pred = tc->bn_joint = 0;
            return false;
        }
        tc->bn_lstm = plan.bn[0];
        tc->bn_pred = plan.bn[1];
        tc->bn_joint = plan.bn[2];
    }
    TcMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    TcBufs xb;
    for (int l = 0; l < w.layers; ++l) {
        maps.xl_hi[l] = tc->m_xl_hi[l].map;
        maps.xl_lo[l] = tc->m_xl_lo[l].map;
        maps.wl_hi[l] = tc->m_wl_hi[l].map;
        maps.wl_lo[l] = tc->m_wl_lo[l].map;
    }
    for (int l = 0; l < 4; ++l) {
        xb.xl_hi[l] = reinterpret_cast<__half*>(tc->xl_hi[l]);
        xb.xl_lo[l] = reinterpret_cast<__half*>(tc->xl_lo[l]);
    }
    maps.xp_hi = tc->m_xp_hi.map;
    maps.xp_lo = tc->m_xp_lo.map;
    maps.wp_hi = tc->m_wp_hi.map;
    maps.wp_lo = tc->m_wp_lo.map;
    maps.xj_hi = tc->m_xj_hi.map;
    maps.xj_lo = tc->m_xj_lo.map;
    maps.wo_hi = tc->m_wo_hi.map;
    maps.wo_lo = tc->m_wo_lo.map;
    xb.xp_hi = reinterpret_cast<__half*>(tc->xp_hi);
    xb.xp_lo = reinterpret_cast<__half*>(tc->xp_lo);
    xb.xj_hi = reinterpret_cast<__half*>(tc->xj_hi);
    xb.xj_lo = reinterpret_cast<__half*>(tc->xj_lo);

    static size_t attr_set[kMaxDevices] = {};
    ensure_dyn_smem(rnnt_tc_kernel, kSmemMax, attr_set);
    cudaMemsetAsync(scr.barrier, 0, sizeof(unsigned long long), s);
    // Cooperative: the runtime refuses the launch unless all G CTAs can be resident at once, so the grid barriers
    // never wait on a CTA that was not scheduled (their bounded waits stay as a second guard).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, rnnt_tc_kernel, maps, w, st, xb, plan, proj, ld_proj, meta, n, tokens, tok_stride,
                           n_tokens, scr, dev_err) != cudaSuccess) {
        cudaGetLastError();   // a refused launch leaves no error behind: the caller decodes with another kernel
        return false;
    }
    return true;
}

}  // namespace ud
