// Epilogue helpers shared by the tcgen05 GEMMs: accumulator columns become
// out_scale * act(acc + bias) + res_scale * residual, stored to the output row-contiguously.
//
// A warp's tcgen05.ld gives each lane one row (its TMEM lane) and consecutive columns, so writing straight from
// registers makes every store instruction touch 32 different rows. For fp32 outputs each warp instead passes
// 16-column blocks through its own shared-memory buffer (32 rows x 16 fp32, row stride 20 floats: conflict-free float4
// writes by row, at most 2-way conflicts on the transposed reads) and then 4 lanes cover one row's 16 columns,
// 8 rows per instruction. The residual is read in the same transposed pattern, by the lane that later writes
// the same elements (so residual may alias out).
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace ud {

constexpr int kEpiStride = 20;                       // floats per staged row
constexpr int kEpiStageFloats = 32 * kEpiStride;     // one warp's buffer
constexpr int kEpiStageBytes = kEpiStageFloats * 4;

// Residual values this lane combines for the 32 x 16 block at (row0, col): rows row0 + 8 it + lane / 4,
// columns col + 4 (lane % 4) .. + 3.
static __device__ __forceinline__ void epi16_load_res(const GemmEpilogue& epi, int row0, int M, int col, int lane,
                                                      float4 (&r)[4]) {
    const int cq = (lane & 3) * 4, rs = lane >> 2;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        const int g = row0 + it * 8 + rs;
        r[it] = (epi.residual && g < M)
                    ? *reinterpret_cast<const float4*>(epi.residual + static_cast<size_t>(g) * epi.ldr + col + cq)
                    : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

static __device__ __forceinline__ float epi_act(int act, float x) {
    if (act == ACT_RELU) return fmaxf(x, 0.f);
    if (act == ACT_SILU) return silu(x);
    return x;
}
// The same for outputs stored as bf16: SiLU with one special-function operation instead of two.
static __device__ __forceinline__ float epi_act_bf16(int act, float x) {
    if (act == ACT_RELU) return fmaxf(x, 0.f);
    if (act == ACT_SILU) return x_sigmoid_bf16out(x, x);
    return x;
}

// v: this lane's row (row0 + lane), columns col .. col + 15. stg: the warp's staging buffer.
static __device__ __forceinline__ void epi16_store(const GemmEpilogue& epi, float* stg, int row0, int M, int col,
                                                   int lane, const float* v, const float4 (&r)[4]) {
    float* mine = stg + lane * kEpiStride;
#pragma unroll
    for (int q = 0; q < 4; ++q)
        *reinterpret_cast<float4*>(mine + 4 * q) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    __syncwarp();
    const int cq = (lane & 3) * 4, rs = lane >> 2;
    const float4 b = epi.bias ? *reinterpret_cast<const float4*>(epi.bias + col + cq) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        const int rr = it * 8 + rs, g = row0 + rr;
        const float4 x = *reinterpret_cast<const float4*>(stg + rr * kEpiStride + cq);
        float e[4] = {x.x, x.y, x.z, x.w};
        if (epi.bias) { e[0] += b.x; e[1] += b.y; e[2] += b.z; e[3] += b.w; }
#pragma unroll
        for (int j = 0; j < 4; ++j) e[j] = (epi.out_bf16 ? epi_act_bf16(epi.act, e[j]) : epi_act(epi.act, e[j])) * epi.out_scale;
        if (epi.residual) {
            e[0] = fmaf(epi.res_scale, r[it].x, e[0]);
            e[1] = fmaf(epi.res_scale, r[it].y, e[1]);
            e[2] = fmaf(epi.res_scale, r[it].z, e[2]);
            e[3] = fmaf(epi.res_scale, r[it].w, e[3]);
        }
        if (g < M) {
            if (epi.out_bf16) {
                __nv_bfloat162 lo = __floats2bfloat162_rn(e[0], e[1]), hi = __floats2bfloat162_rn(e[2], e[3]);
                uint2 u;
                u.x = *reinterpret_cast<uint32_t*>(&lo);
                u.y = *reinterpret_cast<uint32_t*>(&hi);
                *reinterpret_cast<uint2*>(reinterpret_cast<bf16*>(epi.out) + static_cast<size_t>(g) * epi.ldo + col + cq) = u;
            } else {
                *reinterpret_cast<float4*>(reinterpret_cast<float*>(epi.out) + static_cast<size_t>(g) * epi.ldo + col + cq) =
                    make_float4(e[0], e[1], e[2], e[3]);
            }
        }
    }
    __syncwarp();
}

// Direct path: 32 (or 16) consecutive columns of this lane's row stored straight from registers with 16-byte
// writes. Used for bf16 outputs, where staging cost more than the wider writes saved.
template <int NC>
static __device__ __forceinline__ void epi_direct(const GemmEpilogue& epi, int row, int col, float* v, const float* r) {
    if (epi.bias) {
#pragma unroll
        for (int j = 0; j < NC; j += 4) {
            const float4 b = *reinterpret_cast<const float4*>(epi.bias + col + j);
            v[j] += b.x; v[j + 1] += b.y; v[j + 2] += b.z; v[j + 3] += b.w;
        }
    }
    if (epi.out_bf16) {
#pragma unroll
        for (int j = 0; j < NC; ++j) v[j] = epi_act_bf16(epi.act, v[j]) * epi.out_scale;
    } else {
#pragma unroll
        for (int j = 0; j < NC; ++j) v[j] = epi_act(epi.act, v[j]) * epi.out_scale;
    }
    if (epi.residual) {
#pragma unroll
        for (int j = 0; j < NC; ++j) v[j] = fmaf(epi.res_scale, r[j], v[j]);
    }
    if (epi.out_bf16) {
        bf16* o = reinterpret_cast<bf16*>(epi.out) + static_cast<size_t>(row) * epi.ldo + col;
#pragma unroll
        for (int j = 0; j < NC; j += 8) store16<bf16>(o + j, v + j);
    } else {
        float* o = reinterpret_cast<float*>(epi.out) + static_cast<size_t>(row) * epi.ldo + col;
#pragma unroll
        for (int j = 0; j < NC; j += 4) store16<float>(o + j, v + j);
    }
}

template <int NC>
static __device__ __forceinline__ void epi_direct_res(const GemmEpilogue& epi, int row, int col, float* r) {
    const float* p = epi.residual + static_cast<size_t>(row) * epi.ldr + col;
#pragma unroll
    for (int j = 0; j < NC; j += 4) {
        const float4 x = *reinterpret_cast<const float4*>(p + j);
        r[j] = x.x; r[j + 1] = x.y; r[j + 2] = x.z; r[j + 3] = x.w;
    }
}

// Drains 16-column blocks [b0, b1) of one accumulator row range: the warp's 32 TMEM lanes at t_row hold rows
// row0 .. row0 + 31; tile column 16 blk is output column col0 + 16 blk. fp32 outputs go through the staging
// buffer (residual of both 16-column blocks requested before the TMEM load); bf16 outputs are written directly,
// 32 columns at a time with the next chunk's residual in flight.
static __device__ __forceinline__ void epi_drain(const GemmEpilogue& epi, float* stg, uint32_t t_row, int row0, int M,
                                                 int col0, int b0, int b1, int lane) {
    int blk = b0;
    if (!epi.out_bf16) {
#pragma unroll 1
        for (; blk + 2 <= b1; blk += 2) {
            float4 ra[4], rb[4];
            epi16_load_res(epi, row0, M, col0 + blk * 16, lane, ra);
            epi16_load_res(epi, row0, M, col0 + blk * 16 + 16, lane, rb);
            float v[32];
            tmem_ld32(t_row + static_cast<uint32_t>(blk * 16), v);
            epi16_store(epi, stg, row0, M, col0 + blk * 16, lane, v, ra);
            epi16_store(epi, stg, row0, M, col0 + blk * 16 + 16, lane, v + 16, rb);
        }
        if (blk < b1) {
            float4 ra[4];
            epi16_load_res(epi, row0, M, col0 + blk * 16, lane, ra);
            float v[16];
            tmem_ld16(t_row + static_cast<uint32_t>(blk * 16), v);
            epi16_store(epi, stg, row0, M, col0 + blk * 16, lane, v, ra);
        }
        return;
    }
    const int row = row0 + lane;
    const bool live = row < M;
    const bool res = epi.residual != nullptr && live;
    float rnext[32];
    if (res && blk + 2 <= b1) epi_direct_res<32>(epi, row, col0 + blk * 16, rnext);
#pragma unroll 1
    for (; blk + 2 <= b1; blk += 2) {
        float v[32], rcur[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) rcur[j] = rnext[j];
        if (res && blk + 4 <= b1) epi_direct_res<32>(epi, row, col0 + (blk + 2) * 16, rnext);
        tmem_ld32(t_row + static_cast<uint32_t>(blk * 16), v);
        if (live) epi_direct<32>(epi, row, col0 + blk * 16, v, rcur);
    }
    if (blk < b1) {
        float v[16], r16[16];
        if (res) epi_direct_res<16>(epi, row, col0 + blk * 16, r16);
        tmem_ld16(t_row + static_cast<uint32_t>(blk * 16), v);
        if (live) epi_direct<16>(epi, row, col0 + blk * 16, v, r16);
    }
}

}  // namespace ud
