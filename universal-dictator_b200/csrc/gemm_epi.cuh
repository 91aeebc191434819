// Epilogue helpers shared by the tcgen05 GEMMs: 32 consecutive accumulator columns of one row are turned into
// out_scale * act(acc + bias) + res_scale * residual and stored with 16-byte writes.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace ud {

// Applies the epilogue to 32 consecutive columns of one row; `r` holds the residual values (if any).
static __device__ __forceinline__ void epilogue_store32(const GemmEpilogue& epi, int row, int col, float* v, const float* r) {
    if (epi.bias) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const float4 b = *reinterpret_cast<const float4*>(epi.bias + col + j);
            v[j] += b.x; v[j + 1] += b.y; v[j + 2] += b.z; v[j + 3] += b.w;
        }
    }
    if (epi.act == ACT_RELU) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
    } else if (epi.act == ACT_SILU) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = silu(v[j]);
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] *= epi.out_scale;
    if (epi.residual) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = fmaf(epi.res_scale, r[j], v[j]);
    }
    if (epi.out_bf16) {
        bf16* o = reinterpret_cast<bf16*>(epi.out) + static_cast<size_t>(row) * epi.ldo + col;
#pragma unroll
        for (int j = 0; j < 32; j += 8) store16<bf16>(o + j, v + j);
    } else {
        float* o = reinterpret_cast<float*>(epi.out) + static_cast<size_t>(row) * epi.ldo + col;
#pragma unroll
        for (int j = 0; j < 32; j += 4) store16<float>(o + j, v + j);
    }
}

static __device__ __forceinline__ void load_residual32(const GemmEpilogue& epi, int row, int col, float* r) {
    const float* p = epi.residual + static_cast<size_t>(row) * epi.ldr + col;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
        const float4 x = *reinterpret_cast<const float4*>(p + j);
        r[j] = x.x; r[j + 1] = x.y; r[j + 2] = x.z; r[j + 3] = x.w;
    }
}

// The same epilogue for 16 consecutive columns.
static __device__ __forceinline__ void epilogue_store16(const GemmEpilogue& epi, int row, int col, float* v,
                                                        const float* r) {
    if (epi.bias) {
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
            const float4 b = *reinterpret_cast<const float4*>(epi.bias + col + j);
            v[j] += b.x; v[j + 1] += b.y; v[j + 2] += b.z; v[j + 3] += b.w;
        }
    }
    if (epi.act == ACT_RELU) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = fmaxf(v[j], 0.f);
    } else if (epi.act == ACT_SILU) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = silu(v[j]);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] *= epi.out_scale;
    if (epi.residual) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = fmaf(epi.res_scale, r[j], v[j]);
    }
    if (epi.out_bf16) {
        bf16* o = reinterpret_cast<bf16*>(epi.out) + static_cast<size_t>(row) * epi.ldo + col;
        store16<bf16>(o, v);
        store16<bf16>(o + 8, v + 8);
    } else {
        float* o = reinterpret_cast<float*>(epi.out) + static_cast<size_t>(row) * epi.ldo + col;
#pragma unroll
        for (int j = 0; j < 16; j += 4) store16<float>(o + j, v + j);
    }
}

static __device__ __forceinline__ void load_residual16(const GemmEpilogue& epi, int row, int col, float* r) {
    const float* p = epi.residual + static_cast<size_t>(row) * epi.ldr + col;
#pragma unroll
    for (int j = 0; j < 16; j += 4) {
        const float4 x = *reinterpret_cast<const float4*>(p + j);
        r[j] = x.x; r[j + 1] = x.y; r[j + 2] = x.z; r[j + 3] = x.w;
    }
}

}  // namespace ud
