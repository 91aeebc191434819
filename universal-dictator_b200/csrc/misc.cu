// Small utility kernels: fills, dtype conversion, and the bounded-wait probe used by the failure-detection test.
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace ud {
namespace {

__global__ void fill_kernel(float* p, float v, size_t n) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        p[i] = v;
}

__global__ void to_bf16_kernel(const float* in, bf16* out, size_t n) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        out[i] = __float2bfloat16_rn(in[i]);
}

// Waits on a flag that nothing sets, with the same bounded-wait discipline as the pipelined kernels:
// after limit_ns it records DEV_TIMEOUT_TEST in the error word and returns, leaving the context usable.
__global__ void wait_probe_kernel(int* err, uint64_t limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbarrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&bar, 0)) {
            if (global_timer_ns() - t0 > limit_ns) {
                report_error(err, DEV_TIMEOUT_TEST);
                break;
            }
        }
    }
}

}  // namespace

bool pdl_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* v = std::getenv("UD_PDL");
        on = (v && std::atoi(v) == 0) ? 0 : 1;
    }
    return on == 1;
}

void fill_f32(float* p, float v, size_t n, cudaStream_t s) {
    if (!n) return;
    fill_kernel<<<296, 256, 0, s>>>(p, v, n);
}

void f32_to_bf16(const float* in, bf16* out, size_t n, cudaStream_t s) {
    if (!n) return;
    to_bf16_kernel<<<592, 256, 0, s>>>(in, out, n);
}

void test_wait_timeout(int* dev_err, uint64_t limit_ns, cudaStream_t s) { wait_probe_kernel<<<1, 32, 0, s>>>(dev_err, limit_ns); }

}  // namespace ud
