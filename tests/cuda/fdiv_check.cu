// Test program (built by tests/test_gpu_ops.py with nvcc): compares the GELU's
// branch-free division fdiv_markstein(2, b) with IEEE division __fdiv_rn(2, b)
// for every float b in [1, 2^26), the range of the GELU denominator
// 1 + exp(2v), |v| <= 9.  Prints the number of differing quotients.
#include <cstdio>
#include "common.cuh"

__device__ unsigned long long g_bad = 0;

__global__ void check(uint32_t lo, uint32_t hi) {
    unsigned long long bad = 0;
    for (uint32_t u = lo + blockIdx.x * blockDim.x + threadIdx.x; u < hi; u += gridDim.x * blockDim.x) {
        const float b = __uint_as_float(u);
        bad += __float_as_uint(eg2::fdiv_markstein(2.0f, b)) != __float_as_uint(__fdiv_rn(2.0f, b));
    }
    if (bad) atomicAdd(&g_bad, bad);
}

int main() {
    const uint32_t lo = 0x3f800000u, hi = 0x4c800000u;  // 1.0f .. 2^26
    check<<<1184, 256>>>(lo, hi);
    const cudaError_t e = cudaDeviceSynchronize();
    unsigned long long bad = 0;
    cudaMemcpyFromSymbol(&bad, g_bad, sizeof bad);
    std::printf("checked %u divisors, %llu differ, %s\n", hi - lo, bad, cudaGetErrorString(e));
    return e != cudaSuccess || bad != 0;
}
