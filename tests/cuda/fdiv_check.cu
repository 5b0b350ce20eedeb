// Test program (built by tests/test_gpu_ops.py with nvcc): compares the
// branch-free divisions of the kernels with IEEE division __fdiv_rn:
//   fdiv_markstein(2, b) for every float b in [1, 2^26), the range of the GELU
//   denominator 1 + exp(2v), |v| <= 9;
//   div_sqrt512(a) against a / sqrtf(512) for every float bit pattern a.
// Prints the number of differing quotients.
#include <cstdio>
#include "common.cuh"

__device__ unsigned long long g_bad = 0, g_bad512 = 0;

__global__ void check512() {
    unsigned long long bad = 0;
    for (uint64_t u = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; u < (1ull << 32); u += uint64_t(gridDim.x) * blockDim.x) {
        const float a = __uint_as_float(uint32_t(u)), q = eg2::div_sqrt512(a), r = __fdiv_rn(a, 22.627416997969522f);
        bad += __float_as_uint(q) != __float_as_uint(r) && !(q != q && r != r);
    }
    if (bad) atomicAdd(&g_bad512, bad);
}

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
    check512<<<2368, 256>>>();
    const cudaError_t e = cudaDeviceSynchronize();
    unsigned long long bad = 0, bad512 = 0;
    cudaMemcpyFromSymbol(&bad, g_bad, sizeof bad);
    cudaMemcpyFromSymbol(&bad512, g_bad512, sizeof bad512);
    std::printf("checked %u divisors, %llu differ; checked 2^32 dividends of sqrt(512), %llu differ; %s\n", hi - lo,
                bad, bad512, cudaGetErrorString(e));
    return e != cudaSuccess || bad != 0 || bad512 != 0;
}
