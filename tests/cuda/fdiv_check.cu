// Test program (built by tests/test_gpu_ops.py with nvcc): compares the
// branch-free divisions of the kernels with IEEE division __fdiv_rn:
//   fdiv_markstein(2, b) for every float b in [1, 2^26), the range of the GELU
//   denominator 1 + exp(2v), |v| <= 9;
//   div_sqrt512(a) against a / sqrtf(512) for every float bit pattern a;
//   div127(a) and rcp_rn(a) (the Q8_0 quantizer's d = amax / 127 and 1 / d)
//   for every non-negative float a.
// Prints the number of differing quotients.
#include <cstdio>
#include "common.cuh"

__device__ unsigned long long g_bad = 0, g_bad512 = 0, g_bad127 = 0, g_badrcp = 0;
__device__ unsigned int g_rcp_first = 0xFFFFFFFFu;

// div127 and rcp_rn against IEEE division for every non-negative float (the
// quantizer's amax and its scale d are never negative).
__global__ void check_quant() {
    unsigned long long b127 = 0, brcp = 0;
    for (uint32_t u = blockIdx.x * blockDim.x + threadIdx.x; u < 0x80000000u; u += gridDim.x * blockDim.x) {
        const float a = __uint_as_float(u);  // every non-negative float, +inf and NaNs included
        const float q = eg2::div127(a), r = __fdiv_rn(a, 127.0f);
        b127 += __float_as_uint(q) != __float_as_uint(r) && !(q != q && r != r);
        if (u != 0) {
            const float y = eg2::rcp_rn(a), z = __fdiv_rn(1.0f, a);
            const bool differ = __float_as_uint(y) != __float_as_uint(z) && !(y != y && z != z);
            if (differ) atomicMin(&g_rcp_first, u);
            brcp += differ;
        }
    }
    if (b127) atomicAdd(&g_bad127, b127);
    if (brcp) atomicAdd(&g_badrcp, brcp);
}

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
    check_quant<<<2368, 256>>>();
    const cudaError_t e = cudaDeviceSynchronize();
    unsigned long long bad = 0, bad512 = 0, bad127 = 0, badrcp = 0;
    cudaMemcpyFromSymbol(&bad, g_bad, sizeof bad);
    cudaMemcpyFromSymbol(&bad512, g_bad512, sizeof bad512);
    cudaMemcpyFromSymbol(&bad127, g_bad127, sizeof bad127);
    cudaMemcpyFromSymbol(&badrcp, g_badrcp, sizeof badrcp);
    unsigned int rf = 0;
    cudaMemcpyFromSymbol(&rf, g_rcp_first, sizeof rf);
    if (badrcp) std::printf("first differing reciprocal input 0x%08x\n", rf);
    std::printf("checked %u divisors, %llu differ; checked 2^32 dividends of sqrt(512), %llu differ; "
                "checked 2^31 dividends of 127, %llu differ; checked 2^31 - 1 reciprocals, %llu differ; %s\n",
                hi - lo, bad, bad512, bad127, badrcp, cudaGetErrorString(e));
    return e != cudaSuccess || bad != 0 || bad512 != 0 || bad127 != 0 || badrcp != 0;
}
