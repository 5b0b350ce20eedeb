// The reference's operator surface, kernels/abi.h:3-11, with the semantics of
// its AMDGPU kernels (kernels/eg2.c): fp32 activations, weights decoded from
// GGUF F32 / F16 / Q8_0 / BF16 on the fly, fp32 accumulation in k order.
// These serve FFI users of the operator ABI and the port of the reference's
// operator tests; the executor's fast path uses the fused kernels instead.
#pragma once
#include "../../include/eg2_ops.h"
#include "common.cuh"

namespace eg2 {

// eg2.c:9-17 -- element i of a GGUF weight of type 0/1/8/30.
__device__ __forceinline__ float gguf_weight(const void *w, size_t i, unsigned type) {
    if (type == 1) return __half2float(reinterpret_cast<const __half *>(w)[i]);
    if (type == 0) return reinterpret_cast<const float *>(w)[i];
    if (type == 30) return __uint_as_float(uint32_t(reinterpret_cast<const uint16_t *>(w)[i]) << 16);
    const uint8_t *b = reinterpret_cast<const uint8_t *>(w) + (i / 32) * 34;
    const uint16_t bits = uint16_t(b[0]) | uint16_t(b[1]) << 8;
    return __fmul_rn(fp16_bits_to_f32(bits), float(reinterpret_cast<const int8_t *>(b + 2)[i % 32]));
}

__global__ void abi_gather_kernel(EgGather p) {
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < size_t(p.n) * 512)
        p.out[i] = __fmul_rn(gguf_weight(p.weight, size_t(unsigned(p.ids[i / 512])) * 512 + i % 512, 8),
                             22.62741699796952f);
}

// 16x16 output tile per 256 threads; W rows staged through shared memory.
__global__ void abi_mm_kernel(EgMM p) {
    __shared__ float a[16][17], b[16][17];
    const int r = threadIdx.x / 16, c = threadIdx.x % 16;
    const unsigned row = blockIdx.y * 16 + r, col = blockIdx.x * 16 + c;
    float acc = 0.0f;
    for (unsigned base = 0; base < p.k; base += 16) {
        a[r][c] = row < p.n && base + c < p.k ? p.x[size_t(row) * p.k + base + c] : 0.0f;
        const unsigned wr = blockIdx.x * 16 + r;
        b[r][c] = wr < p.m && base + c < p.k ? gguf_weight(p.weight, size_t(wr) * p.k + base + c, p.type) : 0.0f;
        __syncthreads();
#pragma unroll
        for (int j = 0; j < 16; ++j) acc = __fmaf_rn(a[r][j], b[c][j], acc);
        __syncthreads();
    }
    if (row < p.n && col < p.m) p.out[size_t(row) * p.m + col] = acc;
}

// eg2.c:122-133: one warp per row; in place is valid.
__global__ void abi_norm_kernel(EgNorm p) {
    const unsigned row = blockIdx.x, lane = threadIdx.x;
    if (row >= p.rows) return;
    float ss = 0.0f;
    for (unsigned z = lane; z < p.d; z += 32) {
        const float v = p.x[size_t(row) * p.d + z] * p.scale;
        ss += v * v;
    }
    const float inv = rsqrtf(warp_sum_f(ss) / float(p.d) + 1.0e-6f);
    __syncwarp();
    for (unsigned z = lane; z < p.d; z += 32)
        p.out[size_t(row) * p.d + z] = p.x[size_t(row) * p.d + z] * p.scale * inv * (p.weight ? p.weight[z] : 1.0f);
}

// eg2.c:135-143.
__global__ void abi_rope_kernel(EgRope p) {
    const unsigned i = blockIdx.x * blockDim.x + threadIdx.x, half = p.d / 2;
    if (i >= p.n * p.heads * half) return;
    const unsigned z = i % half, row = i / half, t = row / p.heads;
    const float c = p.table[size_t(t) * p.d + z], s = p.table[size_t(t) * p.d + half + z];
    const float a = p.x[size_t(row) * p.d + z], b = p.x[size_t(row) * p.d + half + z];
    p.x[size_t(row) * p.d + z] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    p.x[size_t(row) * p.d + half + z] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
}

// eg2.c:147-170: streaming softmax, one warp per (token, head), K/V row stride 512.
template <int D>
__global__ void abi_attention_kernel(EgAttention p) {
    const unsigned row = blockIdx.x, lane = threadIdx.x;
    const unsigned t = row / 4, h = row % 4, kh = h / (4 / (512 / D));
    if (t >= p.n) return;
    unsigned lo = p.bounds[2 * t], hi = p.bounds[2 * t + 1];
    if (p.window && t > p.window && lo < t - p.window) lo = t - p.window;
    if (p.window && hi > t + p.window + 1) hi = t + p.window + 1;
    float q[D / 32], acc[D / 32];
#pragma unroll
    for (int j = 0; j < D / 32; ++j) q[j] = p.q[size_t(row) * D + lane + j * 32], acc[j] = 0.0f;
    float mx = -INFINITY, den = 0.0f;
    for (unsigned s = lo; s < hi; ++s) {
        float dot = 0.0f;
#pragma unroll
        for (int j = 0; j < D / 32; ++j) dot += q[j] * p.k[size_t(s) * 512 + kh * D + lane + j * 32];
        dot = warp_sum_f(dot);
        const float next = fmaxf(mx, dot), alpha = expf(mx - next), beta = expf(dot - next);
        den = den * alpha + beta;
#pragma unroll
        for (int j = 0; j < D / 32; ++j) acc[j] = acc[j] * alpha + beta * p.v[size_t(s) * 512 + kh * D + lane + j * 32];
        mx = next;
    }
#pragma unroll
    for (int j = 0; j < D / 32; ++j) p.out[size_t(row) * D + lane + j * 32] = acc[j] / den;
}

// eg2.c:24-29 GELU form: x * (1 + tanh(u)) / 2 written as x / (1 + exp(-2u)).
__device__ __forceinline__ float abi_gelu(float x) {
    const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
    return x / (1.0f + expf(-2.0f * u));
}
__global__ void abi_element_kernel(EgElement p) {
    const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= p.n) return;
    if (p.mode == 0) p.out[i] = __fmul_rn(__fadd_rn(p.x[i], p.other[i]), p.scale);
    else if (p.mode == 1) p.out[i] = abi_gelu(p.x[i]) * p.other[i];
    else p.out[i] = abi_gelu(p.x[i]) * p.other[(size_t(i / 512) * 24 + p.layer) * 512 + i % 512];
}

__global__ void abi_pool_kernel(EgPool p) {
    const unsigned i = blockIdx.x * blockDim.x + threadIdx.x, seq = i / 768, z = i % 768;
    if (seq >= p.batch) return;
    const unsigned lo = p.offsets[seq], hi = p.offsets[seq + 1];
    float sum = 0.0f;
    for (unsigned t = lo; t < hi; ++t) sum += p.x[size_t(t) * 768 + z];
    p.out[i] = sum / float(hi - lo);
}

// eg2.c:192-202: the normalised product rounds before the residual add.
__global__ void abi_norm_residual_kernel(EgNormResidual p) {
    const unsigned row = blockIdx.x, lane = threadIdx.x;
    float ss = 0.0f;
    for (unsigned z = lane; z < p.d; z += 32) {
        const float x = p.x[size_t(row) * p.d + z];
        ss = __fmaf_rn(x, x, ss);
    }
    const float inv = rsqrtf(warp_sum_f(ss) / float(p.d) + 1.0e-6f);
    for (unsigned z = lane; z < p.d; z += 32) {
        const size_t i = size_t(row) * p.d + z;
        p.out[i] = __fmul_rn(__fadd_rn(p.out[i], __fmul_rn(__fmul_rn(p.x[i], inv), p.weight[z])), p.scale);
    }
}

// eg2.c:204-217.
__global__ void abi_norm_rope_kernel(EgNormRope p) {
    const unsigned row = blockIdx.x, lane = threadIdx.x, half = p.d / 2;
    float ss = 0.0f;
    for (unsigned z = lane; z < p.d; z += 32) {
        const float x = p.x[size_t(row) * p.d + z];
        ss = __fmaf_rn(x, x, ss);
    }
    const float inv = rsqrtf(warp_sum_f(ss) / float(p.d) + 1.0e-6f);
    __syncwarp();
    for (unsigned z = lane; z < half; z += 32) {
        const float a = __fmul_rn(__fmul_rn(p.x[size_t(row) * p.d + z], inv), p.weight[z]);
        const float b = __fmul_rn(__fmul_rn(p.x[size_t(row) * p.d + half + z], inv), p.weight[half + z]);
        const unsigned t = row / p.heads;
        const float c = p.table[size_t(t) * p.d + z], s = p.table[size_t(t) * p.d + half + z];
        p.x[size_t(row) * p.d + z] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        p.x[size_t(row) * p.d + half + z] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    }
}

}  // namespace eg2
