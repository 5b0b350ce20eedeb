// Bandwidth-bound row kernels of the executor.  Each follows the reference's
// CPU graph operation by operation (vendor/embeddinggemma.c/src/gemma2_fast.c)
// with IEEE-rounded intrinsics and no contraction, so that on identical inputs
// the Q8 codes and scales they emit are the reference's.  One warp owns one
// row; every 32-element Q8_0 block is one coalesced 128-byte access with one
// lane per element, and block amax / row sums are warp shuffles.
#pragma once
#include "common.cuh"

namespace eg2 {

// x[t] = (d * q) * sqrt(512) from the GGUF Q8_0 row (gemma2_fast.c:942-950),
// plus the bf16 hi/lo split of x for the PLE tensor-core GEMM.
__global__ void embed_kernel(float *__restrict__ x, __nv_bfloat16 *__restrict__ x_hi,
                             __nv_bfloat16 *__restrict__ x_lo, const uint8_t *__restrict__ emb,
                             const int *__restrict__ ids, int n) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= n) return;
    const uint8_t *row = emb + size_t(ids[t]) * 16 * 34;
#pragma unroll 4
    for (int b = 0; b < 16; ++b) {
        const uint16_t db = uint16_t(row[b * 34]) | uint16_t(row[b * 34 + 1]) << 8;
        const float d = fp16_bits_to_f32(db);
        const float q = float(int8_t(row[b * 34 + 2 + lane]));
        const float v = __fmul_rn(__fmul_rn(d, q), 22.627416997969522f);
        const size_t i = size_t(t) * 512 + b * 32 + lane;
        x[i] = v;
        if (x_hi) {
            const __nv_bfloat16 hi = __float2bfloat16_rn(v);
            x_hi[i] = hi;
            x_lo[i] = __float2bfloat16_rn(__fsub_rn(v, __bfloat162float(hi)));
        }
    }
}

// ROW_NORM_QUANT / ROW_QUANT (gemma2_fast.c:685-691,728-730): optional RMS norm
// with weight w, then Q8_0 quantization of the row, 32 lanes per block.
template <int WIDTH>
__global__ void norm_quant_kernel(int8_t *__restrict__ q, float *__restrict__ qs, int qs_stride,
                                  float *__restrict__ y, const float *__restrict__ x, const float *__restrict__ w,
                                  int rows) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= rows) return;
    constexpr int NB = WIDTH / 32;
    const float *xr = x + size_t(t) * WIDTH;
    float v[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) v[b] = xr[b * 32 + lane];
    if (w) {
        double ss = 0.0;
#pragma unroll
        for (int b = 0; b < NB; ++b) ss = __dadd_rn(ss, __dmul_rn(double(v[b]), double(v[b])));
        const float sc = rms_scale(warp_sum_d(ss), WIDTH);
#pragma unroll
        for (int b = 0; b < NB; ++b) v[b] = __fmul_rn(v[b], __fmul_rn(sc, w[b * 32 + lane]));
        if (y) {
#pragma unroll
            for (int b = 0; b < NB; ++b) y[size_t(t) * WIDTH + b * 32 + lane] = v[b];
        }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        float s;
        const int8_t c = quant_lane32(v[b], &s);
        q[size_t(t) * WIDTH + b * 32 + lane] = c;
        if (lane == 0) qs[size_t(b) * qs_stride + t] = s;
    }
}

// ROW_QKV_POST (gemma2_fast.c:692-706): warp per (token, head row).  Rows
// 0..3 are q heads (weighted RMS + RoPE), then kv k heads (weighted RMS +
// RoPE), then kv v heads (plain RMS).  RoPE: r[z] = a*c - b*s,
// r[z+d/2] = a*s + b*c with host tables (gemma2_fast.c:672-679).
template <int D>
__global__ void qkv_post_kernel(__half *__restrict__ qo, __half *__restrict__ ko, __half *__restrict__ vo,
                                const float *__restrict__ qkv, const float *__restrict__ qn,
                                const float *__restrict__ kn, const float *__restrict__ rc,
                                const float *__restrict__ rs, const unsigned *__restrict__ pos, int n) {
    constexpr int KV = 512 / D, HR = 4 + 2 * KV, PER = D / 64;  // PER pairs per lane
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (gw >= n * HR) return;
    const int t = gw / HR, hr = gw % HR;
    const float *src;
    const float *w;
    __half *dst;
    bool rope = true;
    if (hr < 4) {
        src = qkv + size_t(t) * (4 * D + 1024) + hr * D, w = qn, dst = qo + (size_t(t) * 4 + hr) * D;
    } else if (hr < 4 + KV) {
        const int h = hr - 4;
        src = qkv + size_t(t) * (4 * D + 1024) + 4 * D + h * D, w = kn, dst = ko + (size_t(t) * KV + h) * D;
    } else {
        const int h = hr - 4 - KV;
        src = qkv + size_t(t) * (4 * D + 1024) + 4 * D + 512 + h * D, w = nullptr;
        dst = vo + (size_t(t) * KV + h) * D, rope = false;
    }
    float a[PER], b[PER];
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        a[i] = src[i * 32 + lane];
        b[i] = src[D / 2 + i * 32 + lane];
        ss = __dadd_rn(ss, __dmul_rn(double(a[i]), double(a[i])));
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) ss = __dadd_rn(ss, __dmul_rn(double(b[i]), double(b[i])));
    const float sc = rms_scale(warp_sum_d(ss), D);
    const size_t p = size_t(pos[t]) * (D / 2);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int z = i * 32 + lane;
        const float ya = __fmul_rn(a[i], __fmul_rn(sc, w ? w[z] : 1.0f));
        const float yb = __fmul_rn(b[i], __fmul_rn(sc, w ? w[z + D / 2] : 1.0f));
        float oa = ya, ob = yb;
        if (rope) {
            const float c = rc[p + z], s = rs[p + z];
            oa = __fsub_rn(__fmul_rn(ya, c), __fmul_rn(yb, s));
            ob = __fadd_rn(__fmul_rn(ya, s), __fmul_rn(yb, c));
        }
        dst[z] = __float2half_rn(oa);
        dst[z + D / 2] = __float2half_rn(ob);
    }
}

// ROW_POST_ADD (gemma2_fast.c:707-713): x = (x + rms(h) * w) * scale, then the
// next GEMM operand from the updated x: RMS-norm with next_w and quantize
// (ROW_NORM_QUANT) or, next_w == nullptr, plain quantization (ROW_QUANT).
__global__ void post_add_kernel(float *__restrict__ x, const float *__restrict__ h, const float *__restrict__ w,
                                const float *__restrict__ scale, int8_t *__restrict__ q, float *__restrict__ qs,
                                int qs_stride, const float *__restrict__ next_w, int rows) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= rows) return;
    float hv[16], xv[16];
    double ss = 0.0;
#pragma unroll
    for (int b = 0; b < 16; ++b) {
        hv[b] = h[size_t(t) * 512 + b * 32 + lane];
        xv[b] = x[size_t(t) * 512 + b * 32 + lane];
        ss = __dadd_rn(ss, __dmul_rn(double(hv[b]), double(hv[b])));
    }
    const float sc = rms_scale(warp_sum_d(ss), 512);
    const float ls = scale ? *scale : 1.0f;
    double ss2 = 0.0;
#pragma unroll
    for (int b = 0; b < 16; ++b) {
        const float hn = __fmul_rn(hv[b], __fmul_rn(sc, w[b * 32 + lane]));
        xv[b] = __fmul_rn(__fadd_rn(xv[b], hn), ls);
        x[size_t(t) * 512 + b * 32 + lane] = xv[b];
        ss2 = __dadd_rn(ss2, __dmul_rn(double(xv[b]), double(xv[b])));
    }
    if (next_w) {
        const float sc2 = rms_scale(warp_sum_d(ss2), 512);
#pragma unroll
        for (int b = 0; b < 16; ++b) xv[b] = __fmul_rn(xv[b], __fmul_rn(sc2, next_w[b * 32 + lane]));
    }
#pragma unroll
    for (int b = 0; b < 16; ++b) {
        float s;
        const int8_t c = quant_lane32(xv[b], &s);
        q[size_t(t) * 512 + b * 32 + lane] = c;
        if (lane == 0) qs[size_t(b) * qs_stride + t] = s;
    }
}

// ROW_GELU_QUANT / ROW_PLE_GATE_QUANT (gemma2_fast.c:714-727):
// g = gelu_tanh(x) * other, then Q8_0.  Warp per (row, 8 blocks).
__global__ void gate_quant_kernel(int8_t *__restrict__ q, float *__restrict__ qs, int qs_stride,
                                  const float *__restrict__ x, const float *__restrict__ other, int rows, int width,
                                  int other_stride, int other_offset) {
    const int nb = width / 32, groups = (nb + 7) / 8;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (gw >= rows * groups) return;
    const int t = gw / groups, b0 = (gw % groups) * 8;
#pragma unroll
    for (int bb = 0; bb < 8; ++bb) {
        const int b = b0 + bb;
        if (b >= nb) break;
        const float g = __fmul_rn(ref_gelu(x[size_t(t) * width + b * 32 + lane]),
                                  other[size_t(t) * other_stride + other_offset + b * 32 + lane]);
        float s;
        const int8_t c = quant_lane32(g, &s);
        q[size_t(t) * width + b * 32 + lane] = c;
        if (lane == 0) qs[size_t(b) * qs_stride + t] = s;
    }
}

// Mean pool then L2 (gemma2_fast.c:1000-1008): o[z] += y[t][z] / len in token
// order, then the SSE2 sum of squares of kernels.c:82-93 (two 4-lane
// accumulators over 8-element chunks) and x *= 1/sqrt(ss) (kernels.c:393-396).
__global__ void pool_l2_kernel(float *__restrict__ out, const float *__restrict__ y,
                               const unsigned *__restrict__ offsets, int width) {
    extern __shared__ float pooled[];  // [width]
    __shared__ float lanes[8];
    __shared__ float inv;
    const int s = blockIdx.x;
    const unsigned lo = offsets[s], hi = offsets[s + 1];
    const float len = float(hi - lo);
    for (int z = threadIdx.x; z < width; z += blockDim.x) {
        float o = 0.0f;
        for (unsigned t = lo; t < hi; ++t) o = __fadd_rn(o, __fdiv_rn(y[size_t(t) * width + z], len));
        pooled[z] = o;
    }
    __syncthreads();
    if (threadIdx.x < 8) {
        const int j = threadIdx.x;  // lanes 0..3 -> sum0, 4..7 -> sum1
        float acc = 0.0f;
        for (int i = 0; i + 7 < width; i += 8) acc = __fadd_rn(acc, __fmul_rn(pooled[i + j], pooled[i + j]));
        lanes[j] = acc;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float v[4];
        for (int j = 0; j < 4; ++j) v[j] = __fadd_rn(lanes[j], lanes[4 + j]);
        const float ss = __fadd_rn(__fadd_rn(v[0], v[2]), __fadd_rn(v[1], v[3]));
        inv = ss != 0.0f ? __fdiv_rn(1.0f, __fsqrt_rn(ss)) : 1.0f;
    }
    __syncthreads();
    for (int z = threadIdx.x; z < width; z += blockDim.x) out[size_t(s) * width + z] = __fmul_rn(pooled[z], inv);
}

// GGUF Q8_0 blocks [rows][k/32] (34 B each) -> int8 codes [rows][k] and fp32
// scales block-major, scales[b * scale_stride + row].
__global__ void repack_q8_kernel(const uint8_t *__restrict__ blocks, int rows, int k, int8_t *__restrict__ codes,
                                 float *__restrict__ scales, int scale_stride) {
    const int kb = k / 32;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // one thread per block
    if (i >= (long long)rows * kb) return;
    const int r = int(i / kb), b = int(i % kb);
    const uint8_t *src = blocks + size_t(i) * 34;
    const uint16_t db = uint16_t(src[0]) | uint16_t(src[1]) << 8;
    scales[size_t(b) * scale_stride + r] = fp16_bits_to_f32(db);
    int8_t *dst = codes + size_t(r) * k + b * 32;
#pragma unroll
    for (int z = 0; z < 32; ++z) dst[z] = int8_t(src[2 + z]);
}

}  // namespace eg2
