// Parity mode at TIER_VNNI512: the Q8_0 GEMM in the float order of the
// reference CPU graph's default tier on an AVX-512 VNNI host, so that a wave
// reproduces that tier bit for bit.
//
// gemm_q8 (vendor/embeddinggemma.c/src/gemma2_fast.c:446-465) takes one of two
// x86 paths by the wave's token count n:
//   n > 8:  g2x_gemm512_tile (gemma2_fast_x86.c:168-204) -- per output 16 fp32
//           lanes; for each pair of blocks (p, p + 1) lane g < 8 gets the int32
//           sum over bytes 4g..4g+3 of block p of (x + 128) * w (vpdpbusd on
//           u8 activations), lane 8 + g the same for block p + 1, and lanes 0
//           and 8 are seeded with -128 * sum(w) of their block (:146-158), which
//           removes the bias; each lane adds float(sum) * (sw * sx) with one
//           fused multiply-add; then _mm512_reduce_add_ps;
//   n <= 8: q8_tile_vnni512 (gemma2_fast_x86.c:66-103) -- 8 lanes, lane g the
//           int32 sum of w * x over bytes 4g..4g+3 of each block, fused into the
//           lane with the scale product (dw * dx), then the 8-lane hsum.
// Every int32 lane sum is below 2^22, so its float conversion is exact, and
// the per-output order does not depend on how outputs are grouped into tasks.
//
// CUDA cores: a CTA owns 32 weight rows x 8 tokens, one output per thread; K
// is staged 256 bytes (8 blocks) at a time in shared memory, weight rows padded
// to 65 words so that the 32 rows of a warp sit in 32 banks.  The path is
// chosen on the device from the wave's real token count (offsets[*count]), as
// the graph is captured for a padded bucket.
#pragma once
#include "common.cuh"

namespace eg2 {

struct Q8VnniCfg {
    static constexpr int BR = 32, BT = 8, KC = 256, THREADS = 256;
    static constexpr int WW = KC / 4 + 1;  // words per staged weight row
};

__device__ __forceinline__ int dp4a_s8s8(int a, int b, int c) { return __dp4a(a, b, c); }
// sum of u8(a_i) * s8(b_i) + c (the unsigned-by-signed form of vpdpbusd).
__device__ __forceinline__ int dp4a_u8s8(unsigned a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// out[t][col] for weight row r of the interleaved GeGLU weight (out_up set:
// rows 128c..128c+63 are gate columns 64c.., the next 64 up columns) or
// out[t][r] (out_up NULL).
__global__ void __launch_bounds__(Q8VnniCfg::THREADS) q8gemm_vnni_kernel(
    float *__restrict__ out, float *__restrict__ out_up, int ldo, const int8_t *__restrict__ wq,
    const float *__restrict__ wsc, const int8_t *__restrict__ xq, const float *__restrict__ xsc, int xs_stride, int T,
    int R, int K, const unsigned *__restrict__ offsets, const unsigned *__restrict__ count) {
    using C = Q8VnniCfg;
    pdl_wait();
    pdl_trigger();
    __shared__ int w_s[C::BR][C::WW];
    __shared__ int x_s[C::BT][C::KC / 4];
    __shared__ float sw_s[C::KC / 32][C::BR];
    __shared__ float sx_s[C::KC / 32][C::BT];
    __shared__ int corr_s[C::KC / 32][C::BR];
    const int r0 = blockIdx.x * C::BR, t0 = blockIdx.y * C::BT;
    const int tid = threadIdx.x, rl = tid & 31, tl = tid >> 5;
    const int n_real = offsets && count ? int(offsets[*count]) : T;
    const bool wide = n_real > 8;
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
    for (int k0 = 0; k0 < K; k0 += C::KC) {
        __syncthreads();  // the previous chunk has been consumed
        for (int i = tid; i < C::BR * C::KC / 4; i += C::THREADS) {
            const int rr = i / (C::KC / 4), c = i % (C::KC / 4);
            w_s[rr][c] = reinterpret_cast<const int *>(wq + size_t(r0 + rr) * K + k0)[c];
        }
        for (int i = tid; i < C::BT * C::KC / 4; i += C::THREADS) {
            const int tt = i / (C::KC / 4), c = i % (C::KC / 4);
            x_s[tt][c] = t0 + tt < T ? reinterpret_cast<const int *>(xq + size_t(t0 + tt) * K + k0)[c] : 0;
        }
        {
            const int b = tid / C::BR, rr = tid % C::BR;  // KC / 32 x BR = THREADS
            sw_s[b][rr] = wsc[size_t(k0 / 32 + b) * R + r0 + rr];
        }
        if (tid < C::KC / 32 * C::BT) {
            const int b = tid / C::BT, tt = tid % C::BT;
            sx_s[b][tt] = t0 + tt < T ? xsc[size_t(k0 / 32 + b) * xs_stride + t0 + tt] : 0.0f;
        }
        __syncthreads();
        {
            const int b = tid / C::BR, rr = tid % C::BR;
            int sum = 0;
#pragma unroll
            for (int g = 0; g < 8; ++g) sum = dp4a_s8s8(0x01010101, w_s[rr][b * 8 + g], sum);
            corr_s[b][rr] = -128 * sum;
        }
        __syncthreads();
        const int *wr = w_s[rl], *xr = x_s[tl];
        if (wide) {
#pragma unroll 1
            for (int b = 0; b < C::KC / 32; b += 2)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float sc = __fmul_rn(sw_s[b + h][rl], sx_s[b + h][tl]);
#pragma unroll
                    for (int g = 0; g < 8; ++g) {
                        const int L = dp4a_u8s8(unsigned(xr[(b + h) * 8 + g]) ^ 0x80808080u, wr[(b + h) * 8 + g],
                                                g == 0 ? corr_s[b + h][rl] : 0);
                        acc[h * 8 + g] = __fmaf_rn(__int2float_rn(L), sc, acc[h * 8 + g]);
                    }
                }
        } else {
#pragma unroll 1
            for (int b = 0; b < C::KC / 32; ++b) {
                const float sc = __fmul_rn(sw_s[b][rl], sx_s[b][tl]);
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                    const int L = dp4a_s8s8(xr[b * 8 + g], wr[b * 8 + g], 0);
                    acc[g] = __fmaf_rn(__int2float_rn(L), sc, acc[g]);
                }
            }
        }
    }
    const int t = t0 + tl, r = r0 + rl;
    if (t >= T) return;
    float y;
    if (wide) {
        y = reduce16(acc);
    } else {
        float a8[8];
#pragma unroll
        for (int g = 0; g < 8; ++g) a8[g] = acc[g];
        y = hsum8(a8);
    }
    if (out_up) {
        const int c = r / 128, within = r % 128;
        (within < 64 ? out : out_up)[size_t(t) * ldo + 64 * c + (within & 63)] = y;
    } else {
        out[size_t(t) * ldo + r] = y;
    }
}

}  // namespace eg2
