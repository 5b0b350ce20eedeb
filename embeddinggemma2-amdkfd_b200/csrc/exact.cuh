// Exact-order kernels of the executor's parity mode.  The fast path runs the
// PLE projection on bf16 tensor cores (x split into hi + lo) and attention on
// fp16 tensor cores; both are accurate to ~1e-4 but sum in a different order
// than the reference, and 24 layers amplify any difference in a Q8_0 rounding
// decision.  These CUDA-core kernels follow the reference's scalar loops
// operation for operation instead (fp32, multiply then add, never contracted),
// so that in parity mode the whole wave reproduces the reference's arithmetic.
#pragma once
#include "common.cuh"
#include "ref_expf.h"

namespace eg2 {

__constant__ uint64_t c_exp2_tab[32] = {EG2_EXP2_TAB};

// ---------------------------------------------------------------- PLE
// y[t][r] = sum_z bf16(W[r][z]) * x[t][z] in ascending z
// (vendor/embeddinggemma.c/src/gemma2_fast.c:482-559 scalar branch, gemm_f).
// CTA tile 32 tokens x 128 rows, K chunks of 64 staged in shared memory; each
// thread owns 4 tokens x 4 rows and walks z in order across the chunks.
struct PleExactCfg {
    static constexpr int BT = 32, BR = 128, KC = 64, THREADS = 256;
};
__global__ void __launch_bounds__(PleExactCfg::THREADS) ple_exact_kernel(float *__restrict__ y,
                                                                         const float *__restrict__ x,
                                                                         const uint16_t *__restrict__ w, int n) {
    using C = PleExactCfg;
    pdl_wait();
    pdl_trigger();
    __shared__ float xs[C::BT][C::KC + 1];
    __shared__ float ws[C::BR][C::KC + 1];
    const int t0 = blockIdx.y * C::BT, r0 = blockIdx.x * C::BR;
    const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;  // rows r0 + tx + 32j, tokens t0 + ty + 8i
    float acc[4][4] = {};
    for (int k0 = 0; k0 < 512; k0 += C::KC) {
        __syncthreads();
        for (int i = threadIdx.x; i < C::BT * C::KC; i += C::THREADS) {
            const int tt = i / C::KC, z = i % C::KC, t = t0 + tt;
            xs[tt][z] = t < n ? x[size_t(t) * 512 + k0 + z] : 0.0f;
        }
        for (int i = threadIdx.x; i < C::BR * C::KC; i += C::THREADS) {
            const int rr = i / C::KC, z = i % C::KC;
            ws[rr][z] = __uint_as_float(uint32_t(w[size_t(r0 + rr) * 512 + k0 + z]) << 16);
        }
        __syncthreads();
        for (int z = 0; z < C::KC; ++z) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float xv = xs[ty + 8 * i][z];
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(ws[tx + 32 * j][z], xv));
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + ty + 8 * i;
        if (t < n)
#pragma unroll
            for (int j = 0; j < 4; ++j) y[size_t(t) * (24 * 512) + r0 + tx + 32 * j] = acc[i][j];
    }
}

// The same projection in the order of the reference's default tier on an
// AVX-512 VNNI host (g2x_dot4x4, gemma2_fast_x86.c:260-279, called from
// gemma2_fast.c:537-545): per output, eight lanes of fused multiply-adds, lane
// i over z = 8m + i in ascending m, then hsum8.  CTA tile 32 tokens x 64 rows;
// each thread owns 4 tokens x 2 rows (eight lanes each).
struct PleVnniCfg {
    static constexpr int BT = 32, BR = 64, KC = 64, THREADS = 256;
};
__global__ void __launch_bounds__(PleVnniCfg::THREADS) ple_vnni_kernel(float *__restrict__ y,
                                                                       const float *__restrict__ x,
                                                                       const uint16_t *__restrict__ w, int n) {
    using C = PleVnniCfg;
    pdl_wait();
    pdl_trigger();
    __shared__ float xs[C::BT][C::KC + 1];
    __shared__ float ws[C::BR][C::KC + 1];
    const int t0 = blockIdx.y * C::BT, r0 = blockIdx.x * C::BR;
    const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;  // rows r0 + tx + 32j, tokens t0 + ty + 8i
    float acc[4][2][8] = {};
    for (int k0 = 0; k0 < 512; k0 += C::KC) {
        __syncthreads();
        for (int i = threadIdx.x; i < C::BT * C::KC; i += C::THREADS) {
            const int tt = i / C::KC, z = i % C::KC, t = t0 + tt;
            xs[tt][z] = t < n ? x[size_t(t) * 512 + k0 + z] : 0.0f;
        }
        for (int i = threadIdx.x; i < C::BR * C::KC; i += C::THREADS) {
            const int rr = i / C::KC, z = i % C::KC;
            ws[rr][z] = __uint_as_float(uint32_t(w[size_t(r0 + rr) * 512 + k0 + z]) << 16);
        }
        __syncthreads();
        for (int z = 0; z < C::KC; z += 8)
#pragma unroll
            for (int l = 0; l < 8; ++l)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float xv = xs[ty + 8 * i][z + l];
#pragma unroll
                    for (int j = 0; j < 2; ++j) acc[i][j][l] = __fmaf_rn(ws[tx + 32 * j][z + l], xv, acc[i][j][l]);
                }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + ty + 8 * i;
        if (t < n)
#pragma unroll
            for (int j = 0; j < 2; ++j) y[size_t(t) * (24 * 512) + r0 + tx + 32 * j] = hsum8(acc[i][j]);
    }
}

// ple /= sqrtf(512), then rms_row with the per-slice weight
// (gemma2_fast.c:952-956, :667-671).  CTA of 128 threads per (token, slice).
// tier TIER_VNNI512: the sum of squares in g2x_sum_squares' order.
__global__ void __launch_bounds__(128) ple_norm_kernel(float *__restrict__ ple, const float *__restrict__ w, int tier) {
    pdl_wait();
    pdl_trigger();
    __shared__ double red[4];
    __shared__ __align__(16) float buf[512];
    float4 *row = reinterpret_cast<float4 *>(ple + size_t(blockIdx.x) * 512);
    const int i = threadIdx.x;
    constexpr float S512 = 22.627416997969522f;  // sqrtf(512.0f)
    float4 v = row[i];
    v = make_float4(__fdiv_rn(v.x, S512), __fdiv_rn(v.y, S512), __fdiv_rn(v.z, S512), __fdiv_rn(v.w, S512));
    double ss = __dadd_rn(__dadd_rn(__dmul_rn(double(v.x), double(v.x)), __dmul_rn(double(v.y), double(v.y))),
                          __dadd_rn(__dmul_rn(double(v.z), double(v.z)), __dmul_rn(double(v.w), double(v.w))));
    if (tier == TIER_VNNI512) {
        reinterpret_cast<float4 *>(buf)[i] = v;
        __syncthreads();
        if (i < 32) {
            const float s = x86_sumsq_warp(buf, 512);
            if (i == 0) red[0] = double(s), red[1] = red[2] = red[3] = 0.0;
        }
    } else {
        ss = warp_sum_d(ss);
        if ((i & 31) == 0) red[i >> 5] = ss;
    }
    __syncthreads();
    const float sc = rms_scale(__dadd_rn(__dadd_rn(red[0], red[1]), __dadd_rn(red[2], red[3])), 512);
    const float4 wv = reinterpret_cast<const float4 *>(w)[i];
    row[i] = make_float4(__fmul_rn(v.x, __fmul_rn(sc, wv.x)), __fmul_rn(v.y, __fmul_rn(sc, wv.y)),
                         __fmul_rn(v.z, __fmul_rn(sc, wv.z)), __fmul_rn(v.w, __fmul_rn(sc, wv.w)));
}

// ---------------------------------------------------------------- attention
// The reference's scalar attention (gemma2_fast.c:768-894) for one (token,
// head) per CTA: keys s in [lo, hi) of the token's sequence, intersected with
// [t - window, t + window] when window != 0; kv head h / (4 / kv).
//   sc[s] = sum_z q[z] * k[s][z]      (ascending z, one thread per key)
//   mx = max sc;  sc[s] = exp(sc[s] - mx);  total = sum sc (ascending s)
//   sc[s] /= total;  o[z] = sum_s sc[s] * v[s][z]   (ascending s)
// exp is the C library's expf algorithm with its exact rounding (ref_expf.h).
// q, k, v are fp32 here.
// VNNI: the order of the reference's default tier on an AVX-512 VNNI host:
// scores by g2x_dot4x4 (eight lanes of fused multiply-adds over z, then
// hsum8; gemma2_fast.c:826-828) and o[z] by g2x_pv (one fused multiply-add per
// key in ascending order; gemma2_fast_x86.c:326-349); the softmax is the same.
template <int D, bool VNNI>
__global__ void __launch_bounds__(128) attention_exact_kernel(float *__restrict__ out, const float *__restrict__ q,
                                                              const float *__restrict__ k, const float *__restrict__ v,
                                                              const unsigned *__restrict__ bounds, int n, int window) {
    constexpr int KV = 512 / D, MAXK = 2048;
    pdl_wait();
    pdl_trigger();
    __shared__ float qs[D];
    __shared__ float sc[MAXK];
    __shared__ float red[4];
    const int t = blockIdx.x, h = blockIdx.y, kh = h / (4 / KV), i = threadIdx.x;
    int lo = int(bounds[2 * t]), hi = int(bounds[2 * t + 1]);
    if (window) {
        if (t - window > lo) lo = t - window;
        if (t + window + 1 < hi) hi = t + window + 1;
    }
    const int nk = hi - lo;  // <= 2048 packed tokens per wave
    for (int z = i; z < D; z += 128) qs[z] = q[(size_t(t) * 4 + h) * D + z];
    __syncthreads();
    float mx = -INFINITY;
    for (int s = i; s < nk; s += 128) {
        const float *kr = k + (size_t(lo + s) * KV + kh) * D;
        float dot = 0.0f;
        if constexpr (VNNI) {
            float acc[8] = {};
            for (int z = 0; z < D; z += 8)
#pragma unroll
                for (int l = 0; l < 8; ++l) acc[l] = __fmaf_rn(qs[z + l], kr[z + l], acc[l]);
            dot = hsum8(acc);
        } else {
            for (int z = 0; z < D; ++z) dot = __fadd_rn(dot, __fmul_rn(qs[z], kr[z]));
        }
        sc[s] = dot;
        mx = fmaxf(mx, dot);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    if ((i & 31) == 0) red[i >> 5] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    for (int s = i; s < nk; s += 128) sc[s] = eg2_ref_expf(__fsub_rn(sc[s], mx), c_exp2_tab);
    __syncthreads();
    if (i == 0) {
        float total = 0.0f;
        for (int s = 0; s < nk; ++s) total = __fadd_rn(total, sc[s]);
        red[0] = total;
    }
    __syncthreads();
    const float total = red[0];
    for (int s = i; s < nk; s += 128) sc[s] = __fdiv_rn(sc[s], total);
    __syncthreads();
    for (int z = i; z < D; z += 128) {
        const float *vc = v + size_t(lo) * KV * D + kh * D + z;
        float acc = 0.0f;
        for (int s = 0; s < nk; ++s)
            acc = VNNI ? __fmaf_rn(vc[size_t(s) * KV * D], sc[s], acc)
                       : __fadd_rn(acc, __fmul_rn(sc[s], vc[size_t(s) * KV * D]));
        out[(size_t(t) * 4 + h) * D + z] = acc;
    }
}

}  // namespace eg2
