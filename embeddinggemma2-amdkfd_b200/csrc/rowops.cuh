// Bandwidth-bound row kernels of the executor.  Each follows the reference's
// CPU graph operation by operation (vendor/embeddinggemma.c/src/gemma2_fast.c)
// with IEEE-rounded intrinsics and no contraction, so that on identical inputs
// the Q8 codes and scales they emit are the reference's.  Row sums of squares
// are accumulated in double like the reference's and reduced with warp
// shuffles.
#pragma once
#include "common.cuh"

namespace eg2 {

// x[t] = (d * q) * sqrt(512) from the GGUF Q8_0 row (gemma2_fast.c:942-950),
// plus the bf16 hi/lo split of x for the PLE tensor-core GEMM.
__global__ void embed_kernel(float *__restrict__ x, __nv_bfloat16 *__restrict__ x_hi,
                             __nv_bfloat16 *__restrict__ x_lo, const uint8_t *__restrict__ emb,
                             const int *__restrict__ ids, int n) {
    pdl_wait();
    pdl_trigger();
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

// Media soft-token waves (gemma2_fast.c:940-941): x = the caller's 512-wide rows
// as given (uploaded by the host into `rows`, which the wave never writes, so a
// staged wave replays identically), plus the bf16 hi/lo split of x for the PLE
// tensor-core GEMM with embed_kernel's arithmetic.
__global__ void input_rows_kernel(float *__restrict__ x, __nv_bfloat16 *__restrict__ x_hi,
                                  __nv_bfloat16 *__restrict__ x_lo, const float *__restrict__ rows, int n) {
    pdl_wait();
    pdl_trigger();
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= size_t(n) * 512) return;
    const float v = rows[i];
    x[i] = v;
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    x_hi[i] = hi;
    x_lo[i] = __float2bfloat16_rn(__fsub_rn(v, __bfloat162float(hi)));
}

// Layout of the quantizing kernels: a warp reads a row 512 bytes at a time,
// each lane 4 consecutive floats (one float4), so one warp-wide access covers
// four Q8_0 blocks and each block lives in an aligned group of 8 lanes.  The
// block's amax is 3 shuffles inside the group, and each lane stores its four
// codes as one 32-bit word.

// One 32-element block held as v in each lane of an aligned 8-lane group
// (gemma2_fast_x86.c:211-234): d = amax/127 (IEEE rounding), the scale stored is the
// reference's fp16 rounding of d, id = 1/d.  Returns the lane's four codes;
// *scale_out receives the widened fp16 scale (uniform over the group).
__device__ __forceinline__ uint32_t quant_oct(const float4 v, float *scale_out, int tier) {
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = div127(amax);
    const float id = d != 0.0f ? rcp_rn(d) : 0.0f;
    *scale_out = fp16_bits_to_f32(ref_fp32_to_fp16(d));
    return q8_code(v.x, id, tier) | q8_code(v.y, id, tier) << 8 | q8_code(v.z, id, tier) << 16 |
           q8_code(v.w, id, tier) << 24;
}
__device__ __forceinline__ double sumsq4(double ss, const float4 v) {
    ss = __dadd_rn(ss, __dmul_rn(double(v.x), double(v.x)));
    ss = __dadd_rn(ss, __dmul_rn(double(v.y), double(v.y)));
    ss = __dadd_rn(ss, __dmul_rn(double(v.z), double(v.z)));
    return __dadd_rn(ss, __dmul_rn(double(v.w), double(v.w)));
}
// v * (sc * w), elementwise, in the reference's order (rms_row: r[z] *= scale * w[z]).
__device__ __forceinline__ float4 scale_w4(const float4 v, float sc, const float4 w) {
    return make_float4(__fmul_rn(v.x, __fmul_rn(sc, w.x)), __fmul_rn(v.y, __fmul_rn(sc, w.y)),
                       __fmul_rn(v.z, __fmul_rn(sc, w.z)), __fmul_rn(v.w, __fmul_rn(sc, w.w)));
}
// Sum of a per-thread double over the CTA: warp shuffles, then the per-warp
// partials added in warp order by every thread.  red holds WARPS doubles.
template <int WARPS>
__device__ __forceinline__ double cta_sum_d(double v, double *red) {
    v = warp_sum_d(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    double s = red[0];
#pragma unroll
    for (int i = 1; i < WARPS; ++i) s = __dadd_rn(s, red[i]);
    return s;
}

// The row sum of squares of a CTA whose threads hold one float4 each (thread
// i: elements 4i..4i+3 of a WIDTH-wide row), as the reference computes it:
// for TIER_VNNI512 in g2x_sum_squares' float order (the row staged in buf,
// then one warp), otherwise in double like the scalar loop.  Returned as a
// double (exact for the float sum).
template <int WIDTH>
__device__ __forceinline__ double cta_row_sumsq(const float4 v, int tier, double *red, float *buf) {
    if (tier != TIER_VNNI512) return cta_sum_d<WIDTH / 128>(sumsq4(0.0, v), red);
    reinterpret_cast<float4 *>(buf)[threadIdx.x] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        const float ss = x86_sumsq_warp(buf, WIDTH);
        if (threadIdx.x == 0) red[0] = double(ss);
    }
    __syncthreads();
    const double ss = red[0];
    __syncthreads();  // buf and red may be reused by a second sum
    return ss;
}
// ROW_NORM_QUANT (gemma2_fast.c:685-691): RMS norm with weight w, then Q8_0.
// CTA per row, one float4 per thread (WIDTH / 4 threads).
template <int WIDTH>
__global__ void __launch_bounds__(WIDTH / 4) norm_quant_kernel(int8_t *__restrict__ q, float *__restrict__ qs,
                                                               int qs_stride, float *__restrict__ y,
                                                               const float *__restrict__ x,
                                                               const float *__restrict__ w, int tier) {
    pdl_wait();
    pdl_trigger();
    constexpr int WARPS = WIDTH / 128;
    __shared__ double red[WARPS];
    __shared__ __align__(16) float buf[WIDTH];
    const int t = blockIdx.x, i = threadIdx.x, lane = i & 31;
    float4 v = reinterpret_cast<const float4 *>(x + size_t(t) * WIDTH)[i];
    const float sc = rms_scale(cta_row_sumsq<WIDTH>(v, tier, red, buf), WIDTH);
    v = scale_w4(v, sc, reinterpret_cast<const float4 *>(w)[i]);
    if (y) reinterpret_cast<float4 *>(y + size_t(t) * WIDTH)[i] = v;
    float s;
    reinterpret_cast<uint32_t *>(q + size_t(t) * WIDTH)[i] = quant_oct(v, &s, tier);
    if ((lane & 7) == 0) qs[size_t(i >> 3) * qs_stride + t] = s;
}

// ROW_QUANT (gemma2_fast.c:728-730): Q8_0 of rows of width `width` (a multiple
// of 128).  Warp per (row, four blocks).
__global__ void quant_rows_kernel(int8_t *__restrict__ q, float *__restrict__ qs, int qs_stride,
                                  const float *__restrict__ x, int rows, int width, int tier) {
    pdl_wait();
    pdl_trigger();
    const int steps = width / 128;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (gw >= rows * steps) return;  // warp-uniform
    const int t = gw / steps, st = gw % steps;
    const size_t c = size_t(t) * (width / 4) + st * 32 + lane;
    float s;
    reinterpret_cast<uint32_t *>(q)[c] = quant_oct(reinterpret_cast<const float4 *>(x)[c], &s, tier);
    if ((lane & 7) == 0) qs[size_t(4 * st + (lane >> 3)) * qs_stride + t] = s;
}

// ROW_QKV_POST (gemma2_fast.c:692-706): warp per (token, head row).  Rows
// 0..3 are q heads (weighted RMS + RoPE), then kv k heads (weighted RMS +
// RoPE), then kv v heads (plain RMS).  RoPE: r[z] = a*c - b*s,
// r[z+d/2] = a*s + b*c with host tables (gemma2_fast.c:672-679).  Each lane
// handles 4 consecutive z of each half.
// OutT is __half (the fast path's attention operands) or float (parity mode).
template <int D, typename OutT>
__global__ void qkv_post_kernel(OutT *__restrict__ qo, OutT *__restrict__ ko, OutT *__restrict__ vo,
                                const float *__restrict__ qkv, const float *__restrict__ qn,
                                const float *__restrict__ kn, const float *__restrict__ rc,
                                const float *__restrict__ rs, const unsigned *__restrict__ pos, int n, int tier) {
    pdl_wait();
    pdl_trigger();
    constexpr int KV = 512 / D, HR = 4 + 2 * KV, PER = D / 256;  // float4 chunks per lane per half
    __shared__ __align__(16) float rowbuf[8][D];  // TIER_VNNI512: the warp's row, for the x86 sum order
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (gw >= n * HR) return;
    const int t = gw / HR, hr = gw % HR;
    const float *src;
    const float *w;
    OutT *dst;
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
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    float4 a[PER], b[PER];
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        a[i] = s4[i * 32 + lane];
        b[i] = s4[D / 8 + i * 32 + lane];
        ss = sumsq4(ss, a[i]);
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) ss = sumsq4(ss, b[i]);
    if (tier == TIER_VNNI512) {
        float4 *rb = reinterpret_cast<float4 *>(rowbuf[(threadIdx.x >> 5) & 7]);
#pragma unroll
        for (int i = 0; i < PER; ++i) rb[i * 32 + lane] = a[i], rb[D / 8 + i * 32 + lane] = b[i];
        __syncwarp();
        ss = double(x86_sumsq_warp(rowbuf[(threadIdx.x >> 5) & 7], D));
        __syncwarp();
    } else {
        ss = warp_sum_d(ss);
    }
    const float sc = rms_scale(ss, D);
    const size_t p = size_t(pos[t]) * (D / 2);
    const float4 one = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int z = 4 * (i * 32 + lane);
        const float4 ya = scale_w4(a[i], sc, w ? *reinterpret_cast<const float4 *>(w + z) : one);
        const float4 yb = scale_w4(b[i], sc, w ? *reinterpret_cast<const float4 *>(w + z + D / 2) : one);
        float4 oa = ya, ob = yb;
        if (rope) {
            const float4 c = *reinterpret_cast<const float4 *>(rc + p + z);
            const float4 s = *reinterpret_cast<const float4 *>(rs + p + z);
            oa = make_float4(__fsub_rn(__fmul_rn(ya.x, c.x), __fmul_rn(yb.x, s.x)),
                             __fsub_rn(__fmul_rn(ya.y, c.y), __fmul_rn(yb.y, s.y)),
                             __fsub_rn(__fmul_rn(ya.z, c.z), __fmul_rn(yb.z, s.z)),
                             __fsub_rn(__fmul_rn(ya.w, c.w), __fmul_rn(yb.w, s.w)));
            ob = make_float4(__fadd_rn(__fmul_rn(ya.x, s.x), __fmul_rn(yb.x, c.x)),
                             __fadd_rn(__fmul_rn(ya.y, s.y), __fmul_rn(yb.y, c.y)),
                             __fadd_rn(__fmul_rn(ya.z, s.z), __fmul_rn(yb.z, c.z)),
                             __fadd_rn(__fmul_rn(ya.w, s.w), __fmul_rn(yb.w, c.w)));
        }
        if constexpr (sizeof(OutT) == 4) {
            *reinterpret_cast<float4 *>(dst + z) = oa;
            *reinterpret_cast<float4 *>(dst + z + D / 2) = ob;
        } else {
            __half2 h0 = __floats2half2_rn(oa.x, oa.y), h1 = __floats2half2_rn(oa.z, oa.w);
            __half2 h2 = __floats2half2_rn(ob.x, ob.y), h3 = __floats2half2_rn(ob.z, ob.w);
            *reinterpret_cast<uint2 *>(dst + z) =
                make_uint2(*reinterpret_cast<uint32_t *>(&h0), *reinterpret_cast<uint32_t *>(&h1));
            *reinterpret_cast<uint2 *>(dst + z + D / 2) =
                make_uint2(*reinterpret_cast<uint32_t *>(&h2), *reinterpret_cast<uint32_t *>(&h3));
        }
    }
}

// ROW_POST_ADD (gemma2_fast.c:707-713): x = (x + rms(h) * w) * scale, then the
// next GEMM operand from the updated x: RMS-norm with next_w and quantize
// (ROW_NORM_QUANT) or, next_w == nullptr, plain quantization (ROW_QUANT).
// CTA of 128 threads per 512-wide row, one float4 per thread.
__global__ void __launch_bounds__(128) post_add_kernel(float *__restrict__ x, const float *__restrict__ h,
                                                       const float *__restrict__ w, const float *__restrict__ scale,
                                                       int8_t *__restrict__ q, float *__restrict__ qs, int qs_stride,
                                                       const float *__restrict__ next_w, int tier) {
    pdl_wait();
    pdl_trigger();
    __shared__ double red[2][4];
    __shared__ __align__(16) float buf[512];
    const int t = blockIdx.x, i = threadIdx.x, lane = i & 31;
    float4 *xp = reinterpret_cast<float4 *>(x + size_t(t) * 512) + i;
    const float4 hv = reinterpret_cast<const float4 *>(h + size_t(t) * 512)[i];
    float4 xv = *xp;
    const float sc = rms_scale(cta_row_sumsq<512>(hv, tier, red[0], buf), 512);
    const float ls = scale ? *scale : 1.0f;
    const float4 hn = scale_w4(hv, sc, reinterpret_cast<const float4 *>(w)[i]);
    xv = make_float4(__fmul_rn(__fadd_rn(xv.x, hn.x), ls), __fmul_rn(__fadd_rn(xv.y, hn.y), ls),
                     __fmul_rn(__fadd_rn(xv.z, hn.z), ls), __fmul_rn(__fadd_rn(xv.w, hn.w), ls));
    *xp = xv;
    if (next_w) {
        const float sc2 = rms_scale(cta_row_sumsq<512>(xv, tier, red[1], buf), 512);
        xv = scale_w4(xv, sc2, reinterpret_cast<const float4 *>(next_w)[i]);
    }
    float s;
    reinterpret_cast<uint32_t *>(q + size_t(t) * 512)[i] = quant_oct(xv, &s, tier);
    if ((lane & 7) == 0) qs[size_t(i >> 3) * qs_stride + t] = s;
}

// ROW_GELU_QUANT / ROW_PLE_GATE_QUANT (gemma2_fast.c:714-727):
// g = gelu_tanh(x) * other, then Q8_0.  Warp per (row, four blocks); width,
// other_stride and other_offset are multiples of 128, 4 and 4.  TIER selects
// the GELU and rounding at compile time (no branch per element).
template <int TIER>
__global__ void gate_quant_kernel(int8_t *__restrict__ q, float *__restrict__ qs, int qs_stride,
                                  const float *__restrict__ x, const float *__restrict__ other, int rows, int width,
                                  int other_stride, int other_offset) {
    constexpr int tier = TIER;
    pdl_wait();
    pdl_trigger();
    constexpr int PER = 1;  // float4 steps (4 blocks each) per warp
    const int steps = width / 128, wpr = (steps + PER - 1) / PER;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (gw >= rows * wpr) return;  // warp-uniform
    const int t = gw / wpr, i0 = (gw % wpr) * PER;
    const float4 *xr = reinterpret_cast<const float4 *>(x + size_t(t) * width);
    const float4 *orow = reinterpret_cast<const float4 *>(other + size_t(t) * other_stride + other_offset);
    uint32_t *qr = reinterpret_cast<uint32_t *>(q + size_t(t) * width);
    float4 xv[PER], ov[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i)
        if (i0 + i < steps) xv[i] = xr[(i0 + i) * 32 + lane], ov[i] = orow[(i0 + i) * 32 + lane];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        if (i0 + i >= steps) break;  // warp-uniform
        const float4 g = make_float4(__fmul_rn(gelu_tier(xv[i].x, tier), ov[i].x),
                                     __fmul_rn(gelu_tier(xv[i].y, tier), ov[i].y),
                                     __fmul_rn(gelu_tier(xv[i].z, tier), ov[i].z),
                                     __fmul_rn(gelu_tier(xv[i].w, tier), ov[i].w));
        float sc;
        qr[(i0 + i) * 32 + lane] = quant_oct(g, &sc, tier);
        if ((lane & 7) == 0) qs[size_t(4 * (i0 + i) + (lane >> 3)) * qs_stride + t] = sc;
    }
}

// g[z] = gelu_tanh(g[z]) * (u ? u[z] : 1) for z < n: the reference's GELU rows
// (x86 tiers: g2x_gelu_mul_row, gemma2_fast_x86.c:308-319, whose vector form the
// host restricts to whole 8-element groups; scalar tier: ei_gelu_mul_inplace
// with tanhf, kernels.c:367-371).  Grid-stride over elements.
template <int TIER>
__global__ void gelu_mul_kernel(float *__restrict__ g, const float *__restrict__ u, size_t n) {
    pdl_wait();
    pdl_trigger();
    for (size_t z = size_t(blockIdx.x) * blockDim.x + threadIdx.x; z < n; z += size_t(gridDim.x) * blockDim.x) {
        const float gl = gelu_tier(g[z], TIER);
        g[z] = u ? __fmul_rn(gl, u[z]) : gl;
    }
}

// Mean pool then L2 (gemma2_fast.c:1000-1008), in two launches.
// pool_mean_kernel: o[z] = sum over the sequence's tokens, in token order, of
// y[t][z] / len.  The adds are one serial chain per column in the reference's
// order, so a CTA owns a (32-column chunk, sequence) item: its 256 threads
// load POOL_T tokens x 32 columns (eight float4 each, all in flight at once),
// form the quotients and stage them in shared memory, and warp 0 adds them
// in token order while the next POOL_T tokens are being loaded.  The grid is
// bounded (at most POOL_SEQ CTAs per chunk) and strides over the sequences;
// with count set, sequences from *count on (beyond the wave's batch) are
// skipped.  The result goes straight into out.
constexpr int POOL_T = 256, POOL_SEQ = 64;
__global__ void __launch_bounds__(256) pool_mean_kernel(float *__restrict__ out, const float *__restrict__ y,
                                                        const unsigned *__restrict__ offsets, int width, int batch,
                                                        const unsigned *__restrict__ count) {
    pdl_wait();
    pdl_trigger();
    __shared__ float4 stage[POOL_T][8];  // [token][column / 4] of the chunk
    const int c0 = blockIdx.x * 32, tid = threadIdx.x, j = tid & 7, lane = tid & 31;
    const int nseq = count ? min(int(*count), batch) : batch;
    const bool col_ok = c0 + 4 * j < width;  // width is a multiple of 8
    for (int s = blockIdx.y; s < nseq; s += gridDim.y) {
        const unsigned lo = offsets[s], hi = offsets[s + 1];
        const float len = float(hi - lo);
        float o = 0.0f;
        float4 v[POOL_T / 32];
        auto load = [&](unsigned t0) {
#pragma unroll
            for (int k = 0; k < POOL_T / 32; ++k) {
                const unsigned t = t0 + (tid >> 3) + 32 * k;
                v[k] = t < hi && col_ok ? *reinterpret_cast<const float4 *>(y + size_t(t) * width + c0 + 4 * j)
                                        : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
        };
        load(lo);
        for (unsigned t0 = lo; t0 < hi; t0 += POOL_T) {
            __syncthreads();  // the previous stage has been added up
#pragma unroll
            for (int k = 0; k < POOL_T / 32; ++k)
                stage[(tid >> 3) + 32 * k][j] = make_float4(__fdiv_rn(v[k].x, len), __fdiv_rn(v[k].y, len),
                                                            __fdiv_rn(v[k].z, len), __fdiv_rn(v[k].w, len));
            __syncthreads();
            if (t0 + POOL_T < hi) load(t0 + POOL_T);  // in flight during the adds below
            if (tid < 32) {
                const int nt = int(min(hi - t0, unsigned(POOL_T)));
                const float *col = reinterpret_cast<const float *>(&stage[0][0]) + lane;
                for (int i = 0; i < nt; ++i) o = __fadd_rn(o, col[i * 32]);
            }
        }
        if (tid < 32 && c0 + lane < width) out[size_t(s) * width + c0 + lane] = o;
    }
}
// pool_l2_kernel: one warp per sequence; the SSE2 sum of squares of
// kernels.c:82-93 (lanes 0..7 are its two 4-lane accumulators over 8-element
// chunks, each summed in chunk order), then x *= 1/sqrt(ss) (kernels.c:393-396).
// One warp per sequence of the grid's batch; with count set, sequences from
// *count on are skipped.
__global__ void pool_l2_kernel(float *__restrict__ out, int width, int batch, const unsigned *__restrict__ count) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x;
    const int nseq = count ? min(int(*count), batch) : batch;
    for (int s = blockIdx.x; s < nseq; s += gridDim.x) {  // warp-uniform
        float *o = out + size_t(s) * width;
        float acc = 0.0f;
        if (lane < 8)
            for (int i = 0; i + 7 < width; i += 8) acc = __fadd_rn(acc, __fmul_rn(o[i + lane], o[i + lane]));
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            v[j] = __fadd_rn(__shfl_sync(0xffffffffu, acc, j), __shfl_sync(0xffffffffu, acc, 4 + j));
        const float ss = __fadd_rn(__fadd_rn(v[0], v[2]), __fadd_rn(v[1], v[3]));
        const float inv = ss != 0.0f ? __fdiv_rn(1.0f, __fsqrt_rn(ss)) : 1.0f;
        for (int z = lane; z < width; z += 32) o[z] = __fmul_rn(o[z], inv);
    }
}

// GGUF Q8_0 blocks [rows][k/32] (34 B each) -> int8 codes [rows][k] and fp32
// scales block-major, scales[b * scale_stride + row].  With chunk > 0, source
// row r goes to destination row (r / chunk) * 2 * chunk + phase * chunk +
// r % chunk (two matrices interleaved in chunk-row blocks).
__global__ void repack_q8_kernel(const uint8_t *__restrict__ blocks, int rows, int k, int8_t *__restrict__ codes,
                                 float *__restrict__ scales, int scale_stride, int chunk, int phase) {
    const int kb = k / 32;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // one thread per block
    if (i >= (long long)rows * kb) return;
    const int r = int(i / kb), b = int(i % kb);
    const int dr = chunk > 0 ? (r / chunk) * 2 * chunk + phase * chunk + r % chunk : r;
    const uint8_t *src = blocks + size_t(i) * 34;
    const uint16_t db = uint16_t(src[0]) | uint16_t(src[1]) << 8;
    scales[size_t(b) * scale_stride + dr] = fp16_bits_to_f32(db);
    int8_t *dst = codes + size_t(dr) * k + b * 32;
#pragma unroll
    for (int z = 0; z < 32; ++z) dst[z] = int8_t(src[2 + z]);
}

}  // namespace eg2
