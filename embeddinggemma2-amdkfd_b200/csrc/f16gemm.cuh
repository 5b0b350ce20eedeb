// Q8_0 x Q8_0 GEMM of the fast path on the fp16 tensor cores (tcgen05
// kind::f16) -- the reference's gemm_q8 (vendor/embeddinggemma.c/src/
// gemma2_fast.c:242-253):
//
//     out[t][r] = sum_b ws[b][r] * xs[b][t] * D_b[r][t],   D_b = int32 dot of block b
//
// computed as one plain GEMM of dequantized operands, so that no per-block
// work is left for the CUDA cores.  Every activation x = xs * q and every
// weight w = ws * q is the exact product of an fp16 scale and a 7-bit code (at
// most 18 significant bits), and splits exactly into two fp16 values:
//   x = Xh + Xl        written by the quantizing kernels (rowops.cuh, the
//                      attention epilogue, the GeGLU epilogue below);
//   w * 2^s_r = Wh + Wl  made once at load time (split_q8_kernel), with a
//                      power of two per weight row that keeps the planes in
//                      fp16's range; rowscale[r] = 2^-s_r.
// Then out = rowscale * (Xh.Wh + Xh.Wl + Xl.Wh): three fp16 MMAs per K step
// with exact fp16 x fp16 products accumulated in fp32 in tensor memory.  The
// term left out, Xl.Wl, is below 2^-22 of the product; the sums are the
// reference's up to fp32 accumulation order (the tests bound it at 2e-6 of
// the output range, like the int8 kernel's fast mode).
//
// Tile: 128 tokens (the MMA's M side: one TMEM lane per token) x BN weight
// rows (N = 128 or 256), the K range walked in stages of 64 elements (one
// 128-byte swizzle row of each plane).  A unit is a tile and a contiguous
// range of its K: with splits > 1 unit u covers K range u / tiles and writes
// its partial sum to out + (u / tiles) * split_stride; the consumer adds the
// partials in order.  Two accumulator buffers in TMEM (2 x BN columns) let the
// epilogue of one unit overlap the MMAs of the next.
//
// Warp roles (persistent CTAs, one per SM):
//   warp 0      TMA producer: per stage Xh, Xl (128 x 128 B each) and Wh, Wl
//               (BN x 128 B each), 128-byte swizzle, into a ring of stages;
//   warp 1      TMEM owner and MMA issuer;
//   warps 2..9  epilogue: warp w reads TMEM lane quadrant w % 4 (32 tokens)
//               and column half (w - 2) / 4 (BN / 2 weight rows), scales by
//               rowscale and stores -- or, in GeGLU mode, pairs each 32-column
//               gate block with the up block beside it (weight rows are
//               interleaved in 32-row chunks), so one thread holds a whole
//               Q8_0 output block: gelu(gate) * up, its amax, codes and the
//               dequantized Xh / Xl of the ffn_down operand, all in registers.
// Every wait is a bounded mbarrier wait (common.cuh); TMEM is freed after all
// epilogue warps arrived on epilogue_done.
#pragma once
#include "common.cuh"

namespace eg2 {

struct F16GemmParams {
    float *out;           // plain mode: partial `split` at out + split * split_stride, rows [T][ldo]
    int ldo;
    size_t split_stride;
    const float *rowscale;  // [R] = 2^-s_r
    int T, R, K;          // tokens, weight rows (a multiple of BN), depth (a multiple of 64)
    int tiles_m, num_tiles, splits, units, kstages;  // kstages: 64-deep K stages per unit
    __half *xh, *xl;      // GeGLU mode: the ffn_down operand, dequantized fp16 planes [T][R/2]
    float *q8s;           // and the Q8_0 block scales q8s[b * q8s_stride + t] (fp32)
    int q8s_stride, tier;
};

template <int BN_>
struct F16Cfg {
    static constexpr int BM = 128, BN = BN_, BK = 64;  // BK fp16 = one 128-B swizzle row
    static constexpr int EPI_WARPS = 8, THREADS = (2 + EPI_WARPS) * 32;
    static constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;  // one plane of each
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int STAGES = (227 * 1024 - 2048) / STAGE_BYTES;  // 2 at BN = 256, 3 at BN = 128
    static constexpr int TMEM_COLS = 2 * BN;                           // two accumulator buffers
    static constexpr size_t SMEM = 1024 + size_t(STAGES) * STAGE_BYTES + 1024;
    static_assert(STAGES >= 2, "stage ring");
};

// GeGLU tail of one thread (ROW_GELU_QUANT, gemma2_fast.c:714-720): the 32
// gate and 32 up values of one token's Q8_0 output block -> g = gelu(gate) *
// up, d = amax / 127, codes, and the dequantized fp16 split d * q = hi + lo
// written to 32 consecutive elements of xh / xl; the scale (widened fp16)
// goes to *so.  TIER selects the GELU and the rounding at compile time.
template <int TIER>
__device__ __forceinline__ void geglu_block(const float *gate, const float *up, __half *xh, __half *xl, float *so,
                                            bool store) {
    float g[32];
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        g[j] = __fmul_rn(gelu_tier(gate[j], TIER), up[j]);
        amax = fmaxf(amax, fabsf(g[j]));
    }
    const float d = div127(amax);
    const float id = d != 0.0f ? rcp_rn(d) : 0.0f;
    const float ds = fp16_bits_to_f32(ref_fp32_to_fp16(d));
    if (!store) return;
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float v0 = __fmul_rn(ds, float(int(int8_t(uint8_t(q8_code(g[j + 2 * e], id, TIER)))))),
                        v1 = __fmul_rn(ds, float(int(int8_t(uint8_t(q8_code(g[j + 2 * e + 1], id, TIER))))));
            const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
            const __half2 hh = __halves2half2(h0, h1);
            const __half2 ll = __halves2half2(__float2half_rn(__fsub_rn(v0, __half2float(h0))),
                                              __float2half_rn(__fsub_rn(v1, __half2float(h1))));
            hw[e] = *reinterpret_cast<const uint32_t *>(&hh);
            lw[e] = *reinterpret_cast<const uint32_t *>(&ll);
        }
        *reinterpret_cast<uint4 *>(xh + j) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4 *>(xl + j) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
    *so = ds;
}

template <int BN, bool GEGLU>
__global__ void __launch_bounds__(F16Cfg<BN>::THREADS, 1)
    f16gemm_kernel(const __grid_constant__ CUtensorMap tmXh, const __grid_constant__ CUtensorMap tmXl,
                   const __grid_constant__ CUtensorMap tmWh, const __grid_constant__ CUtensorMap tmWl,
                   const F16GemmParams p) {
    using C = F16Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = align_smem_1024(smem_raw);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + size_t(C::STAGES) * C::STAGE_BYTES);
    uint64_t *full = bars, *empty = bars + C::STAGES, *accf = empty + C::STAGES, *acce = accf + 2;
    uint64_t *mdone = acce + 2, *edone = mdone + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(edone + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    auto stage = [&](int s) { return smem + size_t(s) * C::STAGE_BYTES; };
    // Stage layout: Xh | Xl | Wh | Wl.
    auto unit_coords = [&](int u, int &m0, int &n0, int &ks0) {
        const int tile = u % p.num_tiles;
        m0 = (tile % p.tiles_m) * C::BM, n0 = (tile / p.tiles_m) * BN, ks0 = (u / p.num_tiles) * p.kstages;
    };

    if (threadIdx.x == 0) {
        tma_prefetch(&tmXh), tma_prefetch(&tmXl), tma_prefetch(&tmWh), tma_prefetch(&tmWl);
        *abort = 0;
        for (int s = 0; s < C::STAGES; ++s) bar_init(&full[s], 1), bar_init(&empty[s], 1);
        for (int b = 0; b < 2; ++b) bar_init(&accf[b], 1), bar_init(&acce[b], C::EPI_WARPS);
        bar_init(mdone, 1), bar_init(edone, C::EPI_WARPS);
        fence_bar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    pdl_wait();  // the prologue above overlaps the previous kernel's tail
    pdl_trigger();
    tc_fence_before();
    cta_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (elect_one()) {
            int g = 0, issued = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
                int m0, n0, ks0;
                unit_coords(u, m0, n0, ks0);
                for (int ks = 0; ks < p.kstages; ++ks, ++g) {
                    const int s = g % C::STAGES;
                    if (!wait_bar(&empty[s], ((g / C::STAGES) & 1) ^ 1, abort)) {
                        ok = false;
                        break;
                    }
                    // x coordinate: a multiple of 64 fp16 elements (128 B).
                    const int k_el = (ks0 + ks) * C::BK;
                    uint8_t *st = stage(s);
                    bar_expect_tx(&full[s], C::STAGE_BYTES);
                    tma_load_2d(st, &tmXh, &full[s], k_el, m0);
                    tma_load_2d(st + C::A_BYTES, &tmXl, &full[s], k_el, m0);
                    tma_load_2d(st + 2 * C::A_BYTES, &tmWh, &full[s], k_el, n0);
                    tma_load_2d(st + 2 * C::A_BYTES + C::B_BYTES, &tmWl, &full[s], k_el, n0);
                    ++issued;
                }
            }
            // Drain: the last load into every stage has landed before exit.
            for (int k = issued > C::STAGES ? issued - C::STAGES : 0; k < issued; ++k)
                wait_bar(&full[k % C::STAGES], (k / C::STAGES) & 1, nullptr);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (elect_one() && !*abort) {
            constexpr uint32_t idesc = idesc_f16(C::BM, BN);
            int g = 0, it = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++it) {
                const int buf = it & 1;
                // The epilogue has drained this accumulator buffer's previous unit.
                if (!wait_bar(&acce[buf], ((it >> 1) & 1) ^ 1, abort)) break;
                tc_fence_after();
                const uint32_t d = tmem + uint32_t(buf * BN);
                for (int ks = 0; ks < p.kstages; ++ks, ++g) {
                    const int s = g % C::STAGES;
                    if (!wait_bar(&full[s], (g / C::STAGES) & 1, abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t xh = smem_u32(stage(s)), xl = xh + C::A_BYTES, wh = xh + 2 * C::A_BYTES,
                                   wl = wh + C::B_BYTES;
#pragma unroll
                    for (int kk = 0; kk < C::BK / 16; ++kk) {  // K = 16 steps: 32 bytes along each row
                        const uint32_t off = uint32_t(kk * 32);
                        mma_f16(d, desc_sw128(xh + off), desc_sw128(wh + off), idesc, (ks | kk) ? 1u : 0u);
                        mma_f16(d, desc_sw128(xh + off), desc_sw128(wl + off), idesc, 1u);
                        mma_f16(d, desc_sw128(xl + off), desc_sw128(wh + off), idesc, 1u);
                    }
                    tc_commit(&empty[s]);
                }
                tc_commit(&accf[buf]);
            }
            // Drain: every MMA issued above has completed before TMEM is freed.
            tc_commit(mdone);
            wait_bar(mdone, 0, nullptr);
        }
        __syncwarp();
        wait_bar(edone, 0, nullptr);
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    } else {
        // ------------------------------------------------------------ epilogue
        const int quad = warp & 3, hf = (warp - 2) >> 2;
        constexpr int COLS = BN / 2;  // weight rows (columns) per warp
        int it = 0;
        for (int u = blockIdx.x; u < p.units; u += gridDim.x, ++it) {
            const int buf = it & 1;
            int m0, n0, ks0;
            unit_coords(u, m0, n0, ks0);
            const int t = m0 + quad * 32 + lane, c0 = n0 + hf * COLS;
            if (!__all_sync(0xffffffffu, wait_bar(&accf[buf], (it >> 1) & 1, abort))) break;  // tcgen05.ld is warp-collective
            tc_fence_after();
            const uint32_t taddr = tmem + (uint32_t(quad * 32) << 16) + uint32_t(buf * BN + hf * COLS);
            if constexpr (GEGLU) {
                // Columns come in 64-wide pairs: 32 gate rows, then the 32 up
                // rows of the same output columns.
#pragma unroll 1
                for (int c = 0; c < COLS; c += 64) {
                    uint32_t gr[32], ur[32];
                    tmem_ld32(taddr + uint32_t(c), gr);
                    tmem_ld32(taddr + uint32_t(c + 32), ur);
                    tmem_wait_ld();
                    reg_fence(gr);
                    reg_fence(ur);
                    float gate[32], up[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        gate[j] = __uint_as_float(gr[j]) * p.rowscale[c0 + c + j];
                        up[j] = __uint_as_float(ur[j]) * p.rowscale[c0 + c + 32 + j];
                    }
                    const int oc = (c0 + c) / 2;  // first output column of the block
                    __half *xh = p.xh + size_t(t) * (p.R / 2) + oc, *xl = p.xl + size_t(t) * (p.R / 2) + oc;
                    float *so = p.q8s + size_t(oc / 32) * p.q8s_stride + t;
                    if (p.tier == TIER_SCALAR)
                        geglu_block<TIER_SCALAR>(gate, up, xh, xl, so, t < p.T);
                    else
                        geglu_block<TIER_X86>(gate, up, xh, xl, so, t < p.T);
                }
            } else {
                float *o = p.out + size_t(u / p.num_tiles) * p.split_stride + size_t(t) * p.ldo + c0;
#pragma unroll 1
                for (int c = 0; c < COLS; c += 32) {
                    uint32_t r[32];
                    tmem_ld32(taddr + uint32_t(c), r);
                    tmem_wait_ld();
                    reg_fence(r);
                    if (t < p.T) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4) {
                            const float4 rs = *reinterpret_cast<const float4 *>(p.rowscale + c0 + c + j);
                            *reinterpret_cast<float4 *>(o + c + j) =
                                make_float4(__uint_as_float(r[j]) * rs.x, __uint_as_float(r[j + 1]) * rs.y,
                                            __uint_as_float(r[j + 2]) * rs.z, __uint_as_float(r[j + 3]) * rs.w);
                        }
                    }
                }
            }
            // This buffer may take the next unit's MMAs once every warp has read it.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&acce[buf]);
        }
        __syncwarp();
        tc_fence_before();
        if (lane == 0) bar_arrive(edone);
    }
}

// Load-time weight preparation for f16gemm_kernel: one warp per weight row of
// the SoA Q8 weight (codes [rows][k], fp32 scales [k/32][scale_stride]):
// w = ws * q exactly, s_r such that max |w| * 2^s_r lies in [2^14, 2^15) (or 0
// for an all-zero row), Wh = fp16(w * 2^s_r), Wl = fp16(w * 2^s_r - Wh), and
// rowscale[r] = 2^-s_r.  w * 2^s_r has at most 18 significant bits, so
// Wh + Wl == w * 2^s_r exactly unless Wl falls below fp16's subnormal step
// (only for a block scale more than 2^20 times smaller than the row's largest
// weight).
__global__ void split_q8_kernel(const int8_t *__restrict__ codes, const float *__restrict__ scales, int scale_stride,
                                int rows, int k, __half *__restrict__ wh, __half *__restrict__ wl,
                                float *__restrict__ rowscale) {
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= rows) return;
    const int8_t *q = codes + size_t(r) * k;
    float amax = 0.0f;
    for (int z = lane; z < k; z += 32) amax = fmaxf(amax, fabsf(scales[size_t(z / 32) * scale_stride + r] * float(q[z])));
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    int e = 0;
    if (amax > 0.0f) frexpf(amax, &e);  // amax = m * 2^e, m in [0.5, 1)
    const int s = amax > 0.0f ? max(-120, min(120, 15 - e)) : 0;
    const float up = ldexpf(1.0f, s);
    for (int z = lane; z < k; z += 32) {
        const float v = scales[size_t(z / 32) * scale_stride + r] * float(q[z]) * up;  // both products exact
        const __half h = __float2half_rn(v);
        wh[size_t(r) * k + z] = h;
        wl[size_t(r) * k + z] = __float2half_rn(v - __half2float(h));
    }
    if (lane == 0) rowscale[r] = ldexpf(1.0f, -s);
}

}  // namespace eg2
