// Q8_0 x Q8_0 GEMM of the fast path on the fp16 tensor cores (tcgen05
// kind::f16) -- the reference's gemm_q8 (vendor/embeddinggemma.c/src/
// gemma2_fast.c:242-253) with the same block structure:
//
//     out[t][r] = sum_b ws[b][r] * xs[b][t] * D_b[r][t],   D_b = int32 dot of block b
//
// The weight scale goes into the operand instead of the epilogue: at load time
// every weight w = ws * q (an exact product of an fp16 scale and a 7-bit code,
// at most 18 significant bits) is scaled by a per-row power of two 2^s_r and
// split exactly into two fp16 values, w * 2^s_r = Wh + Wl (Wh = w rounded to
// 11 bits, Wl = the remaining <= 7 bits; split_q8_kernel).  Activation codes
// are exact in fp16 (|q| <= 128).  Per Q8_0 block the MMA warp issues
// D(+)= Wh . q and D += Wl . q (two K = 16 steps each) into that block's own
// TMEM slot, so
//     P_b[r][t] = 2^s_r * ws_b[r] * D_b[r][t]
// up to the fp32 accumulation of 64 exact products, and the epilogue needs one
// FMA per block and element, acc += P_b * xs_b[t] (the int8 kernel, q8gemm.cuh,
// needs a conversion and two multiply-adds), and one exact multiply by
// 2^-s_r at the end.
//
// Tiles are 128 weight rows (the MMA's M side, TMEM lanes) x 128 tokens (N,
// the full-rate MMA width).  A unit is a tile and a contiguous range of its K
// blocks: with splits > 1 (GEMMs with few output tiles) unit u covers blocks
// [kbu * (u / tiles), kbu * (u / tiles + 1)) and writes its partial sum to
// out + (u / tiles) * split_stride; the consumer adds the partials in order.
//
// Persistent CTAs (one per SM) walk the units; warp roles:
//   warp 0      TMA producer: per unit the activation-scale panel [kbu][128]
//               into a double buffer, then per stage of two Q8_0 blocks the
//               Wh and Wl tiles (128 rows x 128 B each) and the code tile
//               (128 tokens x 128 B), 128-byte swizzle;
//   warp 1      TMEM owner (512 columns = 4 block slots x 128) and MMA issuer;
//               slots go in groups of two (one stage), one handshake per group;
//   warps 2..9  epilogue: warp w reads TMEM lane quadrant w % 4 and token half
//               (w - 2) / 4, i.e. 32 weight rows x 64 tokens, accumulating in
//               registers in ascending block order.
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
    int T, R, K;          // tokens, weight rows (a multiple of 128), depth (a multiple of 64)
    int tiles_t, num_tiles, splits, units, kbu;  // kbu: Q8_0 blocks per unit
    __half *q16;          // GeGLU mode: fp16 codes [T][R/2] of gelu(gate) * up
    float *q8s;           // and their block-major scales q8s[b * q8s_stride + t]
    int q8s_stride, tier;
};

struct F16Cfg {
    static constexpr int BM = 128, BN = 128, BK = 64;  // BK fp16 = two Q8_0 blocks = one 128-B swizzle row
    static constexpr int SLOT = 128, NSLOT = 4, GROUP = 2, HALF = 64;
    static constexpr int EPI_WARPS = 8, THREADS = (2 + EPI_WARPS) * 32;
    static constexpr int MAX_STAGES = 6;
    static constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = 2 * A_BYTES + B_BYTES;  // Wh, Wl, codes
};

struct F16Smem {
    int stages, pbufs;
    size_t panel_bytes, gbuf_bytes, total;
    __host__ __device__ size_t panel(int b) const { return size_t(stages) * F16Cfg::STAGE_BYTES + size_t(b) * panel_bytes; }
    __host__ __device__ size_t gbuf() const { return panel(pbufs); }
    __host__ __device__ size_t bars() const { return gbuf() + gbuf_bytes; }
};
__host__ __device__ inline F16Smem f16gemm_smem(int kbu, bool geglu) {
    F16Smem s;
    s.panel_bytes = (size_t(kbu) * F16Cfg::BN * 4 + 1023) / 1024 * 1024;
    s.gbuf_bytes = geglu ? (size_t(F16Cfg::BN) * (F16Cfg::BM + 1) * 4 + 1023) / 1024 * 1024 : 0;
    const size_t limit = 227 * 1024, fixed = 1024 + 512 + s.gbuf_bytes;
    for (s.stages = F16Cfg::MAX_STAGES; s.stages > 2; --s.stages)
        if (fixed + size_t(s.stages) * F16Cfg::STAGE_BYTES + s.panel_bytes <= limit) break;
    s.pbufs = fixed + size_t(s.stages) * F16Cfg::STAGE_BYTES + 2 * s.panel_bytes <= limit ? 2 : 1;
    s.total = fixed + size_t(s.stages) * F16Cfg::STAGE_BYTES + size_t(s.pbufs) * s.panel_bytes;
    return s;
}

// GeGLU tail unit (ROW_GELU_QUANT, gemma2_fast.c:714-720): g = gelu(gate) * up
// for 16 columns of one (token, 32-column block) -- gate at gr[0..15], up at
// gr[64..79] -- then the block's Q8_0 codes, the lane pair (part 0, 1) sharing
// the block's amax by one shuffle; stores only when `store` is set.
template <int TIER, typename CodeT>
__device__ __forceinline__ void geglu_unit_codes(const float *gr, int part, bool store, CodeT *q8, float *q8s) {
    float g[16];
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        g[j] = __fmul_rn(gelu_tier(gr[j], TIER), gr[64 + j]);
        amax = fmaxf(amax, fabsf(g[j]));
    }
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    const float d = div127(amax);
    const float id = d != 0.0f ? rcp_rn(d) : 0.0f;
    if (!store) return;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        store_codes4(q8, j, q8_code(g[4 * j], id, TIER) | q8_code(g[4 * j + 1], id, TIER) << 8 |
                                q8_code(g[4 * j + 2], id, TIER) << 16 | q8_code(g[4 * j + 3], id, TIER) << 24);
    if (part == 0) *q8s = fp16_bits_to_f32(ref_fp32_to_fp16(d));
}

// GEGLU: every 128-row weight tile is 64 gate rows followed by the 64 up rows
// of the same output columns; the epilogue pairs them through shared memory
// and writes the fp16 Q8_0 codes of gelu_tanh(gate) * up (the ffn_down operand).
template <bool GEGLU>
__global__ void __launch_bounds__(F16Cfg::THREADS, 1)
    f16gemm_kernel(const __grid_constant__ CUtensorMap tmWh, const __grid_constant__ CUtensorMap tmWl,
                   const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmSX,
                   const F16GemmParams p) {
    using C = F16Cfg;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = align_smem_1024(smem_raw);
    const F16Smem L = f16gemm_smem(p.kbu, GEGLU);
    const int STAGES = L.stages, PBUFS = L.pbufs, kstages = p.kbu / 2;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars());
    uint64_t *full = bars, *empty = bars + C::MAX_STAGES, *accf = bars + 2 * C::MAX_STAGES;
    uint64_t *acce = accf + 2, *pfull = acce + 2, *pempty = pfull + 2, *mdone = pempty + 2, *edone = mdone + 1;
    uint64_t *gfull = edone + 1, *gdone = gfull + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gdone + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    auto wh_tile = [&](int s) { return smem + size_t(s) * C::STAGE_BYTES; };
    auto wl_tile = [&](int s) { return smem + size_t(s) * C::STAGE_BYTES + C::A_BYTES; };
    auto x_tile = [&](int s) { return smem + size_t(s) * C::STAGE_BYTES + 2 * C::A_BYTES; };
    auto panel = [&](int b) { return reinterpret_cast<float *>(smem + L.panel(b)); };

    if (threadIdx.x == 0) {
        tma_prefetch(&tmWh), tma_prefetch(&tmWl), tma_prefetch(&tmX), tma_prefetch(&tmSX);
        *abort = 0;
        for (int s = 0; s < STAGES; ++s) bar_init(&full[s], 1), bar_init(&empty[s], 1);
        for (int b = 0; b < 2; ++b) bar_init(&accf[b], 1), bar_init(&acce[b], C::EPI_WARPS);
        for (int b = 0; b < PBUFS; ++b) bar_init(&pfull[b], 1), bar_init(&pempty[b], C::EPI_WARPS);
        bar_init(mdone, 1), bar_init(edone, C::EPI_WARPS);
        bar_init(gfull, C::EPI_WARPS), bar_init(gdone, C::EPI_WARPS);
        fence_bar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
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
            int g = 0, issued = 0, it = 0, panels = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++it) {
                const int tile = u % p.num_tiles, kb0 = (u / p.num_tiles) * p.kbu;
                const int r0 = (tile / p.tiles_t) * C::BM, t0 = (tile % p.tiles_t) * C::BN;
                const int pb = it % PBUFS;
                for (int ks = 0; ks < kstages; ++ks, ++g) {
                    const int s = g % STAGES;
                    if (!wait_bar(&empty[s], ((g / STAGES) & 1) ^ 1, abort)) {
                        ok = false;
                        break;
                    }
                    // x coordinate: a multiple of 64 fp16 elements (128 B).
                    const int k_el = (kb0 + 2 * ks) * 32;
                    bar_expect_tx(&full[s], C::STAGE_BYTES);
                    tma_load_2d(wh_tile(s), &tmWh, &full[s], k_el, r0);
                    tma_load_2d(wl_tile(s), &tmWl, &full[s], k_el, r0);
                    tma_load_2d(x_tile(s), &tmX, &full[s], k_el, t0);
                    ++issued;
                    if (ks == 0) {  // first needed by the epilogue: after the first stage
                        if (!wait_bar(&pempty[pb], ((it / PBUFS) & 1) ^ 1, abort)) {
                            ok = false;
                            break;
                        }
                        bar_expect_tx(&pfull[pb], uint32_t(p.kbu * C::BN * 4));
                        tma_load_2d(panel(pb), &tmSX, &pfull[pb], t0, kb0);
                        ++panels;
                    }
                }
            }
            // Drain: the last load into every stage / panel buffer has landed before exit.
            for (int k = issued > STAGES ? issued - STAGES : 0; k < issued; ++k)
                wait_bar(&full[k % STAGES], (k / STAGES) & 1, nullptr);
            for (int k = panels > PBUFS ? panels - PBUFS : 0; k < panels; ++k)
                wait_bar(&pfull[k % PBUFS], (k / PBUFS) & 1, nullptr);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (elect_one() && !*abort) {
            constexpr uint32_t idesc = idesc_f16(C::BM, C::BN);
            int g = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
                for (int ks = 0; ks < kstages && ok; ++ks, ++g) {
                    const int s = g % STAGES, grp = g & 1;
                    if (!wait_bar(&full[s], (g / STAGES) & 1, abort) ||
                        !wait_bar(&acce[grp], ((g >> 1) & 1) ^ 1, abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t ah = smem_u32(wh_tile(s)), al = smem_u32(wl_tile(s)), b = smem_u32(x_tile(s));
#pragma unroll
                    for (int j = 0; j < C::GROUP; ++j) {  // Q8_0 block j of the stage: bytes 64j .. 64j + 63 of each row
                        const uint32_t d = tmem + uint32_t((grp * C::GROUP + j) * C::SLOT);
#pragma unroll
                        for (int kk = 0; kk < 2; ++kk)
                            mma_f16(d, desc_sw128(ah + j * 64 + kk * 32), desc_sw128(b + j * 64 + kk * 32), idesc,
                                    kk ? 1u : 0u);
#pragma unroll
                        for (int kk = 0; kk < 2; ++kk)
                            mma_f16(d, desc_sw128(al + j * 64 + kk * 32), desc_sw128(b + j * 64 + kk * 32), idesc, 1u);
                    }
                    tc_commit(&accf[grp]);
                    tc_commit(&empty[s]);
                }
            }
            // Drain: every MMA issued above has completed before TMEM is freed.
            tc_commit(mdone);
            wait_bar(mdone, 0, nullptr);
        }
        __syncwarp();
        wait_bar(edone, 0, nullptr);
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    } else {
        // ------------------------------------------------------------ epilogue
        const int quad = warp & 3, hf = (warp - 2) >> 2, r_local = quad * 32 + lane;
        const uint32_t tbase = tmem + (uint32_t(quad * 32) << 16) + uint32_t(hf * C::HALF);
        int grp_count = 0, it = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++it) {
            const int tile = u % p.num_tiles, split = u / p.num_tiles;
            const int r0 = (tile / p.tiles_t) * C::BM, t0 = (tile % p.tiles_t) * C::BN;
            const int pb = it % PBUFS;
            if (!__all_sync(0xffffffffu, wait_bar(&pfull[pb], (it / PBUFS) & 1, abort))) break;
            const float4 *sx = reinterpret_cast<const float4 *>(panel(pb) + hf * C::HALF);  // block j: sx[j * 32 + c]
            float2 acc[C::HALF / 2];
#pragma unroll
            for (int c = 0; c < C::HALF / 2; ++c) acc[c] = make_float2(0.0f, 0.0f);
            auto math = [&](const uint32_t(&r)[C::HALF], int j) {
                const float4 *xs = sx + j * (C::BN / 4);
#pragma unroll
                for (int c4 = 0; c4 < C::HALF / 4; ++c4) {
                    const float4 x4 = xs[c4];
                    acc[2 * c4] = __ffma2_rn(make_float2(__uint_as_float(r[4 * c4]), __uint_as_float(r[4 * c4 + 1])),
                                             make_float2(x4.x, x4.y), acc[2 * c4]);
                    acc[2 * c4 + 1] =
                        __ffma2_rn(make_float2(__uint_as_float(r[4 * c4 + 2]), __uint_as_float(r[4 * c4 + 3])),
                                   make_float2(x4.z, x4.w), acc[2 * c4 + 1]);
                }
            };
            uint32_t r[C::HALF];
            for (int ks = 0; ks < kstages; ++ks, ++grp_count) {
                const int grp = grp_count & 1, use = grp_count >> 1;
                if (!__all_sync(0xffffffffu, wait_bar(&accf[grp], use & 1, abort))) {  // tcgen05.ld is warp-collective
                    ok = false;
                    break;
                }
                tc_fence_after();
                tmem_ld64(tbase + uint32_t(grp * C::GROUP * C::SLOT), r);
                tmem_wait_ld();
                reg_fence(r);
                math(r, 2 * ks);
                tmem_ld64(tbase + uint32_t((grp * C::GROUP + 1) * C::SLOT), r);
                tmem_wait_ld();
                reg_fence(r);
                tc_fence_before();
                if (lane == 0) bar_arrive(&acce[grp]);
                math(r, 2 * ks + 1);
            }
            __syncwarp();
            if (lane == 0) bar_arrive(&pempty[pb]);
            if (!ok) break;
            const float rs = p.rowscale[r0 + r_local];
            if (GEGLU) {
                // Pair gate (lanes 0..63) and up (lanes 64..127) of each output
                // column through G[token][row] (row stride GS against bank
                // conflicts); then lane pairs own (token, 32-column block) units,
                // 16 columns per lane, two units per pair.
                constexpr int GS = C::BM + 1;
                float *G = reinterpret_cast<float *>(smem + L.gbuf());
#pragma unroll
                for (int c = 0; c < C::HALF / 2; ++c) {
                    const int tok = hf * C::HALF + 2 * c;
                    G[tok * GS + r_local] = acc[c].x * rs;
                    G[(tok + 1) * GS + r_local] = acc[c].y * rs;
                }
                __syncwarp();
                if (lane == 0) bar_arrive(gfull);
                if (!__all_sync(0xffffffffu, wait_bar(gfull, it & 1, abort))) {
                    ok = false;
                    break;
                }
                const int e = (warp - 2) * 32 + lane, part = e & 1, col0 = r0 / 2;
#pragma unroll
                for (int pass = 0; pass < 2; ++pass) {
                    const int unit = pass * 128 + (e >> 1), tok = unit >> 1, cb = unit & 1, t = t0 + tok;
                    const float *gr = G + tok * GS + cb * 32 + part * 16;
                    __half *qo = p.q16 + size_t(t) * (p.R / 2) + col0 + cb * 32 + part * 16;
                    float *so = p.q8s + size_t(col0 / 32 + cb) * p.q8s_stride + t;
                    if (p.tier == TIER_SCALAR)
                        geglu_unit_codes<TIER_SCALAR>(gr, part, t < p.T, qo, so);
                    else
                        geglu_unit_codes<TIER_X86>(gr, part, t < p.T, qo, so);
                }
                __syncwarp();
                if (lane == 0) bar_arrive(gdone);
                if (!__all_sync(0xffffffffu, wait_bar(gdone, it & 1, abort))) {  // G is rewritten next unit
                    ok = false;
                    break;
                }
                continue;
            }
            // out[t][r]: for each token the warp's 32 lanes write 128 consecutive bytes.
            float *o = p.out + size_t(split) * p.split_stride + size_t(t0 + hf * C::HALF) * p.ldo + r0 + r_local;
            const int tmax = p.T - (t0 + hf * C::HALF);
#pragma unroll
            for (int c = 0; c < C::HALF / 2; ++c) {
                if (2 * c < tmax) o[size_t(2 * c) * p.ldo] = acc[c].x * rs;
                if (2 * c + 1 < tmax) o[size_t(2 * c + 1) * p.ldo] = acc[c].y * rs;
            }
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
