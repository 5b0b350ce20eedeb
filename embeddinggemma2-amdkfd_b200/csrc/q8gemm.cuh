// Q8_0 x Q8_0 GEMM on the 5th-generation tensor cores (tcgen05 kind::i8).
//
// out[t][r] = sum_b D_b[r][t] * ws[b][r] * xs[b][t],  D_b = int32 dot of the
// 32-element block b of weight row r and activation row t -- the reference's
// gemm_q8 (vendor/embeddinggemma.c/src/gemma2_fast.c:242-253, scalar tile
// :193-204).  One tcgen05.mma with K = 32 is exactly one Q8_0 block, so each
// block's int32 dot lands exactly in its own TMEM slot; the epilogue warps
// rescale and accumulate in fp32 registers, blocks in ascending order:
//     t   = round(D_b * ws)            (one FMA, see below)
//     acc = acc + round(t * xs)        EXACT: the reference scalar tile's order,
//                                      ((float)dot * dw) * dx then sum +=
//     acc = fma(t, xs, acc)            otherwise (one rounding fewer)
// The int32 -> fp32 conversion uses the exact bias trick: with
// B = 1.5 * 2^23, the bits of D + 0x4B400000 are the float B + D for
// |D| < 2^22 (|D| <= 32 * 128 * 128 here), and fma(B + D, ws, -B * ws) rounds
// (B + D) * ws - B * ws = D * ws once; -B * ws is exact because ws is an fp16
// value.  Pairs of tokens go through fma.rn.f32x2.
//
// Operand roles: the 128 weight rows of a tile are the MMA's M side (TMEM
// lanes) and its 64 activation tokens the N side (TMEM columns).  An epilogue
// thread therefore owns one output column r: its weight scale is one scalar
// per block, and only the activation scales (one per token column, the same
// for every lane) are broadcast from shared memory.
//
// Persistent CTAs (one per SM) walk the 128 x 64 output tiles; warp roles:
//   warp 0      TMA producer: per tile the scale panels (weight scales
//               [K/32][128], activation scales [K/32][64]) into a double
//               buffer, then int8 weight/token tiles of 128 B (one 128-byte
//               swizzle row = four Q8_0 blocks) per stage of a ring of up
//               to six stages;
//   warp 1      TMEM owner and MMA issuer: block j is two N=32 MMAs (token
//               halves h = 0, 1) into TMEM columns h*256 + (j % 8)*32.  The
//               eight slots form two groups of four, one stage's blocks each:
//               the warp waits once per stage for its group to be free and
//               commits once per stage -> acc_full[group];
//   warps 2..9  epilogue: warp w reads TMEM lanes 32*(w%4).. (its hardware
//               quadrant) of token half h = (w-2)/4.  Per group it waits once,
//               fetches the four blocks as two 64-column tcgen05.ld, frees the
//               group after the second, and rescales from registers.
// Barrier round trips cost on the order of 100 ns each, so they are paid per
// stage of four blocks, not per block.
// The stage ring, TMEM slots and panel buffers continue across tiles, so loads
// and MMAs of the next tile overlap the epilogue of the current one.  Every
// wait is a bounded mbarrier wait that sets the device error word and exits;
// the MMA warp frees TMEM once the epilogue warps have all arrived on
// epilogue_done (there is no CTA-wide barrier after the roles diverge).
#pragma once
#include "common.cuh"

namespace eg2 {

struct Q8GemmParams {
    float *out;   // [T][ldo] fp32 (plain mode)
    int ldo;
    int T, R, K;  // tokens, weight rows (= output columns, a multiple of 128), depth
    int tiles_t, num_tiles;
    int8_t *q8;   // GeGLU mode: Q8_0 codes [T][R/2] of gelu(gate) * up
    float *q8s;   // and their block-major scales, q8s[b * q8s_stride + t]
    int q8s_stride;
};

struct Q8Cfg {
    static constexpr int BM = 128;   // weight rows per tile = TMEM lanes
    static constexpr int BN = 64;    // tokens per tile
    static constexpr int BK = 128;   // bytes of K per stage: four Q8_0 blocks
    static constexpr int HALF = 32;  // token columns of one epilogue warp (one N=32 MMA)
    static constexpr int NBUF = 8;   // block slots: 2 halves x 8 slots x 32 columns = 512
    static constexpr int GROUP = 4;  // slots per handshake group = Q8_0 blocks per stage
    static constexpr int EPI_WARPS = 8, THREADS = (2 + EPI_WARPS) * 32;
    static constexpr int MAX_STAGES = 6;  // depth of the TMA ring when shared memory allows
    static constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, STAGE_BYTES = A_BYTES + B_BYTES;
};

// Shared-memory plan (offsets from the 1024-aligned base) for depth K; the
// GeGLU mode adds the 64 x 128 fp32 tile used to pair gate and up rows.
struct Q8Smem {
    int stages, pbufs, kb;
    size_t stage_bytes, sw_bytes, sx_bytes, panel_bytes, gbuf_bytes, total;
    __host__ __device__ size_t panel(int b) const { return size_t(stages) * stage_bytes + size_t(b) * panel_bytes; }
    __host__ __device__ size_t gbuf() const { return size_t(stages) * stage_bytes + size_t(pbufs) * panel_bytes; }
    __host__ __device__ size_t bars() const { return gbuf() + gbuf_bytes; }
};
__host__ __device__ inline Q8Smem q8gemm_smem(int K, bool geglu = false) {
    Q8Smem s;
    s.kb = K / 32;
    s.stage_bytes = size_t(Q8Cfg::STAGE_BYTES);
    s.sw_bytes = size_t(s.kb) * Q8Cfg::BM * 4;
    s.sx_bytes = size_t(s.kb) * Q8Cfg::BN * 4;
    s.panel_bytes = (s.sw_bytes + s.sx_bytes + 1023) / 1024 * 1024;
    s.gbuf_bytes = geglu ? (size_t(Q8Cfg::BN) * (Q8Cfg::BM + 1) * 4 + 1023) / 1024 * 1024 : 0;
    // The deepest ring (MAX_STAGES down to 2) that fits, with two panel buffers
    // when they fit beside it, else one.
    const size_t limit = 227 * 1024, fixed = 1024 + 512 + s.gbuf_bytes;
    for (s.stages = Q8Cfg::MAX_STAGES; s.stages > 2; --s.stages)
        if (fixed + size_t(s.stages) * s.stage_bytes + s.panel_bytes <= limit) break;
    s.pbufs = fixed + size_t(s.stages) * s.stage_bytes + 2 * s.panel_bytes <= limit ? 2 : 1;
    s.total = fixed + size_t(s.stages) * s.stage_bytes + size_t(s.pbufs) * s.panel_bytes;
    return s;
}

// One unit of the GeGLU tail: g = gelu(gate) * up for 16 columns of one
// (token, 32-column block) -- gate at gr[0..15], up at gr[64..79] -- then the
// block's Q8_0 codes, the lane pair (part 0, 1) sharing its amax by one
// shuffle; stores only when store is set (all lanes take part in the shuffle).
// The tier is a template argument so the 16 independent chains compile without
// a branch per element.
template <int TIER>
__device__ __forceinline__ void geglu_unit(const float *gr, int part, bool store, int8_t *q8, float *q8s) {
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
    uint32_t w4[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
        w4[j] = q8_code(g[4 * j], id, TIER) | q8_code(g[4 * j + 1], id, TIER) << 8 |
                q8_code(g[4 * j + 2], id, TIER) << 16 | q8_code(g[4 * j + 3], id, TIER) << 24;
    *reinterpret_cast<uint4 *>(q8) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
    if (part == 0) *q8s = fp16_bits_to_f32(ref_fp32_to_fp16(d));
}

// GEGLU: the weight rows of every 128-row tile are 64 gate rows followed by
// the 64 up rows of the same output columns (ROW_GELU_QUANT fused,
// gemma2_fast.c:714-720): the epilogue pairs them through shared memory and
// writes Q8_0 codes of gelu_tanh(gate) * up instead of fp32 outputs, with
// TIER's GELU and quantizer rounding (TIER_X86 or TIER_SCALAR).  The tier is
// a template argument so that each kernel carries one tail: the unrolled
// GELU chains of a second tier beside the main loop cost instruction fetch.
template <bool EXACT, bool GEGLU, int TIER = TIER_X86>
__global__ void __launch_bounds__(Q8Cfg::THREADS, 1)
    q8gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                  const __grid_constant__ CUtensorMap tmSW, const __grid_constant__ CUtensorMap tmSX,
                  const Q8GemmParams p) {
    using C = Q8Cfg;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = align_smem_1024(smem_raw);
    const Q8Smem L = q8gemm_smem(p.K, GEGLU);
    const int Kb = L.kb, ksteps = p.K / C::BK, STAGES = L.stages, PBUFS = L.pbufs;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars());
    uint64_t *full = bars, *empty = bars + C::MAX_STAGES, *accf = bars + 2 * C::MAX_STAGES;
    uint64_t *acce = accf + 2;  // accf/acce: per slot group
    uint64_t *pfull = acce + 2, *pempty = pfull + 2, *mdone = pempty + 2, *edone = mdone + 1;
    uint64_t *gfull = edone + 1, *gdone = gfull + 1;  // GeGLU pairing tile written / consumed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gdone + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    auto w_tile = [&](int s) { return smem + size_t(s) * L.stage_bytes; };
    auto x_tile = [&](int s) { return smem + size_t(s) * L.stage_bytes + C::A_BYTES; };
    auto sw_pan = [&](int b) { return reinterpret_cast<float *>(smem + L.panel(b)); };
    auto sx_pan = [&](int b) { return reinterpret_cast<float *>(smem + L.panel(b) + L.sw_bytes); };

    if (threadIdx.x == 0) {
        // Descriptor fetches overlap the rest of the prologue.
        tma_prefetch(&tmW), tma_prefetch(&tmX), tma_prefetch(&tmSW), tma_prefetch(&tmSX);
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
            for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++it) {
                const int r0 = (tile / p.tiles_t) * C::BM, t0 = (tile % p.tiles_t) * C::BN;
                const int pb = it % PBUFS;
                for (int ks = 0; ks < ksteps; ++ks, ++g) {
                    const int s = g % STAGES;
                    if (!wait_bar(&empty[s], ((g / STAGES) & 1) ^ 1, abort)) {
                        ok = false;
                        break;
                    }
                    bar_expect_tx(&full[s], C::STAGE_BYTES);
                    tma_load_2d(w_tile(s), &tmW, &full[s], ks * C::BK, r0);
                    tma_load_2d(x_tile(s), &tmX, &full[s], ks * C::BK, t0);
                    ++issued;
                    if (ks == 0) {  // the scale panel is first needed by the epilogue: after the first stage
                        if (!wait_bar(&pempty[pb], ((it / PBUFS) & 1) ^ 1, abort)) {
                            ok = false;
                            break;
                        }
                        bar_expect_tx(&pfull[pb], uint32_t(L.sw_bytes + L.sx_bytes));
                        tma_load_2d(sw_pan(pb), &tmSW, &pfull[pb], r0, 0);
                        tma_load_2d(sx_pan(pb), &tmSX, &pfull[pb], t0, 0);
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
            constexpr uint32_t idesc = idesc_i8(C::BM, C::HALF);
            int g = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
                for (int ks = 0; ks < ksteps && ok; ++ks, ++g) {
                    const int s = g % STAGES;
                    if (!wait_bar(&full[s], (g / STAGES) & 1, abort)) {
                        ok = false;
                        break;
                    }
                    const int grp = g & 1;  // this stage's blocks use TMEM slots 4*grp .. 4*grp+3
                    if (!wait_bar(&acce[grp], ((g >> 1) & 1) ^ 1, abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t w_addr = smem_u32(w_tile(s)), x_addr = smem_u32(x_tile(s));
#pragma unroll
                    for (int kk = 0; kk < C::GROUP; ++kk) {
                        const int slot = grp * C::GROUP + kk;
                        const uint64_t wd = desc_sw128(w_addr + kk * 32);
#pragma unroll
                        for (int h = 0; h < 2; ++h)  // token half h: rows 32h.. of the token tile, 4 KB in
                            mma_i8(tmem + uint32_t(h * C::NBUF * C::HALF + slot * C::HALF), wd,
                                   desc_sw128(x_addr + h * C::HALF * 128 + kk * 32), idesc, 0u);
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
        // TMEM is released only after every epilogue warp has finished reading it.
        wait_bar(edone, 0, nullptr);
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    } else {
        // ------------------------------------------------------------ epilogue
        const int quad = warp & 3, half = (warp - 2) >> 2;
        const int r_local = quad * 32 + lane;
        const uint32_t tbase = tmem + (uint32_t(quad * 32) << 16) + uint32_t(half * C::NBUF * C::HALF);
        constexpr float BIAS = 12582912.0f;  // 1.5 * 2^23
        int blk = 0, it = 0;
        bool ok = true;

        // Blocks b, b+1 of a completed group into r (64 columns).
        auto load2 = [&](uint32_t(&r)[2 * C::HALF], int b) {
            tmem_ld64(tbase + uint32_t((b % C::NBUF) * C::HALF), r);
            tmem_wait_ld();
            reg_fence(r);
        };
        for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++it) {
            const int r0 = (tile / p.tiles_t) * C::BM, t0 = (tile % p.tiles_t) * C::BN;
            const int pb = it % PBUFS;
            if (!__all_sync(0xffffffffu, wait_bar(&pfull[pb], (it / PBUFS) & 1, abort))) break;
            const float *sw = sw_pan(pb) + r_local;  // ws of block j: sw[j * 128]
            const float4 *sx = reinterpret_cast<const float4 *>(sx_pan(pb) + half * C::HALF);  // xs: sx[j * 16 + c / 4]
            float2 acc[C::HALF / 2];
#pragma unroll
            for (int c = 0; c < C::HALF / 2; ++c) acc[c] = make_float2(0.0f, 0.0f);

            // Rescale and accumulate block j held in r.
            auto math = [&](const uint32_t(&r)[C::HALF], int j) {
                const float ws = sw[j * C::BM];
                const float2 w2 = make_float2(ws, ws), c2 = make_float2(-BIAS * ws, -BIAS * ws);
                const float4 *xs = sx + j * (C::BN / 4);
#pragma unroll
                for (int c4 = 0; c4 < C::HALF / 4; ++c4) {
                    const float4 x4 = xs[c4];
                    const uint32_t *d = r + 4 * c4;
                    const float2 xa = make_float2(__int_as_float(int(d[0]) + 0x4B400000),
                                                  __int_as_float(int(d[1]) + 0x4B400000));
                    const float2 xb = make_float2(__int_as_float(int(d[2]) + 0x4B400000),
                                                  __int_as_float(int(d[3]) + 0x4B400000));
                    const float2 ta = __ffma2_rn(xa, w2, c2), tb = __ffma2_rn(xb, w2, c2);
                    float2 &aa = acc[2 * c4], &ab = acc[2 * c4 + 1];
                    if (EXACT) {  // scalar _rn intrinsics are never contracted into an FMA
                        aa.x = __fadd_rn(aa.x, __fmul_rn(ta.x, x4.x));
                        aa.y = __fadd_rn(aa.y, __fmul_rn(ta.y, x4.y));
                        ab.x = __fadd_rn(ab.x, __fmul_rn(tb.x, x4.z));
                        ab.y = __fadd_rn(ab.y, __fmul_rn(tb.y, x4.w));
                    } else {
                        aa = __ffma2_rn(ta, make_float2(x4.x, x4.y), aa);
                        ab = __ffma2_rn(tb, make_float2(x4.z, x4.w), ab);
                    }
                }
            };

            // Per group of four blocks (one stage): one wait, two 64-column loads,
            // the group handed back to the MMA warp before the last two blocks
            // are rescaled from registers.  Kb is a multiple of 4.
            uint32_t r2[2 * C::HALF];
            for (int j = 0; j < Kb; j += C::GROUP, blk += C::GROUP) {
                const int grp = (blk / C::GROUP) & 1, use = blk / (2 * C::GROUP);
                if (!__all_sync(0xffffffffu, wait_bar(&accf[grp], use & 1, abort))) {  // tcgen05.ld is warp-collective
                    ok = false;
                    break;
                }
                tc_fence_after();
                load2(r2, blk);
                math(*reinterpret_cast<uint32_t(*)[C::HALF]>(r2), j);
                math(*reinterpret_cast<uint32_t(*)[C::HALF]>(r2 + C::HALF), j + 1);
                load2(r2, blk + 2);
                tc_fence_before();
                if (lane == 0) bar_arrive(&acce[grp]);
                math(*reinterpret_cast<uint32_t(*)[C::HALF]>(r2), j + 2);
                math(*reinterpret_cast<uint32_t(*)[C::HALF]>(r2 + C::HALF), j + 3);
            }
            __syncwarp();
            if (lane == 0) bar_arrive(&pempty[pb]);
            if (!ok) break;
            if (GEGLU) {
                // Pair gate (lanes 0..63) and up (lanes 64..127) of each output
                // column through shared memory G[token][row] (row stride GS,
                // padded against bank conflicts).  Then each lane pair owns one
                // (token, 32-column block) of the tile's 64 tokens x 64 output
                // columns: each lane computes g = gelu(gate) * up for 16
                // columns (16 independent chains), the pair exchanges its amax
                // with one shuffle, and each lane stores its 16 codes.
                constexpr int GS = C::BM + 1;
                float *G = reinterpret_cast<float *>(smem + L.gbuf());
#pragma unroll
                for (int c = 0; c < C::HALF / 2; ++c) {
                    const int tok = half * C::HALF + 2 * c;
                    G[tok * GS + r_local] = acc[c].x;
                    G[(tok + 1) * GS + r_local] = acc[c].y;
                }
                __syncwarp();
                if (lane == 0) bar_arrive(gfull);
                if (!__all_sync(0xffffffffu, wait_bar(gfull, it & 1, abort))) {
                    ok = false;
                    break;
                }
                const int u = ((warp - 2) * 32 + lane) >> 1, part = lane & 1;  // 128 units, 2 lanes each
                const int tok = u >> 1, cb = u & 1, t = t0 + tok, col0 = r0 / 2;
                const float *gr = G + tok * GS + cb * 32 + part * 16;
                int8_t *qo = p.q8 + size_t(t) * (p.R / 2) + col0 + cb * 32 + part * 16;
                float *so = p.q8s + size_t(col0 / 32 + cb) * p.q8s_stride + t;
                geglu_unit<TIER>(gr, part, t < p.T, qo, so);
                __syncwarp();
                if (lane == 0) bar_arrive(gdone);
                if (!__all_sync(0xffffffffu, wait_bar(gdone, it & 1, abort))) {  // G is rewritten next tile
                    ok = false;
                    break;
                }
                continue;
            }
            // out[t][r]: for each token the warp's 32 lanes write 128 consecutive bytes.
            float *o = p.out + size_t(t0 + half * C::HALF) * p.ldo + r0 + r_local;
            const int tmax = p.T - (t0 + half * C::HALF);
#pragma unroll
            for (int c = 0; c < C::HALF / 2; ++c) {
                if (2 * c < tmax) o[size_t(2 * c) * p.ldo] = acc[c].x;
                if (2 * c + 1 < tmax) o[size_t(2 * c + 1) * p.ldo] = acc[c].y;
            }
        }
        __syncwarp();
        tc_fence_before();
        if (lane == 0) bar_arrive(edone);
    }
}

}  // namespace eg2
