// Q8_0 x Q8_0 GEMM on the 5th-generation tensor cores (tcgen05 kind::i8).
//
// out[t][r] = sum_b D_b[t][r] * xs[b][t] * ws[b][r],  D_b = int32 dot of the
// 32-element block b of activation row t and weight row r -- the reference's
// gemm_q8 (vendor/embeddinggemma.c/src/gemma2_fast.c:242-253, scalar tile
// :193-204).  One tcgen05.mma with K = 32 is exactly one Q8_0 block, so each
// block's int32 dot lands exactly in its own TMEM buffer; the epilogue warps
// rescale and accumulate in fp32 registers, blocks in ascending order:
//     t   = round(D_b * ws)            (one FMA, see below)
//     acc = acc + round(t * xs)        EXACT: the reference scalar tile's order,
//                                      ((float)dot * dw) * dx then sum +=
//     acc = fma(t, xs, acc)            otherwise (one rounding fewer)
// The int32 -> fp32 conversion uses the exact bias trick: with
// B = 1.5 * 2^23, the bits of D + 0x4B400000 are the float B + D for
// |D| < 2^22 (|D| <= 32 * 128 * 128 here), and fma(B + D, ws, -B * ws) rounds
// (B + D) * ws - B * ws = D * ws once; -B * ws is exact because ws is an fp16
// value.  So D * ws costs one integer add and one FMA, computed in pairs with
// fma.rn.f32x2.
//
// Persistent CTAs (one per SM) walk the 128 x 64 output tiles; warp roles:
//   warp 0      TMA producer: per tile the scale panels (activation scales
//               [K/32][128], weight scales [K/32][64]) into a double buffer, then
//               int8 A/B tiles of 128 B (one 128-byte swizzle row) per stage;
//   warp 1      TMEM owner and MMA issuer: each Q8 block j is four N=16 MMAs,
//               one per 16-column sub-tile q, into TMEM columns
//               q*128 + (j % 8)*16; commit -> acc_full[j % 8];
//   warps 2..17 epilogue: warp w reads TMEM lanes 32*(w%4).. (its hardware
//               quadrant) of sub-tile q = (w-2)/4.
// Because a sub-tile's eight block slots are adjacent TMEM columns, one
// 32-column tcgen05.ld brings a warp the accumulators of two consecutive
// blocks: the load latency that follows an MMA's completion is paid once per
// two blocks instead of once per block.  The stage ring, TMEM slots and panel
// buffers continue across tiles, so loads and MMAs of the next tile overlap the
// epilogue of the current one.
#pragma once
#include "common.cuh"

namespace eg2 {

struct Q8GemmParams {
    float *out;  // [M][ldo] fp32
    int ldo;
    int M, N, K;
    int tiles_n, num_tiles;
};

template <int BN>
struct Q8Cfg {
    static constexpr int BM = 128, BK = 128, STAGES = 4, CW = 16, NSUB = BN / CW, NBUF = 512 / BN;
    static constexpr int GRP = 2;  // blocks fetched by one epilogue TMEM load (registers: 18 warps -> 96/thread)
    static constexpr int EPI_WARPS = 4 * (BN / CW), EPI_THREADS = EPI_WARPS * 32;
    static constexpr int THREADS = (2 + EPI_WARPS) * 32;
    static constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, STAGE_BYTES = A_BYTES + B_BYTES;
    static_assert(BN == 64, "tuned for N = 64: 8 TMEM accumulator buffers, 16 epilogue warps");
};

// Shared-memory plan (offsets from the 1024-aligned base) for BN and K.
struct Q8Smem {
    int stages, pbufs, kb;
    size_t stage_bytes, sa_bytes, sb_bytes, prep_bytes, panel_bytes, total;
    __host__ __device__ size_t panel(int b) const { return size_t(stages) * stage_bytes + size_t(b) * panel_bytes; }
    __host__ __device__ size_t bars() const { return size_t(stages) * stage_bytes + size_t(pbufs) * panel_bytes; }
};
__host__ __device__ inline Q8Smem q8gemm_smem(int bn, int K) {
    Q8Smem s;
    s.stages = 4;
    s.kb = K / 32;
    s.stage_bytes = size_t(128) * 128 + size_t(bn) * 128;
    s.sa_bytes = size_t(s.kb) * 128 * 4;
    s.sb_bytes = size_t(s.kb) * bn * 4;
    s.prep_bytes = size_t(s.kb) * bn * 8;  // {ws pair, -B*ws pair} per column pair
    s.panel_bytes = (s.sa_bytes + s.sb_bytes + s.prep_bytes + 1023) / 1024 * 1024;
    const size_t limit = 227 * 1024, fixed = 1024 + 512;
    s.pbufs = 2;
    if (fixed + 4 * s.stage_bytes + 2 * s.panel_bytes > limit) s.pbufs = 1;
    if (fixed + 4 * s.stage_bytes + s.pbufs * s.panel_bytes > limit) s.stages = 3;
    s.total = fixed + size_t(s.stages) * s.stage_bytes + size_t(s.pbufs) * s.panel_bytes;
    return s;
}

template <int BN, bool EXACT>
__global__ void __launch_bounds__(Q8Cfg<BN>::THREADS, 1)
    q8gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmSA, const __grid_constant__ CUtensorMap tmSB,
                  const Q8GemmParams p) {
    using C = Q8Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = align_smem_1024(smem_raw);
    const Q8Smem L = q8gemm_smem(BN, p.K);
    const int Kb = L.kb, ksteps = p.K / C::BK, STAGES = L.stages, PBUFS = L.pbufs;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars());
    uint64_t *full = bars, *empty = bars + 4, *accf = bars + 8, *acce = accf + C::NBUF;
    uint64_t *pfull = acce + C::NBUF, *pempty = pfull + 2, *pprep = pempty + 2, *mdone = pprep + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mdone + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    auto a_tile = [&](int s) { return smem + size_t(s) * L.stage_bytes; };
    auto b_tile = [&](int s) { return smem + size_t(s) * L.stage_bytes + C::A_BYTES; };
    auto sa_pan = [&](int b) { return reinterpret_cast<float *>(smem + L.panel(b)); };
    auto sb_pan = [&](int b) { return reinterpret_cast<float *>(smem + L.panel(b) + L.sa_bytes); };
    auto prep_pan = [&](int b) { return reinterpret_cast<float4 *>(smem + L.panel(b) + L.sa_bytes + L.sb_bytes); };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) bar_init(&full[s], 1), bar_init(&empty[s], 1);
        for (int b = 0; b < C::NBUF; ++b) bar_init(&accf[b], 1), bar_init(&acce[b], C::EPI_WARPS);
        for (int b = 0; b < PBUFS; ++b)
            bar_init(&pfull[b], 1), bar_init(&pempty[b], C::EPI_WARPS), bar_init(&pprep[b], C::EPI_WARPS);
        bar_init(mdone, 1);
        *abort = g_error != 0;
        fence_bar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (elect_one() && !*abort) {
            tma_prefetch(&tmA), tma_prefetch(&tmB), tma_prefetch(&tmSA), tma_prefetch(&tmSB);
            int g = 0, issued = 0, it = 0, panels = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++it) {
                const int m0 = (tile / p.tiles_n) * C::BM, n0 = (tile % p.tiles_n) * BN;
                const int pb = it % PBUFS;
                if (!wait_bar(&pempty[pb], ((it / PBUFS) & 1) ^ 1, abort)) break;
                bar_expect_tx(&pfull[pb], uint32_t(L.sa_bytes + L.sb_bytes));
                tma_load_2d(sa_pan(pb), &tmSA, &pfull[pb], m0, 0);
                tma_load_2d(sb_pan(pb), &tmSB, &pfull[pb], n0, 0);
                ++panels;
                for (int ks = 0; ks < ksteps; ++ks, ++g) {
                    const int s = g % STAGES;
                    if (!wait_bar(&empty[s], ((g / STAGES) & 1) ^ 1, abort)) {
                        ok = false;
                        break;
                    }
                    bar_expect_tx(&full[s], C::STAGE_BYTES);
                    tma_load_2d(a_tile(s), &tmA, &full[s], ks * C::BK, m0);
                    tma_load_2d(b_tile(s), &tmB, &full[s], ks * C::BK, n0);
                    ++issued;
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
            constexpr uint32_t idesc = idesc_i8(128, C::CW);
            int g = 0, blk = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
                for (int ks = 0; ks < ksteps && ok; ++ks, ++g) {
                    const int s = g % STAGES;
                    if (!wait_bar(&full[s], (g / STAGES) & 1, abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(a_tile(s)), b_addr = smem_u32(b_tile(s));
#pragma unroll
                    for (int kk = 0; kk < C::BK / 32; ++kk, ++blk) {
                        const int buf = blk % C::NBUF;
                        if (!wait_bar(&acce[buf], ((blk / C::NBUF) & 1) ^ 1, abort)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint64_t ad = desc_sw128(a_addr + kk * 32);
#pragma unroll
                        for (int q = 0; q < C::NSUB; ++q)  // sub-tile q: weight rows 16q.., 2 KB into the B tile
                            mma_i8(tmem + uint32_t(q * C::NBUF * C::CW + buf * C::CW), ad,
                                   desc_sw128(b_addr + q * C::CW * 128 + kk * 32), idesc, 0u);
                        tc_commit(&accf[buf]);
                    }
                    tc_commit(&empty[s]);
                }
            }
            // Drain: every MMA issued above has completed before TMEM is freed.
            tc_commit(mdone);
            wait_bar(mdone, 0, nullptr);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue
        const int ew = warp - 2, quad = warp & 3, sub = ew >> 2;
        const int row = quad * 32 + lane, colbase = sub * C::CW;
        const uint32_t taddr = tmem + (uint32_t(quad * 32) << 16) + uint32_t(sub * C::NBUF * C::CW);
        const int et = threadIdx.x - 64;  // 0 .. EPI_THREADS-1
        constexpr float BIAS = 12582912.0f;  // 1.5 * 2^23
        int blk = 0, it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++it) {
            const int m0 = (tile / p.tiles_n) * C::BM, n0 = (tile % p.tiles_n) * BN;
            const int pb = it % PBUFS;
            if (!__all_sync(0xffffffffu, wait_bar(&pfull[pb], (it / PBUFS) & 1, abort))) break;
            // Column constants of this tile: {ws[c], ws[c+1], -B*ws[c], -B*ws[c+1]} per pair.
            {
                const float *sb = sb_pan(pb);
                float4 *prep = prep_pan(pb);
                for (int i = et; i < Kb * BN / 2; i += C::EPI_THREADS) {
                    const int j = i / (BN / 2), c2 = i % (BN / 2);
                    const float w0 = sb[j * BN + 2 * c2], w1 = sb[j * BN + 2 * c2 + 1];
                    prep[i] = make_float4(w0, w1, -BIAS * w0, -BIAS * w1);
                }
                // Bounded barrier among the epilogue warps (an mbarrier, not bar.sync, so
                // that a warp leaving on a timeout cannot strand the others).
                __syncwarp();
                if (lane == 0) bar_arrive(&pprep[pb]);
                if (!__all_sync(0xffffffffu, wait_bar(&pprep[pb], (it / PBUFS) & 1, abort))) break;
            }
            const float *sa_p = sa_pan(pb);
            const float4 *prep = prep_pan(pb) + colbase / 2;
            float2 acc[C::CW / 2];
#pragma unroll
            for (int c = 0; c < C::CW / 2; ++c) acc[c] = make_float2(0.0f, 0.0f);
            // One 32-column TMEM load per two blocks (GRP); the per-block column
            // constants are read after the load completed, so no shared-memory
            // access queues behind an outstanding TMEM load.
            for (int j = 0; j < Kb && ok; j += C::GRP) {
                bool ready = true;
#pragma unroll
                for (int g = 0; g < C::GRP; ++g)
                    ready = ready && wait_bar(&accf[(blk + g) % C::NBUF], ((blk + g) / C::NBUF) & 1, abort);
                // tcgen05.ld is warp-collective: decide as a whole warp.
                if (!__all_sync(0xffffffffu, ready)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t d[C::GRP * C::CW];
                tmem_ld32(taddr + uint32_t((blk % C::NBUF) * C::CW), d);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
#pragma unroll
                    for (int g = 0; g < C::GRP; ++g) bar_arrive(&acce[(blk + g) % C::NBUF]);
                }
#pragma unroll
                for (int g = 0; g < C::GRP; ++g) {
                    const float sa = sa_p[(j + g) * C::BM + row];
                    const float2 sa2 = make_float2(sa, sa);
                    const float4 *pj = prep + (j + g) * (BN / 2);
#pragma unroll
                    for (int c = 0; c < C::CW / 2; ++c) {
                        const float4 w = pj[c];
                        const uint32_t *dc = d + g * C::CW;
                        const float2 x = make_float2(__int_as_float(int(dc[2 * c]) + 0x4B400000),
                                                     __int_as_float(int(dc[2 * c + 1]) + 0x4B400000));
                        const float2 t = __ffma2_rn(x, make_float2(w.x, w.y), make_float2(w.z, w.w));
                        if (EXACT) {  // scalar _rn intrinsics are never contracted into an FMA
                            acc[c].x = __fadd_rn(acc[c].x, __fmul_rn(t.x, sa));
                            acc[c].y = __fadd_rn(acc[c].y, __fmul_rn(t.y, sa));
                        } else {
                            acc[c] = __ffma2_rn(t, sa2, acc[c]);
                        }
                    }
                }
                blk += C::GRP;
            }
            __syncwarp();
            if (lane == 0) bar_arrive(&pempty[pb]);
            const int m = m0 + row;
            if (ok && m < p.M) {
                float4 *o = reinterpret_cast<float4 *>(p.out + size_t(m) * p.ldo + n0 + colbase);
#pragma unroll
                for (int c = 0; c < C::CW / 4; ++c)
                    o[c] = make_float4(acc[2 * c].x, acc[2 * c].y, acc[2 * c + 1].x, acc[2 * c + 1].y);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace eg2
