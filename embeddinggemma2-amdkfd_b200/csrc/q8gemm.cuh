// Q8_0 x Q8_0 GEMM on the 5th-generation tensor cores (tcgen05 kind::i8).
//
// out[t][r] = sum_b D_b[t][r] * xs[b][t] * ws[b][r],  D_b = int32 dot of the
// 32-element block b of activation row t and weight row r -- the reference's
// gemm_q8 (vendor/embeddinggemma.c/src/gemma2_fast.c:242-253, scalar tile
// :193-204).  One tcgen05.mma with K = 32 is exactly one Q8_0 block, so each
// block's int32 dot lands exactly (no rounding) in its own TMEM buffer; the
// epilogue warps convert, scale by the two fp16-exact block scales and
// accumulate in fp32 registers, in ascending block order.
//
// CTA tile 128 tokens x BN weight rows.  Warp roles:
//   warp 0       TMA producer: int8 tiles [128 x 128 B] of A and [BN x 128 B] of
//                B per stage, 128-byte swizzle, STAGES-deep ring;
//   warp 1       TMEM owner and MMA issuer (one elected lane): 4 MMAs per stage,
//                block j into TMEM buffer j % NBUF, commit -> acc_full[buf];
//   warps 2..9   epilogue: warp w reads TMEM lanes 32*(w%4).. (its hardware
//                quadrant) and half (w-2)/4 of the BN columns.
// The scale panels of the tile (activations [Kb][128], weights [Kb][BN]) are
// staged in shared memory once per CTA.
#pragma once
#include "common.cuh"

namespace eg2 {

struct Q8GemmParams {
    const float *sa;  // activation block scales, [K/32][sa_stride]
    int sa_stride;
    const float *sb;  // weight block scales, [K/32][N]
    float *out;       // [M][ldo] fp32
    int ldo;
    int M, N, K;
};

template <int BN>
struct Q8Cfg {
    static constexpr int BM = 128, BK = 128, STAGES = 4, NBUF = 4;
    static constexpr int EPI_WARPS = 8, THREADS = (2 + EPI_WARPS) * 32;
    static constexpr int CW = BN / 2;  // columns per epilogue thread
    static constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = NBUF * BN;
    static_assert(BN == 64 || BN == 128, "BN");
    static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation must be a power of two");
};

__host__ __device__ inline size_t q8gemm_smem_bytes(int bn, int K) {
    const int kb = K / 32;
    return 1024 /*alignment slack*/ + size_t(4) * (128 * 128 + bn * 128) + size_t(kb) * 128 * 4 +
           size_t(kb) * bn * 4 + 256;
}

template <int BN>
__global__ void __launch_bounds__(Q8Cfg<BN>::THREADS, 1)
    q8gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const Q8GemmParams p) {
    using C = Q8Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int Kb = p.K / 32, ksteps = p.K / C::BK;
    float *sa_s = reinterpret_cast<float *>(smem + C::STAGES * C::STAGE_BYTES);
    float *sb_s = sa_s + Kb * C::BM;
    uint64_t *full = reinterpret_cast<uint64_t *>(sb_s + Kb * BN);
    uint64_t *empty = full + C::STAGES;
    uint64_t *accf = empty + C::STAGES;
    uint64_t *acce = accf + C::NBUF;
    uint64_t *mdone = acce + C::NBUF;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mdone + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * C::BM, n0 = blockIdx.x * BN;
    auto a_tile = [&](int s) { return smem + s * C::STAGE_BYTES; };
    auto b_tile = [&](int s) { return smem + s * C::STAGE_BYTES + C::A_BYTES; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) bar_init(&full[s], 1), bar_init(&empty[s], 1);
        for (int b = 0; b < C::NBUF; ++b) bar_init(&accf[b], 1), bar_init(&acce[b], C::EPI_WARPS);
        bar_init(mdone, 1);
        *abort = g_error != 0;
        fence_bar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    // Scale panels of this tile (coalesced rows of the block-major planes).
    for (int i = threadIdx.x; i < Kb * C::BM; i += C::THREADS) {
        const int j = i / C::BM, r = i % C::BM;
        sa_s[i] = (m0 + r < p.M) ? p.sa[size_t(j) * p.sa_stride + m0 + r] : 0.0f;
    }
    for (int i = threadIdx.x; i < Kb * BN; i += C::THREADS) {
        const int j = i / BN, c = i % BN;
        sb_s[i] = p.sb[size_t(j) * p.N + n0 + c];
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (elect_one() && !*abort) {
            tma_prefetch(&tmA);
            tma_prefetch(&tmB);
            int issued = 0;
            for (int ks = 0; ks < ksteps; ++ks, ++issued) {
                const int s = ks % C::STAGES;
                const uint32_t ph = (ks / C::STAGES) & 1;
                if (!wait_bar(&empty[s], ph ^ 1, abort)) break;
                bar_expect_tx(&full[s], C::STAGE_BYTES);
                tma_load_2d(a_tile(s), &tmA, &full[s], ks * C::BK, m0);
                tma_load_2d(b_tile(s), &tmB, &full[s], ks * C::BK, n0);
            }
            // Drain: the last load into each stage has landed before exit.
            for (int ks = issued > C::STAGES ? issued - C::STAGES : 0; ks < issued; ++ks)
                wait_bar(&full[ks % C::STAGES], (ks / C::STAGES) & 1, nullptr);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (elect_one() && !*abort) {
            constexpr uint32_t idesc = idesc_i8(128, BN);
            int blk = 0;
            bool ok = true;
            for (int ks = 0; ks < ksteps && ok; ++ks) {
                const int s = ks % C::STAGES;
                const uint32_t ph = (ks / C::STAGES) & 1;
                if (!wait_bar(&full[s], ph, abort)) break;
                tc_fence_after();
                const uint32_t a_addr = smem_u32(a_tile(s)), b_addr = smem_u32(b_tile(s));
#pragma unroll
                for (int kk = 0; kk < C::BK / 32; ++kk, ++blk) {
                    const int buf = blk % C::NBUF;
                    const uint32_t bph = (blk / C::NBUF) & 1;
                    if (!wait_bar(&acce[buf], bph ^ 1, abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    mma_i8(tmem + uint32_t(buf * BN), desc_sw128(a_addr + kk * 32), desc_sw128(b_addr + kk * 32),
                           idesc, 0u);
                    tc_commit(&accf[buf]);
                }
                tc_commit(&empty[s]);
            }
            // Drain: every MMA issued above has completed before TMEM is freed.
            tc_commit(mdone);
            wait_bar(mdone, 0, nullptr);
        }
        __syncwarp();
    } else {
        const int ew = warp - 2, quad = warp & 3, half = ew >> 2;
        const int row = quad * 32 + lane, colbase = half * C::CW;
        const uint32_t taddr = tmem + (uint32_t(quad * 32) << 16) + uint32_t(colbase);
        float acc[C::CW];
#pragma unroll
        for (int c = 0; c < C::CW; ++c) acc[c] = 0.0f;
        bool ok = true;
        for (int blk = 0; blk < Kb; ++blk) {
            const int buf = blk % C::NBUF;
            const uint32_t bph = (blk / C::NBUF) & 1;
            // tcgen05.ld is warp-collective: leave the loop as a whole warp.
            if (!__all_sync(0xffffffffu, wait_bar(&accf[buf], bph, abort))) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t d[C::CW];
#pragma unroll
            for (int c = 0; c < C::CW; c += 32) tmem_ld32(taddr + uint32_t(buf * BN + c), &d[c]);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&acce[buf]);
            const float sa = sa_s[blk * C::BM + row];
            const float4 *sb4 = reinterpret_cast<const float4 *>(sb_s + blk * BN + colbase);
#pragma unroll
            for (int c = 0; c < C::CW; c += 4) {
                const float4 s4 = sb4[c / 4];
                acc[c + 0] = __fmaf_rn(float(int32_t(d[c + 0])), __fmul_rn(sa, s4.x), acc[c + 0]);
                acc[c + 1] = __fmaf_rn(float(int32_t(d[c + 1])), __fmul_rn(sa, s4.y), acc[c + 1]);
                acc[c + 2] = __fmaf_rn(float(int32_t(d[c + 2])), __fmul_rn(sa, s4.z), acc[c + 2]);
                acc[c + 3] = __fmaf_rn(float(int32_t(d[c + 3])), __fmul_rn(sa, s4.w), acc[c + 3]);
            }
        }
        const int m = m0 + row;
        if (ok && m < p.M) {
            float4 *o = reinterpret_cast<float4 *>(p.out + size_t(m) * p.ldo + n0 + colbase);
#pragma unroll
            for (int c = 0; c < C::CW; c += 4) o[c / 4] = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

}  // namespace eg2
