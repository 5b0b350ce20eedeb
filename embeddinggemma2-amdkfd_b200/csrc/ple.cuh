// Per-layer-embedding projection on tcgen05 kind::f16 (bf16 operands, fp32
// accumulation in TMEM), with the scale and RMS normalisation fused into the
// epilogue:
//     ple[t][l][:] = rms(x[t] . W[l*512 .. l*512+511]^T / sqrt(512)) * w
// (vendor/embeddinggemma.c/src/gemma2_fast.c:951-956).  The reference multiplies
// fp32 activations by BF16 weights; here x is split as x ~= hi + lo with
// hi = bf16(x), lo = bf16(x - hi) (relative error < 2^-17), and both halves are
// multiplied by the same BF16 weight tile: the products are exact in the fp32
// accumulator.
//
// CTA tile: 128 tokens x one 512-wide PLE slice (two N=256 MMAs), K = 512 in
// 8 stages of 64 bf16 (128-byte swizzled rows).  Warp 0 TMA, warp 1 MMA,
// warps 2..9 epilogue (quadrant = warp % 4, column half = (warp-2)/4).
#pragma once
#include "common.cuh"

namespace eg2 {

struct PleParams {
    float *ple;         // [n][24*512]
    const float *norm;  // per_layer_proj_norm [512]
    int M;
};

struct PleCfg {
    static constexpr int BM = 128, BN = 512, BK = 64, K = 512, STAGES = 2, EPI_WARPS = 8;
    static constexpr int THREADS = (2 + EPI_WARPS) * 32;
    static constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = 2 * A_BYTES + B_BYTES;  // hi, lo, weights
    static constexpr size_t SMEM = 1024 + size_t(STAGES) * STAGE_BYTES + 2 * BM * 8 + 256;
};

__global__ void __launch_bounds__(PleCfg::THREADS, 1)
    ple_kernel(const __grid_constant__ CUtensorMap tmHi, const __grid_constant__ CUtensorMap tmLo,
               const __grid_constant__ CUtensorMap tmW, const PleParams p) {
    using C = PleCfg;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = align_smem_1024(smem_raw);
    double *partial = reinterpret_cast<double *>(smem + C::STAGES * C::STAGE_BYTES);  // [2][128]
    uint64_t *full = reinterpret_cast<uint64_t *>(partial + 2 * C::BM);
    uint64_t *empty = full + C::STAGES;
    uint64_t *accf = empty + C::STAGES, *edone = accf + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(edone + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * C::BM, slice = blockIdx.x;
    auto hi_tile = [&](int s) { return smem + s * C::STAGE_BYTES; };
    auto lo_tile = [&](int s) { return smem + s * C::STAGE_BYTES + C::A_BYTES; };
    auto w_tile = [&](int s) { return smem + s * C::STAGE_BYTES + 2 * C::A_BYTES; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) bar_init(&full[s], 1), bar_init(&empty[s], 1);
        bar_init(accf, 1), bar_init(edone, C::EPI_WARPS);
        fence_bar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    pdl_wait();  // the prologue above overlaps the previous kernel's tail
    pdl_trigger();
    if (threadIdx.x == 0) *abort = 0;
    tc_fence_before();
    cta_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    constexpr int KSTEPS = C::K / C::BK;

    if (warp == 0) {
        if (elect_one() && !*abort) {
            tma_prefetch(&tmHi);
            tma_prefetch(&tmLo);
            tma_prefetch(&tmW);
            int issued = 0;
            for (int ks = 0; ks < KSTEPS; ++ks, ++issued) {
                const int s = ks % C::STAGES;
                if (!wait_bar(&empty[s], ((ks / C::STAGES) & 1) ^ 1, abort)) break;
                bar_expect_tx(&full[s], C::STAGE_BYTES);
                tma_load_2d(hi_tile(s), &tmHi, &full[s], ks * C::BK, m0);
                tma_load_2d(lo_tile(s), &tmLo, &full[s], ks * C::BK, m0);
                tma_load_2d(w_tile(s), &tmW, &full[s], ks * C::BK, slice * C::BN);
                tma_load_2d(w_tile(s) + C::B_BYTES / 2, &tmW, &full[s], ks * C::BK, slice * C::BN + 256);
            }
            for (int ks = issued > C::STAGES ? issued - C::STAGES : 0; ks < issued; ++ks)
                wait_bar(&full[ks % C::STAGES], (ks / C::STAGES) & 1, nullptr);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (elect_one() && !*abort) {
            constexpr uint32_t idesc = idesc_bf16(128, 256);
            for (int ks = 0; ks < KSTEPS; ++ks) {
                const int s = ks % C::STAGES;
                if (!wait_bar(&full[s], (ks / C::STAGES) & 1, abort)) break;
                tc_fence_after();
                const uint32_t hi = smem_u32(hi_tile(s)), lo = smem_u32(lo_tile(s)), w = smem_u32(w_tile(s));
#pragma unroll
                for (int kk = 0; kk < C::BK / 16; ++kk) {
#pragma unroll
                    for (int nh = 0; nh < 2; ++nh) {
                        const uint64_t bd = desc_sw128(w + nh * (C::B_BYTES / 2) + kk * 32);
                        mma_f16(tmem + nh * 256, desc_sw128(hi + kk * 32), bd, idesc, (ks | kk) ? 1u : 0u);
                        mma_f16(tmem + nh * 256, desc_sw128(lo + kk * 32), bd, idesc, 1u);
                    }
                }
                tc_commit(&empty[s]);
            }
            tc_commit(accf);
            wait_bar(accf, 0, nullptr);
        }
        __syncwarp();
        // TMEM is released only after every epilogue warp has finished reading it.
        wait_bar(edone, 0, nullptr);
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    } else {
        const int quad = warp & 3, half = (warp - 2) >> 2;
        const int row = quad * 32 + lane, colbase = half * 256;
        const uint32_t taddr = tmem + (uint32_t(quad * 32) << 16) + uint32_t(colbase);
        const bool ok = __all_sync(0xffffffffu, wait_bar(accf, 0, abort));  // warp-uniform before tcgen05.ld
        tc_fence_after();
        auto scaled = [](uint32_t bits) { return div_sqrt512(__uint_as_float(bits)); };  // = v / sqrtf(512)
        double ss = 0.0;
        if (ok) {
            double s4[4] = {0.0, 0.0, 0.0, 0.0};
            for (int c = 0; c < 256; c += 32) {
                uint32_t d[32];
                tmem_ld32(taddr + uint32_t(c), d);
                tmem_wait_ld();
                reg_fence(d);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const double v = double(scaled(d[i]));
                    s4[i & 3] = __dadd_rn(s4[i & 3], __dmul_rn(v, v));
                }
            }
            ss = __dadd_rn(__dadd_rn(s4[0], s4[1]), __dadd_rn(s4[2], s4[3]));
        }
        partial[half * C::BM + row] = ss;
        named_sync(1, C::EPI_WARPS * 32);
        const float scale = rms_scale(partial[row] + partial[C::BM + row], 512);
        if (ok) {
            // Each 32-column chunk of the warp's 32 token rows goes through a
            // padded shared-memory tile (the stage buffers are free once every MMA
            // has completed) so that each store instruction writes four whole
            // 128-byte row segments.
            float *st = reinterpret_cast<float *>(smem) + (warp - 2) * (32 * 33);
            const int srow = lane >> 3, scol = (lane & 7) * 4;
            const float *w = p.norm + colbase;
            for (int c = 0; c < 256; c += 32) {
                uint32_t d[32];
                tmem_ld32(taddr + uint32_t(c), d);
                tmem_wait_ld();
                reg_fence(d);
#pragma unroll
                for (int i = 0; i < 32; ++i) st[lane * 33 + i] = __fmul_rn(scaled(d[i]), __fmul_rn(scale, w[c + i]));
                __syncwarp();
#pragma unroll
                for (int rr = 0; rr < 32; rr += 4) {
                    const int r = rr + srow, m = m0 + quad * 32 + r;
                    const float *src = st + r * 33 + scol;
                    if (m < p.M)
                        *reinterpret_cast<float4 *>(p.ple + size_t(m) * (24 * 512) + slice * 512 + colbase + c + scol) =
                            make_float4(src[0], src[1], src[2], src[3]);
                }
                __syncwarp();
            }
        }
        __syncwarp();
        tc_fence_before();
        if (lane == 0) bar_arrive(edone);
    }
}

}  // namespace eg2
