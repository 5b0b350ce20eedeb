// Packed-varlen bidirectional GQA attention for d = 256 on the 5th-generation
// tensor cores -- the reference's attention_rows
// (vendor/embeddinggemma.c/src/gemma2_fast.c:768-894) for the sliding-window
// layers: for token t and head h, keys s in [lo_t, hi_t) of its own sequence,
// intersected with [t - window, t + window]; KV head h / 2; scale 1.
//
// A CTA owns 128 query tokens of one head (the TMEM lanes).  Per key block of 64:
//   S = Q . K^T         tcgen05.mma kind::f16, M = 128, N = 64, K = 256, fp32 in TMEM
//   softmax             one thread per query row reads its 64 scores from TMEM and
//                       writes P (fp16, packed in pairs) back over the first 32
//                       columns of the same S stage
//   O += P . V          A = P from TMEM, B = V as an MN-major shared-memory
//                       operand, M = 128, N = 256, K = 64, fp32 accumulator in TMEM
// TMEM: S/P stages at columns 0, 64, 128; O at 256..511.  The MMA warp keeps S
// two blocks ahead (S0 S1 PV0 S2 PV1 S3 ...), so the softmax of block j never
// waits for its scores, and P needs no shared memory, proxy fence or buffer of
// its own.  K and V have separate double-buffered stages: K(j+2) loads as soon
// as S(j) completed, V(j+2) once P.V(j) did.
// Warps: 0 TMA for Q and K, 6 TMA for V, 1 TMEM owner and MMA issuer, 2..5
// softmax and epilogue (TMEM lane quadrant = warp % 4; fp32 rows leave through
// a padded shared-memory tile as whole 128-byte segments).  With a Q8 output
// each thread quantizes its row's eight 32-element blocks straight from the
// accumulator: the block scale and codes are those the row quantizer computes
// from the same fp32 values, so the fp32 row never goes to memory.
//
// Online softmax with a lazily updated reference maximum: a row's weights are
// 2^(s log2e - m log2e) against its running reference m; when a block raises
// the row maximum by more than 8 (natural log), O and the row sum are rescaled
// by exp(m_old - m_new) in TMEM and m moves, so P <= e^8 always fits fp16.  O
// is only touched (after the previous P.V completed) on such a move, and not
// for a row whose first key this is (its O and sum are still zero).
//
// Key blocks start at multiples of 64 from the start of each sequence in the
// tile, and a block's keys past its sequence's end are masked (they are counted
// in the next sequence's own blocks), so a row's keys are grouped and summed
// the same way wherever its sequence sits in the packed wave (packed and solo
// results are identical).  Q, K and V are addressed through 3-D tensor maps
// (element, head, token), the token being an outer coordinate.
#pragma once
#include "common.cuh"

namespace eg2 {

struct AttnTcParams {
    float *out;              // [n][4][256] fp32 (when q is null)
    const unsigned *bounds;  // [n][2] = sequence [lo, hi)
    int n, window;
    // Optional Q8_0 output instead of out (ROW_QUANT of the attention row,
    // gemma2_fast.c:728-730, fused): codes [n][1024], scales block-major
    // [32][q_stride]; quantizer rounding of `tier`.
    int8_t *q;
    float *qs;
    int q_stride, tier;
};

struct AttnTcCfg {
    static constexpr int D = 256, BQ = 128, BKEY = 64, KV_STAGES = 2, S_STAGES = 3, MAXB = 256;
    static constexpr int THREADS = 7 * 32;
    static constexpr int Q_BYTES = BQ * D * 2;    // 4 K-chunks of [128 rows][128 B]
    static constexpr int K_BYTES = BKEY * D * 2;  // 4 K-chunks of [64 rows][128 B]
    static constexpr int V_BYTES = BKEY * D * 2;  // 4 d-chunks of [64 keys][128 B] (MN-major)
    static constexpr size_t K_OFF = Q_BYTES, V_OFF = K_OFF + size_t(KV_STAGES) * K_BYTES;
    static constexpr size_t BLK_OFF = V_OFF + size_t(KV_STAGES) * V_BYTES;
    static constexpr size_t SMEM = 1024 + BLK_OFF + MAXB * 8 + 256;
    static constexpr float RESCALE = 8.0f;
    static constexpr uint32_t O_COL = 256;
};

template <int D_ = 256>
__global__ void __launch_bounds__(AttnTcCfg::THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const AttnTcParams p) {
    using C = AttnTcCfg;
    static_assert(D_ == C::D, "d = 256 only");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = align_smem_1024(smem_raw);
    uint8_t *qs = smem;
    int2 *blocks = reinterpret_cast<int2 *>(smem + C::BLK_OFF);  // (first key, sequence end)
    uint64_t *bars = reinterpret_cast<uint64_t *>(blocks + C::MAXB);
    uint64_t *qfull = bars, *kfull = bars + 1, *kempty = kfull + 2, *vfull = kempty + 2, *vempty = vfull + 2;
    uint64_t *sfull = vempty + 2, *pfull = sfull + 3, *pvdone = pfull + 3, *edone = pvdone + 3, *mdone = edone + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mdone + 1);
    int *nblocks = reinterpret_cast<int *>(tmem_slot + 1);
    volatile int *abort = nblocks + 1;
    auto k_tile = [&](int s) { return smem + C::K_OFF + s * C::K_BYTES; };
    auto v_tile = [&](int s) { return smem + C::V_OFF + s * C::V_BYTES; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * C::BQ, head = blockIdx.y, kh = head / 2;
    // Block j's K (V) into stage j & 1; the caller has made sure the stage is free.
    auto load_k = [&](int j) {
        const int s = j & 1;
        bar_expect_tx(&kfull[s], C::K_BYTES);
        for (int c = 0; c < 4; ++c)
            tma_load_3d(k_tile(s) + c * (C::K_BYTES / 4), &tmK, &kfull[s], c * 64, kh, blocks[j].x);
    };
    auto load_v = [&](int j) {
        const int s = j & 1;
        bar_expect_tx(&vfull[s], C::V_BYTES);
        for (int c = 0; c < 4; ++c)
            tma_load_3d(v_tile(s) + c * (C::V_BYTES / 4), &tmV, &vfull[s], c * 64, kh, blocks[j].x);
    };
    if (threadIdx.x == 0) {
        tma_prefetch(&tmQ), tma_prefetch(&tmK), tma_prefetch(&tmV);
        *abort = 0;
        bar_init(qfull, 1), bar_init(edone, 4), bar_init(mdone, 1);
        for (int s = 0; s < C::KV_STAGES; ++s)
            bar_init(&kfull[s], 1), bar_init(&kempty[s], 1), bar_init(&vfull[s], 1), bar_init(&vempty[s], 1);
        for (int s = 0; s < C::S_STAGES; ++s) bar_init(&sfull[s], 1), bar_init(&pfull[s], 4), bar_init(&pvdone[s], 1);
        fence_bar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) {
        // Q first (it needs no bounds), then the tile's key blocks: per
        // sequence present in [t0, tlast), blocks of 64 from the sequence start
        // covering its rows' key range; the first two blocks' K and V go out
        // as soon as they are known.
        bar_expect_tx(qfull, C::Q_BYTES);
        for (int c = 0; c < 4; ++c) tma_load_3d(qs + c * (C::Q_BYTES / 4), &tmQ, qfull, c * 64, head, t0);
        const int tlast = min(t0 + C::BQ, p.n);
        int nb = 0;
        // Row t0's lo and hi as two independent loads: the first sequence needs
        // no dependent read (later ones read their end from their first row).
        const int lo0 = int(p.bounds[2 * t0]), hi0 = int(p.bounds[2 * t0 + 1]);
        for (int seq_lo = lo0; seq_lo < tlast;) {
            const int seq_hi = seq_lo == lo0 ? hi0 : int(p.bounds[2 * seq_lo + 1]);
            if (seq_hi <= seq_lo) break;  // malformed bounds: never loop without progress
            int kmin = seq_lo, kmax = seq_hi;
            if (p.window) {
                const int r_first = max(seq_lo, t0), r_last = min(seq_hi, tlast);
                kmin = max(seq_lo, r_first - p.window);
                kmax = min(seq_hi, r_last + p.window);
            }
            for (int kb = seq_lo + (kmin - seq_lo) / C::BKEY * C::BKEY; kb < kmax; kb += C::BKEY) {
                if (nb == C::MAXB) {
                    // More key blocks than the list holds (only reachable past the
                    // host-checked token limit): record it and compute nothing.
                    atomicExch(&g_error, ERR_RANGE);
                    nb = -1;
                    break;
                }
                blocks[nb] = make_int2(kb, seq_hi);
                if (nb < C::KV_STAGES) load_k(nb), load_v(nb);
                ++nb;
            }
            if (nb < 0) break;
            seq_lo = seq_hi;
        }
        // On overflow the loads already issued still land (drained below) and
        // nothing consumes them.
        *nblocks = nb < 0 ? -C::MAXB : nb;
    }
    tc_fence_before();
    cta_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int nb_raw = *nblocks, nb = nb_raw < 0 ? 0 : nb_raw;
    const int listed = nb_raw < 0 ? C::MAXB : nb;  // blocks whose first loads may be in flight

    if (warp == 0 || warp == 6) {
        // ------------------------------------------------------------ TMA producers (K: warp 0, V: warp 6)
        if (lane == 0) {
            const bool is_k = warp == 0;
            uint64_t *empty = is_k ? kempty : vempty, *full = is_k ? kfull : vfull;
            int issued = min(listed, C::KV_STAGES);
            for (int j = C::KV_STAGES; j < nb; ++j) {
                if (!wait_bar(&empty[j & 1], ((j >> 1) & 1) ^ 1, abort)) break;
                if (is_k) load_k(j);
                else load_v(j);
                ++issued;
            }
            // Drain: the last loads into each stage (and Q) have landed before exit.
            if (is_k) wait_bar(qfull, 0, nullptr);
            for (int k = issued > 2 ? issued - 2 : 0; k < issued; ++k) wait_bar(&full[k & 1], (k >> 1) & 1, nullptr);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0 && nb > 0) {
            constexpr uint32_t idesc_s = idesc_f16(C::BQ, C::BKEY), idesc_o = idesc_f16(C::BQ, C::D, true);
            const uint32_t qa = smem_u32(qs);
            auto issue_s = [&](int j) -> bool {
                const int ks = j & 1, st = j % C::S_STAGES;
                // Stage st last held P of block j - 3, whose P.V must have completed.
                if (!wait_bar(&kfull[ks], (j >> 1) & 1, abort) ||
                    (j >= C::S_STAGES && !wait_bar(&pvdone[st], ((j - C::S_STAGES) / C::S_STAGES) & 1, abort)))
                    return false;
                tc_fence_after();
                const uint32_t ka = smem_u32(k_tile(ks));
#pragma unroll
                for (int kk = 0; kk < C::D / 16; ++kk)
                    mma_f16(tmem + uint32_t(st * C::BKEY),
                            desc_sw128(qa + (kk >> 2) * (C::Q_BYTES / 4) + (kk & 3) * 32),
                            desc_sw128(ka + (kk >> 2) * (C::K_BYTES / 4) + (kk & 3) * 32), idesc_s, kk ? 1u : 0u);
                tc_commit(&sfull[st]);
                tc_commit(&kempty[ks]);
                return true;
            };
            auto issue_pv = [&](int i) -> bool {
                const int vs = i & 1, st = i % C::S_STAGES;
                if (!wait_bar(&pfull[st], (i / C::S_STAGES) & 1, abort) || !wait_bar(&vfull[vs], (i >> 1) & 1, abort))
                    return false;
                tc_fence_after();
                const uint32_t va = smem_u32(v_tile(vs));
#pragma unroll
                for (int kk = 0; kk < C::BKEY / 16; ++kk)
                    mma_f16_ts(tmem + C::O_COL, tmem + uint32_t(st * C::BKEY + kk * 8),
                               desc_mn_sw128(va + kk * 2048, C::V_BYTES / 4), idesc_o, (i > 0 || kk > 0) ? 1u : 0u);
                tc_commit(&pvdone[st]);
                tc_commit(&vempty[vs]);
                return true;
            };
            bool ok = wait_bar(qfull, 0, abort) && issue_s(0) && (nb < 2 || issue_s(1));
            for (int j = 0; ok && j < nb; ++j) ok = issue_pv(j) && (j + 2 >= nb || issue_s(j + 2));
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
        // ------------------------------------------------------------ softmax + epilogue
        constexpr float L2E = 1.4426950408889634f;
        const int quad = warp & 3, row = quad * 32 + lane, t = t0 + row;
        const uint32_t lane_base = tmem + (uint32_t(quad * 32) << 16);
        int lo = 0, hi = 0;
        if (t < p.n) {
            lo = int(p.bounds[2 * t]), hi = int(p.bounds[2 * t + 1]);
            if (p.window) {
                if (t - p.window > lo) lo = t - p.window;
                if (t + p.window + 1 < hi) hi = t + p.window + 1;
            }
        }
        float m = -INFINITY, m2 = -INFINITY, l = 0.0f;  // m2 = m * log2e
        bool ok = true;
        for (int j = 0; j < nb; ++j) {
            const int st = j % C::S_STAGES;
            const uint32_t scol = lane_base + uint32_t(st * C::BKEY);
            if (!__all_sync(0xffffffffu, wait_bar(&sfull[st], (j / C::S_STAGES) & 1, abort))) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sr[64];
            tmem_ld32(scol, reinterpret_cast<uint32_t *>(sr));
            tmem_ld32(scol + 32, reinterpret_cast<uint32_t *>(sr + 32));
            tmem_wait_ld();
            const int kb = blocks[j].x, kend = min(hi, blocks[j].y);
            if (!(kb >= lo && kb + C::BKEY <= kend)) {
#pragma unroll
                for (int c = 0; c < 64; ++c)
                    if (kb + c < lo || kb + c >= kend) sr[c] = -INFINITY;
            }
            float mx8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) mx8[e] = sr[e];
#pragma unroll
            for (int c = 8; c < 64; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], sr[c]);
            const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                   fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
            const bool raise = mx > m + C::RESCALE;  // false while the row has no key (mx = -inf)
            // Rows seeing their first key (m = -inf) still have O = 0 and l = 0.
            const bool rescale = raise && m != -INFINITY;
            if (__any_sync(0xffffffffu, rescale)) {
                // O holds the sum through block j - 1 once that P.V completed.
                const int pj = j - 1, pst = pj % C::S_STAGES;
                if (!__all_sync(0xffffffffu, wait_bar(&pvdone[pst], (pj / C::S_STAGES) & 1, abort))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const float f = rescale ? ex2_approx((m - mx) * L2E) : 1.0f;
                for (int c = 0; c < C::D; c += 32) {
                    uint32_t o[32];
                    tmem_ld32(lane_base + C::O_COL + uint32_t(c), o);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
                    tmem_st32(lane_base + C::O_COL + uint32_t(c), o);
                }
                l *= f;
            }
            if (raise) m = mx, m2 = mx * L2E;
            // P = 2^(s log2e - m log2e) in fp16 pairs over the stage's first 32
            // columns.  Before the row's first key (m = -inf) every score of the
            // block is masked, and the offset 0 makes each weight 2^-inf = 0.
            const float nm2 = m2 == -INFINITY ? 0.0f : -m2;
            uint32_t pk[32];
            float l4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                const float p0 = ex2_approx(fmaf(sr[2 * c], L2E, nm2)), p1 = ex2_approx(fmaf(sr[2 * c + 1], L2E, nm2));
                l4[c & 3] += p0 + p1;
                const __half2 h = __floats2half2_rn(p0, p1);
                pk[c] = *reinterpret_cast<const uint32_t *>(&h);
            }
            l += (l4[0] + l4[1]) + (l4[2] + l4[3]);
            tmem_st32(scol, pk);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&pfull[st]);
        }
        if (ok && nb > 0) {
            const int pj = nb - 1, pst = pj % C::S_STAGES;
            if (__all_sync(0xffffffffu, wait_bar(&pvdone[pst], (pj / C::S_STAGES) & 1, abort))) {
                tc_fence_after();
                // Every MMA has completed, so the Q tile is free: each 32-column
                // chunk of the warp's 32 rows goes through a padded tile there and
                // each store instruction writes four whole 128-byte row segments.
                const float il = l > 0.0f ? 1.0f / l : 0.0f;
                if (p.q) {
                    for (int c = 0; c < C::D; c += 32) {
                        uint32_t r[32];
                        tmem_ld32(lane_base + C::O_COL + uint32_t(c), r);
                        tmem_wait_ld();
                        float amax = 0.0f;
#pragma unroll
                        for (int e = 0; e < 32; ++e) amax = fmaxf(amax, fabsf(__uint_as_float(r[e]) * il));
                        const float d = div127(amax), id = d != 0.0f ? rcp_rn(d) : 0.0f;
                        uint32_t w[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            w[e] = 0;
#pragma unroll
                            for (int b = 0; b < 4; ++b)
                                w[e] |= q8_code(__uint_as_float(r[4 * e + b]) * il, id, p.tier) << (8 * b);
                        }
                        if (t < p.n) {
                            uint4 *dst = reinterpret_cast<uint4 *>(p.q + size_t(t) * 1024 + head * C::D + c);
                            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
                            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
                            p.qs[size_t(head * 8 + c / 32) * p.q_stride + t] = fp16_bits_to_f32(ref_fp32_to_fp16(d));
                        }
                    }
                } else {
                    float *stg = reinterpret_cast<float *>(qs) + (warp - 2) * (32 * 33);
                    const int srow = lane >> 3, scol4 = (lane & 7) * 4;
                    for (int c = 0; c < C::D; c += 32) {
                        uint32_t r[32];
                        tmem_ld32(lane_base + C::O_COL + uint32_t(c), r);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) stg[lane * 33 + e] = __uint_as_float(r[e]) * il;
                        __syncwarp();
#pragma unroll
                        for (int rr = 0; rr < 32; rr += 4) {
                            const int r8 = rr + srow, tt = t0 + quad * 32 + r8;
                            const float *src = stg + r8 * 33 + scol4;
                            if (tt < p.n)
                                *reinterpret_cast<float4 *>(p.out + (size_t(tt) * 4 + head) * C::D + c + scol4) =
                                    make_float4(src[0], src[1], src[2], src[3]);
                        }
                        __syncwarp();
                    }
                }
            }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) bar_arrive(edone);
    }
}

}  // namespace eg2
