// Packed-varlen bidirectional GQA attention on the 5th-generation tensor cores
// -- the reference's attention_rows (vendor/embeddinggemma.c/src/gemma2_fast.c:
// 768-894): for token t and head h, keys s in [lo_t, hi_t) of its own sequence,
// intersected with [t - window, t + window] when window != 0; scale 1.
// d = 256 (sliding-window layers, KV head h / 2) and d = 512 (global layers,
// one KV head).  At d = 512 the 512 output columns would fill the whole tensor
// memory, so a CTA computes one 256-column half of O (blockIdx.z) and the full
// score S = Q.K^T over d = 512 from two 256-wide K pieces per key block; Q is a
// 128 KB tile and one key block of K and V is in flight.
//
// A CTA owns 128 query tokens of one head (the TMEM lanes).  Per key block of 64:
//   S = Q . K^T         tcgen05.mma kind::f16, M = 128, N = 64, K = 256, fp32 in TMEM
//   softmax             one thread per query row reads its 64 scores from TMEM and
//                       writes P (fp16, packed in pairs) back over the first 32
//                       columns of the same S stage
//   O += P . V          A = P from TMEM, B = V as an MN-major shared-memory
//                       operand, M = 128, N = 256, K = 64, fp32 accumulator in TMEM
// TMEM: S/P stages at columns 0, 64, 128; O (256 columns) at 256..511.  At
// d = 256 the MMA warp keeps S two blocks ahead (S0 S1 PV0 S2 PV1 S3 ...), so
// the softmax of block j never waits for its scores, and P needs no shared
// memory, proxy fence or buffer of its own; K and V have separate
// double-buffered stages: K(j+2) loads as soon as S(j) completed, V(j+2) once
// P.V(j) did.  At d = 512 the two K stages hold the two 256-wide halves of one
// block (each reloaded as soon as its half of S completed) and V has one stage,
// so the order is S0 PV0 S1 PV1 ...
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
    float *out;              // [n][4][d] fp32 (when q is null)
    const unsigned *bounds;  // [n][2] = sequence [lo, hi)
    int n, window;
    // Optional Q8_0 output instead of out (ROW_QUANT of the attention row,
    // gemma2_fast.c:728-730, fused): codes [n][4d], scales block-major
    // [4d/32][q_stride]; quantizer rounding of `tier`.
    int8_t *q;
    float *qs;
    int q_stride, tier;
};

template <int D_>
struct AttnTcCfgD {
    static constexpr int D = D_, DV = 256, BQ = 128, BKEY = 64, S_STAGES = 3, MAXB = 256;
    // K arrives in pieces of 64 keys x 256 d (KPB per key block) through a ring
    // of K_STAGES; V in pieces of 64 keys x this CTA's 256 output columns.
    static constexpr int KPB = D / 256, K_STAGES = 2, V_STAGES = D == 256 ? 2 : 1;
    static constexpr int AHEAD = D == 256 ? 2 : 1;  // S blocks issued ahead of P.V
    static constexpr int THREADS = 7 * 32;
    static constexpr int Q_BYTES = BQ * D * 2;      // D/64 K-chunks of [128 rows][128 B]
    static constexpr int K_BYTES = BKEY * 256 * 2;  // 4 K-chunks of [64 rows][128 B]
    static constexpr int V_BYTES = BKEY * DV * 2;   // 4 d-chunks of [64 keys][128 B] (MN-major)
    static constexpr size_t K_OFF = Q_BYTES, V_OFF = K_OFF + size_t(K_STAGES) * K_BYTES;
    static constexpr size_t BLK_OFF = V_OFF + size_t(V_STAGES) * V_BYTES;
    static constexpr size_t SMEM = 1024 + BLK_OFF + MAXB * 4 + 256;
    static constexpr float RESCALE = 8.0f;
    static constexpr uint32_t O_COL = 256;
};
using AttnTcCfg = AttnTcCfgD<256>;
static_assert(AttnTcCfgD<512>::SMEM <= 227 * 1024, "shared memory");

template <int D_>
__global__ void __launch_bounds__(AttnTcCfgD<D_>::THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const AttnTcParams p) {
    using C = AttnTcCfgD<D_>;
    static_assert(D_ == 256 || D_ == 512, "d = 256 or 512");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = align_smem_1024(smem_raw);
    uint8_t *qs = smem;
    // Key blocks: first key | sequence end << 16 (both below 2^16 for n <= 8192).
    uint32_t *blocks = reinterpret_cast<uint32_t *>(smem + C::BLK_OFF);
    uint64_t *bars = reinterpret_cast<uint64_t *>(blocks + C::MAXB);
    uint64_t *qfull = bars, *kfull = bars + 1, *kempty = kfull + 2, *vfull = kempty + 2, *vempty = vfull + 2;
    uint64_t *sfull = vempty + 2, *pfull = sfull + 3, *pvdone = pfull + 3, *edone = pvdone + 3, *mdone = edone + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mdone + 1);
    int *nblocks = reinterpret_cast<int *>(tmem_slot + 1);
    volatile int *abort = nblocks + 1;
    auto k_tile = [&](int s) { return smem + C::K_OFF + s * C::K_BYTES; };
    auto v_tile = [&](int s) { return smem + C::V_OFF + s * C::V_BYTES; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // dh: this CTA's 256 output columns (d = 512; always 0 at d = 256).
    const int t0 = blockIdx.x * C::BQ, head = blockIdx.y, dh = blockIdx.z, kh = C::D == 256 ? head / 2 : 0;
    // K piece kp = block kp / KPB, d columns 256 (kp % KPB) .., into stage
    // kp % 2; block j's V (this CTA's columns) into stage j % V_STAGES.  The
    // caller has made sure the stage is free.
    auto load_k = [&](int kp) {
        const int s = kp % C::K_STAGES, key = int(blocks[kp / C::KPB] & 0xFFFFu), d0 = (kp % C::KPB) * 256;
        bar_expect_tx(&kfull[s], C::K_BYTES);
        for (int c = 0; c < 4; ++c)
            tma_load_3d(k_tile(s) + c * (C::K_BYTES / 4), &tmK, &kfull[s], d0 + c * 64, kh, key);
    };
    auto load_v = [&](int j) {
        const int s = j % C::V_STAGES, key = int(blocks[j] & 0xFFFFu);
        bar_expect_tx(&vfull[s], C::V_BYTES);
        for (int c = 0; c < 4; ++c)
            tma_load_3d(v_tile(s) + c * (C::V_BYTES / 4), &tmV, &vfull[s], dh * 256 + c * 64, kh, key);
    };
    if (threadIdx.x == 0) {
        tma_prefetch(&tmQ), tma_prefetch(&tmK), tma_prefetch(&tmV);
        *abort = 0;
        bar_init(qfull, 1), bar_init(edone, 4), bar_init(mdone, 1);
        for (int s = 0; s < 2; ++s)
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
        // covering its rows' key range; the first K pieces and V blocks that
        // fit the stages go out as soon as they are known.
        bar_expect_tx(qfull, C::Q_BYTES);
        for (int c = 0; c < C::D / 64; ++c)
            tma_load_3d(qs + c * (C::Q_BYTES / (C::D / 64)), &tmQ, qfull, c * 64, head, t0);
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
                blocks[nb] = uint32_t(kb) | uint32_t(seq_hi) << 16;
                for (int kp = nb * C::KPB; kp < (nb + 1) * C::KPB && kp < C::K_STAGES; ++kp) load_k(kp);
                if (nb < C::V_STAGES) load_v(nb);
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
            // Units: K pieces (warp 0) or V blocks (warp 6).
            const bool is_k = warp == 0;
            const int stages = is_k ? C::K_STAGES : C::V_STAGES, units = is_k ? nb * C::KPB : nb;
            uint64_t *empty = is_k ? kempty : vempty, *full = is_k ? kfull : vfull;
            int issued = min(is_k ? listed * C::KPB : listed, stages);
            for (int u = stages; u < units; ++u) {
                if (!wait_bar(&empty[u % stages], ((u / stages) & 1) ^ 1, abort)) break;
                if (is_k) load_k(u);
                else load_v(u);
                ++issued;
            }
            // Drain: the last loads into each stage (and Q) have landed before exit.
            if (is_k) wait_bar(qfull, 0, nullptr);
            for (int k = issued > stages ? issued - stages : 0; k < issued; ++k)
                wait_bar(&full[k % stages], (k / stages) & 1, nullptr);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0 && nb > 0) {
            constexpr uint32_t idesc_s = idesc_f16(C::BQ, C::BKEY), idesc_o = idesc_f16(C::BQ, C::DV, true);
            constexpr int QCH = C::Q_BYTES / (C::D / 64);  // bytes of one 64-column Q chunk
            const uint32_t qa = smem_u32(qs);
            auto issue_s = [&](int j) -> bool {
                const int st = j % C::S_STAGES;
                // Stage st last held P of block j - 3, whose P.V must have completed.
                if (j >= C::S_STAGES && !wait_bar(&pvdone[st], ((j - C::S_STAGES) / C::S_STAGES) & 1, abort))
                    return false;
                for (int h = 0; h < C::KPB; ++h) {
                    const int kp = j * C::KPB + h, ks = kp % C::K_STAGES;
                    if (!wait_bar(&kfull[ks], (kp / C::K_STAGES) & 1, abort)) return false;
                    tc_fence_after();
                    const uint32_t ka = smem_u32(k_tile(ks));
#pragma unroll
                    for (int kk = 0; kk < 16; ++kk)
                        mma_f16(tmem + uint32_t(st * C::BKEY),
                                desc_sw128(qa + (h * 4 + (kk >> 2)) * QCH + (kk & 3) * 32),
                                desc_sw128(ka + (kk >> 2) * (C::K_BYTES / 4) + (kk & 3) * 32), idesc_s,
                                (h > 0 || kk > 0) ? 1u : 0u);
                    tc_commit(&kempty[ks]);  // this K piece is free once its MMAs completed
                }
                tc_commit(&sfull[st]);
                return true;
            };
            auto issue_pv = [&](int i) -> bool {
                const int vs = i % C::V_STAGES, st = i % C::S_STAGES;
                if (!wait_bar(&pfull[st], (i / C::S_STAGES) & 1, abort) ||
                    !wait_bar(&vfull[vs], (i / C::V_STAGES) & 1, abort))
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
            bool ok = wait_bar(qfull, 0, abort);
            for (int j = 0; ok && j < C::AHEAD && j < nb; ++j) ok = issue_s(j);
            for (int j = 0; ok && j < nb; ++j) ok = issue_pv(j) && (j + C::AHEAD >= nb || issue_s(j + C::AHEAD));
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
            const int kb = int(blocks[j] & 0xFFFFu), kend = min(hi, int(blocks[j] >> 16));
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
                for (int c = 0; c < C::DV; c += 32) {
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
                // This CTA's columns of the token's 4 x D attention row.
                const int col0 = head * C::D + dh * C::DV;
                if (p.q) {
                    for (int c = 0; c < C::DV; c += 32) {
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
                            uint4 *dst = reinterpret_cast<uint4 *>(p.q + size_t(t) * (4 * C::D) + col0 + c);
                            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
                            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
                            p.qs[size_t((col0 + c) / 32) * p.q_stride + t] = fp16_bits_to_f32(ref_fp32_to_fp16(d));
                        }
                    }
                } else {
                    float *stg = reinterpret_cast<float *>(qs) + (warp - 2) * (32 * 33);
                    const int srow = lane >> 3, scol4 = (lane & 7) * 4;
                    for (int c = 0; c < C::DV; c += 32) {
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
                                *reinterpret_cast<float4 *>(p.out + size_t(tt) * (4 * C::D) + col0 + c + scol4) =
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
