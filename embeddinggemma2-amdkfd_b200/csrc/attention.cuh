// Packed-varlen bidirectional GQA attention (scale 1) -- the reference's
// attention_rows (vendor/embeddinggemma.c/src/gemma2_fast.c:768-894): for token
// t and head h, keys s in [lo_t, hi_t) of its own sequence, intersected with
// [t - window, t + window] on sliding-window layers (window 512), global layers
// window 0; KV head h / (4 / kv); softmax in fp32.
//
// Flash-style: a CTA owns 64 query tokens of one head and one 256-wide slice of
// the value dimension (d = 512 uses two slices, each recomputing Q.K^T).  Its
// two groups of four warps split the key blocks (even / odd block of each
// sequence), each warp holding 16 queries; Q.K^T and P.V run on fp16
// tensor-core MMAs with fp32 accumulation and an online softmax, and the two
// groups' partial states are merged at the end.  The CTA visits the sequences
// present in its query tile one after another, and each sequence's key blocks
// of 64 start at multiples of 64 from the sequence's first token: a row's keys
// are therefore grouped and summed the same way wherever its sequence sits in
// the packed wave (blocks of other sequences are fully masked for it and leave
// its state bit-for-bit unchanged), so packed and solo results are identical.
// Shared-memory rows are XOR-swizzled in 16-byte chunks so ldmatrix is
// conflict-free.  The executor's fast path runs the tcgen05 kernel of
// attention_tc.cuh on both layer kinds; this one is the eg2_launch_attention_f16
// operator.
#pragma once
#include "common.cuh"

namespace eg2 {

struct AttnParams {
    float *out;               // [n][4][d]
    const __half *q, *k, *v;  // q [n][4][d], k/v [n][kv][d]
    const unsigned *bounds;   // [n][2] = sequence [lo, hi)
    int n, window;
};

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid) {
    const int bytes = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

// Byte offset of element (row, col) in a swizzled tile with `chunks` 16-byte
// chunks per row.
__device__ __forceinline__ uint32_t swz(int row, int col, int chunks) {
    return uint32_t(row * chunks * 16 + (((col >> 3) ^ (row & 7)) << 4) + (col & 7) * 2);
}

template <int D>
struct AttnCfg {
    // Key blocks of BKEY alternate between the CTA's two warp groups; each group
    // owns one K/V buffer, so one group's loads overlap the other's MMAs.
    static constexpr int BQ = 64, BKEY = D == 256 ? 64 : 32, DV = 256, GROUP_WARPS = 4;
    static constexpr int WARPS = 2 * GROUP_WARPS, THREADS = WARPS * 32;
    static constexpr int QCH = D / 8, VCH = DV / 8;  // 16-byte chunks per row
    static constexpr int Q_BYTES = BQ * D * 2, K_BYTES = BKEY * D * 2, V_BYTES = BKEY * DV * 2;
    static constexpr int KV_BYTES = K_BYTES + V_BYTES;
    // The merge of the two groups' partial states reuses the K/V buffers: per
    // thread of group 1, DV/8 float4 of o and one float4 (m0, m1, l0, l1).
    static constexpr int MERGE_BYTES = (DV / 8 + 1) * GROUP_WARPS * 32 * 16;
    static_assert(MERGE_BYTES <= 2 * KV_BYTES, "merge area exceeds the K/V buffers");
    static constexpr size_t SMEM = size_t(Q_BYTES) + 2 * KV_BYTES + 2 * BQ * 4 + 16;
};

template <int D>
__global__ void __launch_bounds__(AttnCfg<D>::THREADS, 1) attention_kernel(const AttnParams p) {
    using C = AttnCfg<D>;
    constexpr int KV = 512 / D, NB = C::BKEY / 8;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *qs = smem, *kvs = smem + C::Q_BYTES;
    int *qlo = reinterpret_cast<int *>(kvs + 2 * C::KV_BYTES), *qhi = qlo + C::BQ;
    pdl_wait();
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = warp / C::GROUP_WARPS, wl = warp % C::GROUP_WARPS, gt = threadIdx.x % (C::GROUP_WARPS * 32);
    const int t0 = blockIdx.x * C::BQ, head = blockIdx.y, dv0 = blockIdx.z * C::DV;
    const int kh = head / (4 / KV);
    uint8_t *ks = kvs + grp * C::KV_BYTES, *vs = ks + C::K_BYTES;

    // Per-query key ranges.
    if (threadIdx.x < C::BQ) {
        const int t = t0 + threadIdx.x;
        int lo = 0, hi = 0;
        if (t < p.n) {
            lo = int(p.bounds[2 * t]), hi = int(p.bounds[2 * t + 1]);
            if (p.window) {
                if (t - p.window > lo) lo = t - p.window;
                if (t + p.window + 1 < hi) hi = t + p.window + 1;
            }
        }
        qlo[threadIdx.x] = lo, qhi[threadIdx.x] = hi;
    }
    // Q tile (64 x D) -> shared.
    for (int i = threadIdx.x; i < C::BQ * C::QCH; i += C::THREADS) {
        const int r = i / C::QCH, ch = i % C::QCH, t = t0 + r;
        cp_async16(qs + swz(r, ch * 8, C::QCH), p.q + (size_t(t < p.n ? t : 0) * 4 + head) * D + ch * 8, t < p.n);
    }
    cp_async_wait_all();
    __syncthreads();
    const int tlast = min(t0 + C::BQ, p.n);

    // Each thread: query rows g and g+8 of its warp's 16 (the same rows in both groups).
    const int g = lane >> 2, tq = lane & 3;
    const int r0 = wl * 16 + g, r1 = r0 + 8;
    const int lo0 = qlo[r0], hi0 = qhi[r0], lo1 = qlo[r1], hi1 = qhi[r1];
    float o[C::DV / 8][4];
#pragma unroll
    for (int j = 0; j < C::DV / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    float m0 = -1e30f, m1 = -1e30f, l0 = 0.0f, l1 = 0.0f;
    const uint32_t qbase = smem_u32(qs), kbase = smem_u32(ks), vbase = smem_u32(vs);

    for (int seq_lo = int(p.bounds[2 * t0]); seq_lo < tlast;) {
      const int seq_hi = int(p.bounds[2 * seq_lo + 1]);
      if (seq_hi <= seq_lo) break;  // malformed bounds: never loop without progress
      int kmin = seq_lo, kmax = seq_hi;
      if (p.window) {
          const int r_first = max(seq_lo, t0), r_last = min(seq_hi, tlast);
          kmin = max(seq_lo, r_first - p.window);
          kmax = min(seq_hi, r_last + p.window);
      }
      // Blocks at multiples of BKEY from the sequence start; block b goes to
      // group b % 2.
      const int b_first = (kmin - seq_lo) / C::BKEY;
      for (int b = b_first + ((b_first & 1) != grp); seq_lo + b * C::BKEY < kmax; b += 2) {
        const int kb = seq_lo + b * C::BKEY;
        named_sync(1 + grp, C::GROUP_WARPS * 32);  // this group's previous tile fully consumed
        for (int i = gt; i < C::BKEY * C::QCH; i += C::GROUP_WARPS * 32) {
            const int r = i / C::QCH, ch = i % C::QCH, s = kb + r;
            const bool ok = s < p.n;
            cp_async16(ks + swz(r, ch * 8, C::QCH), p.k + (size_t(ok ? s : 0) * KV + kh) * D + ch * 8, ok);
        }
        for (int i = gt; i < C::BKEY * C::VCH; i += C::GROUP_WARPS * 32) {
            const int r = i / C::VCH, ch = i % C::VCH, s = kb + r;
            const bool ok = s < p.n;
            cp_async16(vs + swz(r, ch * 8, C::VCH), p.v + (size_t(ok ? s : 0) * KV + kh) * D + dv0 + ch * 8, ok);
        }
        cp_async_wait_all();
        named_sync(1 + grp, C::GROUP_WARPS * 32);

        // S = Q K^T for this warp's 16 queries x BKEY keys.
        float sacc[NB][4];
#pragma unroll
        for (int j = 0; j < NB; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.0f;
#pragma unroll 4
        for (int kk = 0; kk < D; kk += 16) {
            uint32_t a0, a1, a2, a3;
            {
                const int row = wl * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, col = kk + (lane >> 4) * 8;
                ldsm_x4(qbase + swz(row, col, C::QCH), a0, a1, a2, a3);
            }
#pragma unroll
            for (int nb = 0; nb < NB; nb += 2) {
                uint32_t b0, b1, b2, b3;
                const int key = nb * 8 + (lane & 7) + (lane >> 4) * 8, col = kk + ((lane >> 3) & 1) * 8;
                ldsm_x4(kbase + swz(key, col, C::QCH), b0, b1, b2, b3);
                mma16816(sacc[nb], a0, a1, a2, a3, b0, b1);
                mma16816(sacc[nb + 1], a0, a1, a2, a3, b2, b3);
            }
        }
        // Mask, online softmax.
        float mx0 = m0, mx1 = m1;
#pragma unroll
        for (int j = 0; j < NB; ++j) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                // Keys past the current sequence belong to the next one: they are
                // counted in that sequence's own pass, never here.
                const int s = kb + j * 8 + tq * 2 + e;
                if (s < lo0 || s >= hi0 || s >= seq_hi) sacc[j][e] = -INFINITY;
                if (s < lo1 || s >= hi1 || s >= seq_hi) sacc[j][2 + e] = -INFINITY;
                mx0 = fmaxf(mx0, sacc[j][e]);
                mx1 = fmaxf(mx1, sacc[j][2 + e]);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float c0 = expf(m0 - mx0), c1 = expf(m1 - mx1);
        m0 = mx0, m1 = mx1;
        l0 *= c0, l1 *= c1;
#pragma unroll
        for (int j = 0; j < C::DV / 8; ++j) o[j][0] *= c0, o[j][1] *= c0, o[j][2] *= c1, o[j][3] *= c1;
        uint32_t pa[NB / 2][4];  // P as fp16 A fragments, k-steps of 16 keys
#pragma unroll
        for (int j = 0; j < NB; ++j) {
            const float p0 = expf(sacc[j][0] - m0), p1 = expf(sacc[j][1] - m0);
            const float p2 = expf(sacc[j][2] - m1), p3 = expf(sacc[j][3] - m1);
            l0 += p0 + p1, l1 += p2 + p3;
            const int ks2 = j >> 1, hi = j & 1;
            pa[ks2][hi * 2 + 0] = pack_h2(p0, p1);
            pa[ks2][hi * 2 + 1] = pack_h2(p2, p3);
        }
        // O += P V over the 256-wide value slice.
#pragma unroll
        for (int k2 = 0; k2 < NB / 2; ++k2) {
#pragma unroll
            for (int db = 0; db < C::DV / 8; db += 2) {
                uint32_t b0, b1, b2, b3;
                const int key = k2 * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, col = db * 8 + (lane >> 4) * 8;
                ldsm_x4_t(vbase + swz(key, col, C::VCH), b0, b1, b2, b3);
                mma16816(o[db], pa[k2][0], pa[k2][1], pa[k2][2], pa[k2][3], b0, b1);
                mma16816(o[db + 1], pa[k2][0], pa[k2][1], pa[k2][2], pa[k2][3], b2, b3);
            }
        }
      }
      seq_lo = seq_hi;
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

    // Merge: group 1 hands its (m, l, o) to the thread of group 0 that holds the
    // same fragment positions, through the (now free) K/V buffers.
    __syncthreads();
    float4 *mo = reinterpret_cast<float4 *>(kvs);
    constexpr int GT = C::GROUP_WARPS * 32;
    if (grp == 1) {
#pragma unroll
        for (int j = 0; j < C::DV / 8; ++j) mo[j * GT + gt] = make_float4(o[j][0], o[j][1], o[j][2], o[j][3]);
        mo[(C::DV / 8) * GT + gt] = make_float4(m0, m1, l0, l1);
    }
    __syncthreads();
    if (grp == 1) return;
    const float4 st = mo[(C::DV / 8) * GT + gt];
    const float n0 = fmaxf(m0, st.x), n1 = fmaxf(m1, st.y);
    const float a0 = expf(m0 - n0), b0 = expf(st.x - n0), a1 = expf(m1 - n1), b1 = expf(st.y - n1);
    const float il0 = 1.0f / (l0 * a0 + st.z * b0), il1 = 1.0f / (l1 * a1 + st.w * b1);
    const int ta = t0 + r0, tb = t0 + r1;
#pragma unroll
    for (int j = 0; j < C::DV / 8; ++j) {
        const float4 ob = mo[j * GT + gt];
        const int col = dv0 + j * 8 + tq * 2;
        if (ta < p.n)
            *reinterpret_cast<float2 *>(p.out + (size_t(ta) * 4 + head) * D + col) =
                make_float2((o[j][0] * a0 + ob.x * b0) * il0, (o[j][1] * a0 + ob.y * b0) * il0);
        if (tb < p.n)
            *reinterpret_cast<float2 *>(p.out + (size_t(tb) * 4 + head) * D + col) =
                make_float2((o[j][2] * a1 + ob.z * b1) * il1, (o[j][3] * a1 + ob.w * b1) * il1);
    }
}

}  // namespace eg2
