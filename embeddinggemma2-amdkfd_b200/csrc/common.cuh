// Device helpers shared by the sm_100a kernels: mbarriers with bounded waits,
// TMA tile loads, tcgen05 (TMEM allocation, MMA, commit, loads) and the exact
// scalar arithmetic the reference CPU graph uses.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "launch.h"
#include "ref_tanhf.h"

namespace eg2 {

// Set by any bounded wait that ran out (see wait_bar); read by the host after a
// wave, which then reports the wave as failed.  Kernels do not read it: every
// wait is bounded, so a kernel that follows a failed one still terminates.
// Defined here: the library has a single device translation unit (kernels.cu).
__device__ int g_error = 0;
enum : int { ERR_NONE = 0, ERR_WAIT_TIMEOUT = 1, ERR_RANGE = 2 };

// ---------------------------------------------------------------- basics
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// Rounds the dynamic shared-memory base up to a 1024-byte boundary (the
// 128-byte swizzle atom repeats every 1024 bytes) by pointer arithmetic on the
// shared array itself, so the compiler still knows every derived pointer is
// shared memory and emits LDS/STS (an integer round trip would turn each access
// into a generic load tracked on the long scoreboard).
__device__ __forceinline__ uint8_t *align_smem_1024(uint8_t *raw) {
    return raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u);
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// CTA-wide and named barriers in their non-aligned form: arrivals are counted
// per thread, so they stay correct when a warp reaches them diverged (after an
// elect_one() role or a lane-0 branch).  __syncthreads() is the aligned form,
// whose count is undefined for a diverged warp.
__device__ __forceinline__ void cta_sync() { asm volatile("barrier.sync 0;" ::: "memory"); }
__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("barrier.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// Programmatic dependent launch: every kernel of the wave is launched so that
// it may start while its predecessor in the stream is still running.
// pdl_wait() blocks until that predecessor has completed and its memory is
// visible; nothing that reads or overwrites its inputs/outputs may come
// before it.  pdl_trigger() lets the successor be scheduled.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .b32 r;\n\t.reg .pred p;\n\t"
        "elect.sync r|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void bar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_bar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool bar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Every wait on a barrier is bounded: after ~2 s (or, when abort is given,
// once another thread of the CTA gave up) it returns false and records
// ERR_WAIT_TIMEOUT, so a lost arrival can never hang the GPU.  Waits used to
// drain this CTA's own in-flight copies / MMAs before exit pass abort = nullptr.
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, volatile int *abort) {
    if (bar_try_wait(bar, parity)) return true;
    const uint64_t start = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (bar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (abort && *abort) return false;
            if (globaltimer_ns() - start > 2000000000ull) {
                if (abort) *abort = 1;
                atomicExch(&g_error, ERR_WAIT_TIMEOUT);
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// 2-D tiled load into this CTA's shared memory; c0 is the innermost coordinate in elements and
// every caller passes a multiple of the 128-byte swizzle row, so c0 * element
// size is always a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

// 3-D tiled load into this CTA's shared memory; c0 (innermost, elements) is always a multiple
// of 64 16-bit elements here, so c0 * element size is a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// D[tmem] (+)= A[smem] . B[smem]^T, int8 x int8 -> int32, one K=32 step.
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A . B^T, bf16 x bf16 -> fp32, one K=16 step.
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// As mma_f16 with the A operand (M rows x K 16-bit elements) in tensor memory:
// row i in lane i, elements 2c and 2c + 1 packed (low, high) in column c.
__device__ __forceinline__ void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 2^x by the MUFU approximation (relative error about 2^-22; -inf -> +0).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// Instruction descriptors (tcgen05 instruction-descriptor bit layout):
// [4,6) D format, [7,10) A format, [10,13) B format, [15] A MN-major,
// [16] B MN-major, [17,23) N>>3, [24,29) M>>4.  A and B always share a type.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}
// kind::f16 with fp16 A and B and fp32 D; b_mn: B is MN-major (its N
// dimension contiguous in shared memory).
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool b_mn = false) {
    return (1u << 4) | (b_mn ? (1u << 16) : 0u) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}
// Shared-memory descriptor for an MN-major 16-bit operand with 128-byte
// swizzle: 64-element (128-byte) rows along MN, 8 consecutive K rows per
// 1024-byte atom (SBO = 1024), and lbo bytes between successive 64-element
// blocks along MN.  Advancing along K by 16 rows adds 2048 bytes to saddr.
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t saddr, uint32_t lbo) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Shared-memory matrix descriptor for a K-major operand written by TMA with
// 128-byte swizzle: rows of 128 B, 8-row atoms of 1024 B (SBO), version 1,
// layout type 2 (SWIZZLE_128B).  Advancing along K inside the 128-byte row is
// done by adding the byte offset to the start address (atom bases stay
// 1024-byte aligned).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// 32 registers per thread -> 32 lanes x 32 consecutive 32-bit TMEM columns.
// Warp-collective; complete with tmem_wait_st().
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t *r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 32 lanes x 32 consecutive 32-bit TMEM columns -> 32 registers per thread.
// Warp-collective: every lane of the warp must execute it.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t *r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
          "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
          "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
// 32 lanes x 64 consecutive 32-bit TMEM columns -> 64 registers per thread.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t *r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
        "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
        "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
          "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
          "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]),
          "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]),
          "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]),
          "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]),
          "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr));
}
// 32 lanes x 16 consecutive 32-bit TMEM columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t *r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// After tcgen05.wait::ld: marks the destination registers of the completed
// loads as redefined here, so the compiler cannot move their first use above
// the wait (the tcgen05.ld statement itself only names them as outputs).
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// ---------------------------------------------------------------- exact scalar math
// fp32 -> fp16 bits with the reference's rounding (quants.c:13-37): ties on
// bit 12 round up in magnitude, which is not round-to-nearest-even.
__device__ __forceinline__ uint16_t ref_fp32_to_fp16(float f) {
    const uint32_t x = __float_as_uint(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t mant = x & 0x7FFFFFu;
    const int32_t e = int32_t((x >> 23) & 0xFFu) - 112;
    if (e <= 0) {
        if (e < -10) return uint16_t(sign);
        mant |= 0x800000u;
        const uint32_t shift = uint32_t(14 - e);
        uint32_t half = sign | (mant >> shift);
        if ((mant >> (shift - 1u)) & 1u) half++;
        return uint16_t(half);
    }
    if (e >= 31) return uint16_t(sign | 0x7C00u | (mant ? ((mant >> 13) | 1u) : 0u));
    uint32_t half = sign | (uint32_t(e) << 10) | (mant >> 13);
    if (mant & 0x1000u) half++;
    return uint16_t(half);
}
__device__ __forceinline__ float fp16_bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// The reference CPU tier to reproduce (TIER_X86, TIER_SCALAR, TIER_VNNI512) is
// declared in launch.h.

// Q8_0 code of x with id = 1/d: trunc(x*id +- 0.5) on the x86 tiers
// (gemma2_fast_x86.c:225-230), roundf(x*id) on the scalar tier (quants.c:97-177
// generic branch); both clamp to [-128, 127].
__device__ __forceinline__ uint32_t q8_code(float x, float id, int tier = TIER_X86) {
    const float v = __fmul_rn(x, id);
    int q = tier == TIER_SCALAR ? int(roundf(v)) : __float2int_rz(__fadd_rn(v, copysignf(0.5f, v)));
    q = q < -128 ? -128 : (q > 127 ? 127 : q);
    return uint32_t(q) & 0xFFu;
}
// exp(x) by Cody-Waite reduction and a degree-6 polynomial: the reference's own
// x86 GELU helper (gemma2_fast_x86.c:291-306), evaluated with the same fused
// and unfused operations so that results match it bit for bit.
__device__ __forceinline__ float ref_exp8(float x) {
    x = fminf(fmaxf(x, -87.0f), 88.0f);
    const float n = rintf(__fmul_rn(x, 1.44269504088896341f));
    float r = __fmaf_rn(-n, 0.693359375f, x);
    r = __fmaf_rn(-n, -2.12194440e-4f, r);
    float p = 1.0f / 720;
    p = __fmaf_rn(p, r, 1.0f / 120);
    p = __fmaf_rn(p, r, 1.0f / 24);
    p = __fmaf_rn(p, r, 1.0f / 6);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    return __fmul_rn(p, __uint_as_float(uint32_t(int32_t(n) + 127) << 23));
}
// a / b without a branch, by Markstein's sequence (P. Markstein, "IA-64 and
// Elementary Functions", 2000, ch. 8): y ~ 1/b from the hardware reciprocal
// approximation, one Newton step y += y (1 - b y), then the quotient q = a y
// corrected once with its exact FMA residual, q += (a - b q) y.  IEEE division
// compiles to a range check and a slow-path branch per quotient, which keeps
// the compiler from interleaving a thread's independent GELU chains.  Used only
// where it equals the correctly rounded quotient: a = 2 and b in [1, 2^26), the
// GELU's 1 + exp(2v) with |v| <= 9, checked against IEEE division on B200 for
// every float b in that range (tests/test_gpu_ops.py).
__device__ __forceinline__ float fdiv_markstein(float a, float b) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(b));
    y = __fmaf_rn(y, __fmaf_rn(-b, y, 1.0f), y);
    const float q = __fmul_rn(a, y);
    return __fmaf_rn(__fmaf_rn(-b, q, a), y, q);
}
// v / sqrtf(512) with the rounding of IEEE division, without its branch: the
// double product with RN(1/b) is within 2^-52 of the quotient, and a quotient
// of two floats lies at least 2^-49 (relative) from any float rounding
// midpoint (b's odd 24-bit significand makes an exact midpoint impossible), so
// rounding the product to float gives the correctly rounded quotient.  Checked
// on B200 against IEEE division for every float v (tests/test_gpu_ops.py).
__device__ __forceinline__ float div_sqrt512(float v) {
    constexpr double INV = 1.0 / double(22.627416997969522f);
    return __double2float_rn(__dmul_rn(double(v), INV));
}
// a / 127 rounded as IEEE division rounds it (same argument as div_sqrt512:
// 127 has an odd significand).  Checked for every non-negative float.
__device__ __forceinline__ float div127(float a) {
    constexpr double INV = 1.0 / 127.0;
    return __double2float_rn(__dmul_rn(double(a), INV));
}
// 1 / d rounded as IEEE division rounds it, for d > 0, without the division's
// slow-path branch: the double reciprocal approximation refined by two Newton
// steps is within 2^-52 of 1/d, which lies at least 2^-49 (relative) from any
// float rounding midpoint, so its rounding to float is the correctly rounded
// reciprocal.  Checked against IEEE division for every positive float and +inf.
__device__ __forceinline__ float rcp_rn(float d) {
    const double x = double(d);
    double y;
    asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(y) : "d"(x));
    y = __fma_rn(y, __fma_rn(-x, y, 1.0), y);
    y = __fma_rn(y, __fma_rn(-x, y, 1.0), y);
    return d == INFINITY ? 0.0f : __double2float_rn(y);  // the Newton steps turn 1/inf into NaN
}
// gelu_tanh(x) with tanh(v) = 1 - 2/(exp(2v)+1) (gemma2_fast_x86.c:308-325).
__device__ __forceinline__ float ref_gelu(float x) {
    float inner = __fmul_rn(__fmul_rn(0.79788456080286535588f, x), __fmaf_rn(__fmul_rn(0.044715f, x), x, 1.0f));
    inner = fminf(fmaxf(inner, -9.0f), 9.0f);
    const float t = __fsub_rn(1.0f, fdiv_markstein(2.0f, __fadd_rn(ref_exp8(__fmul_rn(2.0f, inner)), 1.0f)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
}
// gelu_tanh(x) = 0.5 x (1 + tanh(0.7978845608 x (1 + 0.044715 x^2))) with the C
// library's tanhf, in the scalar tier's operation order (kernels.c:367-371).
__device__ __forceinline__ float ref_gelu_scalar(float x) {
    const float inner = __fmul_rn(__fmul_rn(0.79788456080286535587989211986876f, x),
                                  __fadd_rn(1.0f, __fmul_rn(__fmul_rn(0.044715f, x), x)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, eg2_ref_tanhf(inner)));
}
__device__ __forceinline__ float gelu_tier(float x, int tier) {
    return tier == TIER_SCALAR ? ref_gelu_scalar(x) : ref_gelu(x);
}

// RMS scale 1/sqrt(sum/d + 1e-6) from a double sum of squares rounded to
// float, as gemma2_fast.c:587-590,667-671 computes it.
__device__ __forceinline__ float rms_scale(double sumsq, int d) {
    const float s = __double2float_rn(sumsq);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, float(d)), 1e-6f)));
}
// Horizontal sum of 8 lanes as the reference's hsum and 4-row Q8 tile end it
// (gemma2_fast_x86.c:95-101, :239-244): (a_j + a_{j+4}) for j < 4, then
// (s0 + s2) + (s1 + s3).
__device__ __forceinline__ float hsum8(const float (&a)[8]) {
    const float s0 = __fadd_rn(a[0], a[4]), s1 = __fadd_rn(a[1], a[5]);
    const float s2 = __fadd_rn(a[2], a[6]), s3 = __fadd_rn(a[3], a[7]);
    return __fadd_rn(__fadd_rn(s0, s2), __fadd_rn(s1, s3));
}
// _mm512_reduce_add_ps as the reference's build expands it
// (gemma2_fast_x86.c:203): 256-bit halves added lane by lane, then 128-bit
// halves, then lanes 0 + 2 and 1 + 3, then those two.
__device__ __forceinline__ float reduce16(const float (&a)[16]) {
    float t[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) t[i] = __fadd_rn(a[i], a[i + 8]);
    const float u0 = __fadd_rn(t[0], t[4]), u1 = __fadd_rn(t[1], t[5]);
    const float u2 = __fadd_rn(t[2], t[6]), u3 = __fadd_rn(t[3], t[7]);
    return __fadd_rn(__fadd_rn(u0, u2), __fadd_rn(u1, u3));
}
// g2x_sum_squares (gemma2_fast_x86.c:280-289) of row[0, d) in shared memory,
// d a multiple of 16, by one whole warp: lane i < 16 runs the fused
// multiply-add chain over z = 16m + i (the 8-lane accumulators s0 and s1 of
// 16-element chunks), then hsum8 of s0 + s1.  Every lane gets the sum.
__device__ __forceinline__ float x86_sumsq_warp(const float *row, int d) {
    const int lane = threadIdx.x & 31;
    float c = 0.0f;
    if (lane < 16)
        for (int z = lane; z < d; z += 16) c = __fmaf_rn(row[z], row[z], c);
    const float v = __fadd_rn(c, __shfl_down_sync(0xffffffffu, c, 8));  // lane i < 8: s0_i + s1_i
    const float s = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4));  // lane j < 4: v_j + v_{j+4}
    const float u = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, 2));  // lanes 0, 1: s0 + s2, s1 + s3
    return __shfl_sync(0xffffffffu, __fadd_rn(u, __shfl_down_sync(0xffffffffu, u, 1)), 0);
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace eg2
